// score.cuh -- HBM-streaming LUT scorer with a fused selection histogram.
//
// Reference: the grouped scorer aq_kernels/aq_lut_gqa.cu:157-212
// (lut_gather_grouped_interleaved_kernel) and the fp32 CPU path
// laprune/llm/aq_kv.py:614-630: score[h][t] = sum_{m<32} LUT_h[m][code[t][m]].
//
// Design (M = 32 codebooks, K = 256 entries, one code row = 32 bytes):
//   * Code rows stream HBM -> shared memory through a ring of 1-D bulk (TMA)
//     copies, one tile of THREADS rows per stage, L2 evict-first.
//   * Each thread scores one token of the tile.  Lane l handles codebook
//     m = 4*((i + l/4) & 7) + ((s + l) & 3) at step (i, s): over its 32 steps
//     a lane visits every m once, and at any step the 32 lanes of a warp
//     visit 32 DIFFERENT m.  With the table laid out so that the bank of an
//     entry is fixed by m, every shared-memory gather is conflict-free.
//     The rotated byte is extracted from the code word with one PRMT that
//     also builds the table address.
//   * GROUP tables (one per KV head, built from the summed query) are stored
//     [k][m'] with m' in [0,64) holding LUT[m' & 31][k] (row duplicated) so
//     the per-step address is "register + immediate": one PRMT, one LDS and
//     one FADD per (token, m).
//   * HEADS tables hold the G <= 4 query heads of a KV group interleaved
//     (16 bytes per (k, m)); one 128-bit conflict-free gather per (token, m).
//   * Table entries are staged into shared memory as int32 fixed point with
//     a power-of-two scale 2^S chosen from the table bound (every entry
//     below 2^25 / 2^23 in magnitude, so 32 / 128 terms cannot overflow), and
//     the gathered entries are summed EXACTLY in integers.  The score is
//     therefore independent of the (rotated) summation order: tokens with
//     identical code rows get identical scores, and ties are real ties.
//   * The selection score of every candidate token is written (fp32) and
//     counted into a per-unit histogram over the hard score bound [lo, hi]
//     derived from the table's per-m min/max, for the radix select that
//     follows.
#pragma once
#include "common.cuh"
#include "lut_build.cuh"

namespace lp {

constexpr int kNB = 2048;  // selection histogram bins per unit

struct ScoreParams {
    const float* lut;      // GROUP: [U][256][32]   HEADS: [U][256][32][4]
    const float* bounds;   // [U][Gb][32][2]
    const uint8_t* codes;  // codes[b][hkv][t][32] (row stride 32 bytes)
    int64_t codes_stride_b, codes_stride_h;  // bytes
    int Hkv, G, U;
    int c0, c1;            // candidate window [c0, c1)
    float* sel_scores;     // [Usel][sel_stride]
    int64_t sel_stride;
    float* head_scores;    // HEADS: optional per-query-head scores [B][Hq][hs_stride]
    int64_t hs_stride;
    uint32_t* hist;        // [Usel][kNB]
    int sel_per_head;      // HEADS: 1 -> unit per query head, 0 -> per KV group
    uint32_t* err;
};

// Hard bound [lo, hi] of the selection score of unit `usel` and the bin
// scale.  Shared by the scorer and the select kernel so both derive the
// identical bins.
struct BinParams {
    float lo, inv_w;
};

// Executed by ONE full warp (lane m handles codebook m; M == 32): the hard
// score bound of a selection unit summed over g in [g_first, g_first+g_count)
// and the bin scale.  The reduction tree is fixed, so every kernel that calls
// this gets bit-identical bins.
__device__ __forceinline__ BinParams bin_params_warp(const float* bounds, int u, int Gb, int g_first,
                                                     int g_count) {
    const int lane = threadIdx.x & 31;
    float lo = 0.f, hi = 0.f;
    for (int g = g_first; g < g_first + g_count; ++g) {
        const float* bd = bounds + (((int64_t)u * Gb + g) * 32 + lane) * kLutParts * 2;
        float mn = bd[0], mx = bd[1];
#pragma unroll
        for (int q = 1; q < kLutParts; ++q) {
            mn = fminf(mn, bd[2 * q]);
            mx = fmaxf(mx, bd[2 * q + 1]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = __fadd_rn(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = __fadd_rn(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        lo = __fadd_rn(lo, mn);
        hi = __fadd_rn(hi, mx);
    }
    // widen by a relative margin so rounding of the scores cannot leave the
    // range (values outside are clamped anyway; this only keeps bins even)
    const float span = __fsub_rn(hi, lo);
    const float pad = __fmul_rn(fmaxf(fabsf(lo), fabsf(hi)), 1e-5f);
    lo = __fsub_rn(lo, pad);
    hi = __fadd_rn(hi, pad);
    BinParams bp;
    bp.lo = lo;
    bp.inv_w = (span > 0.f) ? __fdiv_rn((float)kNB, __fsub_rn(hi, lo)) : 0.f;
    return bp;
}

// Executed by ONE full warp: power-of-two fixed-point scale of a unit's
// tables, S such that every entry |v| < 2^(limit_bits - S).
__device__ __forceinline__ int fixed_shift_warp(const float* bounds, int u, int Gb, int limit_bits) {
    const int lane = threadIdx.x & 31;
    float mx = 0.f;
    for (int g = 0; g < Gb; ++g) {
        const float* bd = bounds + (((int64_t)u * Gb + g) * 32 + lane) * kLutParts * 2;
#pragma unroll
        for (int i = 0; i < 2 * kLutParts; ++i) {
            const float v = fabsf(bd[i]);
            if (isfinite(v)) mx = fmaxf(mx, v);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (!(mx > 0.f)) return 0;
    int e;
    frexpf(mx, &e);  // mx < 2^e
    const int S = limit_bits - e;
    return S < -100 ? -100 : (S > 100 ? 100 : S);
}

__device__ __forceinline__ int to_fixed(float v, float scale) {
    return __float2int_rn(__fmul_rn(v, scale));
}

// Shared-memory footprint of the scorer.
template <bool HEADS, int THREADS, int STAGES>
struct ScoreSmem {
    static constexpr int kLutBytes = HEADS ? 256 * 32 * 16 : 256 * 64 * 4;
    static constexpr int kTileBytes = THREADS * 32;  // one code row per thread
    static constexpr int kRingBytes = STAGES * kTileBytes;
    static constexpr int kHistHeads = HEADS ? 4 : 1;
    static constexpr int kHistBytes = kHistHeads * kNB * 4;
    static constexpr int kBarBytes = (STAGES + 1) * 8;
    static constexpr int kTotal = kLutBytes + kRingBytes + kHistBytes + kBarBytes + 128;
};

// CTA -> (unit, token range).  The nctas CTAs are spread over the U units as
// evenly as possible (units u < nctas % U get one more CTA).
__device__ __forceinline__ void score_cta_range(int cta, int nctas, int U, int c0, int ncand,
                                                int* unit, int* t_begin, int* t_end) {
    const int base = nctas / U, extra = nctas % U;
    int u, j, n;
    if (cta < extra * (base + 1)) {
        u = cta / (base + 1); j = cta - u * (base + 1); n = base + 1;
    } else {
        const int i = cta - extra * (base + 1);
        u = extra + i / base; j = i - (u - extra) * base; n = base;
    }
    *unit = u;
    *t_begin = c0 + (int)((int64_t)ncand * j / n);
    *t_end = c0 + (int)((int64_t)ncand * (j + 1) / n);
}

template <bool HEADS, int THREADS, int STAGES>
__global__ void __launch_bounds__(THREADS, 1) score_kernel(ScoreParams p) {
    using S = ScoreSmem<HEADS, THREADS, STAGES>;
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* s_lut = smem;
    unsigned char* s_ring = smem + S::kLutBytes;
    uint32_t* s_hist = reinterpret_cast<uint32_t*>(s_ring + S::kRingBytes);
    uint64_t* s_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(s_hist) + S::kHistBytes);
    uint64_t* s_lut_bar = s_bar + STAGES;

    const int tid = threadIdx.x, lane = tid & 31;
    int u, t_begin, t_end;
    score_cta_range(blockIdx.x, gridDim.x, p.U, p.c0, p.c1 - p.c0, &u, &t_begin, &t_end);
    const int b = u / p.Hkv, hkv = u - b * p.Hkv;
    const int ntiles = t_end > t_begin ? (t_end - t_begin + THREADS - 1) / THREADS : 0;
    const uint8_t* src = p.codes + (int64_t)b * p.codes_stride_b + (int64_t)hkv * p.codes_stride_h;
    const float* lut_g = p.lut + (int64_t)u * (HEADS ? 256 * 32 * 4 : 256 * 32);

    if (tid == 0) {
        for (int s = 0; s < STAGES + 1; ++s) mbar_init(&s_bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // Code tiles do not depend on the table-build kernel: start streaming them
    // before waiting for it (programmatic dependent launch).
    uint64_t policy = 0;
    const int npre = ntiles < STAGES ? ntiles : STAGES;
    if (tid == 0) {
        policy = policy_evict_first();
        for (int i = 0; i < npre; ++i) {
            const int t0 = t_begin + i * THREADS;
            const int n = min(THREADS, t_end - t0);
            mbar_arrive_expect_tx(&s_bar[i], (uint32_t)n * 32u);
            bulk_g2s_stream(s_ring + i * S::kTileBytes, src + (int64_t)t0 * 32, (uint32_t)n * 32u,
                            &s_bar[i], policy);
        }
    }
    for (int i = tid; i < S::kHistHeads * kNB; i += THREADS) s_hist[i] = 0u;
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (HEADS && tid == 0) {
        mbar_arrive_expect_tx(s_lut_bar, S::kLutBytes);
        bulk_g2s(s_lut, lut_g, S::kLutBytes, s_lut_bar);
    }
    const int Gb = HEADS ? p.G : 1;
    // per-unit constants, computed by warp 0 and broadcast
    __shared__ BinParams s_bp[4];
    __shared__ int s_shift;
    if (tid < 32) {
        const int sh = fixed_shift_warp(p.bounds, u, Gb, HEADS ? 23 : 25);
        if (HEADS && p.sel_per_head) {
            for (int g = 0; g < p.G; ++g) {
                const BinParams b_ = bin_params_warp(p.bounds, u, Gb, g, 1);
                if (tid == 0) s_bp[g] = b_;
            }
        } else {
            const BinParams b_ = bin_params_warp(p.bounds, u, Gb, 0, Gb);
            if (tid == 0) s_bp[0] = b_;
        }
        if (tid == 0) s_shift = sh;
    }
    __syncthreads();
    const int S_fx = s_shift;
    const float to_fx = ldexpf(1.f, S_fx), from_fx = ldexpf(1.f, -S_fx);
    if (!HEADS) {
        // [k][m] (32 floats per k) -> int32 [k][m'] with m' and m'+32 both LUT[m'][k]
        const float4* g4 = reinterpret_cast<const float4*>(lut_g);
        int4* d4 = reinterpret_cast<int4*>(s_lut);
#pragma unroll 4
        for (int f = tid; f < 256 * 8; f += THREADS) {
            const float4 v = __ldcg(g4 + f);
            const int4 iv = make_int4(to_fixed(v.x, to_fx), to_fixed(v.y, to_fx), to_fixed(v.z, to_fx),
                                      to_fixed(v.w, to_fx));
            const int k = f >> 3, m4 = f & 7;
            d4[k * 16 + m4] = iv;
            d4[k * 16 + 8 + m4] = iv;
        }
    }

    // selection-unit bin parameters
    BinParams bp[S::kHistHeads];
#pragma unroll
    for (int g = 0; g < S::kHistHeads; ++g) bp[g] = s_bp[(HEADS && p.sel_per_head && g < p.G) ? g : 0];

    // per-lane constants of the rotated gather
    const uint32_t L = (uint32_t)lane >> 2;
    uint32_t off[4], sel[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint32_t bs = (uint32_t)(s + lane) & 3u;
        if (HEADS) {
            off[s] = 16u * bs;
            sel[s] = 0x4440u | bs;  // byte bs of the code word -> low byte, rest zero
        } else {
            off[s] = 16u * L + 4u * bs;
            sel[s] = 0x5504u | (bs << 4);  // [0][0][code][off] = code*256 + off
        }
    }
    int issued = npre;
    bool ok = true;
    if (HEADS) ok = mbar_wait(s_lut_bar, 0, p.err);
    if (__syncthreads_or(!ok)) {
        for (int j = 0; j < issued; ++j) mbar_wait(&s_bar[j], 0u, nullptr);
        return;
    }
    if (HEADS) {
        float4* l4 = reinterpret_cast<float4*>(s_lut);
        for (int i = tid; i < S::kLutBytes / 16; i += THREADS) {
            const float4 v = l4[i];
            reinterpret_cast<int4*>(l4)[i] = make_int4(to_fixed(v.x, to_fx), to_fixed(v.y, to_fx),
                                                       to_fixed(v.z, to_fx), to_fixed(v.w, to_fx));
        }
        __syncthreads();
    }

    for (int i = 0; i < ntiles; ++i) {
        const int slot = i % STAGES;
        ok = mbar_wait(&s_bar[slot], (uint32_t)(i / STAGES) & 1u, p.err);
        if (__syncthreads_or(!ok)) {
            // drain our own copies still in flight (bounded), then give up
            for (int j = i; j < issued; ++j) mbar_wait(&s_bar[j % STAGES], (uint32_t)(j / STAGES) & 1u, nullptr);
            return;
        }
        const int t = t_begin + i * THREADS + tid;
        if (t < t_end) {
            const uint32_t* row = reinterpret_cast<const uint32_t*>(s_ring + slot * S::kTileBytes + tid * 32);
            if (!HEADS) {
                int iacc = 0;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    const uint32_t cw = row[(w + L) & 7u];
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t a = __byte_perm(cw, off[s], sel[s]);
                        iacc += *reinterpret_cast<const int*>(s_lut + a + 16 * w);
                    }
                }
                const float acc = __fmul_rn(__int2float_rn(iacc), from_fx);
                p.sel_scores[(int64_t)u * p.sel_stride + t] = acc;
                atomicAdd(&s_hist[score_bin(acc, bp[0].lo, bp[0].inv_w, kNB)], 1u);
            } else {
                int i0 = 0, i1 = 0, i2 = 0, i3 = 0;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    const uint32_t wi = (w + L) & 7u;
                    const uint32_t cw = row[wi];
                    const uint32_t rot = wi << 6;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint32_t code = __byte_perm(cw, 0u, sel[s]);
                        const int4 v = *reinterpret_cast<const int4*>(s_lut + (code << 9) + rot + off[s]);
                        i0 += v.x;
                        i1 += v.y;
                        i2 += v.z;
                        i3 += v.w;
                    }
                }
                const float a0 = __fmul_rn(__int2float_rn(i0), from_fx);
                const float a1 = __fmul_rn(__int2float_rn(i1), from_fx);
                const float a2 = __fmul_rn(__int2float_rn(i2), from_fx);
                const float a3 = __fmul_rn(__int2float_rn(i3), from_fx);
                const float hs[4] = {a0, a1, a2, a3};
                if (p.head_scores) {
#pragma unroll
                    for (int g = 0; g < 4; ++g)
                        if (g < p.G) p.head_scores[((int64_t)u * p.G + g) * p.hs_stride + t] = hs[g];
                }
                if (p.sel_per_head) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        if (g < p.G) {
                            p.sel_scores[((int64_t)u * p.G + g) * p.sel_stride + t] = hs[g];
                            atomicAdd(&s_hist[g * kNB + score_bin(hs[g], bp[g].lo, bp[g].inv_w, kNB)], 1u);
                        }
                    }
                } else {
                    const float sum = __fmul_rn(__int2float_rn(((i0 + i1) + i2) + i3), from_fx);
                    p.sel_scores[(int64_t)u * p.sel_stride + t] = sum;
                    atomicAdd(&s_hist[score_bin(sum, bp[0].lo, bp[0].inv_w, kNB)], 1u);
                }
            }
        }
        __syncthreads();
        if (tid == 0 && i + STAGES < ntiles) {
            const int j = i + STAGES;
            const int t0 = t_begin + j * THREADS;
            const int n = min(THREADS, t_end - t0);
            mbar_arrive_expect_tx(&s_bar[slot], (uint32_t)n * 32u);
            bulk_g2s_stream(s_ring + slot * S::kTileBytes, src + (int64_t)t0 * 32, (uint32_t)n * 32u,
                            &s_bar[slot], policy);
            ++issued;
        }
    }

    const int nh = (HEADS && p.sel_per_head) ? p.G : 1;
    const int64_t hbase = (int64_t)u * nh;
    for (int i = tid; i < nh * kNB; i += THREADS) {
        const uint32_t c = s_hist[i];
        if (c) atomicAdd(&p.hist[(hbase + i / kNB) * kNB + (i % kNB)], c);
    }
}

}  // namespace lp
