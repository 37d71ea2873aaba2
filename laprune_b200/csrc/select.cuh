// select.cuh -- exact top-k of the candidate scores of every selection unit.
//
// Reference: torch.topk(scores_cand, k, sorted=False) over the candidate
// window, laprune/llm/modifiers/aq_evaluation.py:185-201.  Here the result
// is a bitmap of the selected tokens (ascending order is implicit), with the
// tie rule fixed: larger score first, lower token index among equal scores.
//
// Two-level radix select:
//   1. the scorer histogrammed every score into kNB monotone bins;
//   2. every CTA of this kernel finds the bin b* holding the k-th largest
//      score, writes the bitmap words of its token range for bins > b*
//      (warp ballots, no atomics), and appends the tokens of bin b* to a
//      per-unit tie buffer;
//   3. the last CTA of the unit (completion counter, no waiting) orders the
//      tie-buffer tokens by (score desc, index asc) and sets the bits of the
//      first `need` of them.  If bin b* held more tokens than the tie buffer
//      (degenerate inputs, e.g. many equal scores), the same CTA runs an
//      exact 4 x 8-bit radix select on the float keys of bin b* instead.
#pragma once
#include <cub/block/block_scan.cuh>
#include <cub/block/block_reduce.cuh>
#include "score.cuh"

namespace lp {

constexpr int kTieCap = 4096;

struct SelectParams {
    const float* sel_scores;
    int64_t sel_stride;
    const float* bounds;
    int Gb;            // heads per bounds unit (1 GROUP table, G HEADS tables)
    int per_head;      // selection unit = query head (g within the bounds unit)
    const uint32_t* hist;  // [Usel][kNB]
    uint32_t* bitmap;  // [Usel][bm_stride]
    int64_t bm_stride;
    float2* tie_buf;   // [Usel][kTieCap] (score, index bits)
    uint32_t* tie_count;
    uint32_t* done;
    int4* info;        // [Usel] {b*, count_above, need, n_tie}
    int c0, c1, k;
    int words_per_cta;
    uint32_t* err;
};

__device__ __forceinline__ uint32_t ordered_key(float s) {
    const uint32_t b = __float_as_uint(s);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// a precedes b in selection order
__device__ __forceinline__ bool sel_before(float sa, int ia, float sb, int ib) {
    return sa > sb || (sa == sb && ia < ib);
}

template <int THREADS>
__device__ void find_threshold_bin(const uint32_t* hist_s, int k, int* out_bstar, int* out_above) {
    // thread t owns bins [kNB - PER*(t+1), kNB - PER*t) (top bins first)
    constexpr int PER = kNB / THREADS;
    using Scan = cub::BlockScan<uint32_t, THREADS>;
    __shared__ typename Scan::TempStorage tmp;
    const int t = threadIdx.x;
    const int hi_bin = kNB - PER * t;  // exclusive
    uint32_t local = 0;
#pragma unroll
    for (int j = 1; j <= PER; ++j) local += hist_s[hi_bin - j];
    uint32_t before;
    Scan(tmp).ExclusiveSum(local, before);
    if ((int)before < k && k <= (int)(before + local)) {
        uint32_t acc = before;
        for (int j = 1; j <= PER; ++j) {
            const uint32_t c = hist_s[hi_bin - j];
            if ((int)(acc + c) >= k) {
                *out_bstar = hi_bin - j;
                *out_above = (int)acc;
                break;
            }
            acc += c;
        }
    }
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) select_kernel(SelectParams p) {
    __shared__ uint32_t s_hist[kNB];
    __shared__ int s_bstar, s_above, s_last;
    extern __shared__ __align__(16) unsigned char dsm[];  // last CTA: tie sort (kTieCap x 8 B)

    const int usel = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NWARP = THREADS / 32;
    const int bu = p.per_head ? usel / p.Gb : usel;
    const int g0 = p.per_head ? usel - bu * p.Gb : 0;
    __shared__ BinParams s_bp;
    if (tid < 32) {
        const BinParams b_ = bin_params_warp(p.bounds, bu, p.Gb, g0, p.per_head ? 1 : p.Gb);
        if (tid == 0) s_bp = b_;
    }
    for (int i = tid; i < kNB; i += THREADS) s_hist[i] = __ldcg(p.hist + (int64_t)usel * kNB + i);
    if (tid == 0) { s_bstar = kNB; s_above = 0; }
    __syncthreads();
    const BinParams bp = s_bp;
    if (p.k > 0) find_threshold_bin<THREADS>(s_hist, p.k, &s_bstar, &s_above);
    __syncthreads();
    const int bstar = s_bstar;
    const int above = s_above;

    const float* sc = p.sel_scores + (int64_t)usel * p.sel_stride;
    uint32_t* bm = p.bitmap + (int64_t)usel * p.bm_stride;
    const int wlo = p.c0 >> 5, whi = (p.c1 + 31) >> 5;
    const int wb = wlo + blockIdx.x * p.words_per_cta;
    const int we = min(whi, wb + p.words_per_cta);
    constexpr int BATCH = 8;  // words per warp whose scores are loaded together
    for (int w0 = wb + warp; w0 < we; w0 += NWARP * BATCH) {
      float sv[BATCH];
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const int t = (w0 + j * NWARP) * 32 + lane;
        sv[j] = (w0 + j * NWARP < we && t >= p.c0 && t < p.c1) ? __ldcg(sc + t) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < BATCH; ++j) {
        const int w = w0 + j * NWARP;
        if (w >= we) break;
        const int t = w * 32 + lane;
        const bool valid = t >= p.c0 && t < p.c1;
        const float s = sv[j];
        const int bin = score_bin(s, bp.lo, bp.inv_w, kNB);
        const bool sel = valid && bin > bstar;
        const bool tie = valid && bin == bstar;
        const uint32_t bits = __ballot_sync(0xffffffffu, sel);
        if (lane == 0) bm[w] = bits;
        const uint32_t tmask = __ballot_sync(0xffffffffu, tie);
        if (tmask) {
            uint32_t base = 0;
            if (lane == 0) base = atomicAdd(&p.tie_count[usel], (uint32_t)__popc(tmask));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (tie) {
                const uint32_t pos = base + __popc(tmask & ((1u << lane) - 1u));
                if (pos < (uint32_t)kTieCap)
                    p.tie_buf[(int64_t)usel * kTieCap + pos] = make_float2(s, __int_as_float(t));
            }
        }
      }
    }

    // completion: the last CTA of this unit resolves bin b*
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t ticket = atomicAdd(&p.done[usel], 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    const int need = p.k - above;
    const int ntie = (int)atomicAdd(&p.tie_count[usel], 0u);
    if (tid == 0 && p.info) p.info[usel] = make_int4(bstar, above, need, ntie);
    if (need <= 0) return;

    if (ntie <= kTieCap) {
        float* ks = reinterpret_cast<float*>(dsm);
        int* is = reinterpret_cast<int*>(dsm + kTieCap * sizeof(float));
        int n = 1;
        while (n < ntie) n <<= 1;
        for (int i = tid; i < n; i += THREADS) {
            if (i < ntie) {
                const float2 e = p.tie_buf[(int64_t)usel * kTieCap + i];
                ks[i] = e.x;
                is[i] = __float_as_int(e.y);
            } else {
                ks[i] = -INFINITY;
                is[i] = 0x7fffffff;
            }
        }
        // bitonic sort into selection order
        for (int size = 2; size <= n; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                __syncthreads();
                for (int i = tid; i < (n >> 1); i += THREADS) {
                    const int a = 2 * i - (i & (stride - 1));
                    const int c = a + stride;
                    const bool up = (a & size) == 0;
                    const float ka = ks[a], kc = ks[c];
                    const int ia = is[a], ic = is[c];
                    const bool c_first = sel_before(kc, ic, ka, ia);
                    if (c_first == up) {
                        ks[a] = kc; ks[c] = ka;
                        is[a] = ic; is[c] = ia;
                    }
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < need; i += THREADS) {
            const int t = is[i];
            if (t >= p.c0 && t < p.c1) atomicOr(&bm[t >> 5], 1u << (t & 31));
        }
        return;
    }

    // ---- exact slow path: radix select on the float keys of bin b* ----
    if (tid == 0) atomicOr(p.err, LP_DEVERR_TIE_OVERFLOW);
    uint32_t* h256 = reinterpret_cast<uint32_t*>(dsm);
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_remaining, s_gt;
    if (tid == 0) { s_prefix = 0; s_mask = 0; s_remaining = need; s_gt = 0; }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += THREADS) h256[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        for (int t = p.c0 + tid; t < p.c1; t += THREADS) {
            const float s = sc[t];
            if (score_bin(s, bp.lo, bp.inv_w, kNB) != bstar) continue;
            const uint32_t key = ordered_key(s);
            if ((key & mask) != prefix) continue;
            atomicAdd(&h256[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining;
            int acc = 0;
            for (int d = 255; d >= 0; --d) {
                const int c = (int)h256[d];
                if (acc + c >= rem) {
                    s_prefix = prefix | ((uint32_t)d << shift);
                    s_mask = mask | (255u << shift);
                    s_remaining = rem - acc;
                    s_gt += acc;
                    break;
                }
                acc += c;
            }
        }
        __syncthreads();
    }
    // s_prefix is the exact key of the need-th element; s_remaining of the
    // tokens with that key are taken, lowest index first.
    const uint32_t kstar = s_prefix;
    const int take_eq = s_remaining;
    using Scan = cub::BlockScan<int, THREADS>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int s_eq_base;
    if (tid == 0) s_eq_base = 0;
    __syncthreads();
    for (int base = p.c0; base < p.c1; base += THREADS) {
        const int t = base + tid;
        int gt = 0, eq = 0;
        if (t < p.c1) {
            const float s = sc[t];
            if (score_bin(s, bp.lo, bp.inv_w, kNB) == bstar) {
                const uint32_t key = ordered_key(s);
                gt = key > kstar;
                eq = key == kstar;
            }
        }
        int rank, total;
        Scan(tmp).ExclusiveSum(eq, rank, total);
        const int r = s_eq_base + rank;
        if (gt || (eq && r < take_eq)) atomicOr(&bm[t >> 5], 1u << (t & 31));
        __syncthreads();
        if (tid == 0) s_eq_base += total;
        __syncthreads();
    }
}

// The same compaction in parallel, two launches of (chunks, units) CTAs:
// selected-token counts per 256-word chunk of the candidate window, then
// every chunk writes its tokens at the count of the chunks before it.
constexpr int kCompactWords = 256;  // bitmap words per chunk (one per thread)

__device__ __forceinline__ uint32_t window_bits(const uint32_t* bm, int w, int c0, int c1) {
    uint32_t bits = bm[w];
    const int lo = w * 32, hi = lo + 32;
    if (lo < c0) bits &= ~0u << (c0 - lo);
    if (hi > c1) bits &= (c1 - lo) >= 32 ? ~0u : ((1u << (c1 - lo)) - 1u);
    return bits;
}

__global__ void __launch_bounds__(kCompactWords) bitmap_chunk_count_kernel(const uint32_t* bitmap, int64_t bm_stride,
                                                                           int c0, int c1, int nchunk, int* cnt) {
    using Reduce = cub::BlockReduce<int, kCompactWords>;
    __shared__ typename Reduce::TempStorage tmp;
    const int usel = blockIdx.y, ch = blockIdx.x;
    const int wlo = c0 >> 5, whi = (c1 + 31) >> 5;
    const int w = wlo + ch * kCompactWords + threadIdx.x;
    const uint32_t bits = w < whi ? window_bits(bitmap + (int64_t)usel * bm_stride, w, c0, c1) : 0u;
    const int total = Reduce(tmp).Sum(__popc(bits));
    if (threadIdx.x == 0) cnt[(int64_t)usel * nchunk + ch] = total;
}

__global__ void __launch_bounds__(kCompactWords) bitmap_compact_kernel(const uint32_t* bitmap, int64_t bm_stride,
                                                                       int c0, int c1, int k, int nchunk,
                                                                       const int* cnt, int32_t* out) {
    using Scan = cub::BlockScan<int, kCompactWords>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int s_base;
    const int usel = blockIdx.y, ch = blockIdx.x;
    if (threadIdx.x < 32) {
        int b = 0;
        for (int j = threadIdx.x; j < ch; j += 32) b += cnt[(int64_t)usel * nchunk + j];
        b = __reduce_add_sync(0xffffffffu, b);
        if (threadIdx.x == 0) s_base = b;
    }
    const int wlo = c0 >> 5, whi = (c1 + 31) >> 5;
    const int w = wlo + ch * kCompactWords + threadIdx.x;
    uint32_t bits = w < whi ? window_bits(bitmap + (int64_t)usel * bm_stride, w, c0, c1) : 0u;
    int rank, total;
    Scan(tmp).ExclusiveSum(__popc(bits), rank, total);
    __syncthreads();  // s_base
    int r = s_base + rank;
    int32_t* o = out + (int64_t)usel * k;
    while (bits) {
        const int bit = __ffs(bits) - 1;
        bits &= bits - 1;
        if (r < k) o[r] = w * 32 + bit;
        ++r;
    }
}


}  // namespace lp
