// attention.cuh -- GQA K/V gather + split-K flash-decode over the kept rows.
//
// Reference: the keep set of laprune/llm/modifiers/aq_evaluation.py:206-237
// (top-k + sink [0,sink) + local window [T-local, T)), the GQA gather of
// aq_kernels/aq_lut_gqa.cu:277-323 (gqa_gather_kv_half8_kernel) and the
// SDPA of aq_evaluation.py:251 (one query row, no mask).
//
// The reference copies the kept rows of every QUERY head into a [B,Hq,N,D]
// tensor (4x the bytes under GQA) and then runs SDPA over it.  Here one CTA
// handles a contiguous slice (in ascending token order) of the kept rows of
// one selection unit, gathers each K/V row ONCE into shared memory with
// 16-byte cp.async, and attends every query head that shares the unit
// (all G heads of the KV group in KV_GROUP mode).  Partial softmax states
// (max, sum, P.V) of the slices are merged by the unit's last CTA.
//
// The row list of a slice comes from the units' compacted selections (made
// in parallel before this kernel), or, without them, from the selection
// bitmap with a block-wide prefix popcount.
#pragma once
#include <cub/block/block_scan.cuh>
#include "common.cuh"

namespace lp {

constexpr int kAttnRows = 64;  // kept rows per CTA (max)

struct AttnParams {
    const void* q;
    int64_t q_stride_b, q_stride_h;
    const void* keys;
    const void* vals;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    const uint32_t* bitmap;
    int64_t bm_stride;
    const int32_t* toplist;  // [U][k] selected tokens in ascending order (NULL: recover them from the bitmap)
    int Hkv, G, HG;     // HG = query heads attended per unit (G or 1)
    int c0, c1;         // candidate window (bitmap range)
    int n_sink, k, local_start, n_local;
    int n_rows;         // n_sink + k + n_local
    int T_total;        // K/V rows valid in [0, T_total)
    int nsplit;
    float scale_log2;   // softmax scale * log2(e)
    float* part;        // [U][nsplit][HG][2 + 128]
    uint32_t* done;     // [U]
    void* out;
    int64_t out_stride_b, out_stride_h;
};

template <typename T>
struct Vec4;
template <>
struct Vec4<__nv_bfloat16> {
    static __device__ __forceinline__ float4 load(const __nv_bfloat16* p) {
        const uint2 r = *reinterpret_cast<const uint2*>(p);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    static __device__ __forceinline__ float2 load2(const __nv_bfloat16* p) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    }
};
template <>
struct Vec4<__half> {
    static __device__ __forceinline__ float4 load(const __half* p) {
        const uint2 r = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    static __device__ __forceinline__ float2 load2(const __half* p) {
        return __half22float2(*reinterpret_cast<const __half2*>(p));
    }
};

// D = 128.  One CTA = (slice, unit); unit = (b, hkv[, g]).
template <typename QT, typename KT, typename OT, int THREADS>
__global__ void __launch_bounds__(THREADS) sparse_attn_kernel(AttnParams p) {
    constexpr int D = 128;
    constexpr int R = kAttnRows;
    constexpr int NW = THREADS / 32;
    __shared__ __align__(16) KT s_k[R][D];
    __shared__ __align__(16) KT s_v[R][D];
    __shared__ int s_rows[R];
    __shared__ float s_q[8][D];
    __shared__ float s_p[8][R];
    __shared__ float s_m[8], s_l[8];
    __shared__ int s_last;
    using Scan = cub::BlockScan<int, THREADS>;
    __shared__ typename Scan::TempStorage scan_tmp;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int u = blockIdx.y;               // attention unit
    const int split = blockIdx.x;
    const int per_kv = p.G / p.HG;          // units per KV head (1 or G)
    const int ukv = u / per_kv;             // b*Hkv + hkv
    const int g0 = (u - ukv * per_kv) * p.HG;
    const int b = ukv / p.Hkv, hkv = ukv - b * p.Hkv;
    const int rows_per = (p.n_rows + p.nsplit - 1) / p.nsplit;
    const int r0 = split * rows_per;
    const int r1 = min(p.n_rows, r0 + rows_per);
    const int nr = r1 - r0;

    // ---- 1. row list of this slice ----
    // (pre-filled with a valid row so that no gather can leave the cache even
    // if the bitmap held fewer selected tokens than expected)
    for (int i = tid; i < R; i += THREADS) s_rows[i] = 0;
    __syncthreads();
    // sink part: rank r in [0, n_sink) -> token r
    for (int r = r0 + tid; r < min(r1, p.n_sink); r += THREADS) s_rows[r - r0] = r;
    // local part: rank in [n_sink + k, n_rows) -> local_start + offset
    for (int r = max(r0, p.n_sink + p.k) + tid; r < r1; r += THREADS)
        s_rows[r - r0] = p.local_start + (r - p.n_sink - p.k);
    // selected part: ranks [n_sink, n_sink + k) are the set bits in order
    const int j0 = max(r0, p.n_sink) - p.n_sink;
    const int j1 = min(r1, p.n_sink + p.k) - p.n_sink;
    if (j0 < j1 && p.toplist) {
        const int32_t* tl = p.toplist + (int64_t)u * p.k;
        for (int j = j0 + tid; j < j1; j += THREADS) s_rows[p.n_sink + j - r0] = tl[j];
    } else if (j0 < j1) {
        const uint32_t* bm = p.bitmap + (int64_t)u * p.bm_stride;
        const int wlo = p.c0 >> 5, whi = (p.c1 + 31) >> 5;
        const int nwords = whi - wlo;
        // each thread owns a contiguous run of words; runs are scanned in
        // rounds of WB words held in registers (loads issued together)
        constexpr int WB = 16;
        const int per = (nwords + THREADS - 1) / THREADS;
        const int wa = wlo + tid * per, wb = min(whi, wa + per);
        int base_round = 0;  // selected tokens before this round (block-wide)
        for (int r = 0; r < per; r += WB) {
            uint32_t words[WB];
            int cnt = 0;
#pragma unroll
            for (int j = 0; j < WB; ++j) {
                const int w = wa + r + j;
                words[j] = (r + j < per && w < wb) ? __ldcg(bm + w) : 0u;
            }
#pragma unroll
            for (int j = 0; j < WB; ++j) cnt += __popc(words[j]);
            int before, total;
            Scan(scan_tmp).ExclusiveSum(cnt, before, total);
            __syncthreads();
            int rank = base_round + before;
            if (rank < j1 && rank + cnt > j0) {
#pragma unroll
                for (int j = 0; j < WB; ++j) {
                    uint32_t bits = words[j];
                    const int c = __popc(bits);
                    if (rank + c <= j0 || rank >= j1) { rank += c; continue; }
                    while (bits) {
                        const int bit = __ffs(bits) - 1;
                        bits &= bits - 1;
                        if (rank >= j0 && rank < j1) s_rows[p.n_sink + rank - r0] = (wa + r + j) * 32 + bit;
                        ++rank;
                    }
                }
            }
            base_round += total;
        }
    }
    // queries (fp32)
    const QT* qb = reinterpret_cast<const QT*>(p.q) + (int64_t)b * p.q_stride_b;
    for (int i = tid; i < p.HG * D; i += THREADS) {
        const int g = i / D, d = i - g * D;
        s_q[g][d] = to_f32(qb[(int64_t)(hkv * p.G + g0 + g) * p.q_stride_h + d]);
    }
    __syncthreads();

    // ---- 2. gather K and V rows (16-byte cp.async) ----
    const KT* kb = reinterpret_cast<const KT*>(p.keys) + (int64_t)b * p.k_stride_b + (int64_t)hkv * p.k_stride_h;
    const KT* vb = reinterpret_cast<const KT*>(p.vals) + (int64_t)b * p.v_stride_b + (int64_t)hkv * p.v_stride_h;
    constexpr int CH = D * (int)sizeof(KT) / 16;  // 16-byte chunks per row
    for (int c = tid; c < nr * CH; c += THREADS) {
        const int r = c / CH, part = c - r * CH;
        const int64_t t = min(max(s_rows[r], 0), p.T_total - 1);
        cp_async16(&s_k[r][part * (16 / sizeof(KT))], kb + t * p.k_stride_t + part * (16 / sizeof(KT)));
        cp_async16(&s_v[r][part * (16 / sizeof(KT))], vb + t * p.v_stride_t + part * (16 / sizeof(KT)));
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();

    // ---- 3. logits (log2 domain) ----
    for (int r = warp; r < nr; r += NW) {
        const float4 kv = Vec4<KT>::load(&s_k[r][lane * 4]);
        for (int g = 0; g < p.HG; ++g) {
            const float4 qv = *reinterpret_cast<const float4*>(&s_q[g][lane * 4]);
            float a = qv.x * kv.x;
            a = fmaf(qv.y, kv.y, a);
            a = fmaf(qv.z, kv.z, a);
            a = fmaf(qv.w, kv.w, a);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == g) s_p[g][r] = a * p.scale_log2;
        }
    }
    __syncthreads();
    // ---- 4. slice softmax state per head ----
    for (int g = warp; g < p.HG; g += NW) {
        float mx = -INFINITY;
        for (int r = lane; r < nr; r += 32) mx = fmaxf(mx, s_p[g][r]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int r = lane; r < nr; r += 32) {
            const float e = exp2f(s_p[g][r] - mx);
            s_p[g][r] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { s_m[g] = mx; s_l[g] = sum; }
    }
    __syncthreads();
    // ---- 5. P.V and partial state ----
    float* part = p.part + ((int64_t)u * p.nsplit + split) * p.HG * (2 + D);
    for (int o = tid; o < p.HG * (D / 2); o += THREADS) {
        const int g = o / (D / 2), dp = o - g * (D / 2);
        float ax = 0.f, ay = 0.f;
        for (int r = 0; r < nr; ++r) {
            const float2 v = Vec4<KT>::load2(&s_v[r][2 * dp]);
            const float w = s_p[g][r];
            ax = fmaf(w, v.x, ax);
            ay = fmaf(w, v.y, ay);
        }
        float* pg = part + g * (2 + D);
        pg[2 + 2 * dp] = ax;
        pg[3 + 2 * dp] = ay;
        if (dp == 0) { pg[0] = s_m[g]; pg[1] = s_l[g]; }
    }

    // ---- 6. the last CTA of the unit merges the slices ----
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t ticket = atomicAdd(&p.done[u], 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* pu = p.part + (int64_t)u * p.nsplit * p.HG * (2 + D);
    OT* ob = reinterpret_cast<OT*>(p.out) + (int64_t)b * p.out_stride_b;
    // slice weights 2^(m_s - M) / L per head, computed once into shared memory
    float* s_w = &s_p[0][0];  // reuse: needs nsplit * HG floats (<= 8 * R)
    const bool wfit = p.nsplit * p.HG <= 8 * R;
    if (wfit) {
        for (int g = warp; g < p.HG; g += NW) {
            float M = -INFINITY;
            for (int s = lane; s < p.nsplit; s += 32) M = fmaxf(M, __ldcg(pu + ((int64_t)s * p.HG + g) * (2 + D)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.f;
            for (int s = lane; s < p.nsplit; s += 32) {
                const float* ps = pu + ((int64_t)s * p.HG + g) * (2 + D);
                const float f = exp2f(__ldcg(ps) - M);
                s_w[g * p.nsplit + s] = f;
                L = fmaf(__ldcg(ps + 1), f, L);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
            __syncwarp();
            const float invL = 1.f / L;
            for (int s = lane; s < p.nsplit; s += 32) s_w[g * p.nsplit + s] *= invL;
        }
        __syncthreads();
        for (int o = tid; o < p.HG * D; o += THREADS) {
            const int g = o / D, d = o - g * D;
            const float* pg = pu + (int64_t)g * (2 + D) + 2 + d;
            const int64_t sstride = (int64_t)p.HG * (2 + D);
            float acc = 0.f;
            int s = 0;
            for (; s + 8 <= p.nsplit; s += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldcg(pg + (s + j) * sstride);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc = fmaf(v[j], s_w[g * p.nsplit + s + j], acc);
            }
            for (; s < p.nsplit; ++s) acc = fmaf(__ldcg(pg + s * sstride), s_w[g * p.nsplit + s], acc);
            ob[(int64_t)(hkv * p.G + g0 + g) * p.out_stride_h + d] = from_f32<OT>(acc);
        }
    } else {
        for (int o = tid; o < p.HG * D; o += THREADS) {
            const int g = o / D, d = o - g * D;
            float M = -INFINITY;
            for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, __ldcg(pu + ((int64_t)s * p.HG + g) * (2 + D)));
            float L = 0.f, acc = 0.f;
            for (int s = 0; s < p.nsplit; ++s) {
                const float* ps = pu + ((int64_t)s * p.HG + g) * (2 + D);
                const float f = exp2f(__ldcg(ps) - M);
                L = fmaf(__ldcg(ps + 1), f, L);
                acc = fmaf(__ldcg(ps + 2 + d), f, acc);
            }
            ob[(int64_t)(hkv * p.G + g0 + g) * p.out_stride_h + d] = from_f32<OT>(acc / L);
        }
    }
}

}  // namespace lp
