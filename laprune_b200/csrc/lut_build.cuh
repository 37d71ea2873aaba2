// lut_build.cuh -- per-query lookup tables LUT[m][k] = q . C_m[k] (fp32).
//
// Reference: laprune/llm/aq_kv.py:681-682 (cuBLAS q @ C^T, fp16) and the CPU
// path aq_kv.py:620 (einsum, fp32).  Here the table is built in fp32 on CUDA
// cores from fp32 codebooks, or from fp16 / bf16 copies (the reference's
// fp16 manager dtype; their elements widen to fp32 exactly).  The work is a skinny GEMV that is bound by
// the codebook bytes (33.5 MB for per-KV-head fp32 codebooks at Llama-3.1-8B
// geometry), so the kernel is organised for memory-level parallelism: one
// CTA per (codebook m, quarter of the K codewords, unit), each warp keeps 8
// coalesced 512-byte codeword rows in flight, and the 8 dot products of a
// batch are reduced across the warp with a 9-shuffle transpose-reduction.
//
// Two table forms:
//   GROUP: one table per KV head built from q_sum = sum_g q_g (fp32, g in
//          order).  score_sum(t) = sum_m LUT_sum[m][code_m] equals the
//          GQA-summed score sum_g sum_m q_g . C_m[code_m], so top-k per KV
//          head on summed scores needs ONE lookup per (token, m) instead of G.
//          Stored [unit][k][m] (k-major so the scorer can stage it into a
//          bank-conflict-free shared-memory layout with plain vector copies).
//   HEADS: one table per query head, the G <= 4 heads of a KV group
//          interleaved: [unit][k][m][4] fp32 (16 bytes per (k, m)), unused
//          slots zero.
// Each CTA also writes the min and max over its codewords of every table
// (partial bounds [unit][head][m][part][2]); consumers reduce the parts into
// a hard bound [lo, hi] of every score.
#pragma once
#include "common.cuh"

namespace lp {

constexpr int kLutParts = 4;     // CTAs per (m, unit), each covering K/4 codewords
constexpr int kLutThreads = 128; // 4 warps

struct LutBuildParams {
    const void* q;
    int64_t q_stride_b, q_stride_h;
    const void* cb;    // [Hkv or 1][M][K][D] of cb_dtype
    int cb_dtype;      // LP_F32 | LP_F16 | LP_BF16
    int cb_per_kv_head;
    int Hkv, G, D, M, K;
    float* lut;      // GROUP: [U][K][M]; HEADS: [U][K][M][4]
    float* bounds;   // [U][Gb][M][kLutParts][2]  (Gb = 1 for GROUP, G for HEADS)
    uint32_t* zero;  // per-call state cleared by this kernel
    int64_t zero_words;
};

// Sum over the 32 lanes of v[0..7] (8 independent values); afterwards lane l
// holds the total of value index (l >> 2) & 7.
__device__ __forceinline__ float transpose_reduce8(float v[8], int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float keep = b4 ? v[4 + j] : v[j];
        const float send = b4 ? v[j] : v[4 + j];
        w[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float x[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float keep = b3 ? w[2 + j] : w[j];
        const float send = b3 ? w[j] : w[2 + j];
        x[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    const float keep = b2 ? x[1] : x[0];
    const float send = b2 ? x[0] : x[1];
    float y = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    return y;
}

template <typename QT, bool HEADS>
__global__ void __launch_bounds__(kLutThreads) lut_build_kernel(LutBuildParams p) {
    constexpr int NW = kLutThreads / 32;
    constexpr int GQ = HEADS ? 4 : 1;  // tables built per CTA
    extern __shared__ float qf[];      // [GQ][D]
    __shared__ float s_min[NW][GQ], s_max[NW][GQ];

    const int m = blockIdx.x / kLutParts;
    const int part = blockIdx.x - m * kLutParts;
    const int u = blockIdx.y;
    const int b = u / p.Hkv;
    const int hkv = u - b * p.Hkv;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the scorer may be scheduled now: it only streams codes until it waits
    // for this grid's completion (griddepcontrol.wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // clear the per-call counters / histograms of the following kernels
    {
        const int64_t nthreads = (int64_t)gridDim.x * gridDim.y * blockDim.x;
        const int64_t start = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid;
        for (int64_t i = start; i < p.zero_words; i += nthreads) p.zero[i] = 0u;
    }

    const int esz = cb_elem_bytes(p.cb_dtype);
    const unsigned char* cbm = static_cast<const unsigned char*>(p.cb) +
                               ((int64_t)(p.cb_per_kv_head ? hkv : 0) * p.M * p.K * p.D + (int64_t)m * p.K * p.D) * esz;
    const int kper = (p.K + kLutParts - 1) / kLutParts;
    const int kbeg = part * kper, kend = min(p.K, kbeg + kper);
    // pull this CTA's whole codebook slice toward L2 before anything else
    if (tid == 0 && kend > kbeg) {
        const uint32_t bytes = (uint32_t)((kend - kbeg) * p.D * esz);
        const unsigned char* src = cbm + (int64_t)kbeg * p.D * esz;
        if ((bytes & 15u) == 0 && (((uintptr_t)src) & 15u) == 0)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
    }

    const QT* qb = reinterpret_cast<const QT*>(p.q) + (int64_t)b * p.q_stride_b;
    for (int d = tid; d < p.D; d += blockDim.x) {
        if (HEADS) {
#pragma unroll
            for (int g = 0; g < 4; ++g)
                qf[g * p.D + d] =
                    g < p.G ? to_f32(qb[(int64_t)(hkv * p.G + g) * p.q_stride_h + d]) : 0.f;
        } else {
            float acc = 0.f;
            for (int g = 0; g < p.G; ++g) acc += to_f32(qb[(int64_t)(hkv * p.G + g) * p.q_stride_h + d]);
            qf[d] = acc;
        }
    }
    __syncthreads();

    const int nchunk = (p.D + 127) / 128;

    float vmin[GQ], vmax[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g) { vmin[g] = INFINITY; vmax[g] = -INFINITY; }

    for (int k0 = kbeg + warp * 8; k0 < kend; k0 += NW * 8) {
        float part_[GQ][8];
#pragma unroll
        for (int g = 0; g < GQ; ++g)
#pragma unroll
            for (int j = 0; j < 8; ++j) part_[g][j] = 0.f;
        for (int c = 0; c < nchunk; ++c) {
            const int d = c * 128 + lane * 4;
            if (d < p.D) {
                float4 cv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int k = k0 + j;
                    cv[j] = k < kend ? cb_load4(cbm, (int64_t)k * p.D + d, p.cb_dtype)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int g = 0; g < GQ; ++g) {
                    const float4 qv = *reinterpret_cast<const float4*>(qf + g * p.D + d);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float a = part_[g][j];
                        a = fmaf(qv.x, cv[j].x, a);
                        a = fmaf(qv.y, cv[j].y, a);
                        a = fmaf(qv.z, cv[j].z, a);
                        a = fmaf(qv.w, cv[j].w, a);
                        part_[g][j] = a;
                    }
                }
            }
        }
        float tot[GQ];
#pragma unroll
        for (int g = 0; g < GQ; ++g) tot[g] = transpose_reduce8(part_[g], lane);
        const int k = k0 + ((lane >> 2) & 7);
        if ((lane & 3) == 0 && k < kend) {
            if (HEADS) {
                reinterpret_cast<float4*>(p.lut)[((int64_t)u * p.K + k) * p.M + m] =
                    make_float4(tot[0], tot[1], tot[2], tot[3]);
            } else {
                p.lut[((int64_t)u * p.K + k) * p.M + m] = tot[0];
            }
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
                vmin[g] = fminf(vmin[g], tot[g]);
                vmax[g] = fmaxf(vmax[g], tot[g]);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            vmin[g] = fminf(vmin[g], __shfl_xor_sync(0xffffffffu, vmin[g], o));
            vmax[g] = fmaxf(vmax[g], __shfl_xor_sync(0xffffffffu, vmax[g], o));
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < GQ; ++g) { s_min[warp][g] = vmin[g]; s_max[warp][g] = vmax[g]; }
    }
    __syncthreads();
    const int Gb = HEADS ? p.G : 1;
    if (tid < Gb) {
        const int g = tid;
        float mn = s_min[0][g], mx = s_max[0][g];
        for (int w = 1; w < NW; ++w) { mn = fminf(mn, s_min[w][g]); mx = fmaxf(mx, s_max[w][g]); }
        float* bd = p.bounds + ((((int64_t)u * Gb + g) * p.M + m) * kLutParts + part) * 2;
        bd[0] = mn;
        bd[1] = mx;
    }
}

}  // namespace lp
