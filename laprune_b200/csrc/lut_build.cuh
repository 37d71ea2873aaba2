// lut_build.cuh -- per-query lookup tables LUT[m][k] = q . C_m[k] (fp32).
//
// Reference: laprune/llm/aq_kv.py:681-682 (cuBLAS q @ C^T, fp16) and the CPU
// path aq_kv.py:620 (einsum, fp32).  Here the table is built in fp32 from
// fp32 codebooks on CUDA cores: one CTA per (codebook m, unit), one warp per
// codeword row (coalesced 512-byte row reads, HBM-bound on the codebooks).
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
// Each CTA also writes the per-(head, m) min and max over k, from which the
// scorer derives a hard bound [lo, hi] of every score for its histogram.
#pragma once
#include "common.cuh"

namespace lp {

struct LutBuildParams {
    const void* q;
    int64_t q_stride_b, q_stride_h;
    const float* cb;
    int cb_per_kv_head;
    int Hkv, G, D, M, K;
    float* lut;      // GROUP: [U][K][M]; HEADS: [U][K][M][4]
    float* bounds;   // [U][Gb][M][2]  (Gb = 1 for GROUP, G for HEADS)
    uint32_t* zero;  // per-call state cleared by this kernel
    int64_t zero_words;
};

template <typename QT, bool HEADS>
__global__ void __launch_bounds__(256) lut_build_kernel(LutBuildParams p) {
    constexpr int NW = 8;
    constexpr int GQ = HEADS ? 4 : 1;  // tables built per CTA
    extern __shared__ float qf[];      // [GQ][D]
    __shared__ float s_min[NW][GQ], s_max[NW][GQ];

    const int m = blockIdx.x;
    const int u = blockIdx.y;
    const int b = u / p.Hkv;
    const int hkv = u - b * p.Hkv;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // clear the per-call counters / histograms of the following kernels
    {
        const int64_t nthreads = (int64_t)gridDim.x * gridDim.y * blockDim.x;
        const int64_t start = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid;
        for (int64_t i = start; i < p.zero_words; i += nthreads) p.zero[i] = 0u;
    }

    const QT* qb = reinterpret_cast<const QT*>(p.q) + (int64_t)b * p.q_stride_b;
    for (int d = tid; d < p.D; d += blockDim.x) {
        if (HEADS) {
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

    const float* cbm = p.cb + (int64_t)(p.cb_per_kv_head ? hkv : 0) * p.M * p.K * p.D +
                       (int64_t)m * p.K * p.D;
    const int nchunk = (p.D + 127) / 128;

    float vmin[GQ], vmax[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g) { vmin[g] = INFINITY; vmax[g] = -INFINITY; }

    for (int k0 = warp * 4; k0 < p.K; k0 += NW * 4) {
        float part[4][GQ];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int g = 0; g < GQ; ++g) part[j][g] = 0.f;
        for (int c = 0; c < nchunk; ++c) {
            const int d = c * 128 + lane * 4;
            if (d < p.D) {
                float4 cv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int k = k0 + j;
                    cv[j] = k < p.K ? __ldg(reinterpret_cast<const float4*>(cbm + (int64_t)k * p.D + d))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int g = 0; g < GQ; ++g) {
                    const float4 qv = *reinterpret_cast<const float4*>(qf + g * p.D + d);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float a = part[j][g];
                        a = fmaf(qv.x, cv[j].x, a);
                        a = fmaf(qv.y, cv[j].y, a);
                        a = fmaf(qv.z, cv[j].z, a);
                        a = fmaf(qv.w, cv[j].w, a);
                        part[j][g] = a;
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int g = 0; g < GQ; ++g)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) part[j][g] += __shfl_xor_sync(0xffffffffu, part[j][g], o);
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int k = k0 + j;
                if (k >= p.K) break;
                if (HEADS) {
                    float4 v = make_float4(part[j][0], part[j][1], part[j][2], part[j][3]);
                    reinterpret_cast<float4*>(p.lut)[((int64_t)u * p.K + k) * p.M + m] = v;
                } else {
                    p.lut[((int64_t)u * p.K + k) * p.M + m] = part[j][0];
                }
#pragma unroll
                for (int g = 0; g < GQ; ++g) {
                    vmin[g] = fminf(vmin[g], part[j][g]);
                    vmax[g] = fmaxf(vmax[g], part[j][g]);
                }
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < GQ; ++g) { s_min[warp][g] = vmin[g]; s_max[warp][g] = vmax[g]; }
    }
    __syncthreads();
    if (tid < GQ) {
        const int g = tid;
        float mn = s_min[0][g], mx = s_max[0][g];
        for (int w = 1; w < NW; ++w) { mn = fminf(mn, s_min[w][g]); mx = fmaxf(mx, s_max[w][g]); }
        const int Gb = HEADS ? p.G : 1;
        if (g < Gb) {
            float* bd = p.bounds + (((int64_t)u * Gb + g) * p.M + m) * 2;
            bd[0] = mn;
            bd[1] = mx;
        }
    }
}

}  // namespace lp
