// compat.cuh -- kernels behind the aq_kernels-named Python surface.
//
// Reference entry points (aq_kernels/__init__.py:1-23):
//   aq_lut_gather_grouped  aq_kernels/aq_lut_gqa.cu:460-534 (kernels :111-212)
//   aq_lut_gather (gqa)    aq_kernels/aq_lut_gqa.cu:350-422 (kernel :20-76)
//   aq_lut_gather_forward  aq_kernels/aq_lut.cu:581-738
//   aq_lut_forward         aq_kernels/aq_lut.cu:37-149, 445-574
//   gqa_gather_kv(_with_tail) aq_kernels/aq_lut_gqa.cu:277-323, 536-664
// The fused decode step does all of this in one kernel; these are the
// building blocks for callers of the individual ops.
#pragma once
#include "common.cuh"

namespace lp {

// out[q][n] = sum_{m in [m0,m1)} lut[q][m][code(q, n, m)] -- fp32 accumulation
// in m order, then the output type.  Row q reads codes head q / G; token
// t = indices ? indices[q][n] : n (outside [0,T): 0).  code_mode 0: clamp
// codes to K-1; 1: codes >= K contribute nothing.
struct LutGatherParams {
    const void* lut;
    int lut_f16;
    int64_t lut_stride_q;
    int M_stride, K, m0, m1;
    const uint8_t* codes;
    int64_t cs_h, cs_t;
    int Q, G, T, N;
    const int64_t* indices;
    int64_t is_q;
    int code_mode;
    void* out;
    int out_f16;
    int64_t os_q;
};

__global__ void __launch_bounds__(256) lut_gather_kernel(LutGatherParams p) {
    extern __shared__ float s_lut[];  // [m1 - m0][K]
    const int q = blockIdx.y;
    const int mr = p.m1 - p.m0;
    for (int i = threadIdx.x; i < mr * p.K; i += blockDim.x) {
        const int64_t src = (int64_t)q * p.lut_stride_q + (int64_t)(p.m0 + i / p.K) * p.K + i % p.K;
        s_lut[i] = p.lut_f16 ? __half2float(reinterpret_cast<const __half*>(p.lut)[src])
                             : reinterpret_cast<const float*>(p.lut)[src];
    }
    __syncthreads();
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= p.N) return;
    const int64_t t = p.indices ? p.indices[(int64_t)q * p.is_q + n] : n;
    float acc = 0.f;
    if (t >= 0 && t < p.T) {
        const uint8_t* c = p.codes + (int64_t)(q / p.G) * p.cs_h + t * p.cs_t;
        for (int m = p.m0; m < p.m1; ++m) {
            int k = c[m];
            if (k >= p.K) {
                if (p.code_mode) continue;
                k = p.K - 1;
            }
            acc = __fadd_rn(acc, s_lut[(m - p.m0) * p.K + k]);
        }
    }
    if (p.out_f16) reinterpret_cast<__half*>(p.out)[(int64_t)q * p.os_q + n] = __float2half_rn(acc);
    else reinterpret_cast<float*>(p.out)[(int64_t)q * p.os_q + n] = acc;
}

// lut[q][m][k] = q_row . C[m][k] (fp32, sequential fma over d)
template <typename QT>
__global__ void __launch_bounds__(256) lut_build_rows_kernel(const QT* q, int64_t q_stride, const float* cb, int M,
                                                             int K, int D, float* lut) {
    extern __shared__ float s_q[];
    const int m = blockIdx.x, qi = blockIdx.y;
    for (int d = threadIdx.x; d < D; d += blockDim.x) s_q[d] = to_f32(q[(int64_t)qi * q_stride + d]);
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float* c = cb + ((int64_t)m * K + k) * D;
        float acc = 0.f;
        for (int d = 0; d < D; ++d) acc = __fmaf_rn(s_q[d], __ldg(c + d), acc);
        lut[((int64_t)qi * M + m) * K + k] = acc;
    }
}

// one warp per output row (b, hq, n): K and V rows of token
// n < N_explicit ? indices[b][hq][n] : tail_start + n - N_explicit, zeros
// for tokens outside [0, T)
struct GqaGatherParams {
    const uint16_t* keys;
    const uint16_t* vals;
    int64_t ks_b, ks_h, ks_t, vs_b, vs_h, vs_t;
    const int64_t* indices;
    int64_t is_b, is_h;
    int B, Hkv, G, T, D, N_explicit, tail_start, N;
    uint16_t* out_k;
    uint16_t* out_v;
};

__global__ void __launch_bounds__(256) gqa_gather_kernel(GqaGatherParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int Hq = p.Hkv * p.G;
    const int64_t nrows = (int64_t)p.B * Hq * p.N;
    if (row >= nrows) return;
    const int n = (int)(row % p.N);
    const int64_t bh = row / p.N;
    const int hq = (int)(bh % Hq), b = (int)(bh / Hq);
    const int64_t t = n < p.N_explicit ? p.indices[(int64_t)b * p.is_b + (int64_t)hq * p.is_h + n]
                                       : (int64_t)p.tail_start + (n - p.N_explicit);
    const bool ok = t >= 0 && t < p.T;
    const int hk = hq / p.G;
    uint16_t* ok_ = p.out_k + row * p.D;
    uint16_t* ov_ = p.out_v + row * p.D;
    const uint16_t* sk = p.keys + (int64_t)b * p.ks_b + (int64_t)hk * p.ks_h + (ok ? t : 0) * p.ks_t;
    const uint16_t* sv = p.vals + (int64_t)b * p.vs_b + (int64_t)hk * p.vs_h + (ok ? t : 0) * p.vs_t;
    for (int d = lane; d < p.D; d += 32) {
        ok_[d] = ok ? sk[d] : (uint16_t)0;
        ov_[d] = ok ? sv[d] : (uint16_t)0;
    }
}

}  // namespace lp
