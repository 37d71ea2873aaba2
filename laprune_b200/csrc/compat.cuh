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
    int lut_vec;  // fp16 rows' [m0*K, m1*K) spans 16-byte aligned (8-element loads)
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

// ---- vectorised forms of lut_gather_kernel (same sums, same order) ----
//
// Both read a token's code row with 16-byte loads (rows 16-byte aligned,
// m1 <= 32) and sum its table entries in fp32 in m order, as
// lut_gather_kernel does, so their results are bit-identical to it.

// Byte m (compile-time) of the 32-byte code row held in c[0..7].
__device__ __forceinline__ uint32_t code_byte(const uint32_t* c, int m) { return (c[m >> 2] >> (8 * (m & 3))) & 0xffu; }

__device__ __forceinline__ void load_code_row(const uint8_t* row, int m1, uint32_t* c) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(row));
    c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w;
    if (m1 > 16) {
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(row) + 1);
        c[4] = b.x; c[5] = b.y; c[6] = b.z; c[7] = b.w;
    } else {
        c[4] = c[5] = c[6] = c[7] = 0u;
    }
}

// Dense scan with codes shared by G query rows (rows h*G .. h*G+G-1 read the
// codes of head h = blockIdx.y): each code row is loaded once for all G
// rows.  fp16 tables are staged as half2 pairs of rows (2g, 2g+1), so one
// shared-memory load serves two rows; fp32 tables one row per load.  CTA:
// tokens [blockIdx.x * tile, +tile) of head h, 256 threads, one token per
// thread per step.
constexpr int kScanMaxG = 8;     // fp16 tables
constexpr int kScanMaxG32 = 4;   // fp32 tables
constexpr int kScanThreads = 512;
template <bool F16>
__global__ void __launch_bounds__(kScanThreads, 3) lut_scan_group_kernel(LutGatherParams p, int tile) {
    constexpr int MAXG = F16 ? kScanMaxG : kScanMaxG32;
    extern __shared__ __align__(16) unsigned char s_tab[];
    const int h = blockIdx.y, G = p.G, mr = p.m1 - p.m0, K = p.K;
    const int npair = (G + 1) >> 1;
    // rows' [m0*K, m1*K) spans are contiguous: staged linearly, 8 elements
    // per 16-byte load when the spans are 16-byte aligned
    const int span = mr * K;
    if constexpr (F16) {
        __half2* t2 = reinterpret_cast<__half2*>(s_tab);  // [npair][span]
        const __half* lut = reinterpret_cast<const __half*>(p.lut) + (int64_t)p.m0 * K;
        for (int gp = 0; gp < npair; ++gp) {
            const __half* r0 = lut + ((int64_t)h * G + 2 * gp) * p.lut_stride_q;
            const __half* r1 = r0 + p.lut_stride_q;
            const bool two = 2 * gp + 1 < G;
            __half2* dst = t2 + gp * span;
            if (p.lut_vec) {
                for (int e = threadIdx.x * 8; e < span; e += blockDim.x * 8) {
                    const uint4 a = __ldg(reinterpret_cast<const uint4*>(r0 + e));
                    const uint4 b = two ? __ldg(reinterpret_cast<const uint4*>(r1 + e)) : make_uint4(0u, 0u, 0u, 0u);
                    const __half* ha = reinterpret_cast<const __half*>(&a);
                    const __half* hb = reinterpret_cast<const __half*>(&b);
#pragma unroll
                    for (int j = 0; j < 8; ++j) dst[e + j] = __halves2half2(ha[j], hb[j]);
                }
            } else {
                for (int e = threadIdx.x; e < span; e += blockDim.x)
                    dst[e] = __halves2half2(r0[e], two ? r1[e] : __float2half_rn(0.f));
            }
        }
    } else {
        float* t1 = reinterpret_cast<float*>(s_tab);  // [G][span]
        const float* lut = reinterpret_cast<const float*>(p.lut) + (int64_t)p.m0 * K;
        for (int g = 0; g < G; ++g) {
            const float* r0 = lut + ((int64_t)h * G + g) * p.lut_stride_q;
            for (int e = threadIdx.x; e < span; e += blockDim.x) t1[g * span + e] = __ldg(r0 + e);
        }
    }
    __syncthreads();
    const int t_end = min(p.T, (blockIdx.x + 1) * tile);
    const uint8_t* cbase = p.codes + (int64_t)h * p.cs_h;
    // one token per thread per step; the next step's code row is loaded
    // before this step's lookups, so a load is always in flight
    int t = blockIdx.x * tile + threadIdx.x;
    uint32_t c[8], cn[8];
    if (t < t_end) load_code_row(cbase + (int64_t)t * p.cs_t, p.m1, c);
    for (; t < t_end; t += blockDim.x) {
        const int tn = t + blockDim.x;
        if (tn < t_end) load_code_row(cbase + (int64_t)tn * p.cs_t, p.m1, cn);
        float acc[MAXG];
#pragma unroll
        for (int g = 0; g < MAXG; ++g) acc[g] = 0.f;
#pragma unroll
        for (int m = 0; m < 32; ++m) {
            if (m < p.m0 || m >= p.m1) continue;
            int k = (int)code_byte(c, m);
            if (k >= K) {
                if (p.code_mode) continue;
                k = K - 1;
            }
            const int e = (m - p.m0) * K + k;
            if constexpr (F16) {
                const __half2* t2 = reinterpret_cast<const __half2*>(s_tab);
#pragma unroll
                for (int gp = 0; gp < MAXG / 2; ++gp) {
                    if (gp >= npair) break;
                    const float2 v = __half22float2(t2[gp * mr * K + e]);
                    acc[2 * gp] = __fadd_rn(acc[2 * gp], v.x);
                    acc[2 * gp + 1] = __fadd_rn(acc[2 * gp + 1], v.y);
                }
            } else {
                const float* t1 = reinterpret_cast<const float*>(s_tab);
#pragma unroll
                for (int g = 0; g < MAXG; ++g) {
                    if (g >= G) break;
                    acc[g] = __fadd_rn(acc[g], t1[g * mr * K + e]);
                }
            }
        }
#pragma unroll
        for (int g = 0; g < MAXG; ++g) {
            if (g >= G) break;
            const int64_t o = ((int64_t)h * G + g) * p.os_q + t;
            if (p.out_f16) reinterpret_cast<__half*>(p.out)[o] = __float2half_rn(acc[g]);
            else reinterpret_cast<float*>(p.out)[o] = acc[g];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = cn[j];
    }
}

// Index-list (or per-row dense) gather with 16-byte code-row loads and
// `tile` tokens per CTA (one table staging per tile): row q = blockIdx.y.
__global__ void __launch_bounds__(256) lut_gather_rows_kernel(LutGatherParams p, int tile) {
    extern __shared__ float s_lut1[];  // [m1 - m0][K]
    const int q = blockIdx.y, mr = p.m1 - p.m0, K = p.K, span = mr * K;
    const int64_t r0 = (int64_t)q * p.lut_stride_q + (int64_t)p.m0 * K;  // the row's span is contiguous
    if (p.lut_f16 && p.lut_vec) {
        const __half* src = reinterpret_cast<const __half*>(p.lut) + r0;
        for (int e = threadIdx.x * 8; e < span; e += blockDim.x * 8) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + e));
            const __half* ha = reinterpret_cast<const __half*>(&a);
#pragma unroll
            for (int j = 0; j < 8; ++j) s_lut1[e + j] = __half2float(ha[j]);
        }
    } else {
        for (int e = threadIdx.x; e < span; e += blockDim.x)
            s_lut1[e] = p.lut_f16 ? __half2float(reinterpret_cast<const __half*>(p.lut)[r0 + e])
                                  : reinterpret_cast<const float*>(p.lut)[r0 + e];
    }
    __syncthreads();
    const int n_end = min(p.N, (blockIdx.x + 1) * tile);
    const uint8_t* cbase = p.codes + (int64_t)(q / p.G) * p.cs_h;
    for (int n = blockIdx.x * tile + threadIdx.x; n < n_end; n += blockDim.x) {
        const int64_t t = p.indices ? p.indices[(int64_t)q * p.is_q + n] : n;
        float acc = 0.f;
        if (t >= 0 && t < p.T) {
            uint32_t c[8];
            load_code_row(cbase + t * p.cs_t, p.m1, c);
#pragma unroll
            for (int m = 0; m < 32; ++m) {
                if (m < p.m0 || m >= p.m1) continue;
                int k = (int)code_byte(c, m);
                if (k >= K) {
                    if (p.code_mode) continue;
                    k = K - 1;
                }
                acc = __fadd_rn(acc, s_lut1[(m - p.m0) * K + k]);
            }
        }
        const int64_t o = (int64_t)q * p.os_q + n;
        if (p.out_f16) reinterpret_cast<__half*>(p.out)[o] = __float2half_rn(acc);
        else reinterpret_cast<float*>(p.out)[o] = acc;
    }
}

// lut[q][m][k] = q_row . C[m][k] (fp32, sequential fma over d).  CTA (k
// tile of 32 codewords, m, q tile of 32 rows): the codeword rows and query
// rows are staged in shared memory with coalesced loads (rows padded to
// D + 1 floats, so that the lanes' rows fall in different banks); thread
// (warp w, lane l) computes codeword 32x + l against query rows w, w + 8, ...
template <typename QT>
__global__ void __launch_bounds__(256) lut_build_rows_kernel(const QT* q, int64_t q_stride, const float* cb, int M,
                                                             int K, int D, int Q, float* lut) {
    extern __shared__ float s_buf[];  // codewords [32][D + 1], then queries [32][D + 1]
    const int DP = D + 1;
    float* s_c = s_buf;
    float* s_q = s_buf + 32 * DP;
    const int k0 = blockIdx.x * 32, m = blockIdx.y, q0 = blockIdx.z * 32;
    const int nk = min(32, K - k0), nq = min(32, Q - q0);
    for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) {
        const int r = i / D, d = i - r * D;
        s_c[r * DP + d] = r < nk ? __ldg(cb + ((int64_t)m * K + k0 + r) * D + d) : 0.f;
        s_q[r * DP + d] = r < nq ? to_f32(q[(int64_t)(q0 + r) * q_stride + d]) : 0.f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane >= nk) return;
    const float* c = s_c + lane * DP;
    for (int r = w; r < nq; r += blockDim.x / 32) {
        const float* qq = s_q + r * DP;  // broadcast across the warp
        float acc = 0.f;
        for (int d = 0; d < D; ++d) acc = __fmaf_rn(qq[d], c[d], acc);
        lut[((int64_t)(q0 + r) * M + m) * K + k0 + lane] = acc;
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

// 16-byte form (D * 2 bytes a multiple of 16, 16-byte aligned rows): CTA
// (x, y = b * Hq + hq) moves rows n = 32x .. 32x+31 of query head hq, four
// rows per warp with every row's loads issued before any store; a row's K
// units then its V units go to the warp's lanes, so a warp's loads and
// stores cover whole row segments.
constexpr int kKvRowsPerWarp = 4;
__global__ void __launch_bounds__(256) gqa_gather_vec_kernel(GqaGatherParams p) {
    const int upr = p.D / 8;  // 16-byte units per K (or V) row
    const int Hq = p.Hkv * p.G;
    const int bhq = blockIdx.y, b = bhq / Hq, hq = bhq - b * Hq, hk = hq / p.G;
    const int n0 = (blockIdx.x * 8 + (threadIdx.x >> 5)) * kKvRowsPerWarp, lane = threadIdx.x & 31;
    if (n0 >= p.N) return;
    // lane r < 4 fetches row n0 + r's token, then every lane has all four
    int64_t tl = -1;
    if (lane < kKvRowsPerWarp && n0 + lane < p.N) {
        const int n = n0 + lane;
        tl = n < p.N_explicit ? __ldg(p.indices + (int64_t)b * p.is_b + (int64_t)hq * p.is_h + n)
                              : (int64_t)p.tail_start + (n - p.N_explicit);
    }
    int64_t tr[kKvRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kKvRowsPerWarp; ++r) tr[r] = __shfl_sync(0xffffffffu, tl, r);
    const uint16_t* kb = p.keys + (int64_t)b * p.ks_b + (int64_t)hk * p.ks_h;
    const uint16_t* vb = p.vals + (int64_t)b * p.vs_b + (int64_t)hk * p.vs_h;
    for (int j = lane; j < 2 * upr; j += 32) {
        const bool isv = j >= upr;
        const int part = isv ? j - upr : j;
        uint4 v[kKvRowsPerWarp];
#pragma unroll
        for (int r = 0; r < kKvRowsPerWarp; ++r) {
            const int64_t t = tr[r];
            v[r] = make_uint4(0u, 0u, 0u, 0u);
            if (t >= 0 && t < p.T)
                v[r] = __ldg(reinterpret_cast<const uint4*>(isv ? vb + t * p.vs_t : kb + t * p.ks_t) + part);
        }
#pragma unroll
        for (int r = 0; r < kKvRowsPerWarp; ++r) {
            if (n0 + r >= p.N) break;
            const int64_t row = (int64_t)bhq * p.N + n0 + r;
            reinterpret_cast<uint4*>((isv ? p.out_v : p.out_k) + row * p.D)[part] = v[r];
        }
    }
}

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
