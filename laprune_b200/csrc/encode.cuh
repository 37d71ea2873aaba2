// encode.cuh -- greedy residual additive-quantization encode of new keys.
//
// Reference: laprune/aq_kernels/fused_linear_encode.cu:34-234
// (fused_linear_encode_forward: per stage m, code_m = argmax_k(bias[m,k] +
// r . C_m[k]) with bias = -||C||^2 / 2, then r -= C_m[code_m]) and its CPU
// counterpart laprune/quantizer.py:346-374 (_batch_icm_lut with 0 ICM
// iterations: code_m = first argmin_k ||r||^2 + ||C_m[k]||^2 - 2 r . C_m[k]).
//
// Result: the codes of the CPU arithmetic, exactly -- every sum a sequential
// chain of fp32 fused multiply-adds in index order (the oracle states the
// same), the first minimum on ties.
//
// Work: per stage the residuals of the CTA's 128 vectors meet the stage's
// 256 codewords, R[128 x 128] . C_m^T[128 x 256], on the 5th-generation
// tensor cores (tcgen05.mma, kind::tf32, fp32 accumulators in TMEM).  The
// tf32 products are only a filter: with |approx - exact| <= eps ||r|| ||c_k||
// for every codeword, the exact winner lies among the codewords whose
// approximate distance is within the bounds of the best upper bound; when
// that set has one member it is the code, otherwise its members are
// recomputed exactly on CUDA cores.
//
// Shared memory holds the residuals (A operand, 64 KB) and the stage's
// codewords in two halves of 128 (B operands, 64 KB each), both in the UMMA
// canonical K-major layout without swizzle: 8-row x 16-byte core matrices,
// K-adjacent ones 128 B apart (LBO), 8-row groups 4096 B apart (SBO).  The
// next stage's codewords load (cp.async) while the current stage's
// distances are searched.
#pragma once
#include "common.cuh"

namespace lp {

constexpr int kEncRows = 128;  // vectors per CTA (UMMA M)
constexpr int kEncThreads = 512;
constexpr int kEncD = 128, kEncK = 256, kEncM = 32;

struct EncodeParams {
    const void* x;
    int64_t xs_b, xs_h, xs_t;  // elements
    int B, H, T;               // vectors x[b][h][t][0..128)
    int per_head;              // codebook set of vector (b, h, t) is h (else 0)
    const float* cb;           // [S][32][256][128] fp32
    const float* nrm;          // [S][32][256]  ||C||^2 (sequential fma)
    const float* cnorm;        // [S][32][256]  ||C|| rounded up
    uint8_t* codes;
    int64_t cs_b, cs_h, cs_t;  // bytes
    int ctas_per_set;          // ceil(vectors of a set / 128)
    int force_exact;           // recompute every codeword exactly (testing)
    uint32_t* err;
};

struct EncSmem {
    static constexpr int kA = kEncRows * kEncD * 4;          // 64 KB
    static constexpr int kBHalf = 128 * kEncD * 4;           // 64 KB
    static constexpr int kNorm = 2 * 2 * kEncK * 4;          // nrm + cnorm, double buffered (4 KB)
    static constexpr int kTotal = kA + 2 * kBHalf + kNorm + 64;
};

// byte offset of element (row n, dim d) in the canonical K-major layout
__device__ __forceinline__ uint32_t enc_off(int n, int d) {
    return (uint32_t)((((n >> 3) * (kEncD / 4) + (d >> 2)) << 7) + ((n & 7) << 4) + ((d & 3) << 2));
}

// UMMA shared-memory descriptor: K-major, no swizzle, LBO 128 B, SBO 4096 B
__device__ __forceinline__ uint64_t enc_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(128u >> 4) << 16;
    d |= (uint64_t)(4096u >> 4) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    return d;
}

// instruction descriptor: D fp32, A/B tf32, both K-major, N = 128, M = 128
constexpr uint32_t kEncIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void enc_mma(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
        "l"(da), "l"(db), "r"(kEncIdesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void enc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 64 fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void enc_tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
        "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// ||C||^2 of every codeword (sequential fma over d) and ||C|| rounded up.
__global__ void __launch_bounds__(256) encode_norms_kernel(const float* cb, int64_t n, float* nrm, float* cnorm) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float4* c = reinterpret_cast<const float4*>(cb + i * kEncD);
    float acc = 0.f;
#pragma unroll 8
    for (int j = 0; j < kEncD / 4; ++j) {
        const float4 v = __ldg(c + j);
        acc = __fmaf_rn(v.x, v.x, acc);
        acc = __fmaf_rn(v.y, v.y, acc);
        acc = __fmaf_rn(v.z, v.z, acc);
        acc = __fmaf_rn(v.w, v.w, acc);
    }
    nrm[i] = acc;
    cnorm[i] = __fmul_ru(__fsqrt_ru(acc), 1.0000001f);
}

template <typename XT>
__global__ void __launch_bounds__(kEncThreads, 1) encode_keys_kernel(EncodeParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* sA = smem;
    unsigned char* sB = smem + EncSmem::kA;  // two halves
    float* sNorm = reinterpret_cast<float*>(sB + 2 * EncSmem::kBHalf);  // [2][nrm 256 | cnorm 256]
    uint64_t* s_mbar = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(sNorm) + EncSmem::kNorm);
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int set = blockIdx.x / p.ctas_per_set;
    const int tile = blockIdx.x - set * p.ctas_per_set;
    const int nvec_set = p.per_head ? p.B * p.T : p.B * p.H * p.T;  // vectors of this set
    const int v0 = tile * kEncRows;
    const float* cbs = p.cb + (int64_t)set * kEncM * kEncK * kEncD;
    const float* nrms = p.nrm + (int64_t)set * kEncM * kEncK;
    const float* cns = p.cnorm + (int64_t)set * kEncM * kEncK;

    // vector i of the set -> (b, h, t)
    auto vec_bht = [&](int i, int* b, int* h, int* t) {
        if (p.per_head) {
            *h = set;
            *b = i / p.T;
            *t = i - *b * p.T;
        } else {
            const int ht = p.H * p.T;
            *b = i / ht;
            const int r = i - *b * ht;
            *h = r / p.T;
            *t = r - *h * p.T;
        }
    };

    // stage m's codewords (both halves) and norms -> buffers (cp.async, one group)
    auto load_stage = [&](int m) {
        const float* cm = cbs + (int64_t)m * kEncK * kEncD;
        for (int c = tid; c < kEncK * (kEncD / 4); c += kEncThreads) {
            const int n = c >> 5, d4 = c & 31;  // codeword, 4-float chunk
            unsigned char* dst = sB + (n >> 7) * EncSmem::kBHalf + enc_off(n & 127, d4 * 4);
            cp_async16(dst, cm + (int64_t)n * kEncD + d4 * 4);
        }
        float* nb = sNorm + (m & 1) * 2 * kEncK;
        if (tid < 64) cp_async16(nb + tid * 4, nrms + (int64_t)m * kEncK + tid * 4);
        else if (tid < 128) cp_async16(nb + kEncK + (tid - 64) * 4, cns + (int64_t)m * kEncK + (tid - 64) * 4);
        cp_async_commit();
    };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(s_mbar, 1);
        fence_barrier_init();
        s_abort = 0;
    }
    // the CTA's vectors -> residuals (fp32, canonical layout); rows past the
    // set's end are zero
    for (int e = tid; e < kEncRows * (kEncD / 4); e += kEncThreads) {
        const int n = e >> 5, d = (e & 31) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (v0 + n < nvec_set) {
            int b, h, t;
            vec_bht(v0 + n, &b, &h, &t);
            const XT* xr = reinterpret_cast<const XT*>(p.x) + (int64_t)b * p.xs_b + (int64_t)h * p.xs_h + (int64_t)t * p.xs_t;
            v = make_float4(to_f32(xr[d]), to_f32(xr[d + 1]), to_f32(xr[d + 2]), to_f32(xr[d + 3]));
        }
        *reinterpret_cast<float4*>(sA + enc_off(n, d)) = v;
    }
    load_stage(0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    // epilogue threads: warps 0-3, thread = vector row (TMEM lane)
    const bool epi = warp < 4;
    const int row = tid;  // valid for epi
    bool row_valid = false;
    uint8_t* code_out = nullptr;
    if (epi && v0 + row < nvec_set) {
        int b, h, t;
        vec_bht(v0 + row, &b, &h, &t);
        row_valid = true;
        code_out = p.codes + (int64_t)b * p.cs_b + (int64_t)h * p.cs_h + (int64_t)t * p.cs_t;
    }
    // |exact dist - (approx dist + ||r||^2)| <= kEps ||r|| ||c_k|| + kAbs (||r||^2 + ||c_k||^2 + |approx|):
    // the tf32 operands (10 mantissa bits) and fp32 accumulation give about
    // 2^-8 ||r|| ||c||, the fp32 roundings of the exact formula about 2^-23
    // of the magnitudes; both are taken with a margin of 4 or more
    constexpr float kEps = 1.0f / 64.0f;
    constexpr float kAbs = 1.0f / 1048576.0f;

    uint32_t phase = 0;
    for (int m = 0; m < kEncM; ++m) {
        cp_async_wait<0>();
        fence_proxy_async();  // generic / cp.async shared writes -> async proxy (MMA)
        __syncthreads();
        if (s_abort) break;
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(sA);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const uint32_t b0 = smem_u32(sB + hf * EncSmem::kBHalf);
#pragma unroll
                for (int s = 0; s < kEncD / 8; ++s)
                    enc_mma(tmem + hf * 128, enc_desc(a0 + s * 256), enc_desc(b0 + s * 256), s > 0 ? 1u : 0u);
            }
            enc_commit(s_mbar);
        }
        // meanwhile: ||r||^2 of the row, exactly (sequential fma in d order)
        float rn = 0.f;
        if (epi) {
#pragma unroll 4
            for (int d4 = 0; d4 < kEncD / 4; ++d4) {
                const float4 r4 = *reinterpret_cast<const float4*>(sA + enc_off(row, d4 * 4));
                rn = __fmaf_rn(r4.x, r4.x, rn);
                rn = __fmaf_rn(r4.y, r4.y, rn);
                rn = __fmaf_rn(r4.z, r4.z, rn);
                rn = __fmaf_rn(r4.w, r4.w, rn);
            }
        }
        const bool done = mbar_wait(s_mbar, phase, p.err);
        phase ^= 1u;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__syncthreads_or(!done)) {
            if (tid == 0) s_abort = 1;
            mbar_wait(s_mbar, phase ^ 1u, nullptr);  // the MMA may still run: bounded second wait
            break;
        }
        // the next stage's codewords load while this stage's distances are searched
        if (m + 1 < kEncM) load_stage(m + 1);
        if (epi) {
            const float* nb = sNorm + (m & 1) * 2 * kEncK;
            const float rnorm = __fmul_ru(__fsqrt_ru(rn), 1.0000001f);
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
            // pass 1: U = min_k (approx_k + bound_k)
            float U = INFINITY;
            for (int c0 = 0; c0 < kEncK; c0 += 64) {
                float v[64];
                enc_tmem_ld64(taddr + c0, v);
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const float ap = fmaf(-2.f, v[i], nb[c0 + i]);
                    const float bd = fmaf(kEps * rnorm, nb[kEncK + c0 + i], kAbs * (rn + nb[c0 + i] + fabsf(ap)));
                    U = fminf(U, ap + bd);
                }
            }
            // pass 2: candidates approx_k - bound_k <= U
            int ncand = 0, first = -1;
            int cand[8];
            for (int c0 = 0; c0 < kEncK; c0 += 64) {
                float v[64];
                enc_tmem_ld64(taddr + c0, v);
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const float ap = fmaf(-2.f, v[i], nb[c0 + i]);
                    const float bd = fmaf(kEps * rnorm, nb[kEncK + c0 + i], kAbs * (rn + nb[c0 + i] + fabsf(ap)));
                    if (ap - bd <= U) {
                        if (ncand < 8) cand[ncand] = c0 + i;
                        if (first < 0) first = c0 + i;
                        ++ncand;
                    }
                }
            }
            int code = first < 0 ? 0 : first;
            if (p.force_exact || ncand > 1) {
                // exact distances of the candidates (all codewords if more
                // than 8 or in the exact test mode), first minimum wins
                const float* cm = cbs + (int64_t)m * kEncK * kEncD;
                const bool all = p.force_exact || ncand > 8;
                const int nk = all ? kEncK : ncand;
                float best = INFINITY;
                int best_k = 0;
                for (int i = 0; i < nk; ++i) {
                    const int k = all ? i : cand[i];
                    const float4* c4 = reinterpret_cast<const float4*>(cm + (int64_t)k * kEncD);
                    float dot = 0.f;
#pragma unroll 4
                    for (int d4 = 0; d4 < kEncD / 4; ++d4) {
                        const float4 r4 = *reinterpret_cast<const float4*>(sA + enc_off(row, d4 * 4));
                        const float4 cv = __ldg(c4 + d4);
                        dot = __fmaf_rn(r4.x, cv.x, dot);
                        dot = __fmaf_rn(r4.y, cv.y, dot);
                        dot = __fmaf_rn(r4.z, cv.z, dot);
                        dot = __fmaf_rn(r4.w, cv.w, dot);
                    }
                    const float dist = __fmaf_rn(-2.f, dot, __fadd_rn(rn, nb[k]));
                    if (dist < best) {
                        best = dist;
                        best_k = k;
                    }
                }
                code = best_k;
            }
            if (row_valid) code_out[m] = (uint8_t)code;
            // r -= C_m[code]
            const float4* c4 = reinterpret_cast<const float4*>(cbs + ((int64_t)m * kEncK + code) * kEncD);
#pragma unroll 4
            for (int d4 = 0; d4 < kEncD / 4; ++d4) {
                float4* r4p = reinterpret_cast<float4*>(sA + enc_off(row, d4 * 4));
                float4 r4 = *r4p;
                const float4 cv = __ldg(c4 + d4);
                r4.x = __fsub_rn(r4.x, cv.x);
                r4.y = __fsub_rn(r4.y, cv.y);
                r4.z = __fsub_rn(r4.z, cv.z);
                r4.w = __fsub_rn(r4.w, cv.w);
                *r4p = r4;
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    cp_async_wait<0>();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

}  // namespace lp
