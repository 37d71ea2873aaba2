// encode.cuh -- greedy residual additive-quantization encode of new keys.
//
// Reference: laprune/aq_kernels/fused_linear_encode.cu:34-234
// (fused_linear_encode_forward: per stage m, code_m = argmax_k(bias[m,k] +
// r . C_m[k]) with bias = -||C||^2 / 2, then r -= C_m[code_m]) and its CPU
// counterpart laprune/quantizer.py:346-374 (_batch_icm_lut with 0 ICM
// iterations: code_m = first argmin_k ||r||^2 + ||C_m[k]||^2 - 2 r . C_m[k]).
//
// Result: the codes of the CPU arithmetic, exactly: ||r||^2 and ||c||^2
// sequential chains of fp32 fused multiply-adds in index order, r . c in a
// fixed 32-lane order (lane l a 4-term fma chain over dims 4l..4l+3, then a
// shuffle-xor butterfly at strides 16, 8, 4, 2, 1, whose lanes all end with
// the same bits because fp32 addition is commutative), the first minimum on
// ties.  The oracle states the same order.
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
// Shared memory holds the residuals (A operand, 64 KB) and the stage's 256
// codewords (B operand, 128 KB, one N = 256 MMA per K step), both in the
// UMMA K-major SWIZZLE_128B layout: per 32-dim K chunk (16 KB of residual
// rows, 32 KB of codeword rows), 8-row atoms of 1024 B, rows 128 B apart,
// 16-byte units XOR-swizzled with the row.  The codewords arrive by 2-D TMA
// tensor copies (box 32 dims x 128 rows, the same swizzle); while the MMA
// runs, warps 8-15 compute the stage's ||c||^2 from them.  The exact
// recomputation and the residual update read the codeword rows from there,
// so the next stage's copies start once the chosen codewords are in
// registers.  Rows with several candidates put their (row, codeword) pairs
// on a CTA-wide list, one pair per 8 lanes, so that the sequential 128-term
// chains run side by side; the codes collect in shared memory and leave
// once, 32 bytes per vector.  CTAs of 64, 32 or 16 vectors hold 2, 4 or 8
// copies of their rows in the MMA's 128 rows (see encode_keys_kernel).
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace lp {

constexpr int kEncRows = 128;  // vectors per CTA (UMMA M)
constexpr int kEncThreads = 512;
constexpr int kEncD = 128, kEncK = 256, kEncM = 32;
constexpr int kEncListCap = 2048;  // (row, codeword) pairs refined per round

struct EncodeParams {
    const void* x;
    int64_t xs_b, xs_h, xs_t;  // elements
    int B, H, T;               // vectors x[b][h][t][0..128)
    int per_head;              // codebook set of vector (b, h, t) is h (else 0)
    const float* cb;           // [S][32][256][128] fp32
    uint8_t* codes;
    int64_t cs_b, cs_h, cs_t;  // bytes
    int ctas_per_set;          // ceil(vectors of a set / rows_per_cta)
    int rows_per_cta;          // 128, or 64 / 32 / 16 when the sets have too few vectors to fill the GPU
                               // (the MMA still runs 128 rows; the others are zero)
    int force_exact;           // recompute every codeword exactly (testing)
    uint32_t* err;
};

struct EncSmem {
    static constexpr int kA = kEncRows * kEncD * 4;          // 64 KB
    static constexpr int kBHalf = 128 * kEncD * 4;           // 64 KB
    static constexpr int kNormStride = kEncK + 4;           // the stage's ||C||^2 [256] (+ 4 spare)
    static constexpr int kNorm = 2 * kNormStride * 4;        // double buffered
    static constexpr int kTotal = kA + 2 * kBHalf + kNorm + 64 + 1024;  // + alignment slack
};

// byte offset of (row n, dim d) of a [128][128] fp32 operand in the K-major
// SWIZZLE_128B layout: K chunk d/32 at 16 KB steps, 8-row atoms of 1024 B,
// row r of an atom at 128 r with its 16-byte units XOR-ed with r
__device__ __forceinline__ uint32_t enc_off(int n, int d) {
    const int b = (d & 31) << 2;
    const int u = (b >> 4) ^ (n & 7);
    return (uint32_t)(((d >> 5) << 14) + ((n >> 3) << 10) + ((n & 7) << 7) + (u << 4) + (b & 15));
}

// byte offset of (codeword k < 256, dim d) of the stage's [256][128] fp32
// codewords: the same layout with K chunks of 256 rows at 32 KB steps
__device__ __forceinline__ uint32_t enc_off_cb(int k, int d) {
    const int b = (d & 31) << 2;
    const int u = (b >> 4) ^ (k & 7);
    return (uint32_t)(((d >> 5) << 15) + ((k >> 3) << 10) + ((k & 7) << 7) + (u << 4) + (b & 15));
}

// UMMA shared-memory descriptor: K-major SWIZZLE_128B, SBO 1024 B (8-row
// atoms), LBO unused (1); the start address may step inside an atom by the
// 32 bytes of one K step (the swizzle works on absolute address bits)
__device__ __forceinline__ uint64_t enc_desc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void enc_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// instruction descriptor: D fp32, A/B tf32, both K-major, N = 256, M = 128
constexpr uint32_t kEncIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

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

// 16 fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void enc_tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// float order as unsigned order (NaN-free inputs)
__device__ __forceinline__ uint32_t enc_okey(float x) {
    const uint32_t b = __float_as_uint(x);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float enc_okey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
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

// ||C||^2 of every codeword (sequential fma over d), for the ICM sweeps.
__global__ void __launch_bounds__(256) encode_norms_kernel(const float* cb, int64_t n, float* nrm) {
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
}

// REP = 128 / vectors per CTA.  CTAs of 16, 32 or 64 vectors hold REP copies of
// their residual rows in the MMA's 128 rows (rows otherwise computed on
// zeros), so that every TMEM lane quarter, and with it every warp, holds
// rows: each thread filters 64 / REP of a row's 256 columns, and the
// per-row steps spread over all warps (and schedulers) instead of the
// quarter-0 warps.
template <typename XT, int REP>
__global__ void __launch_bounds__(kEncThreads, 1)
    encode_keys_kernel(const __grid_constant__ CUtensorMap cmap, EncodeParams p) {
    extern __shared__ unsigned char smem_raw[];
    // operands need 1024-byte alignment (SWIZZLE_128B atoms)
    // (offset from the shared array itself, so that the compiler keeps every
    // access below a shared-memory access rather than a generic one)
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* sA = smem;
    unsigned char* sB = smem + EncSmem::kA;  // half hf, K chunk c at hf * 64 KB + c * 16 KB
    float* sNorm = reinterpret_cast<float*>(sB + 2 * EncSmem::kBHalf);  // [2][||C||^2 of 256 codewords | . .]
    uint64_t* s_mbar = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(sNorm) + EncSmem::kNorm);
    uint64_t* s_tbar = s_mbar + 1;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int set = blockIdx.x / p.ctas_per_set;
    const int tile = blockIdx.x - set * p.ctas_per_set;
    const int nvec_set = p.per_head ? p.B * p.T : p.B * p.H * p.T;  // vectors of this set
    const int v0 = tile * p.rows_per_cta;

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
    // stage m's 256 codewords: 8 tensor copies (2 halves x 4 K chunks), one thread
    auto issue_stage = [&](int m) {
        mbar_arrive_expect_tx(s_tbar, (uint32_t)(2 * EncSmem::kBHalf));
        const int row0 = (set * kEncM + m) * kEncK;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int c = 0; c < 4; ++c) enc_tma_2d(sB + c * 32768 + hf * 16384, &cmap, 32 * c, row0 + 128 * hf, s_tbar);
    };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&s_tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(s_mbar, 1);
        mbar_init(s_tbar, 1);
        fence_barrier_init();
        s_abort = 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&cmap)) : "memory");
        issue_stage(0);
    }
    // the CTA's vectors -> residuals (fp32); rows past the set's end are zero
    for (int e = tid; e < kEncRows * (kEncD / 4); e += kEncThreads) {
        const int n = e >> 5, d = (e & 31) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        const int nv = REP > 1 ? n % (kEncRows / REP) : n;  // the vector of row n
        if (nv < p.rows_per_cta && v0 + nv < nvec_set) {
            int b, h, t;
            vec_bht(v0 + nv, &b, &h, &t);
            const XT* xr = reinterpret_cast<const XT*>(p.x) + (int64_t)b * p.xs_b + (int64_t)h * p.xs_h + (int64_t)t * p.xs_t;
            v = make_float4(to_f32(xr[d]), to_f32(xr[d + 1]), to_f32(xr[d + 2]), to_f32(xr[d + 3]));
        }
        *reinterpret_cast<float4*>(sA + enc_off(n, d)) = v;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    // epilogue: warp w reads TMEM lane quarter q = w & 3 (vector rows
    // 32q .. 32q+31) and the 64 columns of group cg = w >> 2
    const int q4 = warp & 3, cg = warp >> 2;
    const int row = q4 * 32 + lane;
    // REP > 1: the thread's copy rep, vector row rr (row of copy 0) and
    // first of its W columns
    constexpr int RP = kEncRows / REP, W = 64 / REP;
    const int rep = row / RP;
    const int rr = row % RP;
    const int c0 = 64 * cg + W * rep;
    const bool row_valid = row < p.rows_per_cta && v0 + row < nvec_set;
    __shared__ uint8_t* s_cptr[kEncRows];         // the row's 32 codes in the output (null: no vector)
    __shared__ __align__(16) uint8_t s_codes[kEncRows][kEncM];
    if (cg == 0) {
        uint8_t* co = nullptr;
        if (row_valid) {
            int b, h, t;
            vec_bht(v0 + row, &b, &h, &t);
            co = p.codes + (int64_t)b * p.cs_b + (int64_t)h * p.cs_h + (int64_t)t * p.cs_t;
        }
        s_cptr[row] = co;
    }
    // |exact dist - (approx dist + ||r||^2)| <= kEps ||r|| ||c_k|| + kAbs (||r||^2 + ||c_k||^2 + |approx|):
    // the tf32 operands (10 mantissa bits) and fp32 accumulation give about
    // 2^-8 ||r|| ||c|| (Cauchy-Schwarz), the fp32 roundings of the exact
    // formula about 2^-23 of the magnitudes; both are taken with a margin of 2
    // or more
    constexpr float kEps = 1.0f / 128.0f;
    constexpr float kAbs = 1.0f / 1048576.0f;
    __shared__ float s_rn[kEncRows];
    __shared__ float s_wmx[kEncK / 32][2];  // per warp of the norm threads: max ||c||^2, max ||c||
    __shared__ float s_u[4][kEncRows];
    __shared__ int s_cnt[4][kEncRows];
    __shared__ int s_bk[4][kEncRows];               // the group's first candidate (-1: none)
    // REP > 1: per vector row the ordered key of the smallest approximation,
    // the candidate count and the smallest candidate (reset every stage)
    __shared__ uint32_t s_umin[REP > 1 ? kEncRows / REP : 1];
    __shared__ int s_cnt1[REP > 1 ? kEncRows / REP : 1];
    __shared__ int s_bk1[REP > 1 ? kEncRows / REP : 1];
    __shared__ unsigned long long s_best[kEncRows];  // (ordered exact distance, codeword), minimum
    __shared__ uint32_t s_list[kEncListCap];         // (row << 8) | codeword
    __shared__ int s_nlist[2];

    for (int m = 0; m < kEncM; ++m) {
        const uint32_t par = (uint32_t)(m & 1);
        // this stage's codewords (tensor copies) and norms have landed
        const bool landed = mbar_wait(s_tbar, par, p.err);
        cp_async_wait<0>();
        fence_proxy_async();  // residual writes (generic) -> async proxy (MMA)
        if (__syncthreads_or(!landed)) {
            if (tid == 0) s_abort = 1;
            mbar_wait(s_tbar, par, nullptr);  // copies may still run: bounded second wait
            break;
        }
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            // K step s: 32 bytes into K chunk s / 4 (16 KB of residual rows,
            // 32 KB of codeword rows); all 256 codewords in one N = 256 MMA
#pragma unroll
            for (int s = 0; s < kEncD / 8; ++s) {
                const uint32_t koa = (uint32_t)((s >> 2) * 16384 + (s & 3) * 32);
                const uint32_t kob = (uint32_t)((s >> 2) * 32768 + (s & 3) * 32);
                enc_mma(tmem, enc_desc(a0 + koa), enc_desc(b0 + kob), s > 0 ? 1u : 0u);
            }
            enc_commit(s_mbar);
        }
        // meanwhile: ||r||^2 of each row, exactly (sequential fma in d order)
        if (cg == 0 && rep == 0) {
            float rn = 0.f;
#pragma unroll 4
            for (int d4 = 0; d4 < kEncD / 4; ++d4) {
                const float4 r4 = *reinterpret_cast<const float4*>(sA + enc_off(row, d4 * 4));
                rn = __fmaf_rn(r4.x, r4.x, rn);
                rn = __fmaf_rn(r4.y, r4.y, rn);
                rn = __fmaf_rn(r4.z, r4.z, rn);
                rn = __fmaf_rn(r4.w, r4.w, rn);
            }
            s_rn[row] = rn;
            if constexpr (REP > 1) {
                s_umin[row] = ~0u;
                s_cnt1[row] = 0;
                s_bk1[row] = 0x7fffffff;
            }
        }
        // meanwhile: the stage's codeword norms ||c||^2 from its copies in
        // shared memory (threads 256..511, one codeword each; the sequential
        // fma chain in d order of the CPU arithmetic) and, per warp, the
        // largest ||c||^2 and ||c|| (rounded up)
        if (tid >= kEncThreads - kEncK) {
            const int k = tid - (kEncThreads - kEncK);
            float acc = 0.f;
#pragma unroll 8
            for (int d4 = 0; d4 < kEncD / 4; ++d4) {
                const float4 c = *reinterpret_cast<const float4*>(sB + enc_off_cb(k, d4 * 4));
                acc = __fmaf_rn(c.x, c.x, acc);
                acc = __fmaf_rn(c.y, c.y, acc);
                acc = __fmaf_rn(c.z, c.z, acc);
                acc = __fmaf_rn(c.w, c.w, acc);
            }
            sNorm[(m & 1) * EncSmem::kNormStride + k] = acc;
            float a = acc, cn = __fmul_ru(__fsqrt_ru(acc), 1.0000001f);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
                cn = fmaxf(cn, __shfl_xor_sync(0xffffffffu, cn, o));
            }
            if (lane == 0) {
                s_wmx[warp - (kEncThreads - kEncK) / 32][0] = a;
                s_wmx[warp - (kEncThreads - kEncK) / 32][1] = cn;
            }
        }
        const bool done = mbar_wait(s_mbar, par, p.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__syncthreads_or(!done)) {
            if (tid == 0) s_abort = 1;
            mbar_wait(s_mbar, par, nullptr);  // the MMAs may still run: bounded second wait
            break;
        }
        const float* nb = sNorm + (m & 1) * EncSmem::kNormStride;
        // the stage's largest ||c||^2 and ||c||
        float nmax = s_wmx[0][0], cmax = s_wmx[0][1];
#pragma unroll
        for (int w = 1; w < kEncK / 32; ++w) {
            nmax = fmaxf(nmax, s_wmx[w][0]);
            cmax = fmaxf(cmax, s_wmx[w][1]);
        }
        int total;
        uint64_t pend;
        if constexpr (REP == 1) {
            const float rn = s_rn[row];
            const float rnorm = __fmul_ru(__fsqrt_ru(rn), 1.0000001f);
            // the bound's absolute part, one upper bound per row: |approx| <=
            // ||c||^2 + 2 ||r|| ||c|| <= nmax + 2 rnorm cmax
            const float slack = kAbs * (rn + 2.f * (nmax + rnorm * cmax));
            // the row's bound for every codeword of the stage: kEps ||r|| max ||c|| + slack
            const float bnd = __fmaf_ru(kEps * rnorm, cmax, slack);
            const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) + 64 * cg;
            float v[64];
            enc_tmem_ld64(taddr, v);
            // pass 1: the row's smallest approximate distance A (less ||r||^2)
            float u = INFINITY;
    #pragma unroll
            for (int i = 0; i < 64; ++i) {
                const float ap = fmaf(-2.f, v[i], nb[64 * cg + i]);
                v[i] = ap;
                u = fminf(u, ap);
            }
            s_u[cg][row] = u;
            __syncthreads();
            // pass 2: candidates approx_k <= A + 2 bnd -- the winner's exact
            // distance is at most A + bnd and its approximation at most bnd below
            // that (bit i of the mask = column 64cg + i)
            const float thr = __fmaf_ru(2.f, bnd, fminf(fminf(s_u[0][row], s_u[1][row]), fminf(s_u[2][row], s_u[3][row])));
            uint32_t cm0 = 0u, cm1 = 0u;
    #pragma unroll
            for (int i = 0; i < 64; ++i) {
                const bool c = p.force_exact || v[i] <= thr;
                if (i < 32) cm0 |= (uint32_t)c << i;
                else cm1 |= (uint32_t)c << (i - 32);
            }
            s_cnt[cg][row] = __popc(cm0) + __popc(cm1);
            s_bk[cg][row] = cm0 ? __ffs(cm0) - 1 + 64 * cg : (cm1 ? __ffs(cm1) + 31 + 64 * cg : -1);
            if (cg == 0) s_best[row] = ~0ull;
            if (tid == 0) {
                s_nlist[0] = 0;
                s_nlist[1] = 0;
            }
            __syncthreads();
            total = s_cnt[0][row] + s_cnt[1][row] + s_cnt[2][row] + s_cnt[3][row];
            // a row with several candidates: their exact distances, one (row,
            // codeword) pair per 8 lanes through a CTA-wide list (rounds of at most
            // kEncListCap pairs); the smallest (distance, codeword) key is the
            // first minimum of the CPU scan
            pend = total > 1 ? ((uint64_t)cm1 << 32) | cm0 : 0ull;
        } else {
            // the same bound and passes over the thread's W columns of row
            // rr; per-row minimum, count and first candidate by shared atomics
            const float rn = s_rn[rr];
            const float rnorm = __fmul_ru(__fsqrt_ru(rn), 1.0000001f);
            const float slack = kAbs * (rn + 2.f * (nmax + rnorm * cmax));
            const float bnd = __fmaf_ru(kEps * rnorm, cmax, slack);
            const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) + c0;
            float v[W];
            if constexpr (W == 8) {
                // two copies per lane quarter: the warp loads their 16
                // columns at one (warp-uniform) address, each half-warp keeps
                // its own 8
                float w[16];
                enc_tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + 64 * cg + 16 * q4, w);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = (lane & 16) ? w[8 + i] : w[i];
            } else {
                enc_tmem_ld16(taddr, v);
                if constexpr (W == 32) enc_tmem_ld16(taddr + 16, v + 16);
            }
            float u = INFINITY;
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float ap = fmaf(-2.f, v[i], nb[c0 + i]);
                v[i] = ap;
                u = fminf(u, ap);
            }
            atomicMin(&s_umin[rr], enc_okey(u));
            __syncthreads();
            const float thr = __fmaf_ru(2.f, bnd, enc_okey_inv(s_umin[rr]));
            uint32_t cm = 0u;
#pragma unroll
            for (int i = 0; i < W; ++i) cm |= (uint32_t)(p.force_exact || v[i] <= thr) << i;
            if (cm) {
                atomicAdd(&s_cnt1[rr], __popc(cm));
                atomicMin(&s_bk1[rr], c0 + __ffs(cm) - 1);
            }
            if (cg == 0 && rep == 0) s_best[rr] = ~0ull;
            if (tid == 0) {
                s_nlist[0] = 0;
                s_nlist[1] = 0;
            }
            __syncthreads();
            total = s_cnt1[rr];
            pend = total > 1 ? (uint64_t)cm : 0ull;
        }
        for (int round = 0;; ++round) {
            int* nl = &s_nlist[round & 1];
            const bool had = pend != 0ull;
            // the warp's pairs take one range of the list (one atomic per warp)
            const int mine = __popcll((long long)pend);
            int incl = mine;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            int base = 0;
            if (lane == 31 && incl > 0) base = atomicAdd(nl, incl);
            base = __shfl_sync(0xffffffffu, base, 31);
            for (int i = base + incl - mine; pend && i < kEncListCap; ++i) {
                s_list[i] = ((uint32_t)rr << 8) | (uint32_t)(__ffsll((long long)pend) - 1 + c0);
                pend &= pend - 1;
            }
            if (!__syncthreads_or(had)) break;
            if (tid == 0) s_nlist[(round + 1) & 1] = 0;  // the next round's counter (last read a round ago)
            const int n = min(*nl, kEncListCap);
            // 8 lanes per pair, 4 pairs per warp: lane l8 of a group holds
            // the order's lanes 8j + l8 (dims 32j + 4 l8 .. +3, j = 0..3), so
            // the strides 16 and 8 of the butterfly are its own additions and
            // 4, 2, 1 are shuffles; each 16-byte load of a group covers one
            // 128-byte row segment.  The loop is warp-uniform: every lane
            // takes part in the shuffles.
            for (int e0 = warp * 4; e0 < n; e0 += kEncThreads / 8) {
                const int e = e0 + (lane >> 3), l8 = lane & 7;
                const bool live = e < n;
                float dot = 0.f;
                int r = 0, k = 0;
                if (live) {
                    const uint32_t it = s_list[e];
                    r = (int)(it >> 8);
                    k = (int)(it & 255u);
                    float pj[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float4 r4 = *reinterpret_cast<const float4*>(sA + enc_off(r, 32 * j + 4 * l8));
                        const float4 cv = *reinterpret_cast<const float4*>(sB + enc_off_cb(k, 32 * j + 4 * l8));
                        float a = __fmaf_rn(r4.x, cv.x, 0.f);
                        a = __fmaf_rn(r4.y, cv.y, a);
                        a = __fmaf_rn(r4.z, cv.z, a);
                        pj[j] = __fmaf_rn(r4.w, cv.w, a);
                    }
                    dot = __fadd_rn(__fadd_rn(pj[0], pj[2]), __fadd_rn(pj[1], pj[3]));
                }
#pragma unroll
                for (int o = 4; o > 0; o >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
                if (live && l8 == 0) {
                    // +0 folds a -0 into +0, so that equal distances have equal keys
                    const float dist = __fadd_rn(__fmaf_rn(-2.f, dot, __fadd_rn(s_rn[r], nb[k])), 0.f);
                    uint32_t key = __float_as_uint(dist);
                    key = (key & 0x80000000u) ? ~key : (key | 0x80000000u);  // float order as unsigned order
                    atomicMin(&s_best[r], ((unsigned long long)key << 32) | (unsigned)k);
                }
            }
            if (!__syncthreads_or(pend != 0ull)) break;
        }
        // the code: the refined minimum, else the one candidate (one group has it)
        const int code = total > 1 ? (int)(s_best[rr] & 0xffu)
                         : REP > 1 ? min(s_bk1[rr], kEncK - 1)
                                   : max(max(max(s_bk[0][row], s_bk[1][row]), max(s_bk[2][row], s_bk[3][row])), 0);
        if (cg == 0 && rep == 0) s_codes[rr][m] = (uint8_t)code;
        // r - C_m[code] into registers (the row's 4 column groups take 32
        // dims each, split over the REP copies' threads): the subtractions
        // consume the codeword loads before the barrier, after which the next
        // stage's copies overwrite the codewords; the stores (into every copy
        // of the row) follow the copies' issue
        constexpr int NF = 8 / REP;  // float4 slices of the thread
        float4 nr[NF];
        {
#pragma unroll
            for (int j = 0; j < NF; ++j) {
                const int d = (8 * cg + NF * rep + j) * 4;
                const float4 cv = *reinterpret_cast<const float4*>(sB + enc_off_cb(code, d));
                const float4 r4 = *reinterpret_cast<const float4*>(sA + enc_off(row, d));
                nr[j] = make_float4(__fsub_rn(r4.x, cv.x), __fsub_rn(r4.y, cv.y), __fsub_rn(r4.z, cv.z),
                                    __fsub_rn(r4.w, cv.w));
                // the differences exist before the barrier (the compiler may
                // not sink them, and with them the wait for the loads, past it)
                asm volatile("" : "+f"(nr[j].x), "+f"(nr[j].y), "+f"(nr[j].z), "+f"(nr[j].w));
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();  // the stage's codewords are no longer read: the next stage's copies start
        if (m + 1 < kEncM) {
            if (tid == 0) issue_stage(m + 1);
        }
        // (visible to the next stage's MMA after the barrier that starts it)
#pragma unroll
        for (int j = 0; j < NF; ++j)
#pragma unroll
            for (int c = 0; c < REP; ++c)
                *reinterpret_cast<float4*>(sA + enc_off(c * (kEncRows / REP) + rr, (8 * cg + NF * rep + j) * 4)) = nr[j];
    }
    cp_async_wait<0>();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // the codes, 32 bytes per vector
    if (!s_abort) {
        for (int e = tid; e < kEncRows * kEncM; e += kEncThreads) {
            uint8_t* co = s_cptr[e >> 5];
            if (co) co[e & 31] = s_codes[e >> 5][e & 31];
        }
    }
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
    }
}

}  // namespace lp
