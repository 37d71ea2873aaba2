// fused_step.cuh -- the whole sparse decode step of one layer in ONE
// persistent cooperative kernel (one CTA per SM).
//
// Reference path replaced: laprune/llm/aq_kv.py:633-699 (LUT build +
// grouped scorer), laprune/llm/modifiers/aq_evaluation.py:185-253 (candidate
// window, top-k, keep set, GQA gather, SDPA) -- here with per-KV-head
// selection on GQA-summed scores (the benchmark configs).
//
// Why one kernel: at decode sizes every stage after the two HBM streams is a
// short chain of dependent L2 round trips (histogram -> threshold -> bitmap
// -> ties -> row list -> gather -> merge).  Separate kernels pay a launch
// ramp, a tail and a global round trip for every intermediate; here the
// intermediates stay in shared memory and the stages are separated by
// four barriers among the CTAs of one unit.  Units never wait for each
// other, so a unit whose LUT is ready streams its codes while others are
// still building theirs.
//
// Phases (CTA c belongs to one selection unit u = (b, kv head)):
//   A  LUT build: the CTAs of the units that read one codebook (a LUT
//      group) split its 32*256 codeword rows evenly, write LUT_sum[u][k][m]
//      = q_sum(u) . C_m[k] (fp32) of every unit u of the group to L2 and
//      raise an epoch-tagged flag each.                   | the unit's flags
//   B  score: the unit's table is staged as int32 fixed point (exact sums,
//      order-independent), the per-m bounds are recomputed from the table in
//      shared memory (identical in every CTA of the unit), the CTA's code
//      rows come straight from global memory into registers (one 256-bit
//      load per token, the next step's rows in flight), scores stay in
//      shared memory (or the L2-resident score buffer for long shares),
//      histogram -> global.                                            | barrier
//   C  select: bin b* of the k-th score from the unit histogram; ballots give
//      the CTA's above-threshold tokens (row list in shared memory) and its
//      tie-bin tokens (written to its own slot of the tie buffer).  The K/V
//      rows known at this point -- above-threshold tokens and the CTA's share
//      of the sink and local-window rows -- start loading (cp.async) before
//      the barrier.                                                     | barrier
//   D  ties: every CTA gathers the unit's tie-bin tokens from the slots of
//      its CTAs and ranks its own ones against all -- no barrier.  If the
//      unit overflowed the tie capacity, its leader runs the exact radix
//      select on the global scores and one more unit barrier follows.
//   E  attention: the tie winners' rows are gathered while the logits of
//      the early rows are computed; all G query heads of the KV head attend
//      the CTA's rows (online softmax); the slice state goes to L2.  | barrier
//   M  merge: each CTA of the unit combines the slice states of a 1/cn share
//      of the unit's G*128 outputs and writes them.
//
// Every wait (TMA ring, unit barrier) is bounded; on timeout the CTA records
// LP_DEVERR_WAIT_TIMEOUT, drains its own copies and exits.
#pragma once
#include <type_traits>
#include <cub/block/block_scan.cuh>
#include "attention.cuh"
#include "lut_build.cuh"
#include "score.cuh"
#include "select.cuh"

namespace lp {

constexpr int kFThreads = 512;
constexpr int kFStages = 6;
constexpr int kFPre0 = 2;                        // ring slots kept free ahead of phase A's group queries
constexpr int kFTile = kFThreads * 32;           // 16 KB of code rows per stage
constexpr int kFScoreCap = 11264;                // tokens per CTA kept in smem
constexpr int kFMaxWords = 8192;                 // bitmap words per unit in smem overlay
constexpr int kFMaxRows = 192;                   // K/V staging rows in the ring (phase C's early rows)
constexpr int kFLutRows = 128;                   // more staging rows in the table region (phase E only)
constexpr int kPubWin = 128;                     // bins in a CTA's published count window
constexpr int kPubMaxCtas = 64;                  // CTAs per unit of the published-candidate path
constexpr int kPubMaxCap = 2048;                 // published candidates per CTA (own copy in shared memory)
constexpr int kFastTieCap = 1024;                // tie-bin entries the fast selection path settles
constexpr int kFusedQMaxG = 8;                   // query heads per unit summed into a LUT query
// spill mode (a CTA's share above kFScoreCap tokens): the scores go to the
// L2-resident global buffer and the shared-memory score region holds the row
// list and the CTA's selection bitmaps instead
constexpr int kFSpillList = 5120;                // row list entries (above-threshold + tie winners <= k)
constexpr int kFSpillWords = 2112;               // own bitmap words of a CTA (tokens <= 32 * 2110)
constexpr int kFSpillMaxTok = 32 * (kFSpillWords - 2);
static_assert((kFSpillList + 2 * kFSpillWords) * 4 <= kFScoreCap * 4, "spill overlays fit the score region");

struct FusedParams {
    const void* q;
    int64_t q_stride_b, q_stride_h;
    const void* cb;      // codebooks of cb_dtype (LP_F32 | LP_F16 | LP_BF16)
    int cb_dtype;
    int cb_per_kv_head;
    const uint8_t* codes;
    int64_t codes_stride_b, codes_stride_h;
    const void* keys;
    const void* vals;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    int Hkv, G, U;     // G: query heads attended per unit
    int B;             // sequences
    int Hu, upk;       // units per sequence, units per KV head (1: KV-group units, G: query-head units)
    int spill;         // 1: the CTAs' shares exceed the shared-memory score buffer; scores live in sel_scores
    int c0, c1, k;
    int n_sink, local_start, n_local, n_rows, T_total;
    float scale_log2;
    void* out;
    int64_t out_stride_b, out_stride_h;
    int32_t* topk_out;
    // workspace
    float* lut;                // [U][256][32] fp32 LUT_sum, plain stores
    unsigned long long* lut_flag;  // [gridDim.x] tagged: CTA j's share of its unit's LUT is written
    float* sel_scores;   // [U][sel_stride]
    int64_t sel_stride;
    uint32_t* chist;     // [gridDim.x][kNB] local score histogram of each CTA (exchange path)
    uint32_t* bitmap;    // [U][bm_stride]
    int64_t bm_stride;
    float2* tie_buf;     // [gridDim.x][kTieCap] tie-bin tokens of each CTA
    uint32_t* cta_ties;  // [gridDim.x] tie-bin token count of each CTA
    uint32_t* cta_count; // [gridDim.x] selected-above-threshold count of each CTA
    unsigned long long* pub;   // [gridDim.x][pub_cap][2] tagged (score, token) candidates of each CTA
    unsigned long long* pwin;  // [gridDim.x][kPubWin + 2] tagged bin-count window, count, threshold bin
    int pub_target;      // candidates each CTA aims to publish
    int pub_cap;         // slot capacity (0: no publishing, exchange path only)
    unsigned long long* part;  // [U][max_split][G][2+128] tagged split-K states (max, sum, P.V)
    int max_split;
    int test_timeout;          // LP_FLAG_TEST_WAIT_TIMEOUT: CTA 0 withholds its LUT flag; short LUT waits
    unsigned long long* bar;  // [U] unit barrier words (persistent; epoch-tagged arrival counts)
    unsigned long long* epoch_ctr;  // persistent launch counter: this call's epoch tags its exchanged words
    uint32_t* err;
    unsigned long long* phase_ns;  // optional [8] globaltimer stamps (CTA 0)
    const char* pf_ptr[2];         // L2 prefetch of the next call's inputs
    int64_t pf_bytes[2], pf_count[2], pf_stride[2];
};

// This CTA's share of an L2 prefetch region (count blocks of `bytes` every
// `stride` bytes), split evenly over the grid in 16-byte granules.
__device__ __forceinline__ void prefetch_share(const char* ptr, int64_t bytes, int64_t count, int64_t stride) {
    if (!ptr || bytes <= 0 || count <= 0) return;
    const int64_t total = bytes * count;
    const int64_t per = ((total + gridDim.x - 1) / gridDim.x + 15) & ~(int64_t)15;
    int64_t a = (int64_t)blockIdx.x * per;
    const int64_t e = min(total, a + per);
    while (a < e) {
        const int64_t blk = a / bytes, off = a - blk * bytes;
        int64_t n = min(e - a, bytes - off);
        n = min(n, (int64_t)65536);
        const int64_t n16 = n & ~(int64_t)15;
        if (n16 > 0) {
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr + blk * stride + off), "r"((uint32_t)n16)
                         : "memory");
        }
        a += n > 0 ? n : 16;
    }
}

struct FusedSmem {
    static constexpr int kLut = 256 * 64 * 4;          // 64 KB (phase B table; reused)
    static constexpr int kRing = kFStages * kFTile;    // 96 KB (phase B ring; reused in E)
    static constexpr int kHist = kNB * 4;              // 8 KB
    static constexpr int kScores = kFScoreCap * 4;     // 48 KB
    static constexpr int kBars = (2 * kFStages + 3) * 8;  // ring full + empty, 3 phase-A stages
    static constexpr int kTotal = kLut + kRing + kHist + kScores + kBars + 128;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Fine-grained timeline for kernel development: built with -DLP_FUSED_TRACE,
// thread 0 of CTA 0 and of the grid's last CTA stamp step i into
// phase_ns[8 + i] and phase_ns[40 + i] (the caller then passes 72 words).
// Off in the library build.
#ifdef LP_FUSED_TRACE
#define LP_FTRACE(i)                                                                          \
    do {                                                                                      \
        if (p.phase_ns && threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1)) \
            p.phase_ns[8 + (blockIdx.x ? 32 : 0) + (i)] = global_ns();                        \
    } while (0)
#else
#define LP_FTRACE(i) \
    do {             \
    } while (0)
#endif


// Words exchanged between the CTAs of a unit carry the call's epoch in their
// upper 32 bits; a reader polls a word until it shows the epoch.  A 64-bit
// access is single-copy atomic, so value and tag arrive together and no
// fence or barrier is needed between writer and reader.  Stale words (earlier
// calls, or zero-filled memory) carry smaller epochs.
__device__ __forceinline__ void st_tag(unsigned long long* p, uint32_t v, uint32_t epoch) {
    const unsigned long long x = ((unsigned long long)epoch << 32) | v;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(x) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tag(const unsigned long long* p) {
    unsigned long long x;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(x) : "l"(p) : "memory");
    return x;
}
__device__ __forceinline__ unsigned long long ld_tag_acquire(const unsigned long long* p) {
    unsigned long long x;
    asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(x) : "l"(p) : "memory");
    return x;
}
__device__ __forceinline__ bool tag_ok(unsigned long long x, uint32_t epoch) {
    return (uint32_t)(x >> 32) == epoch;
}

// Barrier among the n CTAs of one selection unit (all resident: cooperative
// launch).  The unit's 64-bit word holds (epoch << 32 | arrivals of this
// call): the first arrival of a call replaces a word that still shows an
// older epoch, later ones add 1 (compare-and-swap, lock-free: a failed swap
// means another CTA's arrival succeeded).  Barrier number nb of the call is
// complete once the word shows this epoch and nb*n arrivals.  Nothing is
// read before the first arrival and nothing needs a reset between calls,
// also after a call that timed out.  Units never wait for one another.
// Bounded: returns false on timeout (after recording the error bit).
__device__ __forceinline__ bool unit_barrier(unsigned long long* bar, int n, int& nb, uint32_t epoch, uint32_t* err) {
    __shared__ int s_ok;
    ++nb;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();  // the CTA's writes before its arrival
        unsigned long long old = ld_tag(bar);
        while (true) {
            const unsigned long long nv =
                tag_ok(old, epoch) ? old + 1ull : (((unsigned long long)epoch << 32) | 1ull);
            const unsigned long long prev = atomicCAS(bar, old, nv);
            if (prev == old) break;
            old = prev;
        }
        const uint32_t target = (uint32_t)(nb * n);
        int ok = 1;
        const long long t0 = clock64();
        while (true) {
            const unsigned long long v = ld_tag_acquire(bar);
            if (tag_ok(v, epoch) && (uint32_t)v >= target) break;
            if (clock64() - t0 > kWaitCycles) {
                atomicOr(err, LP_DEVERR_WAIT_TIMEOUT);
                ok = 0;
                break;
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// dst[i] = value of src[i] for i in [0, n), each polled until it carries
// `epoch`; the CTA's threads take i = tid + k * blockDim.x, 4 loads in flight
// per thread.  Bounded: false (and the error bit) on timeout.
__device__ __forceinline__ bool poll_copy(uint32_t* dst, const unsigned long long* src, int n, uint32_t epoch,
                                          uint32_t* err) {
    constexpr int UNR = 4;
    const long long t0 = clock64();
    for (int i0 = threadIdx.x; i0 < n; i0 += blockDim.x * UNR) {
        unsigned long long w[UNR];
        uint32_t pend = 0u;
#pragma unroll
        for (int r = 0; r < UNR; ++r) {
            const int i = i0 + r * blockDim.x;
            if (i < n) {
                w[r] = ld_tag(src + i);
                pend |= 1u << r;
            }
        }
        while (true) {
#pragma unroll
            for (int r = 0; r < UNR; ++r) {
                if ((pend >> r & 1u) && tag_ok(w[r], epoch)) {
                    dst[i0 + r * blockDim.x] = (uint32_t)w[r];
                    pend &= ~(1u << r);
                }
            }
            if (!pend) break;
            if (clock64() - t0 > kWaitCycles) {
                atomicOr(err, LP_DEVERR_WAIT_TIMEOUT);
                return false;
            }
#pragma unroll
            for (int r = 0; r < UNR; ++r)
                if (pend >> r & 1u) w[r] = ld_tag(src + i0 + r * blockDim.x);
        }
    }
    return true;
}

// CTA -> (unit, index within unit, CTAs of the unit)
__device__ __forceinline__ void fused_cta_unit(int cta, int nctas, int U, int* u, int* j, int* n) {
    const int base = nctas / U, extra = nctas % U;
    if (cta < extra * (base + 1)) {
        *u = cta / (base + 1); *j = cta - *u * (base + 1); *n = base + 1;
    } else {
        const int i = cta - extra * (base + 1);
        *u = extra + i / base; *j = i - (*u - extra) * base; *n = base;
    }
}
// first CTA of unit u (u == U: one past the last CTA)
__device__ __forceinline__ int fused_unit_first_cta(int u, int nctas, int U) {
    const int base = nctas / U, extra = nctas % U;
    return u < extra ? u * (base + 1) : extra * (base + 1) + (u - extra) * base;
}

// Units are ordered KV head first (v = (hkv * B + b) * upk + g), so the units
// that read one codebook -- every unit of a KV head with per-KV-head
// codebooks, all of them with a shared one -- are consecutive, and so are
// their CTAs.  A LUT group is such a run of at most kFLutGroup units; its
// CTAs split the codebook's rows once and build every member's table.
constexpr int kFLutGroup = 64;
__device__ __forceinline__ void fused_lut_group(int v, int U, int cb_units, int* g0, int* g1) {
    const int c0 = v / cb_units * cb_units;           // this codebook's run of units
    const int cnt = min(cb_units, U - c0);
    const int nsub = (cnt + kFLutGroup - 1) / kFLutGroup;
    const int r = v - c0;
    int s = r * nsub / cnt;                            // sub-run s covers [s*cnt/nsub, (s+1)*cnt/nsub)
    while (s + 1 < nsub && (s + 1) * cnt / nsub <= r) ++s;
    while (s > 0 && s * cnt / nsub > r) --s;
    *g0 = c0 + s * cnt / nsub;
    *g1 = c0 + (s + 1) * cnt / nsub;
}

// ---- warp-level tensor-core tiles for phase E (mma.sync m16n8k16, fp32
//      accumulators; A row-major, B column-major; A and B of one type) ----
template <typename KT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (std::is_same<KT, __nv_bfloat16>::value) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&v);
    } else {
        const __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&v);
    }
}
template <typename KT>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
    if constexpr (std::is_same<KT, __nv_bfloat16>::value) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
    }
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

template <typename QT, typename KT, typename OT>
__global__ void __launch_bounds__(kFThreads, 1) sparse_decode_fused_kernel(FusedParams p) {
    using S = FusedSmem;
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* s_lut = smem;
    unsigned char* s_ring = smem + S::kLut;
    uint32_t* s_hist = reinterpret_cast<uint32_t*>(s_ring + S::kRing);
    float* s_scores = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(s_hist) + S::kHist);
    uint64_t* s_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(s_scores) + S::kScores);

    __shared__ BinParams s_bp;
    __shared__ __align__(16) float s_qu[8 * 128];  // the unit's G query rows (fp32), loaded at start
    __shared__ int s_shift, s_bstar, s_above;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kFThreads / 32;

    int u, cj, cn;
    fused_cta_unit(blockIdx.x, gridDim.x, p.U, &u, &cj, &cn);
    unsigned long long* ubar = p.bar + u;
    int nbar = 0;  // unit barriers passed in this call (uniform over the unit's CTAs)
    __shared__ uint32_t s_epoch;
    // unit u = (KV head hkv, sequence b, unit head hu) in KV-head-major order;
    // its codes, codebook and K/V rows are those of KV head hkv, its query
    // rows hu*G .. hu*G + G - 1; ul is its index in the caller's (b, hu)
    // order (rows of the top-k output)
    const int gi = u % p.upk, hb = u / p.upk, hkv = hb / p.B, b = hb - hkv * p.B;
    const int hu = hkv * p.upk + gi;
    const int ul = b * p.Hu + hu;
    // the CTA's tokens: a run of whole bitmap words of the candidate window
    const int wlo = p.c0 >> 5, whi = (p.c1 + 31) >> 5;
    const int nwu = whi - wlo;
    const int w_begin = wlo + (int)((int64_t)nwu * cj / cn);
    const int w_end = wlo + (int)((int64_t)nwu * (cj + 1) / cn);
    const int t_begin = max(p.c0, w_begin * 32);
    const int t_end = min(p.c1, w_end * 32);
    const int ntok = max(0, t_end - t_begin);
    const int ntiles = (ntok + kFThreads - 1) / kFThreads;
    const bool keep_smem = !p.spill;  // the plan guarantees ntok <= kFScoreCap then
    const uint8_t* src = p.codes + (int64_t)b * p.codes_stride_b + (int64_t)hkv * p.codes_stride_h;

    uint64_t* s_empty = s_bar + kFStages;      // per-slot "all warps done" barriers
    uint64_t* s_abar = s_bar + 2 * kFStages;   // phase-A codebook stages
    // phase A's share of the codebook's 32*256 rows: split evenly over the
    // ncg CTAs of the unit's LUT group (units gv0 .. gv1-1, which read the
    // same codebook), streamed HBM -> shared memory in 64-row (32 KB) chunks
    // through 3 stages; each row is dotted with the summed query of every
    // unit of the group
    constexpr int64_t kRows = 32 * 256;
    int gv0, gv1;
    fused_lut_group(u, p.U, p.cb_per_kv_head ? p.B * p.upk : p.U, &gv0, &gv1);
    const int gc0 = fused_unit_first_cta(gv0, gridDim.x, p.U);
    const int ncg = fused_unit_first_cta(gv1, gridDim.x, p.U) - gc0;
    const int jg = blockIdx.x - gc0, nq = gv1 - gv0;
    const int64_t f_begin = (kRows * jg / ncg) & ~(int64_t)7;
    const int64_t f_end = jg + 1 == ncg ? kRows : ((kRows * (jg + 1) / ncg) & ~(int64_t)7);
    const int nchunk = (int)((f_end - f_begin + 63) / 64);
    const uint32_t row_bytes = 128u * (uint32_t)cb_elem_bytes(p.cb_dtype);  // one codeword row
    const unsigned char* cbu = static_cast<const unsigned char*>(p.cb) +
                               (int64_t)(p.cb_per_kv_head ? hkv : 0) * kRows * row_bytes;
    auto abuf = [&](int c) -> unsigned char* {
        const int b3 = c % 3;
        return b3 == 2 ? reinterpret_cast<unsigned char*>(s_scores) : s_lut + b3 * 32768;
    };
    auto issue_chunk = [&](int c) {
        const int64_t r0 = f_begin + (int64_t)c * 64;
        const int64_t r1 = min(f_end, r0 + 64);
        mbar_arrive_expect_tx(&s_abar[c % 3], (uint32_t)(r1 - r0) * row_bytes);
        bulk_g2s(abuf(c), cbu + r0 * row_bytes, (uint32_t)(r1 - r0) * row_bytes, &s_abar[c % 3]);
    };
    // the first 3 codebook chunks
    auto issue_inputs = [&]() {
        for (int c = 0; c < 3 && c < nchunk; ++c) issue_chunk(c);
    };
    if (tid == 0) {
        for (int s = 0; s < kFStages; ++s) {
            mbar_init(&s_bar[s], 1);
            mbar_init(&s_empty[s], NW);
        }
        for (int s = 0; s < 3; ++s) mbar_init(&s_abar[s], 1);
        fence_barrier_init();
    }
    // launched with programmatic stream serialisation: nothing of this call
    // touches global memory before the previous kernel on the stream has
    // completed.  The next launch on the stream may be scheduled as soon as
    // every CTA of this grid is past this point: its CTAs take the SMs this
    // grid frees and wait here in turn, so the launch gap hides behind this
    // grid's tail.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool stamp = p.phase_ns != nullptr && blockIdx.x == 0 && tid == 0;
    if (stamp) p.phase_ns[0] = global_ns();
    LP_FTRACE(0);
    if (tid == 0) {
        // the input streams first: the epoch's round trip below overlaps them
        issue_inputs();
        // every CTA of every call adds 1: in call n the old values lie in
        // [G*(n-1), G*n) for G = gridDim.x, whatever the order and even if a
        // CTA of an earlier call returned early
        unsigned long long old;
        asm volatile("atom.add.relaxed.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(p.epoch_ctr) : "memory");
        s_epoch = (uint32_t)(old / gridDim.x) + 1u;
    }
    // (the epoch stays in shared memory, s_epoch: a register held across the
    // scorer would spill; the mbarrier inits and s_epoch are visible to all
    // threads after the barrier that completes s_qu below)
    int issued = 0;  // TMA transfers into the ring (none: the ring is staging space only)
    auto drain = [&](int from) {
        for (int j = from; j < issued; ++j) mbar_wait(&s_bar[j % kFStages], (uint32_t)(j / kFStages) & 1u, nullptr);
    };

    // the unit's own query rows (G * 128 <= 1024 values, at most 2 per
    // thread): loaded into registers here, stored after the group's rows
    // below have been issued, so that all query loads share one round trip
    float qown[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int i = tid + r * kFThreads;
        qown[r] = i < p.G * 128
                      ? to_f32(reinterpret_cast<const QT*>(p.q)[(int64_t)b * p.q_stride_b +
                                                                (int64_t)(hu * p.G + (i >> 7)) * p.q_stride_h + (i & 127)])
                      : 0.f;
    }

    // ================= phase A: LUT build of the CTA's LUT group =================
    // The CTA's codeword rows arrive in the 3 chunk stages issued above;
    // warp w dots rows 4w..4w+3 of a chunk with the summed query of each
    // unit of the group and reduces the 4 dot products with a 6-shuffle
    // transpose.
    {
        // the summed query rows of the group's units (fp32, g in order), in
        // the ring's slots 2.. (free until phase B's publish)
        float* s_qs = reinterpret_cast<float*>(s_ring + kFPre0 * kFTile);  // [nq <= kFLutGroup][128]
        static_assert(kFPre0 * kFTile + kFLutGroup * 128 * 4 <= FusedSmem::kRing, "group queries fit the ring");
        // every head's value loaded before any is added (the G <= 8 loads of
        // an entry are independent), then summed in g order
        for (int i = tid; i < nq * 128; i += kFThreads) {
            const int jq = i >> 7, d = i & 127;
            const int v = gv0 + jq;
            const int vgi = v % p.upk, vhb = v / p.upk, vkv = vhb / p.B, vb = vhb - vkv * p.B;
            const QT* qr = reinterpret_cast<const QT*>(p.q) + (int64_t)vb * p.q_stride_b +
                           (int64_t)((vkv * p.upk + vgi) * p.G) * p.q_stride_h + d;
            float x[kFusedQMaxG];
#pragma unroll
            for (int g = 0; g < kFusedQMaxG; ++g) x[g] = g < p.G ? to_f32(qr[(int64_t)g * p.q_stride_h]) : 0.f;
            float acc = 0.f;
#pragma unroll
            for (int g = 0; g < kFusedQMaxG; ++g)
                if (g < p.G) acc += x[g];
            s_qs[i] = acc;
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
            if (tid + r * kFThreads < p.G * 128) s_qu[tid + r * kFThreads] = qown[r];
        __syncthreads();
        LP_FTRACE(1);
        bool okA = true;
        for (int c = 0; c < nchunk; ++c) {
            if (!mbar_wait(&s_abar[c % 3], (uint32_t)(c / 3) & 1u, p.err)) okA = false;
            if (__syncthreads_or(!okA)) {
                for (int j = c; j < min(nchunk, c + 3); ++j) mbar_wait(&s_abar[j % 3], (uint32_t)(j / 3) & 1u, nullptr);
                drain(0);
                return;
            }
            if (c == 0) LP_FTRACE(2);
            const int64_t r0 = f_begin + (int64_t)c * 64;
            const int64_t fr = r0 + warp * 4;  // first row of this warp (4 rows of the same m)
            if (fr < f_end) {
                const int m = (int)((fr >> 8) & 31);
                const int k0 = (int)(fr & 255);
                const unsigned char* rows = abuf(c) + (warp * 4) * row_bytes;
                float4 cv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    cv[j] = (fr + j < f_end) ? cb_lds4(rows + j * row_bytes, lane, p.cb_dtype)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                const int jr = (lane >> 3) & 3;  // the row whose total this lane ends with
                float* dst = p.lut + ((int64_t)gv0 * 256 + k0 + jr) * 32 + m;
#pragma unroll 4
                for (int jq = 0; jq < nq; ++jq) {  // independent reductions: unrolled to overlap their shuffles
                    const float4 qv = *reinterpret_cast<const float4*>(&s_qs[jq * 128 + lane * 4]);
                    float v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float a = qv.x * cv[j].x;
                        a = fmaf(qv.y, cv[j].y, a);
                        a = fmaf(qv.z, cv[j].z, a);
                        a = fmaf(qv.w, cv[j].w, a);
                        v[j] = a;
                    }
                    // transpose-reduce of 4 values: lane l ends with row (l >> 3) & 3
                    const bool b4 = lane & 16, b3 = lane & 8;
                    float w2[2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const float keep = b4 ? v[2 + j] : v[j];
                        const float send = b4 ? v[j] : v[2 + j];
                        w2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                    }
                    const float keep = b3 ? w2[1] : w2[0];
                    const float send = b3 ? w2[0] : w2[1];
                    float tot = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                    tot += __shfl_xor_sync(0xffffffffu, tot, 4);
                    tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                    tot += __shfl_xor_sync(0xffffffffu, tot, 1);
                    if ((lane & 7) == 0 && fr + jr < f_end) dst[(int64_t)jq * 256 * 32] = tot;
                }
            }
            __syncthreads();  // stage c fully consumed
            if (tid == 0 && c + 3 < nchunk) issue_chunk(c + 3);
        }
    }
    // the CTA's LUT share is out: every thread's stores precede the barrier
    // that ended the last chunk; the fence makes them visible GPU-wide
    // before the flag
    if (tid == 0 && !(p.test_timeout && blockIdx.x == 0)) {
        __threadfence();
        st_tag(p.lut_flag + blockIdx.x, 1u, s_epoch);
    }
    if (stamp) p.phase_ns[1] = global_ns();
    LP_FTRACE(3);
    // the ring's other slots: issued once phase A's codebook stream is done,
    // so that the two streams do not share HBM while the LUT is built


    using Scan = cub::BlockScan<int, kFThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;

    // ================= phase B: score =================
    BinParams bp;
    float from_fx;
    {
        // stage the unit table: fp32 -> per-m bounds -> int32 fixed point (dup
        // layout).  Its rows come from all CTAs of the unit: thread j < cn
        // polls CTA j's flag (acquire) until it carries this call's epoch;
        // after the barrier the table is read from L2.
        float4 v[4];
        {
            bool ok = true;
            if (tid < ncg) {
                const unsigned long long* fl = p.lut_flag + gc0 + tid;  // the LUT group's CTAs
                const long long lim = p.test_timeout ? (1ll << 20) : kWaitCycles;
                const long long t0 = clock64();
                while (!tag_ok(ld_tag_acquire(fl), s_epoch)) {
                    if (clock64() - t0 > lim) {
                        atomicOr(p.err, LP_DEVERR_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
                }
            }
            if (__syncthreads_or(!ok)) { drain(0); return; }
            const float4* gl = reinterpret_cast<const float4*>(p.lut + (int64_t)u * 256 * 32);
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = __ldcg(gl + tid + j * kFThreads);
        }
        if (stamp) p.phase_ns[2] = global_ns();
        LP_FTRACE(4);
        // thread's m group is (tid & 7); reduce min/max per m over k
        // (scratch in the score buffer, which is not written yet)
        float (*s_mmin)[32] = reinterpret_cast<float (*)[32]>(s_scores);
        float (*s_mmax)[32] = s_mmin + NW;
        float mn[4], mx[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a0 = (&v[0].x)[e], a1 = (&v[1].x)[e], a2 = (&v[2].x)[e], a3 = (&v[3].x)[e];
            mn[e] = fminf(fminf(a0, a1), fminf(a2, a3));
            mx[e] = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
        }
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                mn[e] = fminf(mn[e], __shfl_xor_sync(0xffffffffu, mn[e], o));
                mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], o));
            }
        if (lane < 8) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s_mmin[warp][lane * 4 + e] = mn[e];
                s_mmax[warp][lane * 4 + e] = mx[e];
            }
        }
        __syncthreads();
        if (tid < 32) {
            // lane = m: reduce over warps, then sum over m with a fixed tree
            float a = s_mmin[0][lane], c = s_mmax[0][lane];
            for (int w = 1; w < NW; ++w) { a = fminf(a, s_mmin[w][lane]); c = fmaxf(c, s_mmax[w][lane]); }
            float amax = fmaxf(fabsf(a), fabsf(c));
            float lo = a, hi = c;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                lo = __fadd_rn(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                hi = __fadd_rn(hi, __shfl_xor_sync(0xffffffffu, hi, o));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            }
            if (lane == 0) {
                const float span = __fsub_rn(hi, lo);
                const float pad = __fmul_rn(fmaxf(fabsf(lo), fabsf(hi)), 1e-5f);
                BinParams q_;
                q_.lo = __fsub_rn(lo, pad);
                const float h2 = __fadd_rn(hi, pad);
                q_.inv_w = (span > 0.f) ? __fdiv_rn((float)kNB, __fsub_rn(h2, q_.lo)) : 0.f;
                s_bp = q_;
                int sh = 0;
                if (amax > 0.f && isfinite(amax)) {
                    int e;
                    frexpf(amax, &e);
                    sh = max(-100, min(100, 25 - e));
                }
                s_shift = sh;
            }
        }
        for (int i = tid; i < kNB; i += kFThreads) s_hist[i] = 0u;
        __syncthreads();
        bp = s_bp;
        const float to_fx = ldexpf(1.f, s_shift);
        from_fx = ldexpf(1.f, -s_shift);
        int4* d4 = reinterpret_cast<int4*>(s_lut);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int f = tid + j * kFThreads;
            const int4 iv = make_int4(to_fixed(v[j].x, to_fx), to_fixed(v[j].y, to_fx), to_fixed(v[j].z, to_fx),
                                      to_fixed(v[j].w, to_fx));
            const int kk = f >> 3, m4 = f & 7;
            d4[kk * 16 + m4] = iv;
            d4[kk * 16 + 8 + m4] = iv;
        }
        __syncthreads();

        const uint32_t L = (uint32_t)lane >> 2;
        uint32_t off[4], sel[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint32_t bs = (uint32_t)(s + lane) & 3u;
            off[s] = 16u * L + 4u * bs;
            sel[s] = 0x5504u | (bs << 4);
        }
        float* gsc = p.sel_scores + (int64_t)u * p.sel_stride;
        __shared__ int s_abort;
        if (tid == 0) s_abort = 0;
        __syncthreads();
        LP_FTRACE(5);
        // scores stay in shared memory (the plan keeps every CTA's share
        // there); global memory gets them only on the exact slow path
        auto commit_score = [&](int lt, float sc) {
            if (keep_smem) s_scores[lt] = sc;
            else gsc[t_begin + lt] = sc;
            atomicAdd(&s_hist[score_bin(sc, bp.lo, bp.inv_w, kNB)], 1u);
        };
        // codes straight from global memory into registers: each thread's
        // token rows (two 16-byte loads each), the next step's rows loaded
        // before this step's lookups; a lane's 8 code words are rotated by L
        // in registers, so the table reads stay bank-conflict free
        const uint4* g4 = reinterpret_cast<const uint4*>(src) + (int64_t)t_begin * 2;
        const bool shared_codes = p.upk > 1;  // the G query-head units of a KV head read the same rows
        // 32-byte rows: one 256-bit load each when the rows are 32-byte
        // aligned (evict-first in L2 unless other units read them too)
        const bool v8ok = (reinterpret_cast<uintptr_t>(g4) & 31u) == 0;
        auto load_row = [&](int lt, uint32_t* c) {
#pragma unroll
            for (int j = 0; j < 8; ++j) c[j] = 0u;
            if (t_begin + lt < t_end) {
                const uint4* pp = g4 + (int64_t)lt * 2;
                if (v8ok && !shared_codes) {
                    asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]),
                                   "=r"(c[7])
                                 : "l"(pp));
                } else if (v8ok) {
                    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]),
                                   "=r"(c[7])
                                 : "l"(pp));
                } else {
                    const uint4 a = __ldg(pp), b2 = __ldg(pp + 1);
                    c[0] = a.x; c[1] = a.y; c[2] = a.z; c[3] = a.w;
                    c[4] = b2.x; c[5] = b2.y; c[6] = b2.z; c[7] = b2.w;
                }
            }
        };
        auto score_regs = [&](const uint32_t* c) {
            // r[w] = c[(w + L) & 7]: rotate by 1, 2, 4 as L's bits say
            uint32_t r1[8], r2[8], r[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) r1[w] = (L & 1u) ? c[(w + 1) & 7] : c[w];
#pragma unroll
            for (int w = 0; w < 8; ++w) r2[w] = (L & 2u) ? r1[(w + 2) & 7] : r1[w];
#pragma unroll
            for (int w = 0; w < 8; ++w) r[w] = (L & 4u) ? r2[(w + 4) & 7] : r2[w];
            int iacc = 0;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const uint32_t a = __byte_perm(r[w], off[s], sel[s]);
                    iacc += *reinterpret_cast<const int*>(s_lut + a + 16 * w);
                }
            }
            return __fmul_rn(__int2float_rn(iacc), from_fx);
        };
        uint32_t c0[8], c1[8];
        load_row(tid, c0);
        load_row(tid + kFThreads, c1);
        LP_FTRACE(6);
        for (int i = 0; i < ntiles; i += 2) {
            const int lt0 = i * kFThreads + tid, lt1 = lt0 + kFThreads;
            uint32_t n0[8], n1[8];
            load_row(lt0 + 2 * kFThreads, n0);
            load_row(lt1 + 2 * kFThreads, n1);
            const bool v0 = t_begin + lt0 < t_end, v1 = t_begin + lt1 < t_end;
            if (v1) {
                const float a0 = score_regs(c0);
                const float a1 = score_regs(c1);
                commit_score(lt0, a0);
                commit_score(lt1, a1);
            } else if (v0) {
                commit_score(lt0, score_regs(c0));
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c0[j] = n0[j];
                c1[j] = n1[j];
            }
        }
        if (__syncthreads_or(s_abort)) { drain(0); return; }
        LP_FTRACE(7);
        // the local histogram, for the exchange path (read after a unit barrier)
        for (int i = tid; i < kNB; i += kFThreads) p.chist[(int64_t)blockIdx.x * kNB + i] = s_hist[i];
        LP_FTRACE(19);
        // ---- publish the CTA's candidates for the unit's selection: every
        //      own token whose bin is at or above b_j, the CTA's threshold
        //      bin for pub_target tokens (all tokens if it has fewer), sorted
        //      by descending window bin w = min(bin - b_j, kPubWin - 1), plus
        //      the window counts (bins b_j .. b_j + kPubWin - 2 exactly, the
        //      last one cumulative).  A count above the slot capacity
        //      publishes nothing and b_j = kNB, which sends the unit to the
        //      exchange path. ----
        if (p.pub_cap > 0) {
            __shared__ int s_bj;
            // s_suf: [kNB + 1] suffix counts (the table is dead now).  The
            // scatter cursors s_cur stay in use until a thread's last slot
            // atomic, while threads that are done already copy the unit's
            // windows into the front of the table region in phase C (no
            // barrier in between): they sit in its last 512 bytes, which
            // phase C does not touch before its first barrier.
            uint32_t* s_suf = reinterpret_cast<uint32_t*>(s_lut);
            uint32_t* s_cur = reinterpret_cast<uint32_t*>(s_lut + FusedSmem::kLut - kPubWin * 4);
            static_assert((kNB + 1) * 4 <= FusedSmem::kLut - kPubWin * 4, "suffix counts end before the cursors");
            float2* s_own = reinterpret_cast<float2*>(s_ring + 64 * 1024);  // own published entries
            // suffix counts s_suf[b] = tokens in bins >= b: thread t owns bins
            // [kNB - 4(t+1), kNB - 4t), the top bins first
            {
                constexpr int PER = kNB / kFThreads;
                const int hi = kNB - PER * tid;
                uint32_t c[PER];
                int loc = 0;
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    c[j] = s_hist[hi - 1 - j];
                    loc += (int)c[j];
                }
                int before;
                Scan(scan_tmp).ExclusiveSum(loc, before);
                int run = before;
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    run += (int)c[j];
                    s_suf[hi - 1 - j] = (uint32_t)run;
                }
                if (tid == 0) {
                    s_suf[kNB] = 0u;
                    s_bj = 0;  // fewer tokens than pub_target: publish them all
                }
            }
            __syncthreads();
            LP_FTRACE(20);
            // b_j: the highest bin whose suffix reaches pub_target
            for (int bb = tid; bb < kNB; bb += kFThreads)
                if ((int)s_suf[bb] >= p.pub_target && (int)s_suf[bb + 1] < p.pub_target) s_bj = bb;
            __syncthreads();
            LP_FTRACE(21);
            const int bj = s_bj;
            const int npub = (int)s_suf[bj];
            const bool pub_ok = npub <= p.pub_cap;
            // window w counts bin bj + w (the last one: all bins >= bj + kPubWin - 1);
            // entries go in descending window order, so window w starts at
            // the count of bins >= bj + w + 1
            unsigned long long* pw = p.pwin + (int64_t)blockIdx.x * (kPubWin + 2);
            if (tid < kPubWin) {
                const int b0 = bj + tid;
                uint32_t cw = 0u, start = 0u;
                if (b0 < kNB) {
                    cw = tid < kPubWin - 1 ? s_hist[b0] : s_suf[b0];
                    start = tid < kPubWin - 1 ? s_suf[b0 + 1] : 0u;
                }
                s_cur[tid] = start;
                st_tag(pw + tid, pub_ok ? cw : 0u, s_epoch);
            }
            if (tid == 0) {
                st_tag(pw + kPubWin, pub_ok ? (uint32_t)npub : 0u, s_epoch);
                st_tag(pw + kPubWin + 1, pub_ok ? (uint32_t)bj : (uint32_t)kNB, s_epoch);
            }
            __syncthreads();
            LP_FTRACE(22);
            if (pub_ok) {
                unsigned long long* slot = p.pub + (int64_t)blockIdx.x * p.pub_cap * 2;
                // PU scores per thread per round, all loads issued before any
                // is used (spilled scores come from L2)
                constexpr int PU = 16;
                for (int base = 0; base < ntok; base += kFThreads * PU) {
                    float scv[PU];
#pragma unroll
                    for (int r = 0; r < PU; ++r) {
                        const int lt = base + r * kFThreads + tid;
                        scv[r] = lt < ntok ? (keep_smem ? s_scores[lt] : __ldcg(gsc + t_begin + lt)) : 0.f;
                    }
#pragma unroll
                    for (int r = 0; r < PU; ++r) {
                        const int lt = base + r * kFThreads + tid;
                        const int bin = score_bin(scv[r], bp.lo, bp.inv_w, kNB);
                        if (lt < ntok && bin >= bj) {
                            const int pos = (int)atomicAdd(&s_cur[min(bin - bj, kPubWin - 1)], 1u);
                            st_tag(slot + 2 * pos, __float_as_uint(scv[r]), s_epoch);
                            st_tag(slot + 2 * pos + 1, (uint32_t)(t_begin + lt), s_epoch);
                            s_own[pos] = make_float2(scv[r], __int_as_float(t_begin + lt));
                        }
                    }
                }
            }
        }
    }
    if (stamp) p.phase_ns[3] = global_ns();
    LP_FTRACE(8);
    if (tid == kFThreads - 32) {  // a lane off the select critical path
        prefetch_share(p.pf_ptr[0], p.pf_bytes[0], p.pf_count[0], p.pf_stride[0]);
        prefetch_share(p.pf_ptr[1], p.pf_bytes[1], p.pf_count[1], p.pf_stride[1]);
    }

    // ---- phase E staging and row order, shared with phase C's early gather:
    //      rows = [above-threshold tokens][sink share][local share][tie winners];
    //      s_list holds the above-threshold tokens followed by the tie winners ----
    constexpr int D = 128;
    constexpr int R = kFMaxRows;
    int* s_list = reinterpret_cast<int*>(s_scores);  // [<= kFScoreCap | kFSpillList] (scores consumed by then)
    KT* s_k = reinterpret_cast<KT*>(s_ring);         // [R][128] (the ring is free after phase B)
    KT* s_v = s_k + R * D;                           // [R][128]
    // phase E's chunks take RE rows: rows R.. sit in the table region, which
    // is free from the start of phase E until the warps' states are combined
    constexpr int RE = R + kFLutRows;
    static_assert(2 * kFLutRows * 128 * sizeof(KT) <= FusedSmem::kLut, "staging rows fit the table region");
    KT* s_k2 = reinterpret_cast<KT*>(s_lut);         // [kFLutRows][128]
    KT* s_v2 = s_k2 + kFLutRows * D;                 // [kFLutRows][128]
    auto stg_k = [&](int r) { return r < R ? s_k + r * D : s_k2 + (r - R) * D; };
    auto stg_v = [&](int r) { return r < R ? s_v + r * D : s_v2 + (r - R) * D; };
    const KT* kb = reinterpret_cast<const KT*>(p.keys) + (int64_t)b * p.k_stride_b + (int64_t)hkv * p.k_stride_h;
    const KT* vb = reinterpret_cast<const KT*>(p.vals) + (int64_t)b * p.v_stride_b + (int64_t)hkv * p.v_stride_h;
    constexpr int CH = D * (int)sizeof(KT) / 16;
    constexpr int EPC = 16 / (int)sizeof(KT);
    // the unit's sink and local-window rows are spread evenly over its CTAs
    const int sk0 = (int)((int64_t)p.n_sink * cj / cn), sk1 = (int)((int64_t)p.n_sink * (cj + 1) / cn);
    const int lc0 = (int)((int64_t)p.n_local * cj / cn), lc1 = (int)((int64_t)p.n_local * (cj + 1) / cn);
    const int n_sink_here = sk1 - sk0;
    const int n_loc_here = lc1 - lc0;
    auto row_token = [&](int rr, int nabove) -> int {
        if (rr < nabove) return s_list[rr];
        rr -= nabove;
        if (rr < n_sink_here) return sk0 + rr;
        rr -= n_sink_here;
        if (rr < n_loc_here) return p.local_start + lc0 + rr;
        return s_list[nabove + rr - n_loc_here];
    };
    // rows c0r + [r_lo, r_hi) of the row list -> staging rows [r_lo, r_hi)
    // (16-byte cp.async; every thread commits one group).  16-byte unit u of
    // staging row r sits at unit u ^ (r & 7), so that the 8 rows an
    // ldmatrix reads at one dim offset fall in 8 different bank groups.
    static_assert(CH == 16, "16 units of 16 bytes per staged row");
    auto issue_rows = [&](int c0r, int r_lo, int r_hi, int nabove) {
        for (int c = r_lo * CH + tid; c < r_hi * CH; c += kFThreads) {
            const int r = c / CH, part = c - r * CH;
            const int64_t t = min(max(row_token(c0r + r, nabove), 0), p.T_total - 1);
            const int sw = (part ^ (r & 7)) * EPC;
            cp_async16(stg_k(r) + sw, kb + t * p.k_stride_t + part * EPC);
            cp_async16(stg_v(r) + sw, vb + t * p.v_stride_t + part * EPC);
        }
        cp_async_commit();
    };
    __shared__ int s_nabove, s_nwin;
    using ListScan = cub::BlockScan<int, kFThreads>;
    // s_list[pos0 ..] = tok0 + 32*i + j for every set bit j of words[i],
    // i < nwords, in ascending order, 512 words per round; returns the count
    // (every thread).  Ends with a block barrier.
    auto list_bits = [&](const uint32_t* words, int nwords, int tok0, int pos0) -> int {
        int run = 0;
        for (int w0 = 0; w0 < nwords; w0 += kFThreads) {
            const int w = w0 + tid;
            const uint32_t bits = w < nwords ? words[w] : 0u;
            int pos, total;
            ListScan(scan_tmp).ExclusiveSum(__popc(bits), pos, total);
            pos += pos0 + run;
            for (uint32_t b2 = bits; b2; b2 &= b2 - 1) s_list[pos++] = tok0 + 32 * w + __ffs(b2) - 1;
            run += total;
            __syncthreads();  // scan_tmp is reused by the next round
        }
        return run;
    };

    // ================= phase C: select =================
    uint32_t* bm = p.bitmap + (int64_t)u * p.bm_stride;
    const float* gsc_c = p.sel_scores + (int64_t)u * p.sel_stride;
    __shared__ int s_cnt_above, s_win_before, s_topk_off, s_ntie_loc, s_ntie, s_fast;
    // own words: selected bits (exchange path: above-threshold bits), and the
    // tie winners of the own range (bit lt); spill mode keeps them after the
    // row list in the (unused) score region
    uint32_t* s_selw = keep_smem ? s_hist + 1024 : reinterpret_cast<uint32_t*>(s_scores) + kFSpillList;
    uint32_t* s_win = keep_smem ? s_hist + 1536 : s_selw + kFSpillWords;
    const int nw_own = w_end - w_begin;
    const int ubase = blockIdx.x - cj;  // first CTA of the unit
    // ---- fast path: the unit's threshold bin from the published windows,
    //      then only the published entries of that bin are exchanged ----
    {
        constexpr int PW = kPubWin + 2;                                      // window, count, b_j per CTA
        uint32_t* s_pw = reinterpret_cast<uint32_t*>(s_lut);                 // [cn][PW]
        int* s_tst = reinterpret_cast<int*>(s_lut + 33792);                  // [cn] entries above b* per slot
        int* s_tcn = s_tst + kPubMaxCtas;                                    // [cn] entries in bin b* per slot
        int* s_toff = s_tcn + kPubMaxCtas;                                   // [cn + 1] combined tie offsets
        float* s_tk = reinterpret_cast<float*>(s_lut + 35840);               // tie keys  [kFastTieCap]
        int* s_ti = reinterpret_cast<int*>(s_lut + 35840 + kFastTieCap * 4); // tie index [kFastTieCap]
        const float2* s_own = reinterpret_cast<const float2*>(s_ring + 64 * 1024);
        if (tid <= kPubWin) s_hist[tid] = 0u;  // the fast path's 128-bin histogram + "above"
        if (tid == 0) { s_fast = 0; s_bstar = -1; s_above = 0; s_ntie = 0; s_win_before = 0; s_topk_off = 0; }
        const bool pub = p.pub_cap > 0;
        if (pub) {
            // the unit's windows and headers, as their CTAs publish them
            const bool ok = poll_copy(s_pw, p.pwin + (int64_t)ubase * PW, cn * PW, s_epoch, p.err);
            if (__syncthreads_or(!ok)) return;
        } else {
            __syncthreads();
        }
        if (stamp) p.phase_ns[4] = global_ns();
        LP_FTRACE(9);
        for (int i = tid; i < nw_own; i += kFThreads) s_selw[i] = 0u;
        for (int i = tid; i < (ntok + 31) / 32; i += kFThreads) s_win[i] = 0u;
        if (pub) {
            // b* can only be usable in [bmax, bmin + kPubWin - 2]: every CTA's
            // window covers those bins exactly.  The unit histogram is built
            // on the 128 bins from bmax; anything above goes to one counter.
            __shared__ int s_bmax, s_bmin, s_nun;
            uint32_t* s_uh = s_hist;  // [kPubWin + 1]: bins bmax .. bmax + 127, then "above"
            if (warp == 0) {
                int n = 0, mx = 0, mn = kNB;
                for (int j = lane; j < cn; j += 32) {
                    n += (int)s_pw[j * PW + kPubWin];
                    mx = max(mx, (int)s_pw[j * PW + kPubWin + 1]);
                    mn = min(mn, (int)s_pw[j * PW + kPubWin + 1]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    n += __shfl_xor_sync(0xffffffffu, n, o);
                    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                }
                if (lane == 0) { s_nun = n; s_bmax = mx; s_bmin = mn; }
            }
            __syncthreads();
            const int bmax = s_bmax, bmin = s_bmin;
            // bin bmax + rb gathers window rb + bmax - b_j of every slot j
            // (4 threads per bin, no atomics); b_j <= bmax, so no window maps
            // above bin bmax + 127 and s_uh[kPubWin] stays 0
            {
                static_assert(kFThreads == 4 * kPubWin, "4 threads per bin");
                const int rb = tid >> 2;
                uint32_t c = 0u;
                for (int j = tid & 3; j < cn; j += 4) {
                    const int w = rb + bmax - (int)s_pw[j * PW + kPubWin + 1];
                    if (w < kPubWin) c += s_pw[j * PW + w];
                }
                c += __shfl_xor_sync(0xffffffffu, c, 1);
                c += __shfl_xor_sync(0xffffffffu, c, 2);
                if ((tid & 3) == 0) s_uh[rb] = c;
            }
            __syncthreads();
            if (warp == 0) {
                // suffix counts over the 128 bins (lane holds bins 4l .. 4l+3)
                uint32_t c[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) c[e] = s_uh[4 * lane + e];
                const uint32_t above_all = s_uh[kPubWin];
                uint32_t loc = c[0] + c[1] + c[2] + c[3];
                uint32_t suf = loc;  // inclusive suffix over lanes >= lane
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_down_sync(0xffffffffu, suf, o);
                    if (lane + o < 32) suf += y;
                }
                uint32_t run = suf - loc + above_all;  // tokens in bins above this lane's 4
                int bs = -1, above = 0;
#pragma unroll
                for (int e = 3; e >= 0; --e) {
                    if (bs < 0 && (int)(run + c[e]) >= p.k && (int)run < p.k) {
                        bs = bmax + 4 * lane + e;
                        above = (int)run;
                    }
                    run += c[e];
                }
                const unsigned found = __ballot_sync(0xffffffffu, bs >= 0);
                if (found) {
                    const int src = __ffs(found) - 1;
                    bs = __shfl_sync(0xffffffffu, bs, src);
                    above = __shfl_sync(0xffffffffu, above, src);
                }
                if (lane == 0) {
                    // exact when b* is at or above every CTA's publishing bin
                    // (each unpublished token then lies in a lower bin than the
                    // k-th published one, so it scores below it) and inside
                    // every window
                    const bool fast = found && p.k > 0 && s_nun >= p.k && bs < bmin + kPubWin - 1 &&
                                      (int)s_uh[bs - bmax] <= kFastTieCap;
                    s_fast = fast ? 1 : 0;
                    s_bstar = bs;
                    s_above = above;
                }
            }
        }
        __syncthreads();
        LP_FTRACE(10);
        if (s_fast) {
            const int bs = s_bstar;
            const int need = p.k - s_above;
            // per slot (16 threads each): entries above b* (they lead its
            // sorted list) and in b*; the own above-threshold tokens, by bin
            for (int j0 = 0; j0 < cn; j0 += kFThreads / 16) {
                const int j = j0 + tid / 16, q = tid & 15;
                uint32_t a = 0u;
                int wb = 0;
                if (j < cn) {
                    wb = bs - (int)s_pw[j * PW + kPubWin + 1];  // 0 <= wb < kPubWin - 1
                    for (int w = wb + 1 + q; w < kPubWin; w += 16) a += s_pw[j * PW + w];
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                if (q == 0 && j < cn) {
                    s_tst[j] = (int)a;
                    s_tcn[j] = (int)s_pw[j * PW + wb];
                }
            }
            const int nown = (int)s_pw[cj * PW + kPubWin];
            for (int i = tid; i < nown; i += kFThreads) {
                const float2 e = s_own[i];
                if (score_bin(e.x, bp.lo, bp.inv_w, kNB) > bs) {
                    const int t = __float_as_int(e.y);
                    atomicOr(&s_selw[(t >> 5) - w_begin], 1u << (t & 31));
                }
            }
            __syncthreads();
            LP_FTRACE(23);
            // offsets of the slots' tie entries (warp 0); the own
            // above-threshold tokens in ascending order -> s_list (all)
            if (warp == 0) {
                int carry = 0;
                for (int j0 = 0; j0 < cn; j0 += 32) {
                    const int j = j0 + lane;
                    const int c = j < cn ? s_tcn[j] : 0;
                    int x = c;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const int y = __shfl_up_sync(0xffffffffu, x, o);
                        if (lane >= o) x += y;
                    }
                    if (j < cn) s_toff[j] = carry + x - c;
                    carry += __shfl_sync(0xffffffffu, x, 31);
                }
                if (lane == 0) {
                    s_toff[cn] = carry;
                    s_ntie = carry;
                }
            }
            if (p.topk_out && tid == 32) {
                int c = 0;
                for (int j = 0; j < cj; ++j) c += s_tst[j];
                s_topk_off = c;
            }
            {
                const int na = list_bits(s_selw, nw_own, w_begin * 32, 0);
                if (tid == 0) s_nabove = na;
            }
            __syncthreads();
            LP_FTRACE(24);
            // the unit's tie-bin entries: loads issued first (up to 2 per
            // thread), then the K/V rows known now (own above-threshold
            // tokens, sink and local shares), while the tie bin is settled
            const int ntie = s_ntie;
            const unsigned long long* tsrc[2];
            unsigned long long tw[2][2];
            uint32_t tpend = 0u;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int i = tid + r * kFThreads;
                tsrc[r] = nullptr;
                if (i < ntie) {
                    int lo = 0, hi = cn - 1;  // slot of combined entry i: the last j with s_toff[j] <= i
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (s_toff[mid] <= i) lo = mid;
                        else hi = mid - 1;
                    }
                    tsrc[r] = p.pub + ((int64_t)(ubase + lo) * p.pub_cap + s_tst[lo] + (i - s_toff[lo])) * 2;
                    tw[r][0] = ld_tag(tsrc[r]);
                    tw[r][1] = ld_tag(tsrc[r] + 1);
                    tpend |= 1u << r;
                }
            }
            issue_rows(0, 0, min(s_nabove + n_sink_here + n_loc_here, R), s_nabove);
            LP_FTRACE(25);
            {
                bool ok = true;
                const long long t0 = clock64();
                while (tpend) {
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        if ((tpend >> r & 1u) && tag_ok(tw[r][0], s_epoch) && tag_ok(tw[r][1], s_epoch)) {
                            const int i = tid + r * kFThreads;
                            s_tk[i] = __uint_as_float((uint32_t)tw[r][0]);
                            s_ti[i] = (int)(uint32_t)tw[r][1];
                            tpend &= ~(1u << r);
                        }
                    }
                    if (!tpend) break;
                    if (clock64() - t0 > kWaitCycles) {
                        atomicOr(p.err, LP_DEVERR_WAIT_TIMEOUT);
                        ok = false;
                        break;
                    }
#pragma unroll
                    for (int r = 0; r < 2; ++r)
                        if (tpend >> r & 1u) {
                            tw[r][0] = ld_tag(tsrc[r]);
                            tw[r][1] = ld_tag(tsrc[r] + 1);
                        }
                }
                if (__syncthreads_or(!ok)) {
                    cp_async_wait<0>();
                    return;
                }
            }
            LP_FTRACE(11);
            // rank (score desc, index asc) of the own tie entries (all of them
            // when the top-k indices are requested): the first `need` win
            const int i0 = p.topk_out ? 0 : s_toff[cj];
            const int i1 = p.topk_out ? ntie : s_toff[cj + 1];
            // one warp per entry, its lanes over the unit's entries (the
            // loop is warp-uniform: every lane takes part in the reduction)
            for (int i = i0 + warp; i < i1; i += NW) {
                const float ki = s_tk[i];
                const int ii = s_ti[i];
                int rank = 0;
                for (int j = lane; j < ntie; j += 32) rank += sel_before(s_tk[j], s_ti[j], ki, ii);
                rank = __reduce_add_sync(0xffffffffu, rank);
                if (lane == 0 && rank < need) {
                    if (ii >= t_begin && ii < t_end) atomicOr(&s_win[(ii - t_begin) >> 5], 1u << ((ii - t_begin) & 31));
                    else if (ii < t_begin) atomicAdd(&s_topk_off, 1);
                }
            }
            __syncthreads();
        }
    }
    if (stamp) p.phase_ns[5] = global_ns();
    LP_FTRACE(12);
    if (!s_fast) {
        // ---- exchange path: threshold bin of the unit histogram, ballots,
        //      tie-bin tokens through the tie slots, one more barrier ----
        float2* s_tloc = reinterpret_cast<float2*>(s_lut);  // this CTA's tie-bin tokens (<= kTieCap)
        // the unit histogram: sum of its CTAs' local histograms (published
        // with plain stores in phase B, visible after this barrier)
        if (!unit_barrier(ubar, cn, nbar, s_epoch, p.err)) return;
        for (int i = tid; i < kNB; i += kFThreads) {
            uint32_t c = 0u;
            for (int j = 0; j < cn; ++j) c += __ldcg(p.chist + (int64_t)(ubase + j) * kNB + i);
            s_hist[i] = c;
        }
        if (tid == 0) { s_bstar = kNB; s_above = 0; s_cnt_above = 0; s_ntie_loc = 0; }
        __syncthreads();
        if (p.k > 0) find_threshold_bin<kFThreads>(s_hist, p.k, &s_bstar, &s_above);
        __syncthreads();
        const int bstar = s_bstar;
        int my_above = 0;
        // 4 words per warp and round, their score loads issued first
        // (spilled scores come from L2)
        for (int w4 = w_begin + warp; w4 < w_end; w4 += 4 * NW) {
            float sv4[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int t = (w4 + r * NW) * 32 + lane;
                const bool valid = w4 + r * NW < w_end && t >= p.c0 && t < p.c1;
                sv4[r] = valid ? (keep_smem ? s_scores[t - t_begin] : __ldcg(gsc_c + t)) : 0.f;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int w = w4 + r * NW;
                if (w >= w_end) break;  // warp-uniform
                const int t = w * 32 + lane;
                const bool valid = t >= p.c0 && t < p.c1;
                const float s = sv4[r];
                const int bin = score_bin(s, bp.lo, bp.inv_w, kNB);
                const bool tie = valid && bin == bstar;
                const uint32_t abv = __ballot_sync(0xffffffffu, valid && bin > bstar);
                my_above += __popc(abv);
                if (lane == 0) {
                    bm[w] = 0u;  // cleared for the exact slow path
                    s_selw[w - w_begin] = abv;
                }
                const uint32_t tmask = __ballot_sync(0xffffffffu, tie);
                if (tmask) {
                    int base = 0;
                    if (lane == 0) base = atomicAdd(&s_ntie_loc, __popc(tmask));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (tie) {
                        const int pos = base + __popc(tmask & ((1u << lane) - 1u));
                        if (pos < kTieCap) s_tloc[pos] = make_float2(s, __int_as_float(t));
                    }
                }
            }
        }
        if (lane == 0 && my_above) atomicAdd(&s_cnt_above, my_above);
        __syncthreads();
        // tie-bin tokens -> this CTA's own slot of the tie buffer (no
        // reservation round trip); a count above kTieCap makes the unit
        // overflow, only the copy is capped
        if (tid == 0) {
            p.cta_count[blockIdx.x] = (uint32_t)s_cnt_above;
            p.cta_ties[blockIdx.x] = (uint32_t)s_ntie_loc;
        }
        const int nloc = min(s_ntie_loc, kTieCap);
        for (int i = tid; i < nloc; i += kFThreads) p.tie_buf[(int64_t)blockIdx.x * kTieCap + i] = s_tloc[i];
        if (!unit_barrier(ubar, cn, nbar, s_epoch, p.err)) return;

        // ---- ties (redundant per CTA, no barrier) ----
        float* s_tk = reinterpret_cast<float*>(s_lut);                      // tie keys  [kTieCap]
        int* s_ti = reinterpret_cast<int*>(s_lut + kTieCap * 4);            // tie index [kTieCap]
        int* s_toff = reinterpret_cast<int*>(s_lut + 2 * kTieCap * 4);      // [cn + 1] tie offsets of the unit's CTAs
        const int need = p.k - s_above;
        for (int i = tid; i < (ntok + 31) / 32; i += kFThreads) s_win[i] = 0u;
        if (warp == 0) {
            int carry = 0;
            for (int j0 = 0; j0 < cn; j0 += 32) {
                const int j = j0 + lane;
                const int c = j < cn ? (int)__ldcg(p.cta_ties + ubase + j) : 0;
                int x = c;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x += y;
                }
                if (j < cn) s_toff[j] = carry + x - c;
                carry += __shfl_sync(0xffffffffu, x, 31);
            }
            if (lane == 0) {
                s_toff[cn] = carry;
                s_ntie = carry;
                s_win_before = 0;
            }
        }
        __syncthreads();
        const int ntie = s_ntie;
        const bool overflow = ntie > kTieCap;  // identical in every CTA of the unit
        if (!overflow && need > 0) {
            for (int i = tid; i < ntie; i += kFThreads) {
                // source CTA of combined entry i: the last j with s_toff[j] <= i
                int lo = 0, hi = cn - 1;
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (s_toff[mid] <= i) lo = mid;
                    else hi = mid - 1;
                }
                const float2 e = __ldcg(p.tie_buf + (int64_t)(ubase + lo) * kTieCap + (i - s_toff[lo]));
                s_tk[i] = e.x;
                s_ti[i] = __float_as_int(e.y);
            }
            __syncthreads();
            // rank of a tie entry in selection order (score desc, index asc):
            // the first `need` ranks win.  Only the CTA's own entries are
            // ranked unless the top-k indices are requested.
            const int i0 = p.topk_out ? 0 : s_toff[cj];
            const int i1 = p.topk_out ? ntie : s_toff[cj + 1];
            for (int i = i0 + warp; i < i1; i += NW) {  // one warp per entry (warp-uniform)
                const float ki = s_tk[i];
                const int ii = s_ti[i];
                int rank = 0;
                for (int j = lane; j < ntie; j += 32) rank += sel_before(s_tk[j], s_ti[j], ki, ii);
                rank = __reduce_add_sync(0xffffffffu, rank);
                if (lane == 0 && rank < need) {
                    const int lt = ii - t_begin;
                    if (ii >= t_begin && ii < t_end) atomicOr(&s_win[lt >> 5], 1u << (lt & 31));
                    if (p.topk_out && ii >= p.c0 && ii < p.c1) {
                        // owner CTA (within the unit) of token ii
                        const int x = (ii >> 5) - wlo;
                        const int owner = (int)(((int64_t)(x + 1) * cn - 1) / nwu);
                        if (owner < cj) atomicAdd(&s_win_before, 1);
                    }
                }
            }
        }
        if (overflow) {
            // exact slow path by the unit leader on the global scores, then
            // one more unit barrier (every CTA of the unit saw the same
            // count).  First every CTA stores its scores, one barrier.
            if (keep_smem) {
                float* gsc_w = p.sel_scores + (int64_t)u * p.sel_stride;
                for (int lt = tid; lt < ntok; lt += kFThreads) gsc_w[t_begin + lt] = s_scores[lt];
            }
            if (!unit_barrier(ubar, cn, nbar, s_epoch, p.err)) return;
            if (cj == 0 && need > 0) {
                if (tid == 0) atomicOr(p.err, LP_DEVERR_TIE_OVERFLOW);
                uint32_t* h256 = reinterpret_cast<uint32_t*>(s_lut);
                __shared__ uint32_t s_prefix, s_mask;
                __shared__ int s_remaining;
                if (tid == 0) { s_prefix = 0; s_mask = 0; s_remaining = need; }
                for (int shift = 24; shift >= 0; shift -= 8) {
                    for (int i = tid; i < 256; i += kFThreads) h256[i] = 0;
                    __syncthreads();
                    const uint32_t prefix = s_prefix, mask = s_mask;
                    for (int t = p.c0 + tid; t < p.c1; t += kFThreads) {
                        const float sv = __ldcg(gsc_c + t);
                        if (score_bin(sv, bp.lo, bp.inv_w, kNB) != s_bstar) continue;
                        const uint32_t key = ordered_key(sv);
                        if ((key & mask) != prefix) continue;
                        atomicAdd(&h256[(key >> shift) & 255u], 1u);
                    }
                    __syncthreads();
                    if (tid == 0) {
                        const int rem = s_remaining;
                        int acc = 0;
                        for (int d = 255; d >= 0; --d) {
                            const int c = (int)h256[d];
                            if (acc + c >= rem) {
                                s_prefix = prefix | ((uint32_t)d << shift);
                                s_mask = mask | (255u << shift);
                                s_remaining = rem - acc;
                                break;
                            }
                            acc += c;
                        }
                    }
                    __syncthreads();
                }
                const uint32_t kstar = s_prefix;
                const int take_eq = s_remaining;
                using Scan = cub::BlockScan<int, kFThreads>;
                __shared__ typename Scan::TempStorage tmp;
                __shared__ int s_eq_base;
                if (tid == 0) s_eq_base = 0;
                __syncthreads();
                for (int base = p.c0; base < p.c1; base += kFThreads) {
                    const int t = base + tid;
                    int gt = 0, eq = 0;
                    if (t < p.c1) {
                        const float sv = __ldcg(gsc_c + t);
                        if (score_bin(sv, bp.lo, bp.inv_w, kNB) == s_bstar) {
                            const uint32_t key = ordered_key(sv);
                            gt = key > kstar;
                            eq = key == kstar;
                        }
                    }
                    int rank, total;
                    Scan(tmp).ExclusiveSum(eq, rank, total);
                    if (gt || (eq && s_eq_base + rank < take_eq)) atomicOr(&bm[t >> 5], 1u << (t & 31));
                    __syncthreads();
                    if (tid == 0) s_eq_base += total;
                    __syncthreads();
                }
            }
            if (!unit_barrier(ubar, cn, nbar, s_epoch, p.err)) return;
            if (ntie > kTieCap && need > 0) {
                // winners of this unit are the bits the leader set
                for (int w = w_begin + tid; w < w_end; w += kFThreads) {
                    const uint32_t bits = __ldcg(bm + w);
                    for (uint32_t b2 = bits; b2; b2 &= b2 - 1) {
                        const int lt = w * 32 + __ffs(b2) - 1 - t_begin;
                        if (lt >= 0 && lt < ntok) atomicOr(&s_win[lt >> 5], 1u << (lt & 31));
                    }
                }
                if (p.topk_out) {
                    int c = 0;
                    for (int w = wlo + tid; w < w_begin; w += kFThreads) c += __popc(__ldcg(bm + w));
                    if (c) atomicAdd(&s_win_before, c);
                }
            }
        }
        __syncthreads();
    }




    // ================= phase E: attention over the CTA's own kept rows =================
    {
        const float* s_q = s_qu;  // [G][128] fp32 query rows
        // ---- row list: above-threshold tokens (built in phase C on the fast
        //      path), then the tie winners (bit lt of s_win = token t_begin + lt),
        //      each in ascending token order ----
        if (!s_fast) {
            const int na = list_bits(s_selw, nw_own, w_begin * 32, 0);
            if (tid == 0) s_nabove = na;
            __syncthreads();
        }
        {
            const int nwin = list_bits(s_win, (ntok + 31) / 32, t_begin, s_nabove);
            if (tid == 0) s_nwin = nwin;
        }
        if (!s_fast && p.topk_out && tid == 0) s_topk_off = s_win_before;
        __syncthreads();
        if (p.topk_out) {
            // the CTA's selected tokens (above-threshold | tie winners) in
            // ascending order, at its rank offset within the unit
            if (!s_fast) {
                int c = 0;
                for (int j = tid; j < cj; j += kFThreads) c += (int)__ldcg(p.cta_count + ubase + j);
                if (c) atomicAdd(&s_topk_off, c);
            }
            const int shift0 = t_begin - w_begin * 32;  // 0 except for the first CTA (c0 % 32)
            __syncthreads();  // s_topk_off complete; scan_tmp free
            const int off = s_topk_off;
            int run = 0;
            for (int w0 = 0; w0 < nw_own; w0 += kFThreads) {  // 512 own words per round
                uint32_t wordsel = 0u;
                const int w = w0 + tid;
                if (w < nw_own) {
                    // winners of tokens 32*(w_begin+w) + i  <->  bit lt = 32*w + i - shift0
                    const int lt0 = 32 * w - shift0;
                    uint32_t r = 0u;
                    if (ntok > 0) {
                        const int wl = lt0 >> 5, sh = lt0 & 31;  // lt0 may be negative for w = 0
                        if (lt0 >= 0) {
                            r = s_win[wl] >> sh;
                            if (sh && wl + 1 < (ntok + 31) / 32) r |= s_win[wl + 1] << (32 - sh);
                        } else {
                            r = s_win[0] << (-lt0);
                        }
                    }
                    wordsel = s_selw[w] | r;
                    const int tb = (w_begin + w) * 32;
                    if (tb < p.c0) wordsel &= ~0u << (p.c0 - tb);
                    if (tb + 32 > p.c1) wordsel &= (p.c1 - tb) >= 32 ? ~0u : ((1u << (p.c1 - tb)) - 1u);
                }
                int pos, total;
                Scan(scan_tmp).ExclusiveSum(__popc(wordsel), pos, total);
                pos += run;
                for (uint32_t b2 = wordsel; b2; b2 &= b2 - 1) {
                    if (off + pos < p.k) p.topk_out[(int64_t)ul * p.k + off + pos] = (w_begin + w) * 32 + __ffs(b2) - 1;
                    ++pos;
                }
                run += total;
                __syncthreads();  // scan_tmp is reused by the next round
            }
        }
        LP_FTRACE(13);
        const int nabove = s_nabove;
        const int n_early = nabove + n_sink_here + n_loc_here;
        const int nrows = n_early + s_nwin;
        const int n_issued = s_fast ? min(n_early, R) : 0;  // rows already loading since phase C

        // ---- per-warp flash-decode on the tensor cores (mma.sync m16n8k16):
        //      warp w takes the 16-row tiles w, w + NW, ... of every chunk.
        //      Per tile: S^T[16 rows x 8 heads] = K_tile . Q^T (8 steps over
        //      the 128 dims), online softmax per head, then
        //      O^T[128 dims x 8 heads] += V_tile^T . P^T (8 blocks of 16 dims).
        //      Lane (gq = lane / 4, tq = lane % 4) keeps heads 2tq, 2tq + 1:
        //      their running max / sum and O^T rows 16mb + gq (+8).  Heads at
        //      or above G have a zero query (finite, never written out). ----
        const int gq = lane >> 2, tq = lane & 3;
        float wm[2] = {-INFINITY, -INFINITY}, wl[2] = {0.f, 0.f};
        float oacc[8][4];
#pragma unroll
        for (int mb = 0; mb < 8; ++mb)
#pragma unroll
            for (int e = 0; e < 4; ++e) oacc[mb][e] = 0.f;
        // Q^T (B operand): b0b1 = Q[head gq][16ks + 2tq, +1], b2b3 = dims +8
        uint32_t qb[8][2];
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            if (gq < p.G) {
                const float* qr = s_q + gq * D + 16 * ks + 2 * tq;
                qb[ks][0] = pack2<KT>(qr[0], qr[1]);
                qb[ks][1] = pack2<KT>(qr[8], qr[9]);
            } else {
                qb[ks][0] = 0u;
                qb[ks][1] = 0u;
            }
        }
        const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: this lane addresses row rr of matrix mi
        auto attend = [&](int r_lo, int r_hi) {
            // warp-uniform loop: every lane takes part in the mma and shuffles
            for (int r0 = r_lo + warp * 16; r0 < r_hi; r0 += NW * 16) {
                // rows past r_hi read row r_lo instead (finite data, masked below)
                int krow = r0 + (mi & 1) * 8 + rr;
                if (krow >= r_hi) krow = r_lo;
                const uint32_t kbase = smem_u32(stg_k(krow));
                float sv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    uint32_t af[4];
                    ldsm_x4(af, kbase + (uint32_t)((((2 * ks + (mi >> 1)) ^ (krow & 7)) * 16)));
                    mma16816<KT>(sv, af, qb[ks]);
                }
                // sv: S[row r0+gq][head 2tq + e] (e = 0, 1), rows +8 in sv[2 + e]
                const bool v0 = r0 + gq < r_hi, v1 = r0 + gq + 8 < r_hi;
                float pv[4];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float s0 = v0 ? sv[e] * p.scale_log2 : -INFINITY;
                    const float s1 = v1 ? sv[2 + e] * p.scale_log2 : -INFINITY;
                    float mx = fmaxf(s0, s1);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float mn = fmaxf(wm[e], mx);  // finite: row r0 is valid
                    const float sc = exp2f(wm[e] - mn);
                    pv[e] = exp2f(s0 - mn);
                    pv[2 + e] = exp2f(s1 - mn);
                    float sm = pv[e] + pv[2 + e];
                    sm += __shfl_xor_sync(0xffffffffu, sm, 4);
                    sm += __shfl_xor_sync(0xffffffffu, sm, 8);
                    sm += __shfl_xor_sync(0xffffffffu, sm, 16);
                    wl[e] = fmaf(wl[e], sc, sm);
                    wm[e] = mn;
#pragma unroll
                    for (int mb = 0; mb < 8; ++mb) {
                        oacc[mb][e] *= sc;
                        oacc[mb][2 + e] *= sc;
                    }
                }
                // P^T (B operand): b0b1 = P[rows 2tq, 2tq+1][head gq], b2b3 =
                // rows +8; P[row r][head h] sits in lane 4 (r % 8) + h / 2,
                // half h % 2 of its (row < 8 ? pv01 : pv23) pair
                const uint32_t m01 = pack2<KT>(pv[0], pv[1]), m23 = pack2<KT>(pv[2], pv[3]);
                const int srcA = 8 * tq + (gq >> 1), srcB = srcA + 4;
                const uint32_t xa01 = __shfl_sync(0xffffffffu, m01, srcA), xb01 = __shfl_sync(0xffffffffu, m01, srcB);
                const uint32_t xa23 = __shfl_sync(0xffffffffu, m23, srcA), xb23 = __shfl_sync(0xffffffffu, m23, srcB);
                const uint32_t selp = (gq & 1) ? 0x7632u : 0x5410u;
                uint32_t pb[2];
                pb[0] = __byte_perm(xa01, xb01, selp);
                pb[1] = __byte_perm(xa23, xb23, selp);
                int vrow = r0 + (mi >> 1) * 8 + rr;
                if (vrow >= r_hi) vrow = r_lo;
                const uint32_t vbase = smem_u32(stg_v(vrow));
#pragma unroll
                for (int mb = 0; mb < 8; ++mb) {
                    uint32_t af[4];
                    ldsm_x4_trans(af, vbase + (uint32_t)((((2 * mb + (mi & 1)) ^ (vrow & 7)) * 16)));
                    mma16816<KT>(oacc[mb], af, pb);
                }
            }
        };
        for (int c0r = 0; c0r < nrows; c0r += RE) {
            const int nr = min(RE, nrows - c0r);
            int r_ready = 0;
            if (c0r == 0 && n_issued > 0) {
                // the chunk's first n_issued rows were issued in phase C; the
                // rest (tie winners) loads while those are attended
                issue_rows(0, n_issued, nr, nabove);
                cp_async_wait<1>();
                __syncthreads();
                attend(0, n_issued);
                r_ready = n_issued;
                LP_FTRACE(14);
            } else {
                issue_rows(c0r, 0, nr, nabove);
            }
            cp_async_wait<0>();
            __syncthreads();
            attend(r_ready, nr);
            __syncthreads();  // staging rows consumed before the next chunk lands
        }
        LP_FTRACE(15);
        // ---- combine the warps' states into the CTA's slice state ----
        {
            float* s_wacc = reinterpret_cast<float*>(s_lut);  // [NW][G][128]
            float* s_wm = reinterpret_cast<float*>(s_hist);   // [NW][8] (the histogram is consumed)
            float* s_wl = s_wm + NW * 8;                       // [NW][8]
            float* s_wf = s_wl + NW * 8;                       // [NW][8] rescale of each warp's state
            float* s_cm = s_wf + NW * 8;                       // [8] slice max
            float* s_cl = s_cm + 8;                            // [8] slice sum
            // warps past nwu never had a tile (16 rows per tile, at most
            // min(nrows, RE) rows per chunk): they hold no state
            const int nwu = min(NW, (min(nrows, RE) + 15) / 16);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int h = 2 * tq + e;
                if (h < p.G && warp < nwu) {
                    float* dst = s_wacc + (warp * p.G + h) * D + gq;
#pragma unroll
                    for (int mb = 0; mb < 8; ++mb) {
                        dst[16 * mb] = oacc[mb][e];
                        dst[16 * mb + 8] = oacc[mb][2 + e];
                    }
                    if (gq == 0) {
                        s_wm[warp * 8 + h] = wm[e];
                        s_wl[warp * 8 + h] = wl[e];
                    }
                }
            }
            __syncthreads();
            // 16 lanes per head (one per warp): max, rescale factors, sum.
            // Whole warps take part in the shuffles (lanes of heads >= G
            // carry neutral values and write nothing).
            if (tid < ((NW * p.G + 31) & ~31)) {
                const int g = tid / NW, w = tid - g * NW;
                const bool live = g < p.G && w < nwu;
                const float m = live ? s_wm[w * 8 + g] : -INFINITY;
                float mx = m;
#pragma unroll
                for (int o = 1; o < NW; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                const float f = m == -INFINITY ? 0.f : exp2f(m - mx);
                float l = live ? s_wl[w * 8 + g] * f : 0.f;
#pragma unroll
                for (int o = 1; o < NW; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
                if (live) s_wf[w * 8 + g] = f;
                if (g < p.G && w == 0) {
                    s_cm[g] = mx;
                    s_cl[g] = l;
                }
            }
            __syncthreads();
            unsigned long long* part = p.part + ((int64_t)u * p.max_split + cj) * p.G * (2 + D);
            for (int o = tid; o < p.G * D; o += kFThreads) {
                const int g = o / D, d = o - g * D;
                float a = 0.f;
                for (int w = 0; w < nwu; ++w) a = fmaf(s_wacc[(w * p.G + g) * D + d], s_wf[w * 8 + g], a);
                st_tag(part + g * (2 + D) + 2 + d, __float_as_uint(a), s_epoch);
                if (d == 0) {
                    st_tag(part + g * (2 + D), __float_as_uint(s_cm[g]), s_epoch);
                    st_tag(part + g * (2 + D) + 1, __float_as_uint(s_cl[g]), s_epoch);
                }
            }
        }
    }
    LP_FTRACE(16);

    // ================= merge: each CTA of the unit finalises a slice of its G*128 outputs =================
    {
        constexpr int D = 128;
        const int nout = p.G * D;
        const int per = (nout + cn - 1) / cn;
        const int o0 = min(nout, cj * per), o1 = min(nout, o0 + per);
        const int npair = (o1 - o0) * cn;  // (output, slice) pairs, <= nout + cn <= 4096
        const unsigned long long* pu = p.part + (int64_t)u * p.max_split * p.G * (2 + D);
        const int64_t sstride = (int64_t)p.G * (2 + D);
        float* s_mm = reinterpret_cast<float*>(s_ring);  // [npair] slice max
        float* s_ll = s_mm + 4096;                       // [npair] slice sum
        float* s_aa = s_ll + 4096;                       // [npair] slice P.V
        // the slice states of the unit's CTAs, polled until this call's
        // epoch shows (no barrier: each word carries its own tag)
        bool ok = true;
        const long long t0 = clock64();
        for (int i = tid; i < npair && ok; i += kFThreads) {
            const int ol = i / cn, sl = i - ol * cn;
            const int o = o0 + ol, g = o / D, d = o - g * D;
            const unsigned long long* ps = pu + sl * sstride + g * (2 + D);
            unsigned long long a = ld_tag(ps), l = ld_tag(ps + 1), x = ld_tag(ps + 2 + d);
            while (!(tag_ok(a, s_epoch) && tag_ok(l, s_epoch) && tag_ok(x, s_epoch))) {
                if (clock64() - t0 > kWaitCycles) {
                    atomicOr(p.err, LP_DEVERR_WAIT_TIMEOUT);
                    ok = false;
                    break;
                }
                a = ld_tag(ps);
                l = ld_tag(ps + 1);
                x = ld_tag(ps + 2 + d);
            }
            s_mm[i] = __uint_as_float((uint32_t)a);
            s_ll[i] = __uint_as_float((uint32_t)l);
            s_aa[i] = __uint_as_float((uint32_t)x);
        }
        if (__syncthreads_or(!ok)) return;
        if (stamp) p.phase_ns[6] = global_ns();
        LP_FTRACE(17);
        OT* ob = reinterpret_cast<OT*>(p.out) + (int64_t)b * p.out_stride_b;
        for (int ol = tid; ol < o1 - o0; ol += kFThreads) {
            const float* mm = s_mm + ol * cn;
            const float* ll = s_ll + ol * cn;
            const float* aa = s_aa + ol * cn;
            float M = -INFINITY;
            for (int sl = 0; sl < cn; ++sl) M = fmaxf(M, mm[sl]);
            float L = 0.f, A = 0.f;
            for (int sl = 0; sl < cn; ++sl) {
                const float f = exp2f(mm[sl] - M);  // 0 for a slice without rows
                L = fmaf(ll[sl], f, L);
                A = fmaf(aa[sl], f, A);
            }
            const int o = o0 + ol, g = o / D, d = o - g * D;
            ob[(int64_t)(hu * p.G + g) * p.out_stride_h + d] = from_f32<OT>(A / L);
        }
        if (p.phase_ns && tid == 0) atomicMax(&p.phase_ns[7], global_ns());
        LP_FTRACE(18);
    }
}

}  // namespace lp
