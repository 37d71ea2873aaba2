// pipeline.cu -- C-ABI entry points of the fused sparse-decode hot path.
#include <algorithm>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "compat.cuh"
#include "encode.cuh"
#include "icm.cuh"
#include "rope_append.cuh"
#include "fused_step.cuh"
#include "lut_build.cuh"
#include "score.cuh"
#include "select.cuh"

namespace lp {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(LP_ERR_CUDA, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
    return LP_OK;
}

int sm_count(int device) {
    static int cache[64] = {0};
    if (device < 0 || device >= 64) return 148;
    if (!cache[device]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
        cache[device] = n;
    }
    return cache[device];
}

// Opt-in to > 48 KB dynamic shared memory, once per (kernel, device).
template <typename F>
static int smem_opt_in(F* kernel, int bytes, int device, bool* done_flags) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64) device = 0;
    if (!done_flags[device]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess)
            return fail(LP_ERR_CUDA, std::string("cudaFuncSetAttribute(max dynamic smem): ") + cudaGetErrorString(e));
        done_flags[device] = true;
    }
    return LP_OK;
}

// ----------------------------------------------------------------------------
// geometry / workspace plan
// ----------------------------------------------------------------------------
struct Plan {
    int U, Usel, Uatt, HG;
    bool heads;      // per-head tables (query-head selection or head scores requested)
    bool per_head;   // selection per query head
    int c0, c1, ncand;
    int n_sink, local_start, n_local, n_rows;
    int score_ctas;
    int sel_ctas_per_unit, sel_words_per_cta;
    int rows_per, nsplit;
    int64_t bm_words;
    bool fused;       // single cooperative kernel path
    int fused_ctas, fused_max_split;
    int fused_units;  // its units: (sequence, KV head), or (sequence, query head) for query-head selection
    bool fused_spill; // its CTAs' shares exceed the shared-memory score buffer
    // workspace regions
    uint32_t* err;
    float* lut;
    float* bounds;
    float* sel_scores;
    uint32_t* bitmap;
    int nchunk;        // multi-kernel path: 256-word chunks of the candidate window
    int* chunk_cnt;    // [Usel][nchunk] selected tokens per chunk
    int32_t* toplist;  // [Usel][k] selected tokens, ascending
    bool compact;      // the multi-kernel path compacts the selection (top-k output, per-head attention)
    float2* tie_buf;
    int4* info;
    float* part;
    uint32_t* zero;  // hist | tie_count | done_sel | done_att
    int64_t zero_words;
    uint32_t* hist;
    uint32_t* tie_count;
    uint32_t* done_sel;
    uint32_t* done_att;
    uint32_t* bar;
    unsigned long long* ubar;
    uint32_t* cta_count;
    uint32_t* cta_ties;
    unsigned long long* fpub;   // fused path: tagged candidates [ctas][pub_cap][2]
    unsigned long long* fwin;   // fused path: tagged windows + headers [ctas][kPubWin + 2]
    float* flut;                // fused path: LUT [U][256][32] (plain, behind per-CTA flags)
    unsigned long long* flutflag;  // fused path: tagged per-CTA "LUT share written" flags
    unsigned long long* fpart;  // fused path: tagged split-K states [U][max_split][G][130]
    uint32_t* chist;            // fused path: local histograms [ctas][kNB]
    int pub_target, pub_cap;
    size_t bytes;
};

static constexpr int kScoreThreads = 512;
static constexpr int kUnitBarWords = 192;     // one 64-bit barrier word per unit of the fused path
static constexpr size_t kPersistBytes = 2048; // error word, grid barrier, unit barriers
static constexpr int kGroupStages = 8;
static constexpr int kHeadsStages = 4;
static constexpr int kFusedMaxG = 8;  // query heads per KV head on the fused path

static int make_plan(const lp_sparse_decode_args* a, void* ws, Plan* P, int device) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->B > 0 && a->Hkv > 0 && a->G > 0, "B, Hkv and G must be positive");
    LP_CHECK(a->M == 32 && a->K == 256, "the fused scorer supports M=32 codebooks of K=256 entries");
    LP_CHECK(a->D > 0 && a->D % 4 == 0 && a->D <= 512, "D must be a positive multiple of 4 (<= 512)");
    LP_CHECK(a->T_codes >= 0 && a->T_total > 0 && a->T_codes <= a->T_total,
             "need 0 <= T_codes <= T_total and T_total > 0");
    LP_CHECK(a->sink >= 0 && a->local >= 0, "sink and local must be non-negative");
    LP_CHECK(a->select_mode == LP_SELECT_KV_GROUP || a->select_mode == LP_SELECT_QUERY_HEAD,
             "select_mode must be LP_SELECT_KV_GROUP or LP_SELECT_QUERY_HEAD");
    Plan& p = *P;
    p.per_head = a->select_mode == LP_SELECT_QUERY_HEAD;
    p.heads = p.per_head || a->head_scores != nullptr;
    LP_CHECK(!p.heads || a->G <= 4, "per-query-head scoring supports G <= 4 query heads per KV head");
    p.U = a->B * a->Hkv;
    p.Usel = p.per_head ? p.U * a->G : p.U;
    p.HG = p.per_head ? 1 : a->G;
    p.Uatt = p.Usel;
    LP_CHECK(p.HG <= 8, "at most 8 query heads per KV head are attended per unit");

    // candidate window and keep set (aq_evaluation.py:189-193, 210-237)
    const int T = a->T_total;
    const int sink_end = a->sink > 0 ? std::min(a->sink, a->T_codes) : 0;
    const int local_start0 = std::max(T - std::max(a->local, 0), 0);
    const int cand_end = a->local > 0 ? std::min(a->T_codes, local_start0) : a->T_codes;
    p.c0 = sink_end;
    p.c1 = std::max(sink_end, cand_end);
    p.ncand = p.c1 - p.c0;
    LP_CHECK(a->topk >= 0 && a->topk <= p.ncand,
             "topk must be in [0, number of candidates] (candidates = [sink, min(T_codes, T_total-local)))");
    int sb = a->sink > 0 ? std::min(a->sink, T) : 0;
    int start = a->local > 0 ? std::max(T - a->local, 0) : T;
    if (start <= 0) sb = 0;
    else if (start < sb) start = sb;
    p.n_sink = sb;
    p.local_start = start;
    p.n_local = T - start;
    p.n_rows = p.n_sink + a->topk + p.n_local;
    if (p.n_rows == 0) {  // reference keeps the last token (aq_evaluation.py:234-235)
        p.local_start = T - 1;
        p.n_local = 1;
        p.n_rows = 1;
    }
    LP_CHECK(p.c0 >= p.n_sink || p.ncand == 0, "internal: candidate window overlaps the sink tokens");

    const int sms = sm_count(device);
    {
        const int tiles_per_unit = (p.ncand + kScoreThreads - 1) / kScoreThreads;
        const int64_t want = std::min<int64_t>((int64_t)sms, (int64_t)p.U * std::max(1, tiles_per_unit));
        p.score_ctas = (int)std::max<int64_t>((int64_t)p.U, want);
    }

    const int nwords_cand = p.ncand > 0 ? ((p.c1 + 31) >> 5) - (p.c0 >> 5) : 0;
    p.sel_ctas_per_unit = std::max(1, std::min(std::max(1, 2 * sms / p.Usel), std::max(1, nwords_cand / 8)));
    p.sel_words_per_cta = std::max(1, (nwords_cand + p.sel_ctas_per_unit - 1) / p.sel_ctas_per_unit);
    p.sel_ctas_per_unit = std::max(1, (nwords_cand + p.sel_words_per_cta - 1) / p.sel_words_per_cta);

    const int split_target = std::max(1, 2 * sms / p.Uatt);
    p.rows_per = std::min(kAttnRows, std::max(1, (p.n_rows + split_target - 1) / split_target));
    p.nsplit = (p.n_rows + p.rows_per - 1) / p.rows_per;

    p.bm_words = (a->T_codes + 31) / 32 + 1;

    // the fused single-kernel path (cooperative, one CTA per SM).  Every
    // fused launch on a device has this grid: a call's CTAs derive its epoch
    // as (launch counter / grid size) from a counter that each CTA of every
    // earlier call advanced by one, which is consistent only if all of them
    // used the same grid size (the counter lives in the workspace, and a
    // workspace is device memory of one device)
    p.fused_ctas = sms;
    LP_CHECK(p.fused_ctas == sm_count(device) && p.fused_ctas > 0,
             "internal: the fused grid must have one CTA per SM of the device");
    {
        // per-KV-head selection: a unit is a (sequence, KV head) pair scoring
        // with the summed query of its G heads; per-query-head selection: a
        // unit is a (sequence, query head) pair, G units per KV head reading
        // the same codes and K/V rows
        p.fused_units = p.per_head ? p.Usel : p.U;
        const int Uf = p.fused_units;
        const int cn_min = Uf > 0 ? p.fused_ctas / Uf : 0;
        const int nwu = p.ncand > 0 ? ((p.c1 + 31) >> 5) - (p.c0 >> 5) : 0;
        const int ntok_max = cn_min > 0 ? (nwu + cn_min - 1) / cn_min * 32 : 0;
        // a CTA keeps the scores of up to kFScoreCap tokens in shared memory;
        // above that (long contexts over few CTAs per unit) they spill to the
        // L2-resident score buffer, with the row list bounded by kFSpillList
        p.fused_spill = ntok_max > kFScoreCap;
        p.fused = !(a->flags & LP_FLAG_NO_FUSED) && a->head_scores == nullptr && a->out != nullptr &&
                  a->D == 128 && (p.per_head || a->G <= kFusedMaxG) && Uf <= p.fused_ctas && Uf <= kUnitBarWords &&
                  p.ncand > 0 && a->topk > 0 && nwu <= kFMaxWords && cn_min >= 1 &&
                  (!p.fused_spill || (ntok_max <= kFSpillMaxTok && a->topk <= kFSpillList));
        p.fused_max_split = cn_min + 1;
        // candidate publishing: each CTA aims at twice its even share of the
        // top-k plus a margin (slot capacity: that plus the population of
        // its threshold bin)
        const int cn_max = Uf > 0 ? (p.fused_ctas + Uf - 1) / Uf : 1;
        p.pub_target = 2 * ((a->topk + cn_max - 1) / cn_max) + 32;
        p.pub_cap = p.pub_target + 64;
        if (p.pub_cap > kPubMaxCap || cn_max > kPubMaxCtas || (a->flags & LP_FLAG_EXCHANGE_SELECT)) p.pub_cap = 0;
    }

    Carver c(ws);
    // fixed offsets, identical for every geometry: the error word (0), the
    // fused kernel's 64-bit launch counter (256 B) and the per-unit barrier
    // words (512 B .. 2048 B), whose values must survive between calls
    p.err = c.take<uint32_t>(64);
    p.bar = c.take<uint32_t>(64);
    p.ubar = c.take<unsigned long long>(kUnitBarWords);
    // the fused kernel's exchange arena: a fixed offset and a fixed size (its
    // worst case for this device).  Its tagged words are accepted once their
    // tag shows the call's epoch, so no plain data of any call (another
    // geometry, the multi-kernel path) may ever land on them: a stale plain
    // word whose upper half equals a later epoch would be taken for that
    // call's data.  The one plain region, the LUT, is read only after the
    // flags of its writers show the call's epoch.
    p.fwin = c.take<unsigned long long>((size_t)sms * (kPubWin + 2));
    p.fpub = c.take<unsigned long long>((size_t)sms * kPubMaxCap * 2);
    p.flutflag = c.take<unsigned long long>((size_t)sms);
    p.flut = c.take<float>((size_t)sms * 256 * 32);  // U <= sms units; plain, read only behind the flags
    p.fpart = c.take<unsigned long long>((size_t)2 * sms * kFusedMaxG * (2 + 128));  // U * (sms/U + 1) * G
    p.lut = c.take<float>((size_t)p.U * 256 * 32 * (p.heads ? 4 : 1));
    p.bounds = c.take<float>((size_t)p.U * (p.heads ? a->G : 1) * 32 * kLutParts * 2);
    p.sel_scores = c.take<float>((size_t)p.Usel * std::max(1, a->T_codes));
    p.bitmap = c.take<uint32_t>((size_t)p.Usel * p.bm_words);
    p.nchunk = std::max(1, (nwords_cand + kCompactWords - 1) / kCompactWords);
    p.chunk_cnt = c.take<int>((size_t)p.Usel * p.nchunk);
    p.toplist = c.take<int32_t>((size_t)p.Usel * std::max(a->topk, 1));
    p.compact = a->topk > 0 && p.ncand > 0 && (a->topk_out != nullptr || (a->out != nullptr && p.per_head));
    p.tie_buf = c.take<float2>((size_t)std::max(p.Usel, p.fused_ctas) * kTieCap);
    p.info = c.take<int4>((size_t)p.Usel);
    p.part = c.take<float>((size_t)std::max((size_t)p.Uatt * p.nsplit * p.HG, (size_t)p.U * p.fused_max_split * a->G) *
                           (2 + 128));
    p.cta_count = c.take<uint32_t>((size_t)p.fused_ctas);
    p.cta_ties = c.take<uint32_t>((size_t)p.fused_ctas);
    if (p.fused) p.chist = c.take<uint32_t>((size_t)p.fused_ctas * kNB);
    p.zero_words = (int64_t)p.Usel * kNB + p.Usel + p.Usel + p.Uatt;
    p.zero = c.take<uint32_t>((size_t)p.zero_words);
    p.hist = p.zero;
    p.tie_count = p.hist + (int64_t)p.Usel * kNB;
    p.done_sel = p.tie_count + p.Usel;
    p.done_att = p.done_sel + p.Usel;
    p.bytes = c.used();
    return LP_OK;
}

template <typename QT>
static int launch_lut(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st) {
    LutBuildParams lp_{};
    lp_.q = a->q;
    lp_.q_stride_b = a->q_stride_b;
    lp_.q_stride_h = a->q_stride_h;
    lp_.cb = a->codebooks;
    lp_.cb_dtype = a->cb_dtype;
    lp_.cb_per_kv_head = a->cb_per_kv_head;
    lp_.Hkv = a->Hkv;
    lp_.G = a->G;
    lp_.D = a->D;
    lp_.M = a->M;
    lp_.K = a->K;
    lp_.lut = p.lut;
    lp_.bounds = p.bounds;
    lp_.zero = p.zero;
    lp_.zero_words = p.zero_words;
    dim3 grid(a->M * kLutParts, p.U);
    if (p.heads)
        lut_build_kernel<QT, true><<<grid, kLutThreads, 4 * a->D * sizeof(float), st>>>(lp_);
    else
        lut_build_kernel<QT, false><<<grid, kLutThreads, a->D * sizeof(float), st>>>(lp_);
    return check_launch("lut_build_kernel");
}

template <typename QT, typename KT, typename OT>
static int launch_attn(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st) {
    AttnParams ap{};
    ap.q = a->q;
    ap.q_stride_b = a->q_stride_b;
    ap.q_stride_h = a->q_stride_h;
    ap.keys = a->keys;
    ap.vals = a->vals;
    ap.k_stride_b = a->k_stride_b;
    ap.k_stride_h = a->k_stride_h;
    ap.k_stride_t = a->k_stride_t;
    ap.v_stride_b = a->v_stride_b;
    ap.v_stride_h = a->v_stride_h;
    ap.v_stride_t = a->v_stride_t;
    ap.bitmap = p.bitmap;
    ap.bm_stride = p.bm_words;
    ap.toplist = p.compact ? (a->topk_out ? a->topk_out : p.toplist) : nullptr;
    ap.Hkv = a->Hkv;
    ap.G = a->G;
    ap.HG = p.HG;
    ap.c0 = p.c0;
    ap.c1 = p.c1;
    ap.n_sink = p.n_sink;
    ap.k = a->topk;
    ap.local_start = p.local_start;
    ap.n_local = p.n_local;
    ap.n_rows = p.n_rows;
    ap.T_total = a->T_total;
    ap.nsplit = p.nsplit;
    const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf((float)a->D);
    ap.scale_log2 = scale * 1.4426950408889634f;
    ap.part = p.part;
    ap.done = p.done_att;
    ap.out = a->out;
    ap.out_stride_b = a->out_stride_b;
    ap.out_stride_h = a->out_stride_h;
    dim3 grid(p.nsplit, p.Uatt);
    sparse_attn_kernel<QT, KT, OT, 256><<<grid, 256, 0, st>>>(ap);
    return check_launch("sparse_attn_kernel");
}

template <typename QT, typename KT>
static int launch_attn_out(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st) {
    switch (a->out_dtype) {
        case LP_BF16: return launch_attn<QT, KT, __nv_bfloat16>(a, p, st);
        case LP_F16: return launch_attn<QT, KT, __half>(a, p, st);
        case LP_F32: return launch_attn<QT, KT, float>(a, p, st);
    }
    return fail(LP_ERR_INVALID, "out_dtype must be LP_BF16, LP_F16 or LP_F32");
}

template <typename QT>
static int launch_attn_kv(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st) {
    switch (a->kv_dtype) {
        case LP_BF16: return launch_attn_out<QT, __nv_bfloat16>(a, p, st);
        case LP_F16: return launch_attn_out<QT, __half>(a, p, st);
    }
    return fail(LP_ERR_INVALID, "kv_dtype must be LP_BF16 or LP_F16");
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <typename QT, typename KT, typename OT>
static int launch_fused(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st, int dev) {
    FusedParams fp{};
    fp.q = a->q;
    fp.q_stride_b = a->q_stride_b;
    fp.q_stride_h = a->q_stride_h;
    fp.cb = a->codebooks;
    fp.cb_dtype = a->cb_dtype;
    fp.cb_per_kv_head = a->cb_per_kv_head;
    fp.codes = a->codes;
    fp.codes_stride_b = a->codes_stride_b;
    fp.codes_stride_h = a->codes_stride_h;
    fp.keys = a->keys;
    fp.vals = a->vals;
    fp.k_stride_b = a->k_stride_b;
    fp.k_stride_h = a->k_stride_h;
    fp.k_stride_t = a->k_stride_t;
    fp.v_stride_b = a->v_stride_b;
    fp.v_stride_h = a->v_stride_h;
    fp.v_stride_t = a->v_stride_t;
    fp.Hkv = a->Hkv;
    fp.G = p.per_head ? 1 : a->G;
    fp.U = p.fused_units;
    fp.B = a->B;
    fp.Hu = p.per_head ? a->Hkv * a->G : a->Hkv;
    fp.upk = p.per_head ? a->G : 1;
    fp.spill = p.fused_spill ? 1 : 0;
    fp.c0 = p.c0;
    fp.c1 = p.c1;
    fp.k = a->topk;
    fp.n_sink = p.n_sink;
    fp.local_start = p.local_start;
    fp.n_local = p.n_local;
    fp.n_rows = p.n_rows;
    fp.T_total = a->T_total;
    const float scale = a->scale > 0.f ? a->scale : 1.0f / sqrtf((float)a->D);
    fp.scale_log2 = scale * 1.4426950408889634f;
    fp.out = a->out;
    fp.out_stride_b = a->out_stride_b;
    fp.out_stride_h = a->out_stride_h;
    fp.topk_out = a->topk_out;
    fp.lut = p.flut;
    fp.lut_flag = p.flutflag;
    fp.sel_scores = p.sel_scores;
    fp.sel_stride = std::max(1, a->T_codes);
    fp.chist = p.chist;
    fp.bitmap = p.bitmap;
    fp.bm_stride = p.bm_words;
    fp.tie_buf = p.tie_buf;
    fp.cta_ties = p.cta_ties;
    fp.pub = p.fpub;
    fp.pwin = p.fwin;
    fp.pub_target = p.pub_target;
    fp.pub_cap = p.pub_cap;
    fp.cta_count = p.cta_count;
    fp.part = p.fpart;
    fp.max_split = p.fused_max_split;
    fp.test_timeout = (a->flags & LP_FLAG_TEST_WAIT_TIMEOUT) ? 1 : 0;
    fp.bar = p.ubar;
    fp.epoch_ctr = reinterpret_cast<unsigned long long*>(p.bar);
    fp.err = p.err;
    fp.phase_ns = reinterpret_cast<unsigned long long*>(a->phase_ns);
    for (int i = 0; i < 2; ++i) {
        fp.pf_ptr[i] = static_cast<const char*>(a->prefetch_ptr[i]);
        fp.pf_bytes[i] = a->prefetch_bytes[i];
        fp.pf_count[i] = a->prefetch_count[i];
        fp.pf_stride[i] = a->prefetch_stride[i];
    }
    auto kernel = sparse_decode_fused_kernel<QT, KT, OT>;
    static bool opt[64] = {false};
    int rc = smem_opt_in(kernel, FusedSmem::kTotal, dev, opt);
    if (rc != LP_OK) return rc;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    // programmatic dependent launch: the grid may be scheduled while the
    // previous kernel on the stream finishes; every CTA's first instruction
    // waits for that kernel to complete (griddepcontrol.wait)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(p.fused_ctas);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = FusedSmem::kTotal;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, fp);
    if (e != cudaSuccess) return fail(LP_ERR_CUDA, std::string("sparse_decode_fused_kernel launch: ") + cudaGetErrorString(e));
    return LP_OK;
}

template <typename QT, typename KT>
static int launch_fused_out(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st, int dev) {
    switch (a->out_dtype) {
        case LP_BF16: return launch_fused<QT, KT, __nv_bfloat16>(a, p, st, dev);
        case LP_F16: return launch_fused<QT, KT, __half>(a, p, st, dev);
        case LP_F32: return launch_fused<QT, KT, float>(a, p, st, dev);
    }
    return fail(LP_ERR_INVALID, "out_dtype must be LP_BF16, LP_F16 or LP_F32");
}

template <typename QT>
static int launch_fused_kv(const lp_sparse_decode_args* a, const Plan& p, cudaStream_t st, int dev) {
    switch (a->kv_dtype) {
        case LP_BF16: return launch_fused_out<QT, __nv_bfloat16>(a, p, st, dev);
        case LP_F16: return launch_fused_out<QT, __half>(a, p, st, dev);
    }
    return fail(LP_ERR_INVALID, "kv_dtype must be LP_BF16 or LP_F16");
}

}  // namespace lp

using namespace lp;

extern "C" {

const char* lp_last_error(void) { return g_last_error.c_str(); }

int lp_version(void) { return 1; }

size_t lp_sizeof_sparse_decode_args(void) { return sizeof(lp_sparse_decode_args); }

size_t lp_sparse_decode_workspace_size(const lp_sparse_decode_args* a) {
    Plan p{};
    int dev = 0;
    cudaGetDevice(&dev);
    if (make_plan(a, nullptr, &p, dev) != LP_OK) return 0;
    return p.bytes;
}

int lp_sparse_decode(const lp_sparse_decode_args* a, void* workspace, size_t workspace_bytes, void* stream) {
    int dev = 0;
    LP_CUDA(cudaGetDevice(&dev));
    Plan p{};
    int rc = make_plan(a, workspace, &p, dev);
    if (rc != LP_OK) return rc;
    if (!workspace || workspace_bytes < p.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(LP_ERR_WORKSPACE, "workspace missing, misaligned (256 B) or smaller than lp_sparse_decode_workspace_size()");
    LP_CHECK(a->q && a->codebooks && a->codes, "q, codebooks and codes must not be NULL");
    LP_CHECK(a->q_dtype == LP_BF16 || a->q_dtype == LP_F16 || a->q_dtype == LP_F32,
             "q_dtype must be LP_BF16, LP_F16 or LP_F32");
    LP_CHECK(aligned16(a->codebooks), "codebooks must be 16-byte aligned");
    LP_CHECK(a->cb_dtype == LP_F32 || a->cb_dtype == LP_F16 || a->cb_dtype == LP_BF16,
             "cb_dtype must be LP_F32, LP_F16 or LP_BF16");
    LP_CHECK(aligned16(a->codes) && a->codes_stride_b % 16 == 0 && a->codes_stride_h % 16 == 0,
             "codes base and batch/head strides must be 16-byte aligned");
    LP_CHECK(a->codes_stride_t == 32, "codes rows must be contiguous 32-byte rows (stride_t == M == 32)");
    if (a->out) {
        LP_CHECK(a->keys && a->vals, "keys and vals must not be NULL when out is requested");
        LP_CHECK(a->D == 128, "the attention stage supports head_dim D=128");
        const int esz = 2;
        LP_CHECK(aligned16(a->keys) && aligned16(a->vals), "keys/vals must be 16-byte aligned");
        LP_CHECK((a->k_stride_b * esz) % 16 == 0 && (a->k_stride_h * esz) % 16 == 0 &&
                     (a->k_stride_t * esz) % 16 == 0 && (a->v_stride_b * esz) % 16 == 0 &&
                     (a->v_stride_h * esz) % 16 == 0 && (a->v_stride_t * esz) % 16 == 0,
                 "K/V strides must be multiples of 16 bytes");
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaEvent_t* ev = reinterpret_cast<cudaEvent_t*>(a->stage_events);
    auto mark = [&](int i) -> int {
        if (ev && ev[i]) {
            cudaError_t e = cudaEventRecord(ev[i], st);
            if (e != cudaSuccess) return fail(LP_ERR_CUDA, std::string("cudaEventRecord: ") + cudaGetErrorString(e));
        }
        return LP_OK;
    };
    if ((rc = mark(0)) != LP_OK) return rc;

    if (p.fused) {
        switch (a->q_dtype) {
            case LP_BF16: rc = launch_fused_kv<__nv_bfloat16>(a, p, st, dev); break;
            case LP_F16: rc = launch_fused_kv<__half>(a, p, st, dev); break;
            default: rc = launch_fused_kv<float>(a, p, st, dev); break;
        }
        if (rc != LP_OK) return rc;
        for (int i = 1; i <= 4; ++i)
            if ((rc = mark(i)) != LP_OK) return rc;
        return LP_OK;
    }

    // 1. tables
    switch (a->q_dtype) {
        case LP_BF16: rc = launch_lut<__nv_bfloat16>(a, p, st); break;
        case LP_F16: rc = launch_lut<__half>(a, p, st); break;
        default: rc = launch_lut<float>(a, p, st); break;
    }
    if (rc != LP_OK) return rc;
    if ((rc = mark(1)) != LP_OK) return rc;

    // 2. scores + histogram
    if (p.ncand > 0) {
        ScoreParams sp{};
        sp.lut = p.lut;
        sp.bounds = p.bounds;
        sp.codes = a->codes;
        sp.codes_stride_b = a->codes_stride_b;
        sp.codes_stride_h = a->codes_stride_h;
        sp.Hkv = a->Hkv;
        sp.G = a->G;
        sp.U = p.U;
        sp.c0 = p.c0;
        sp.c1 = p.c1;
        sp.sel_scores = p.sel_scores;
        sp.sel_stride = std::max(1, a->T_codes);
        sp.head_scores = a->head_scores;
        sp.hs_stride = a->T_codes;
        sp.hist = p.hist;
        sp.sel_per_head = p.per_head ? 1 : 0;
        sp.err = p.err;
        // programmatic dependent launch: the scorer starts streaming codes
        // while the table build finishes (it waits before reading tables)
        cudaLaunchConfig_t cfg{};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3(p.score_ctas);
        cfg.blockDim = dim3(kScoreThreads);
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t le;
        if (p.heads) {
            using S = ScoreSmem<true, kScoreThreads, kHeadsStages>;
            static bool opt[64] = {false};
            rc = smem_opt_in(score_kernel<true, kScoreThreads, kHeadsStages>, S::kTotal, dev, opt);
            if (rc != LP_OK) return rc;
            cfg.dynamicSmemBytes = S::kTotal;
            le = cudaLaunchKernelEx(&cfg, score_kernel<true, kScoreThreads, kHeadsStages>, sp);
        } else {
            using S = ScoreSmem<false, kScoreThreads, kGroupStages>;
            static bool opt[64] = {false};
            rc = smem_opt_in(score_kernel<false, kScoreThreads, kGroupStages>, S::kTotal, dev, opt);
            if (rc != LP_OK) return rc;
            cfg.dynamicSmemBytes = S::kTotal;
            le = cudaLaunchKernelEx(&cfg, score_kernel<false, kScoreThreads, kGroupStages>, sp);
        }
        if (le != cudaSuccess) return fail(LP_ERR_CUDA, std::string("score_kernel launch: ") + cudaGetErrorString(le));
        rc = check_launch("score_kernel");
        if (rc != LP_OK) return rc;
        if ((rc = mark(2)) != LP_OK) return rc;

        // 3. selection
        SelectParams sel{};
        sel.sel_scores = p.sel_scores;
        sel.sel_stride = std::max(1, a->T_codes);
        sel.bounds = p.bounds;
        sel.Gb = p.heads ? a->G : 1;
        sel.per_head = p.per_head ? 1 : 0;
        sel.hist = p.hist;
        sel.bitmap = p.bitmap;
        sel.bm_stride = p.bm_words;
        sel.tie_buf = p.tie_buf;
        sel.tie_count = p.tie_count;
        sel.done = p.done_sel;
        sel.info = p.info;
        sel.c0 = p.c0;
        sel.c1 = p.c1;
        sel.k = a->topk;
        sel.words_per_cta = p.sel_words_per_cta;
        sel.err = p.err;
        const int sel_smem = kTieCap * 8;
        static bool opt_sel[64] = {false};
        rc = smem_opt_in(select_kernel<256>, sel_smem, dev, opt_sel);
        if (rc != LP_OK) return rc;
        select_kernel<256><<<dim3(p.sel_ctas_per_unit, p.Usel), 256, sel_smem, st>>>(sel);
        rc = check_launch("select_kernel");
        if (rc != LP_OK) return rc;
        // the selected tokens in ascending order: the caller's top-k output,
        // and the attention's row lists when there are many selection units
        // (per query head: the attention CTAs would each scan a whole bitmap)
        if (p.compact) {
            int32_t* list = a->topk_out ? a->topk_out : p.toplist;
            const dim3 cg(p.nchunk, p.Usel);
            bitmap_chunk_count_kernel<<<cg, kCompactWords, 0, st>>>(p.bitmap, p.bm_words, p.c0, p.c1, p.nchunk,
                                                                   p.chunk_cnt);
            rc = check_launch("bitmap_chunk_count_kernel");
            if (rc != LP_OK) return rc;
            bitmap_compact_kernel<<<cg, kCompactWords, 0, st>>>(p.bitmap, p.bm_words, p.c0, p.c1, a->topk, p.nchunk,
                                                               p.chunk_cnt, list);
            rc = check_launch("bitmap_compact_kernel");
            if (rc != LP_OK) return rc;
        }
    } else {
        if ((rc = mark(2)) != LP_OK) return rc;
    }
    if ((rc = mark(3)) != LP_OK) return rc;

    // 4. attention over the kept rows
    if (a->out) {
        switch (a->q_dtype) {
            case LP_BF16: rc = launch_attn_kv<__nv_bfloat16>(a, p, st); break;
            case LP_F16: rc = launch_attn_kv<__half>(a, p, st); break;
            default: rc = launch_attn_kv<float>(a, p, st); break;
        }
        if (rc != LP_OK) return rc;
    }
    if ((rc = mark(4)) != LP_OK) return rc;
    return LP_OK;
}

size_t lp_sizeof_encode_args(void) { return sizeof(lp_encode_args); }

static int encode_plan(const lp_encode_args* a, size_t* bytes, int64_t* nsets, int64_t* nvec_set) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->D == 128 && a->M == 32 && a->K == 256, "the encoder supports D=128, M=32 codebooks of K=256 entries");
    LP_CHECK(a->B >= 0 && a->H > 0 && a->T >= 0, "need B >= 0, H > 0, T >= 0");
    *nsets = a->cb_per_kv_head ? a->H : 1;
    *nvec_set = a->cb_per_kv_head ? (int64_t)a->B * a->T : (int64_t)a->B * a->H * a->T;
    LP_CHECK(*nvec_set <= (int64_t)1 << 30, "too many vectors");
    LP_CHECK(a->icm_iters >= 0 && a->icm_iters <= 1024, "icm_iters must be in [0, 1024]");
    Carver c(nullptr);
    c.take<unsigned char>(kPersistBytes);
    c.take<float>((size_t)*nsets * 32 * 256);
    if (a->icm_iters > 0) {
        c.take<float>((size_t)*nsets * *nvec_set * 128);
        c.take<uint32_t>((size_t)a->icm_iters * *nsets);
    }
    *bytes = c.used();
    return LP_OK;
}

// Vectors per CTA of the encoder: fewer rows per CTA while that still
// leaves SMs idle (the 32 stages are a serial chain per CTA, so more, smaller
// CTAs finish sooner): 128 (one full UMMA tile), 64, 32 or 16.
static int encode_rows_per_cta(int64_t nsets, int64_t nvec_set, int sms) {
    int rows = kEncRows;
    while (rows > 16 && nsets * ((nvec_set + rows / 2 - 1) / (rows / 2)) <= sms) rows /= 2;
    return rows;
}

int lp_encode_rows_per_cta(const lp_encode_args* a) {
    size_t bytes = 0;
    int64_t ns = 0, nv = 0;
    if (encode_plan(a, &bytes, &ns, &nv) != LP_OK) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    return encode_rows_per_cta(ns, nv, sm_count(dev));
}

size_t lp_encode_workspace_size(const lp_encode_args* a) {
    size_t bytes = 0;
    int64_t ns = 0, nv = 0;
    if (encode_plan(a, &bytes, &ns, &nv) != LP_OK) return 0;
    return bytes;
}

int lp_encode_keys(const lp_encode_args* a, void* workspace, size_t workspace_bytes, void* stream) {
    size_t need = 0;
    int64_t nsets = 0, nvec_set = 0;
    int rc = encode_plan(a, &need, &nsets, &nvec_set);
    if (rc != LP_OK) return rc;
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(LP_ERR_WORKSPACE, "workspace missing, misaligned (256 B) or smaller than lp_encode_workspace_size()");
    LP_CHECK(a->x_dtype == LP_BF16 || a->x_dtype == LP_F16 || a->x_dtype == LP_F32,
             "x_dtype must be LP_BF16, LP_F16 or LP_F32");
    if (nvec_set == 0) return LP_OK;
    LP_CHECK(a->x && a->codebooks && a->codes, "x, codebooks and codes must not be NULL");
    LP_CHECK(aligned16(a->codebooks), "codebooks must be 16-byte aligned");
    int dev = 0;
    LP_CUDA(cudaGetDevice(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    Carver c(workspace);
    uint32_t* err = c.take<uint32_t>(kPersistBytes / 4);
    float* nrm = c.take<float>((size_t)nsets * 32 * 256);  // ||C||^2 for the ICM sweeps
    float* icm_fr = a->icm_iters > 0 ? c.take<float>((size_t)nsets * nvec_set * 128) : nullptr;
    uint32_t* icm_changed = a->icm_iters > 0 ? c.take<uint32_t>((size_t)a->icm_iters * nsets) : nullptr;
    // the ICM sweeps read the codeword norms from the workspace (the greedy
    // kernel computes its own, stage by stage, from its shared-memory copies)
    if (a->icm_iters > 0) {
        const int64_t ncw = nsets * 32 * 256;
        encode_norms_kernel<<<(unsigned)((ncw + 255) / 256), 256, 0, st>>>(a->codebooks, ncw, nrm);
        rc = check_launch("encode_norms_kernel");
        if (rc != LP_OK) return rc;
    }

    EncodeParams ep{};
    ep.x = a->x;
    ep.xs_b = a->x_stride_b;
    ep.xs_h = a->x_stride_h;
    ep.xs_t = a->x_stride_t;
    ep.B = a->B;
    ep.H = a->H;
    ep.T = a->T;
    ep.per_head = a->cb_per_kv_head ? 1 : 0;
    ep.cb = a->codebooks;
    ep.codes = a->codes;
    ep.cs_b = a->codes_stride_b;
    ep.cs_h = a->codes_stride_h;
    ep.cs_t = a->codes_stride_t;
    const int rows = encode_rows_per_cta(nsets, nvec_set, sm_count(dev));
    ep.rows_per_cta = rows;
    ep.ctas_per_set = (int)((nvec_set + rows - 1) / rows);
    ep.force_exact = (a->flags & LP_ENCODE_FLAG_EXACT) ? 1 : 0;
    ep.err = err;
    // the codebooks as a 2-D tensor [S*32*256 rows][128 fp32], copied in boxes
    // of 32 dims x 128 rows with the 128-byte swizzle the UMMA layout expects
    CUtensorMap cmap;
    {
        const cuuint64_t gdim[2] = {128, (cuuint64_t)nsets * 32 * 256};
        const cuuint64_t gstride[1] = {128 * sizeof(float)};
        const cuuint32_t box[2] = {32, 128};
        const cuuint32_t estride[2] = {1, 1};
        // resolved through the runtime, so the library has no link-time
        // dependency on the driver library (it loads on hosts without one)
        using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                           const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                           CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                           CUtensorMapFloatOOBfill);
        static EncodeTiledFn encode_tiled = nullptr;
        static std::once_flag once;
        std::call_once(once, [] {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                encode_tiled = reinterpret_cast<EncodeTiledFn>(fn);
        });
        if (!encode_tiled) return fail(LP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        const CUresult cr = encode_tiled(&cmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                                                   const_cast<float*>(a->codebooks), gdim, gstride, box, estride,
                                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return fail(LP_ERR_CUDA, "cuTensorMapEncodeTiled failed for the codebooks");
    }
    const dim3 grid((unsigned)(nsets * ep.ctas_per_set));
    static bool opt_enc[12][64] = {{false}};
    auto launch_enc = [&](auto kern, int slot) {
        const int r = smem_opt_in(kern, EncSmem::kTotal, dev, opt_enc[slot]);
        if (r != LP_OK) return r;
        kern<<<grid, kEncThreads, EncSmem::kTotal, st>>>(cmap, ep);
        return (int)LP_OK;
    };
    // CTAs of 64, 32 or 16 vectors: the instantiation with 2, 4 or 8 copies
    // of the residual rows in the MMA tile
    const int ri = rows == kEncRows ? 0 : rows == kEncRows / 2 ? 1 : rows == kEncRows / 4 ? 2 : 3;
    switch (a->x_dtype) {
        case LP_BF16:
            rc = ri == 0   ? launch_enc(encode_keys_kernel<__nv_bfloat16, 1>, 0)
                 : ri == 1 ? launch_enc(encode_keys_kernel<__nv_bfloat16, 2>, 1)
                 : ri == 2 ? launch_enc(encode_keys_kernel<__nv_bfloat16, 4>, 2)
                           : launch_enc(encode_keys_kernel<__nv_bfloat16, 8>, 3);
            break;
        case LP_F16:
            rc = ri == 0   ? launch_enc(encode_keys_kernel<__half, 1>, 4)
                 : ri == 1 ? launch_enc(encode_keys_kernel<__half, 2>, 5)
                 : ri == 2 ? launch_enc(encode_keys_kernel<__half, 4>, 6)
                           : launch_enc(encode_keys_kernel<__half, 8>, 7);
            break;
        default:
            rc = ri == 0   ? launch_enc(encode_keys_kernel<float, 1>, 8)
                 : ri == 1 ? launch_enc(encode_keys_kernel<float, 2>, 9)
                 : ri == 2 ? launch_enc(encode_keys_kernel<float, 4>, 10)
                           : launch_enc(encode_keys_kernel<float, 8>, 11);
            break;
    }
    if (rc != LP_OK) return rc;
    rc = check_launch("encode_keys_kernel");
    if (rc != LP_OK || a->icm_iters == 0) return rc;

    // ICM sweeps, one launch each (a sweep reads the previous one's count of
    // changed codes of its set and returns when it is zero)
    LP_CUDA(cudaMemsetAsync(icm_changed, 0, sizeof(uint32_t) * (size_t)a->icm_iters * nsets, st));
    IcmParams ip{};
    ip.x = a->x;
    ip.xs_b = a->x_stride_b;
    ip.xs_h = a->x_stride_h;
    ip.xs_t = a->x_stride_t;
    ip.B = a->B;
    ip.H = a->H;
    ip.T = a->T;
    ip.per_head = a->cb_per_kv_head ? 1 : 0;
    ip.cb = a->codebooks;
    ip.nrm = nrm;
    ip.codes = a->codes;
    ip.cs_b = a->codes_stride_b;
    ip.cs_h = a->codes_stride_h;
    ip.cs_t = a->codes_stride_t;
    ip.fr = icm_fr;
    ip.changed = icm_changed;
    ip.ctas_per_set = (int)((nvec_set + kIcmVec - 1) / kIcmVec);
    ip.err = err;
    const dim3 igrid((unsigned)(nsets * ip.ctas_per_set));
    for (int sweep = 0; sweep < a->icm_iters; ++sweep) {
        ip.sweep = sweep;
        ip.last = sweep + 1 == a->icm_iters ? 1 : 0;
        switch (a->x_dtype) {
            case LP_BF16: icm_sweep_kernel<__nv_bfloat16><<<igrid, kIcmThreads, 0, st>>>(ip); break;
            case LP_F16: icm_sweep_kernel<__half><<<igrid, kIcmThreads, 0, st>>>(ip); break;
            default: icm_sweep_kernel<float><<<igrid, kIcmThreads, 0, st>>>(ip); break;
        }
        rc = check_launch("icm_sweep_kernel");
        if (rc != LP_OK) return rc;
    }
    return LP_OK;
}

int lp_lut_gather(const lp_lut_gather_args* a, void* stream) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->lut_dtype == LP_F16 || a->lut_dtype == LP_F32, "lut must be fp16 or fp32");
    LP_CHECK(a->out_dtype == LP_F16 || a->out_dtype == LP_F32, "out must be fp16 or fp32");
    LP_CHECK(a->Q >= 0 && a->G > 0 && a->T >= 0 && a->N >= 0 && a->K > 0, "invalid sizes");
    LP_CHECK(a->m0 >= 0 && a->m1 > a->m0 && a->m1 <= a->M_stride, "M range must satisfy 0 <= M_start < M_end <= M");
    LP_CHECK((int64_t)(a->m1 - a->m0) * a->K <= 12288, "LUT slice too large (at most 12288 entries per row)");
    if (a->Q == 0 || a->N == 0) return LP_OK;
    LP_CHECK(a->lut && a->codes && a->out, "lut, codes and out must not be NULL");
    LutGatherParams p{};
    p.lut = a->lut;
    p.lut_f16 = a->lut_dtype == LP_F16;
    p.lut_stride_q = a->lut_stride_q;
    p.M_stride = a->M_stride;
    p.K = a->K;
    p.m0 = a->m0;
    p.m1 = a->m1;
    p.codes = a->codes;
    p.cs_h = a->codes_stride_h;
    p.cs_t = a->codes_stride_t;
    p.Q = a->Q;
    p.G = a->G;
    p.T = a->T;
    p.N = a->N;
    p.indices = a->indices;
    p.is_q = a->indices_stride_q;
    p.code_mode = a->code_mode;
    p.out = a->out;
    p.out_f16 = a->out_dtype == LP_F16;
    p.os_q = a->out_stride_q;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = sm_count(dev);
    const int mr = a->m1 - a->m0;
    // 16-byte code-row loads: rows of at most 32 used bytes, 16-byte aligned
    const bool vec = a->m1 <= 32 && (reinterpret_cast<uintptr_t>(a->codes) & 15u) == 0 &&
                     a->codes_stride_h % 16 == 0 && a->codes_stride_t % 16 == 0;
    const bool f16 = a->lut_dtype == LP_F16;
    p.lut_vec = f16 && (reinterpret_cast<uintptr_t>(a->lut) & 15u) == 0 && a->lut_stride_q % 8 == 0 &&
                ((int64_t)a->m0 * a->K) % 8 == 0 && ((int64_t)mr * a->K) % 8 == 0;
    if (vec && a->indices == nullptr && a->G > 1 && a->Q % a->G == 0 && a->G <= (f16 ? kScanMaxG : kScanMaxG32) &&
        a->N == a->T) {
        // dense scan: each code row read once for the G rows that share it
        const int H = a->Q / a->G;
        const int64_t smem64 = (int64_t)(f16 ? (a->G + 1) / 2 : a->G) * mr * a->K * 4;
        if (smem64 <= 200 * 1024) {
            const int smem = (int)smem64;
            // about 3 CTAs per SM (the fp16 G=4 table, 64 KB, allows 3)
            int64_t tile = ((int64_t)a->T * H + 3ll * sms - 1) / (3ll * sms);
            tile = std::min<int64_t>(16384, std::max<int64_t>(kScanThreads, (tile + kScanThreads - 1) / kScanThreads * kScanThreads));
            const dim3 grid((unsigned)((a->T + tile - 1) / tile), (unsigned)H);
            static bool opt16[64] = {false}, opt32[64] = {false};
            if (f16) {
                int rc = smem_opt_in(lut_scan_group_kernel<true>, 200 * 1024, dev, opt16);
                if (rc != LP_OK) return rc;
                lut_scan_group_kernel<true><<<grid, kScanThreads, smem, st>>>(p, (int)tile);
            } else {
                int rc = smem_opt_in(lut_scan_group_kernel<false>, 200 * 1024, dev, opt32);
                if (rc != LP_OK) return rc;
                lut_scan_group_kernel<false><<<grid, kScanThreads, smem, st>>>(p, (int)tile);
            }
            return check_launch("lut_scan_group_kernel");
        }
    }
    const int smem = mr * a->K * 4;
    if (vec) {
        // per-row tables, `tile` tokens per CTA so that a table is staged
        // once for many tokens
        int64_t tile = ((int64_t)a->N * a->Q + 2ll * sms - 1) / (2ll * sms);
        tile = std::min<int64_t>(8192, std::max<int64_t>(256, (tile + 255) / 256 * 256));
        lut_gather_rows_kernel<<<dim3((unsigned)((a->N + tile - 1) / tile), a->Q), 256, smem, st>>>(p, (int)tile);
        return check_launch("lut_gather_rows_kernel");
    }
    lut_gather_kernel<<<dim3((a->N + 255) / 256, a->Q), 256, smem, st>>>(p);
    return check_launch("lut_gather_kernel");
}

int lp_lut_build(const lp_lut_build_args* a, void* stream) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->Q >= 0 && a->M > 0 && a->K > 0 && a->D > 0 && a->D <= 12288, "invalid sizes");
    if (a->Q == 0) return LP_OK;
    LP_CHECK(a->q && a->codebooks && a->lut, "q, codebooks and lut must not be NULL");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    LP_CHECK(a->D <= 320, "lut build: D must be at most 320");
    int dev = 0;
    cudaGetDevice(&dev);
    const dim3 grid((a->K + 31) / 32, a->M, (a->Q + 31) / 32);
    const int smem = 2 * 32 * (a->D + 1) * 4;
    static bool opt[3][64] = {};
    switch (a->q_dtype) {
        case LP_BF16: {
            int rc = smem_opt_in(lut_build_rows_kernel<__nv_bfloat16>, smem, dev, opt[0]);
            if (rc != LP_OK) return rc;
            lut_build_rows_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(
                reinterpret_cast<const __nv_bfloat16*>(a->q), a->q_stride, a->codebooks, a->M, a->K, a->D, a->Q, a->lut);
            break;
        }
        case LP_F16: {
            int rc = smem_opt_in(lut_build_rows_kernel<__half>, smem, dev, opt[1]);
            if (rc != LP_OK) return rc;
            lut_build_rows_kernel<__half><<<grid, 256, smem, st>>>(
                reinterpret_cast<const __half*>(a->q), a->q_stride, a->codebooks, a->M, a->K, a->D, a->Q, a->lut);
            break;
        }
        case LP_F32: {
            int rc = smem_opt_in(lut_build_rows_kernel<float>, smem, dev, opt[2]);
            if (rc != LP_OK) return rc;
            lut_build_rows_kernel<float><<<grid, 256, smem, st>>>(
                reinterpret_cast<const float*>(a->q), a->q_stride, a->codebooks, a->M, a->K, a->D, a->Q, a->lut);
            break;
        }
        default:
            return fail(LP_ERR_INVALID, "q_dtype must be LP_BF16, LP_F16 or LP_F32");
    }
    return check_launch("lut_build_rows_kernel");
}

int lp_gqa_gather_kv(const lp_gqa_gather_args* a, void* stream) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->kv_dtype == LP_F16 || a->kv_dtype == LP_BF16, "K/V must be fp16 or bf16");
    LP_CHECK(a->B >= 0 && a->Hkv > 0 && a->G > 0 && a->T >= 0 && a->D > 0 && a->N_explicit >= 0,
             "invalid sizes");
    LP_CHECK(a->tail_count >= 0 && a->tail_start >= 0 && (int64_t)a->tail_start + a->tail_count <= a->T,
             "invalid implicit tail range");
    const int64_t N = (int64_t)a->N_explicit + a->tail_count;
    const int64_t rows = (int64_t)a->B * a->Hkv * a->G * N;
    if (rows == 0) return LP_OK;
    LP_CHECK(a->keys && a->vals && a->out_k && a->out_v && (a->indices || a->N_explicit == 0),
             "keys, vals, indices and outputs must not be NULL");
    GqaGatherParams p{};
    p.keys = static_cast<const uint16_t*>(a->keys);
    p.vals = static_cast<const uint16_t*>(a->vals);
    p.ks_b = a->k_stride_b;
    p.ks_h = a->k_stride_h;
    p.ks_t = a->k_stride_t;
    p.vs_b = a->v_stride_b;
    p.vs_h = a->v_stride_h;
    p.vs_t = a->v_stride_t;
    p.indices = a->indices;
    p.is_b = a->indices_stride_b;
    p.is_h = a->indices_stride_h;
    p.B = a->B;
    p.Hkv = a->Hkv;
    p.G = a->G;
    p.T = a->T;
    p.D = a->D;
    p.N_explicit = a->N_explicit;
    p.tail_start = a->tail_start;
    p.N = (int)N;
    p.out_k = static_cast<uint16_t*>(a->out_k);
    p.out_v = static_cast<uint16_t*>(a->out_v);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (a->D % 8 == 0 && al16(a->keys) && al16(a->vals) && al16(a->out_k) && al16(a->out_v) &&
        a->k_stride_b % 8 == 0 && a->k_stride_h % 8 == 0 && a->k_stride_t % 8 == 0 && a->v_stride_b % 8 == 0 &&
        a->v_stride_h % 8 == 0 && a->v_stride_t % 8 == 0) {
        // 16-byte units: every K and V row is D/8 of them
        int dev = 0;
        cudaGetDevice(&dev);
        (void)dev;
        const dim3 grid((unsigned)((N + 8 * kKvRowsPerWarp - 1) / (8 * kKvRowsPerWarp)), (unsigned)(a->B * a->Hkv * a->G));
        gqa_gather_vec_kernel<<<grid, 256, 0, st>>>(p);
        return check_launch("gqa_gather_vec_kernel");
    }
    gqa_gather_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(p);
    return check_launch("gqa_gather_kernel");
}

size_t lp_sizeof_rope_append_args(void) { return sizeof(lp_rope_append_args); }

int lp_rope_append(const lp_rope_append_args* a, void* stream) {
    LP_CHECK(a != nullptr, "args must not be NULL");
    LP_CHECK(a->dtype == LP_BF16 || a->dtype == LP_F16, "dtype must be LP_BF16 or LP_F16");
    LP_CHECK(a->B >= 0 && a->Hq > 0 && a->Hkv > 0 && a->D > 0 && a->D % 2 == 0 && a->D <= 1024,
             "need B >= 0, Hq > 0, Hkv > 0 and an even D <= 1024");
    LP_CHECK(a->pos >= 0, "pos must be non-negative");
    if (a->B == 0) return LP_OK;
    LP_CHECK(a->q && a->k && a->v && a->cos && a->sin && a->q_out && a->k_cache && a->v_cache,
             "tensors must not be NULL");
    RopeAppendParams p{};
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.q_sb = a->q_stride_b;
    p.q_sh = a->q_stride_h;
    p.k_sb = a->k_stride_b;
    p.k_sh = a->k_stride_h;
    p.v_sb = a->v_stride_b;
    p.v_sh = a->v_stride_h;
    p.cos = a->cos;
    p.sin = a->sin;
    p.cos_sb = a->cos_stride_b;
    p.sin_sb = a->sin_stride_b;
    p.q_out = a->q_out;
    p.qo_sb = a->q_out_stride_b;
    p.qo_sh = a->q_out_stride_h;
    p.k_cache = a->k_cache;
    p.v_cache = a->v_cache;
    p.kc_sb = a->kc_stride_b;
    p.kc_sh = a->kc_stride_h;
    p.kc_st = a->kc_stride_t;
    p.vc_sb = a->vc_stride_b;
    p.vc_sh = a->vc_stride_h;
    p.vc_st = a->vc_stride_t;
    p.Hq = a->Hq;
    p.Hkv = a->Hkv;
    p.D = a->D;
    p.pos = a->pos;
    const dim3 grid((unsigned)(a->Hq + 2 * a->Hkv), (unsigned)a->B);
    const unsigned threads = (unsigned)((a->D / 2 + 31) / 32 * 32);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (a->dtype == LP_BF16) rope_append_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(p);
    else rope_append_kernel<__half><<<grid, threads, 0, st>>>(p);
    return check_launch("rope_append_kernel");
}

int lp_read_device_errors(void* workspace, size_t workspace_bytes, void* stream, uint32_t* bits_out) {
    LP_CHECK(workspace && workspace_bytes >= 256 && bits_out, "workspace and bits_out must not be NULL");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint32_t v = 0;
    LP_CUDA(cudaMemcpyAsync(&v, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    LP_CUDA(cudaStreamSynchronize(st));
    LP_CUDA(cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st));
    // a timed-out barrier leaves its word mid-count: restore the barrier
    // words (the launch counter at 256 B only ever grows and is kept)
    if (v & LP_DEVERR_WAIT_TIMEOUT) {
        LP_CHECK(workspace_bytes >= kPersistBytes, "workspace smaller than its persistent state");
        LP_CUDA(cudaMemsetAsync(static_cast<char*>(workspace) + 512, 0, kPersistBytes - 512, st));
    }
    LP_CUDA(cudaStreamSynchronize(st));
    *bits_out = v;
    return LP_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of lp_sparse_decode: the workspace is a file-scope
// device array instead of caller-owned memory.
// ---------------------------------------------------------------------------
namespace lp {

// One scratch per device, zero when the module loads.  Host code must not
// pass `g_noalloc_scratch` itself to a kernel (on the host it names a
// stand-in, not device memory): noalloc_scratch() looks up its device
// address once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LP_NOALLOC_SCRATCH_BYTES];

// The identity of the device's current context (0 if the driver cannot say).
// A device reset destroys the primary context and unloads this module with
// it; the scratch then reappears at another address in the next context, so
// the address looked up for a device is only valid while its context lives.
static unsigned long long current_context_id() {
    using GetCurrentFn = CUresult (*)(CUcontext*);
    using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrentFn>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetIdFn>(fn);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS)
        return id;
    return 0;
}

static int noalloc_scratch(void** out) {
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    static unsigned long long ctx_of[64] = {0};
    int dev = 0;
    LP_CUDA(cudaGetDevice(&dev));
    LP_CHECK(dev >= 0 && dev < 64, "device ordinal out of range (at most 64 devices)");
    // 0 before the device's first runtime call (no context yet): the lookup
    // below then creates the context
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx == 0 || ctx != ctx_of[dev]) {
        void* ptr = nullptr;
        LP_CUDA(cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch));
        LP_CHECK(ptr != nullptr && (reinterpret_cast<uintptr_t>(ptr) & 255u) == 0,
                 "built-in scratch has no 256-byte aligned device address");
        addr[dev] = ptr;
        ctx_of[dev] = current_context_id();
    }
    *out = addr[dev];
    return LP_OK;
}

}  // namespace lp

extern "C" int lp_sparse_decode_noalloc(const lp_sparse_decode_args* a, void* stream, uint32_t* device_errors) {
    using namespace lp;
    LP_CHECK(a != nullptr, "args must not be NULL");
    const size_t need = lp_sparse_decode_workspace_size(a);
    if (need == 0) return LP_ERR_INVALID;  // the plan's message is already set
    if (need > (size_t)LP_NOALLOC_SCRATCH_BYTES)
        return fail(LP_ERR_WORKSPACE,
                    "lp_sparse_decode_noalloc: this geometry needs " + std::to_string(need) +
                        " bytes of workspace, more than the built-in scratch of " +
                        std::to_string((size_t)LP_NOALLOC_SCRATCH_BYTES) +
                        " bytes; call lp_sparse_decode with a workspace of your own");
    void* ws = nullptr;
    int rc = noalloc_scratch(&ws);
    if (rc != LP_OK) return rc;
    rc = lp_sparse_decode(a, ws, (size_t)LP_NOALLOC_SCRATCH_BYTES, stream);
    if (rc != LP_OK || device_errors == nullptr) return rc;
    return lp_read_device_errors(ws, (size_t)LP_NOALLOC_SCRATCH_BYTES, stream, device_errors);
}
