/*
 * laprune_b200.h -- C ABI of the B200 (sm_100a) implementation of LAPrune's
 * sparse-decode hot path.
 *
 * Conventions
 *   - Every entry point returns an int status (LP_OK == 0).  On failure the
 *     message is available from lp_last_error() (thread-local); the Python
 *     binding raises RuntimeError with that text, mirroring the reference's
 *     TORCH_CHECK messages where an entry point replaces a reference one.
 *   - Pointers are device pointers unless stated otherwise; sizes and strides
 *     are plain integers (strides in ELEMENTS of the pointed-to type unless
 *     stated as bytes).  No framework types cross this boundary.
 *   - `stream` is a cudaStream_t passed as void*; every kernel is launched on
 *     it and nothing synchronises the host, so calls are stream-ordered and
 *     can be captured in CUDA graphs (except where noted).
 *   - The caller owns every buffer, including `workspace` (size from the
 *     matching *_workspace_size function, 256-byte aligned, device memory,
 *     ZERO-FILLED before its first use).  Its first 2048 bytes hold state
 *     that persists between calls (device error bits, a launch counter,
 *     barrier words), at the same offsets for every geometry; the rest is
 *     scratch.  A workspace must not be shared by calls that may run
 *     concurrently.
 *   - A lp_sparse_decode workspace also holds, after those 2048 bytes, the
 *     fused kernel's exchange arena: words tagged with the call's launch
 *     number, at a fixed offset and of a fixed size for the device, so that
 *     calls of any geometry can share the workspace.  Give lp_encode_keys a
 *     workspace of its own (its scratch would land in that arena).
 */
#ifndef LAPRUNE_B200_H
#define LAPRUNE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define LP_OK 0
#define LP_ERR_INVALID 1     /* bad argument (shape, dtype, stride, size)      */
#define LP_ERR_CUDA 2        /* a CUDA runtime call or kernel launch failed    */
#define LP_ERR_UNSUPPORTED 3 /* valid but not implemented on this path         */
#define LP_ERR_WORKSPACE 4   /* workspace missing, too small or misaligned     */

/* element types */
#define LP_F32 0
#define LP_F16 1
#define LP_BF16 2
#define LP_F64 3
#define LP_U8 4
#define LP_I8 5
#define LP_I64 6
#define LP_I32 7

/* selection modes of the fused pipeline */
#define LP_SELECT_KV_GROUP 0   /* top-k per KV head on GQA-summed scores      */
#define LP_SELECT_QUERY_HEAD 1 /* top-k per query head (reference decode hook) */

/* device-side error bits reported through lp_read_device_errors */
#define LP_DEVERR_WAIT_TIMEOUT 1u  /* a bounded wait gave up                    */
#define LP_DEVERR_TIE_OVERFLOW 2u  /* informational: exact slow select path ran */

const char* lp_last_error(void);
int lp_version(void);
/* sizeof(lp_sparse_decode_args), for bindings to verify their struct layout */
size_t lp_sizeof_sparse_decode_args(void);

/* ======================================================================
 * Fused hot path
 * ====================================================================== */

/* Arguments of the sparse decode step (one decode token, one layer).
 * Geometry: B sequences, Hkv KV heads, G query heads per KV head
 * (Hq = Hkv*G), head_dim D, M codebooks of K entries.                     */
typedef struct lp_sparse_decode_args {
    /* query rows q[b][hq][0..D) at q + b*q_stride_b + hq*q_stride_h (elements) */
    const void* q;
    int32_t q_dtype; /* LP_BF16 | LP_F16 | LP_F32 */
    int32_t _pad0;
    int64_t q_stride_b, q_stride_h;
    /* codebooks, contiguous [Hkv][M][K][D] (cb_per_kv_head=1) or [M][K][D]
     * shared by every KV head (cb_per_kv_head=0), of cb_dtype: LP_F32 (0, the
     * default), or LP_F16 / LP_BF16 copies (half the bytes; the tables are
     * still built in fp32 from their exactly widened elements) */
    const void* codebooks;
    int32_t cb_per_kv_head;
    int32_t cb_dtype;
    /* uint8 codes[b][hkv][t][m] at codes + b*sb + hkv*sh + t*st + m (bytes) */
    const uint8_t* codes;
    int64_t codes_stride_b, codes_stride_h, codes_stride_t;
    /* K/V cache [b][hkv][t][0..D) (elements), dtype LP_BF16 | LP_F16 */
    const void* keys;
    const void* vals;
    int32_t kv_dtype;
    int32_t _pad2;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    int32_t B, Hkv, G, D, M, K;
    int32_t T_codes;  /* tokens with codes (candidate scoring range ends here) */
    int32_t T_total;  /* tokens attended to (K/V rows valid in [0,T_total))   */
    int32_t sink;     /* leading sink tokens always kept                      */
    int32_t local;    /* trailing local window always kept                    */
    int32_t topk;     /* tokens selected per selection unit                   */
    int32_t select_mode; /* LP_SELECT_KV_GROUP | LP_SELECT_QUERY_HEAD          */
    float scale;      /* softmax scale; <= 0 selects 1/sqrt(D)                */
    int32_t out_dtype; /* LP_BF16 | LP_F16 | LP_F32                           */
    /* attention output out[b][hq][0..D) at out + b*out_stride_b + hq*out_stride_h;
     * NULL skips the attention stage (scoring + selection only) */
    void* out;
    int64_t out_stride_b, out_stride_h;
    /* optional fp32 per-query-head scores [B][Hq][T_codes] (contiguous); only
     * the candidate window is written.  NULL: not produced. */
    float* head_scores;
    /* optional selected indices [units][topk] in ascending order, int32;
     * units = B*Hkv (KV_GROUP) or B*Hkv*G (QUERY_HEAD).  NULL: not produced. */
    int32_t* topk_out;
    /* optional array of 5 cudaEvent_t recorded on `stream` before the LUT
     * build and after the LUT build, scoring, selection and attention stages
     * (for live per-kernel timing).  NULL: no events. */
    void** stage_events;
    /* LP_FLAG_* bits */
    int32_t flags;
    int32_t _pad3;
    /* optional uint64[8] of device global-timer stamps (ns) at the phase
     * boundaries of the fused single-kernel path (diagnostics).  NULL: none. */
    uint64_t* phase_ns;
    /* optional L2 prefetch of the NEXT call's inputs, issued by the fused
     * kernel once its own HBM streams are done (while its selection and
     * attention stages leave HBM idle): region i covers prefetch_count[i]
     * blocks of prefetch_bytes[i] bytes starting every prefetch_stride[i]
     * bytes from prefetch_ptr[i] (e.g. the next layer's codebooks and the
     * [0,T) rows of every KV head of its code cache).  Bytes and addresses
     * should be multiples of 16.  NULL pointers / zero bytes: nothing. */
    const void* prefetch_ptr[2];
    int64_t prefetch_bytes[2];
    int64_t prefetch_count[2];
    int64_t prefetch_stride[2];
} lp_sparse_decode_args;

/* flags of lp_sparse_decode_args */
#define LP_FLAG_NO_FUSED 1 /* use the multi-kernel path even when the fused kernel applies */
#define LP_FLAG_EXCHANGE_SELECT 2 /* fused kernel: settle the top-k through the tie exchange,
                                    not the published-candidate union */
#define LP_FLAG_TEST_WAIT_TIMEOUT 4 /* for testing the error path (fused kernel only): CTA 0
                                      withholds its share of its unit's table, so the unit's
                                      waits for it give up after about 2^20 cycles and the
                                      call reports LP_DEVERR_WAIT_TIMEOUT (its outputs are
                                      then undefined); no fault, no hang */

/* Workspace bytes needed by lp_sparse_decode for this geometry. */
size_t lp_sparse_decode_workspace_size(const lp_sparse_decode_args* a);

/* LUT build (q . C_m[k], fp32) -> candidate-window scoring -> exact top-k
 * (ties: lower index first) -> union with sink and local window -> GQA K/V
 * gather -> split-K flash-decode.  Reference path this replaces:
 *   laprune/llm/aq_kv.py:633-699 (approx_inner_product_multihead_gqa),
 *   laprune/llm/modifiers/aq_evaluation.py:146-253 (_decode_attention:
 *   candidate window :185-205, keep set :206-237, gather :239-250,
 *   SDPA :251),
 *   aq_kernels/aq_lut_gqa.cu:460-534 (aq_lut_gather_grouped) and
 *   :536-664 (gqa_gather_kv / gqa_gather_kv_with_tail). */
int lp_sparse_decode(const lp_sparse_decode_args* a, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Reads and clears the device-side error bits accumulated in `workspace`
 * by earlier calls (synchronises `stream`); after a wait timeout it also
 * restores the workspace's barrier words. */
int lp_read_device_errors(void* workspace, size_t workspace_bytes, void* stream,
                          uint32_t* bits_out);

/* ======================================================================
 * Key encode: greedy residual additive quantization of new keys
 * ====================================================================== */

/* Arguments of lp_encode_keys.  Vectors x[b][h][t][0..D) (post-RoPE keys of
 * the code cache's encode buffer); codes[b][h][t][0..M) may point straight
 * into a code cache [B][Hkv][cap][M] at the buffer's first position. */
typedef struct lp_encode_args {
    const void* x;              /* at x + b*x_stride_b + h*x_stride_h + t*x_stride_t (elements) */
    int32_t x_dtype;            /* LP_BF16 | LP_F16 | LP_F32 */
    int32_t cb_per_kv_head;     /* 1: codebooks [H][M][K][D], vector (b,h,t) uses set h;
                                   0: one set [M][K][D] for every vector */
    int64_t x_stride_b, x_stride_h, x_stride_t;
    const float* codebooks;     /* fp32, contiguous, 16-byte aligned */
    uint8_t* codes;             /* at codes + b*sb + h*sh + t*st + m (bytes) */
    int64_t codes_stride_b, codes_stride_h, codes_stride_t;
    int32_t B, H, T, D, M, K;   /* D = 128, M = 32, K = 256 */
    int32_t flags;              /* LP_ENCODE_FLAG_* bits */
    int32_t icm_iters;          /* ICM sweeps after the greedy pass (0: greedy codes only) */
} lp_encode_args;

#define LP_ENCODE_FLAG_EXACT 1 /* compute every distance on CUDA cores (testing) */

/* sizeof(lp_encode_args), for bindings to verify their struct layout */
size_t lp_sizeof_encode_args(void);
/* Workspace bytes needed by lp_encode_keys (first 2048 bytes: error word
 * and reserved state, as for lp_sparse_decode; with icm_iters > 0 also the
 * vectors' reconstructions between sweeps, 512 bytes per vector). */
size_t lp_encode_workspace_size(const lp_encode_args* a);

/* With icm_iters > 0 the greedy codes are then refined by up to icm_iters ICM
 * sweeps (laprune/quantizer.py:356-370): each sweep re-chooses code m =
 * 0..M-1 of every vector against the reconstruction without it
 * (r = x - (full_recon - C_m[prev]), the same distance arithmetic), and a
 * sweep that changes no code of the vectors sharing a codebook set ends that
 * set's refinement.
 *
 * Greedy residual encode: for m = 0..M-1, code_m = the first k minimising
 * ||r||^2 + ||C_m[k]||^2 - 2 r.C_m[k] (fp32: the norms sequential chains of
 * fused multiply-adds in index order, r.C_m[k] 32 four-term chains over
 * dims 4l..4l+3 folded pairwise at strides 16, 8, 4, 2, 1), then
 * r -= C_m[code_m].  The
 * contraction runs on tcgen05 tensor cores (tf32) as a filter under an error
 * bound; near-ties are settled exactly on CUDA cores.  Reference path this
 * replaces: aq_kernels/fused_linear_encode.cu:168-234
 * (fused_linear_encode_forward), laprune/llm/aq_kv.py:44-75
 * (_fast_greedy_encode) and laprune/quantizer.py:346-374
 * (AdditiveQuantizer._batch_icm_lut with 0 ICM iterations). */
int lp_encode_keys(const lp_encode_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* Vectors per CTA that lp_encode_keys uses for this geometry on the current
 * device: 128 (one M=128 tensor-core tile per stage), 64, 32 or 16
 * (smaller CTAs, their rows copied 2, 4 or 8 times into the tile, while
 * larger ones would leave SMs idle); 0 for invalid arguments.
 * A diagnostic for tests that must cover every tile size. */
int lp_encode_rows_per_cta(const lp_encode_args* a);

/* ======================================================================
 * Building blocks behind the aq_kernels-named Python surface
 * ====================================================================== */

/* out[q][n] = sum_{m in [m0,m1)} lut[q][m][codes[q/G][t][m]] (fp32
 * accumulation in m order, then out_dtype), t = indices ? indices[q][n] : n;
 * tokens outside [0,T) give 0.  Replaces aq_kernels/aq_lut_gqa.cu:350-534
 * (aq_lut_gather, aq_lut_gather_grouped) and aq_kernels/aq_lut.cu:581-738
 * (aq_lut_gather_forward). */
typedef struct lp_lut_gather_args {
    const void* lut;          /* LP_F16 | LP_F32, row q: [M_stride][K] contiguous */
    int32_t lut_dtype;
    int32_t code_mode;        /* 0: clamp codes to K-1; 1: codes >= K add nothing */
    int64_t lut_stride_q;     /* elements between rows */
    int32_t M_stride, K, m0, m1;
    const uint8_t* codes;     /* codes[h][t][m] at codes + h*sh + t*st + m (bytes) */
    int64_t codes_stride_h, codes_stride_t;
    int32_t Q, G, T, N;
    const int64_t* indices;   /* optional [Q][N] token indices; NULL: n = t, N = T */
    int64_t indices_stride_q;
    void* out;                /* [Q][N] of out_dtype (LP_F16 | LP_F32) */
    int32_t out_dtype;
    int32_t _pad0;
    int64_t out_stride_q;
} lp_lut_gather_args;
int lp_lut_gather(const lp_lut_gather_args* a, void* stream);

/* lut[q][m][k] = q_q . C[m][k] (fp32, sequential fma over d).  The LUT step
 * of aq_kernels/aq_lut.cu:445-574 (aq_lut_forward). */
typedef struct lp_lut_build_args {
    const void* q;            /* [Q][D] at q + i*q_stride (elements) */
    int32_t q_dtype;          /* LP_BF16 | LP_F16 | LP_F32 */
    int32_t _pad0;
    int64_t q_stride;
    const float* codebooks;   /* fp32 [M][K][D] contiguous */
    int32_t Q, M, K, D;
    float* lut;               /* fp32 [Q][M][K] contiguous */
} lp_lut_build_args;
int lp_lut_build(const lp_lut_build_args* a, void* stream);

/* out_k/out_v[b][hq][n] = K/V[b][hq/G][token] for token = indices[b][hq][n]
 * (n < N_explicit) or tail_start + n - N_explicit (implicit local tail);
 * tokens outside [0,T) give zero rows.  Replaces aq_kernels/aq_lut_gqa.cu:
 * 536-664 (gqa_gather_kv, gqa_gather_kv_with_tail). */
typedef struct lp_gqa_gather_args {
    const void* keys;
    const void* vals;
    int32_t kv_dtype;         /* LP_F16 | LP_BF16 */
    int32_t _pad0;
    int64_t k_stride_b, k_stride_h, k_stride_t, v_stride_b, v_stride_h, v_stride_t;
    const int64_t* indices;   /* [B][Hq][N_explicit] */
    int64_t indices_stride_b, indices_stride_h;
    int32_t B, Hkv, G, T, D, N_explicit, tail_start, tail_count;
    void* out_k;              /* [B][Hq][N_explicit + tail_count][D] contiguous */
    void* out_v;
} lp_gqa_gather_args;
int lp_gqa_gather_kv(const lp_gqa_gather_args* a, void* stream);

/* ======================================================================
 * Decode-token rotary embedding fused with the K/V cache append
 * ====================================================================== */

/* One decode token of B sequences: q_out[b][h] = rope(q[b][h]) for the Hq
 * query rows; k_cache[b][h][pos] = rope(k[b][h]) and v_cache[b][h][pos] =
 * v[b][h] for the Hkv KV rows, rope(x) = x * cos[b] + rotate_half(x) *
 * sin[b] with rotate_half(x) = [-x[D/2:], x[:D/2]] and every product and the
 * sum rounded to the dtype (as HF apply_rotary_pos_emb on bf16/fp16
 * tensors).  Replaces laprune/llm/modifiers/aq_evaluation.py:296-308 (RoPE of
 * the new token, then _kv_cache_append's slice copies, :65-112) for a static
 * cache with room at `pos`.  Strides in elements; every tensor of `dtype`. */
typedef struct lp_rope_append_args {
    const void* q;            /* [B][Hq][D] at q + b*q_stride_b + h*q_stride_h */
    const void* k;            /* [B][Hkv][D] */
    const void* v;            /* [B][Hkv][D] */
    int64_t q_stride_b, q_stride_h, k_stride_b, k_stride_h, v_stride_b, v_stride_h;
    const void* cos;          /* [B][D]: the token's rotary rows */
    const void* sin;
    int64_t cos_stride_b, sin_stride_b;
    void* q_out;              /* [B][Hq][D] */
    int64_t q_out_stride_b, q_out_stride_h;
    void* k_cache;            /* [B][Hkv][cap][D] */
    void* v_cache;
    int64_t kc_stride_b, kc_stride_h, kc_stride_t, vc_stride_b, vc_stride_h, vc_stride_t;
    int32_t dtype;            /* LP_BF16 | LP_F16 */
    int32_t B, Hq, Hkv, D;    /* D even, <= 1024 */
    int32_t pos;              /* cache slot of the token (< cap) */
} lp_rope_append_args;
size_t lp_sizeof_rope_append_args(void);
int lp_rope_append(const lp_rope_append_args* a, void* stream);

/* ======================================================================
 * Allocation-free variant (no counterpart in the reference)
 * ====================================================================== */

/* Size of the library's built-in per-device scratch (32 MiB): enough for one
 * sequence (B = 1) with 8 KV heads up to about 380k tokens; the workspace
 * size lp_sparse_decode_workspace_size() reports must not exceed it. */
#define LP_NOALLOC_SCRATCH_BYTES (32u << 20)

/* lp_sparse_decode for callers that must not allocate device memory: a
 * serving runtime that has handed all of HBM to its own pool (a cudaMalloc
 * there fails or fragments the pool), or a latency-critical decode loop in
 * which cudaMalloc/cudaFree would synchronise the device.  Instead of a
 * caller-owned workspace it uses a scratch array that the library holds in
 * device memory (LP_NOALLOC_SCRATCH_BYTES per GPU that loads the library,
 * kept until the process exits); it calls no cudaMalloc, cudaFree or other
 * allocating routine.  The caller still passes every input and output.
 *   - The first call on a device looks up the scratch's device address
 *     (cudaGetSymbolAddress) with that device current, and so does the first
 *     call after the device's context was recreated (cudaDeviceReset unloads
 *     the library's device code with the context, and the scratch comes back
 *     zeroed at another address); make such a first call before any stream
 *     capture starts on the device.
 *   - Geometries whose workspace exceeds LP_NOALLOC_SCRATCH_BYTES are
 *     rejected with LP_ERR_WORKSPACE (use lp_sparse_decode with a workspace
 *     of your own for those).
 *   - Every call on a device shares the one scratch, which keeps the last
 *     call's contents.  Its first 2048 bytes (error bits, launch counter,
 *     barrier words) must start at zero: the array is zero when the library loads and the calls
 *     leave those words consistent.  Calls whose kernels may overlap on the
 *     GPU (different streams, threads or processes sharing the context) race
 *     on it: order them on one stream.
 *   - device_errors: NULL, or a host pointer that receives the device error
 *     bits (LP_DEVERR_*) of the scratch after this call; the call then
 *     synchronises `stream` and clears the bits, as lp_read_device_errors. */
int lp_sparse_decode_noalloc(const lp_sparse_decode_args* a, void* stream, uint32_t* device_errors);

#ifdef __cplusplus
}
#endif

#endif /* LAPRUNE_B200_H */
