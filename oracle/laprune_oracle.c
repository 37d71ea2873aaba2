/*
 * laprune_oracle.c -- CPU restatement of LAPrune's sparse-decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in laprune_b200/csrc and the timed CPU baseline of bench.py.  The
 * product never links, loads or calls it.
 *
 * Every function restates one step of the reference (LAPrune, Python/PyTorch
 * CPU path) in plain C with fp32 arithmetic, citing the reference file:line it
 * follows.  Parity of this restatement against the reference itself is pinned
 * by tests/test_oracle_golden.py, which compares it with fixtures produced by
 * running the reference code (tests/golden/make_golden.py).
 *
 * Threading: OpenMP over independent heads / vectors / tokens.  Results do not
 * depend on the thread count (each output element is produced by one thread in
 * a fixed order).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* LUT build: lut[q][m][k] = sum_d q[q][d] * cb[m][k][d]  (fp32, d in order).
 * Follows laprune/llm/aq_kv.py:620 (einsum "mkd,qd->qmk") and :500.
 * cb_stride_q: element offset between the codebook sets used by consecutive
 * queries (0 = every query uses the same [M,K,d] codebook, as in the
 * reference's single-group layout; M*K*d*... for per-query-head codebooks). */
void orc_lut(const float* q, const float* cb, int64_t cb_stride_q,
             int Q, int M, int K, int d, float* lut) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int qi = 0; qi < Q; ++qi) {
        for (int m = 0; m < M; ++m) {
            const float* qv = q + (int64_t)qi * d;
            const float* cbm = cb + (int64_t)qi * cb_stride_q + (int64_t)m * K * d;
            float* out = lut + ((int64_t)qi * M + m) * K;
            for (int k = 0; k < K; ++k) {
                const float* c = cbm + (int64_t)k * d;
                float acc = 0.f;
                for (int j = 0; j < d; ++j) acc += qv[j] * c[j];
                out[k] = acc;
            }
        }
    }
}

/* GQA scoring: out[h][t] = sum_{m<M} lut[h][m][codes[h/G][t][m]] (fp32, m in
 * order 0..M-1).  Follows aq_kv.py:621-628 (gather over the codes of the KV
 * head shared by the query head, then sum over m), with the code expansion
 * of aq_kv.py:696-698 done implicitly through h/G.
 * codes are addressed as codes[hkv*stride_h + t*stride_t + m]. */
void orc_score_gqa(const float* lut, const uint8_t* codes,
                   int64_t stride_h, int64_t stride_t,
                   int Hq, int G, int T, int M, int K, float* out) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < Hq; ++h) {
        for (int t = 0; t < T; ++t) {
            const float* l = lut + (int64_t)h * M * K;
            const uint8_t* c = codes + (int64_t)(h / G) * stride_h + (int64_t)t * stride_t;
            float acc = 0.f;
            for (int m = 0; m < M; ++m) acc += l[(int64_t)m * K + c[m]];
            out[(int64_t)h * T + t] = acc;
        }
    }
}

/* Sum the G query-head scores of every KV group: out[u][t] = sum_g s[u*G+g][t]
 * (fp32, g in order).  The per-KV-head selection of the BASELINE configs. */
void orc_group_sum(const float* s, int U, int G, int T, float* out) {
    #pragma omp parallel for schedule(static)
    for (int u = 0; u < U; ++u) {
        for (int t = 0; t < T; ++t) {
            float acc = 0.f;
            for (int g = 0; g < G; ++g) acc += s[((int64_t)u * G + g) * T + t];
            out[(int64_t)u * T + t] = acc;
        }
    }
}

/* ---- exact top-k ------------------------------------------------------ */
typedef struct { float v; int32_t i; } orc_pair;

static int orc_pair_cmp(const void* a, const void* b) {
    const orc_pair* x = (const orc_pair*)a;
    const orc_pair* y = (const orc_pair*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* Top-k of each row of scores[R][n] restricted to [lo, hi): indices (absolute
 * token positions) of the k largest values, ties broken by lower index,
 * written in ascending index order to idx[R][k].  Follows the candidate
 * window + torch.topk of laprune/llm/modifiers/aq_evaluation.py:185-201
 * (torch leaves the order and the tie choice unspecified; this oracle fixes
 * both: largest value first, lowest index among equals). */
static int orc_i32_cmp(const void* a, const void* b) {
    int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

void orc_topk_rows(const float* scores, int R, int n, int lo, int hi, int k,
                   int32_t* idx) {
    #pragma omp parallel for schedule(dynamic)
    for (int r = 0; r < R; ++r) {
        int cnt = hi - lo;
        orc_pair* p = (orc_pair*)malloc(sizeof(orc_pair) * (size_t)(cnt > 0 ? cnt : 1));
        for (int t = 0; t < cnt; ++t) {
            p[t].v = scores[(int64_t)r * n + lo + t];
            p[t].i = lo + t;
        }
        qsort(p, (size_t)cnt, sizeof(orc_pair), orc_pair_cmp);
        int32_t* out = idx + (int64_t)r * k;
        for (int j = 0; j < k; ++j) out[j] = p[j].i;
        qsort(out, (size_t)k, sizeof(int32_t), orc_i32_cmp);
        free(p);
    }
}

/* ---- greedy additive-quantization encode -------------------------------- */
/* r . c in the encoder's fixed order: 32 lanes, lane l a sequential fma chain
 * over its d/32 consecutive dims, then the lanes folded pairwise at strides
 * 16, 8, 4, 2, 1 (p[l] += p[l + s]) -- the order of a warp with a
 * shuffle-xor butterfly, whose every lane ends with the same bits because
 * fp32 addition is commutative.  d must be a multiple of 32. */
static float enc_dot(const float* a, const float* b, int d) {
    float p[32];
    const int per = d / 32;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.f;
        for (int j = l * per; j < (l + 1) * per; ++j) acc = fmaf(a[j], b[j], acc);
        p[l] = acc;
    }
    for (int st = 16; st >= 1; st >>= 1)
        for (int l = 0; l < st; ++l) p[l] = p[l] + p[l + st];
    return p[0];
}

/* Greedy residual encode (icm iters = 0):
 *   for m: dists[k] = (||r||^2 + ||C_m[k]||^2) - 2 * (r . C_m[k]);
 *          code_m = first argmin; r -= C_m[code_m]
 * Follows laprune/quantizer.py:346-355 (with the norms of :315-316).
 * The norms are sequential fma chains in index order, r . C_m[k] is
 * enc_dot's order (the reference's own sums come from BLAS in an
 * implementation-defined order; these are this build's fixed choices).
 * x [N][d] fp32, cb [M][K][d] fp32; codes written as uint8 [N][M].
 * cb_index[n] selects, per vector, which [M,K,d] codebook set of cb to use
 * (NULL = set 0), so per-KV-head codebooks can be encoded in one call. */
void orc_encode_greedy(const float* x, const float* cb, const int32_t* cb_index,
                       int N, int M, int K, int d, uint8_t* codes) {
    /* codebook norms per set: computed lazily for the sets referenced. */
    int nsets = 1;
    if (cb_index) {
        for (int n = 0; n < N; ++n) if (cb_index[n] + 1 > nsets) nsets = cb_index[n] + 1;
    }
    float* norms = (float*)malloc(sizeof(float) * (size_t)nsets * M * K);
    #pragma omp parallel for collapse(2) schedule(static)
    for (int s = 0; s < nsets; ++s) {
        for (int mk = 0; mk < M * K; ++mk) {
            const float* c = cb + ((int64_t)s * M * K + mk) * d;
            float acc = 0.f;
            for (int j = 0; j < d; ++j) acc = fmaf(c[j], c[j], acc);
            norms[(int64_t)s * M * K + mk] = acc;
        }
    }
    #pragma omp parallel
    {
        float* r = (float*)malloc(sizeof(float) * (size_t)d);
        #pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            int s = cb_index ? cb_index[n] : 0;
            const float* cbs = cb + (int64_t)s * M * K * d;
            const float* nrm = norms + (int64_t)s * M * K;
            memcpy(r, x + (int64_t)n * d, sizeof(float) * (size_t)d);
            for (int m = 0; m < M; ++m) {
                /* every sum is written out explicitly (fmaf), so that the
                 * rounding does not depend on the compiler's contraction
                 * choices */
                float rn = 0.f;
                for (int j = 0; j < d; ++j) rn = fmaf(r[j], r[j], rn);
                float best = INFINITY;
                int best_k = 0;
                for (int k = 0; k < K; ++k) {
                    const float* c = cbs + ((int64_t)m * K + k) * d;
                    const float dot = enc_dot(r, c, d);
                    const float dist = fmaf(-2.f, dot, rn + nrm[(int64_t)m * K + k]);
                    if (dist < best) { best = dist; best_k = k; }
                }
                codes[(int64_t)n * M + m] = (uint8_t)best_k;
                const float* cw = cbs + ((int64_t)m * K + best_k) * d;
                for (int j = 0; j < d; ++j) r[j] -= cw[j];
            }
        }
        free(r);
    }
    free(norms);
}

/* ICM refinement after the greedy codes (quantizer.py:356-370, the loop of
 * _batch_icm_lut after its greedy pass): full_recon = x - r_greedy; then up
 * to `iters` sweeps over m = 0..M-1 of
 *     recon_wo = full_recon - C_m[prev];  r = x - recon_wo;
 *     new = first argmin_k ||r||^2 + ||C_m[k]||^2 - 2 r.C_m[k];
 *     full_recon = recon_wo + C_m[new]
 * (elementwise fp32; the norms and r.c in enc_dot's order, as in
 * orc_encode_greedy).  A sweep that changes no code of the batch ends the
 * refinement (quantizer.py:368-369).  The reference runs one quantizer per
 * codebook group, so "the batch" is the set of vectors sharing a codebook
 * set: the early exit is decided per set.  codes [N][M] hold the greedy codes
 * on entry (orc_encode_greedy) and the refined ones on return; sweeps_run
 * [nsets] (optional) receives the number of sweeps each set ran. */
void orc_encode_icm(const float* x, const float* cb, const int32_t* cb_index,
                    int N, int M, int K, int d, int iters, uint8_t* codes, int32_t* sweeps_run) {
    int nsets = 1;
    if (cb_index) {
        for (int n = 0; n < N; ++n) if (cb_index[n] + 1 > nsets) nsets = cb_index[n] + 1;
    }
    for (int s = 0; s < nsets; ++s) if (sweeps_run) sweeps_run[s] = 0;
    if (iters <= 0 || N == 0) return;
    float* norms = (float*)malloc(sizeof(float) * (size_t)nsets * M * K);
    for (int s = 0; s < nsets; ++s) {
        for (int mk = 0; mk < M * K; ++mk) {
            const float* c = cb + ((int64_t)s * M * K + mk) * d;
            float acc = 0.f;
            for (int j = 0; j < d; ++j) acc = fmaf(c[j], c[j], acc);
            norms[(int64_t)s * M * K + mk] = acc;
        }
    }
    /* full reconstruction x - r, r the greedy residual (r -= C_m[code_m]) */
    float* fr = (float*)malloc(sizeof(float) * (size_t)N * d);
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const int s = cb_index ? cb_index[n] : 0;
        const float* cbs = cb + (int64_t)s * M * K * d;
        const float* xn = x + (int64_t)n * d;
        float* f = fr + (int64_t)n * d;
        for (int j = 0; j < d; ++j) f[j] = xn[j];
        for (int m = 0; m < M; ++m) {
            const float* cw = cbs + ((int64_t)m * K + codes[(int64_t)n * M + m]) * d;
            for (int j = 0; j < d; ++j) f[j] -= cw[j];
        }
        for (int j = 0; j < d; ++j) f[j] = xn[j] - f[j];
    }
    int* active = (int*)malloc(sizeof(int) * (size_t)nsets);
    long long* changed = (long long*)malloc(sizeof(long long) * (size_t)nsets);
    for (int s = 0; s < nsets; ++s) active[s] = 1;
    for (int it = 0; it < iters; ++it) {
        for (int s = 0; s < nsets; ++s) changed[s] = 0;
        #pragma omp parallel
        {
            float* rw = (float*)malloc(sizeof(float) * (size_t)d);
            float* r = (float*)malloc(sizeof(float) * (size_t)d);
            #pragma omp for schedule(static)
            for (int n = 0; n < N; ++n) {
                const int s = cb_index ? cb_index[n] : 0;
                if (!active[s]) continue;
                const float* cbs = cb + (int64_t)s * M * K * d;
                const float* nrm = norms + (int64_t)s * M * K;
                const float* xn = x + (int64_t)n * d;
                float* f = fr + (int64_t)n * d;
                long long ch = 0;
                for (int m = 0; m < M; ++m) {
                    const int prev = codes[(int64_t)n * M + m];
                    const float* cp = cbs + ((int64_t)m * K + prev) * d;
                    for (int j = 0; j < d; ++j) { rw[j] = f[j] - cp[j]; r[j] = xn[j] - rw[j]; }
                    float rn = 0.f;
                    for (int j = 0; j < d; ++j) rn = fmaf(r[j], r[j], rn);
                    float best = INFINITY;
                    int best_k = 0;
                    for (int k = 0; k < K; ++k) {
                        const float dot = enc_dot(r, cbs + ((int64_t)m * K + k) * d, d);
                        const float dist = fmaf(-2.f, dot, rn + nrm[(int64_t)m * K + k]);
                        if (dist < best) { best = dist; best_k = k; }
                    }
                    if (best_k != prev) ++ch;
                    codes[(int64_t)n * M + m] = (uint8_t)best_k;
                    const float* cw = cbs + ((int64_t)m * K + best_k) * d;
                    for (int j = 0; j < d; ++j) f[j] = rw[j] + cw[j];
                }
                if (ch) {
                    #pragma omp atomic
                    changed[s] += ch;
                }
            }
            free(rw);
            free(r);
        }
        for (int s = 0; s < nsets; ++s) {
            if (!active[s]) continue;
            if (sweeps_run) sweeps_run[s] += 1;
            if (changed[s] == 0) active[s] = 0;
        }
    }
    free(changed);
    free(active);
    free(fr);
    free(norms);
}

/* Double-precision distances of one vector at one stage, for near-tie
 * classification of encode disagreements: dist[k] = ||r - C_m[k]||^2 with r
 * the residual after the given prefix of codes. */
void orc_encode_stage_dists(const float* x, const float* cb, const uint8_t* prefix,
                            int m, int K, int d, double* dist) {
    double* r = (double*)malloc(sizeof(double) * (size_t)d);
    for (int j = 0; j < d; ++j) r[j] = x[j];
    for (int p = 0; p < m; ++p) {
        const float* cw = cb + ((int64_t)p * K + prefix[p]) * d;
        for (int j = 0; j < d; ++j) r[j] -= cw[j];
    }
    for (int k = 0; k < K; ++k) {
        const float* c = cb + ((int64_t)m * K + k) * d;
        double acc = 0.0;
        for (int j = 0; j < d; ++j) { double e = r[j] - c[j]; acc += e * e; }
        dist[k] = acc;
    }
    free(r);
}

/* ---- sparse attention ------------------------------------------------- */
/* out[h][:] = softmax(q_h . K[idx]^T * scale) . V[idx]   (fp32)
 * Follows the pruned-attention SDPA of aq_evaluation.py:251 (no mask, one
 * query row) over the gathered rows of aq_evaluation.py:239-250.
 * q [H][D]; keys/vals of KV head h/G addressed as base + hkv*stride_h +
 * t*stride_t (+ j); idx [H][n] absolute token positions. */
void orc_sparse_attention(const float* q, const float* keys, const float* vals,
                          int64_t stride_h, int64_t stride_t,
                          const int32_t* idx, int H, int G, int n, int D,
                          float scale, float* out) {
    #pragma omp parallel
    {
        float* w = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
        #pragma omp for schedule(static)
        for (int h = 0; h < H; ++h) {
            const float* qv = q + (int64_t)h * D;
            const int32_t* ih = idx + (int64_t)h * n;
            const int64_t base = (int64_t)(h / G) * stride_h;
            float mx = -INFINITY;
            for (int r = 0; r < n; ++r) {
                const float* kr = keys + base + (int64_t)ih[r] * stride_t;
                float acc = 0.f;
                for (int j = 0; j < D; ++j) acc += qv[j] * kr[j];
                w[r] = acc * scale;
                if (w[r] > mx) mx = w[r];
            }
            float den = 0.f;
            for (int r = 0; r < n; ++r) { w[r] = expf(w[r] - mx); den += w[r]; }
            float* o = out + (int64_t)h * D;
            for (int j = 0; j < D; ++j) o[j] = 0.f;
            for (int r = 0; r < n; ++r) {
                const float* vr = vals + base + (int64_t)ih[r] * stride_t;
                const float p = w[r];
                for (int j = 0; j < D; ++j) o[j] += p * vr[j];
            }
            const float inv = den > 0.f ? 1.f / den : 0.f;
            for (int j = 0; j < D; ++j) o[j] *= inv;
        }
        free(w);
    }
}
