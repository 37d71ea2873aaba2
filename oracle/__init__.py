"""CPU oracle for LAPrune's sparse-decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithm of every step of
the hot path (LUT build, LUT scoring, GQA group sum, candidate window + top-k,
greedy additive-quantization encode, sparse attention) plus the fp16
arithmetic of the reference's CUDA extension entry points.  It is the checker
for the CUDA kernels of ``laprune_b200`` and the timed CPU baseline of
``bench.py``; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import it.  The product never calls it.

The heavy loops live in ``laprune_oracle.c`` (built by ``oracle/Makefile``
into ``oracle/_build``); this module wraps them with numpy.  Parity of this
restatement with the reference itself is pinned by the fixtures under
``tests/golden`` (produced by running the reference code).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liblaprune_oracle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(force: bool = False) -> Path:
    """Compile the C restatement (idempotent)."""
    src = _HERE / "laprune_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        i64 = ctypes.c_int64
        ci = ctypes.c_int
        lib.orc_lut.argtypes = [_f32p, _f32p, i64, ci, ci, ci, ci, _f32p]
        lib.orc_score_gqa.argtypes = [_f32p, _u8p, i64, i64, ci, ci, ci, ci, ci, _f32p]
        lib.orc_group_sum.argtypes = [_f32p, ci, ci, ci, _f32p]
        lib.orc_topk_rows.argtypes = [_f32p, ci, ci, ci, ci, ci, _i32p]
        lib.orc_encode_greedy.argtypes = [_f32p, _f32p, _i32p, ci, ci, ci, ci, _u8p]
        lib.orc_encode_stage_dists.argtypes = [_f32p, _f32p, _u8p, ci, ci, ci, _f64p]
        lib.orc_encode_icm.argtypes = [_f32p, _f32p, _i32p, ci, ci, ci, ci, ci, _u8p, _i32p]
        lib.orc_sparse_attention.argtypes = [_f32p, _f32p, _f32p, i64, i64, _i32p,
                                             ci, ci, ci, ci, ctypes.c_float, _f32p]
        lib.orc_num_threads.restype = ci
        lib.orc_set_num_threads.argtypes = [ci]
        _lib = lib
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def num_threads() -> int:
    return int(_load().orc_num_threads())


def set_num_threads(n: int) -> None:
    _load().orc_set_num_threads(int(n))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


# ---------------------------------------------------------------------------
# fp32 restatement of the reference CPU path
# ---------------------------------------------------------------------------

def lut(q, codebooks, per_query_codebooks: bool = False) -> np.ndarray:
    """LUT[q][m][k] = q . C_m[k] (fp32).  laprune/llm/aq_kv.py:620.

    ``codebooks`` is ``[M,K,d]`` shared by all queries, or (with
    ``per_query_codebooks``) ``[Q,M,K,d]``.
    """
    q = _f32(q)
    cb = _f32(codebooks)
    Q, d = q.shape
    M, K = cb.shape[-3], cb.shape[-2]
    stride = M * K * d if per_query_codebooks else 0
    out = np.empty((Q, M, K), dtype=np.float32)
    _load().orc_lut(_p(q, _f32p), _p(cb, _f32p), stride, Q, M, K, d, _p(out, _f32p))
    return out


def score_gqa(lut_arr, codes, G: int) -> np.ndarray:
    """scores[h][t] = sum_m lut[h][m][codes[h//G][t][m]] (fp32, m order).

    laprune/llm/aq_kv.py:614-630 with the GQA code expansion of :696-698.
    ``codes`` is a uint8 array ``[Hkv, T, M]`` (any strides with M contiguous).
    """
    lut_arr = _f32(lut_arr)
    codes = np.asarray(codes)
    assert codes.dtype == np.uint8 and codes.strides[2] == 1
    Hq, M, K = lut_arr.shape
    Hkv, T, Mc = codes.shape
    assert Mc == M and Hq == Hkv * G
    out = np.empty((Hq, T), dtype=np.float32)
    if T == 0:
        return out
    _load().orc_score_gqa(_p(lut_arr, _f32p), codes.ctypes.data_as(_u8p),
                          codes.strides[0], codes.strides[1], Hq, G, T, M, K,
                          _p(out, _f32p))
    return out


def group_sum(scores, G: int) -> np.ndarray:
    """Sum the G query-head scores of each KV group (fp32, g order)."""
    s = _f32(scores)
    Hq, T = s.shape
    U = Hq // G
    out = np.empty((U, T), dtype=np.float32)
    _load().orc_group_sum(_p(s, _f32p), U, G, T, _p(out, _f32p))
    return out


def topk_rows(scores, lo: int, hi: int, k: int) -> np.ndarray:
    """Exact top-k of each row within [lo, hi): ascending absolute indices.

    Ties at the k-th value are broken by lower index.
    laprune/llm/modifiers/aq_evaluation.py:185-201.
    """
    s = _f32(scores)
    R, n = s.shape
    assert 0 <= lo <= hi <= n and 0 <= k <= hi - lo
    out = np.empty((R, k), dtype=np.int32)
    if k > 0:
        _load().orc_topk_rows(_p(s, _f32p), R, n, lo, hi, k, _p(out, _i32p))
    return out


def num_keep(num_candidate: int, mask_out: float = 0.98, min_remain: int = 20) -> int:
    """Top-k size of the reference decode hook (aq_evaluation.py:193-197)."""
    if num_candidate <= 0:
        return 0
    keep = num_candidate - int(num_candidate * mask_out)
    keep = max(min(num_candidate, min_remain), keep)
    return max(1, min(keep, num_candidate))


def candidate_window(T_codes: int, T_total: int, sink: int, local: int):
    """[cand_start, cand_end) of aq_evaluation.py:189-193."""
    sink_end = min(sink, T_codes) if sink > 0 else 0
    local_start = max(T_total - max(local, 0), 0)
    cand_end = min(T_codes, local_start) if local > 0 else T_codes
    return sink_end, max(sink_end, cand_end)


def keep_positions(topk_idx, T_total: int, sink: int, local: int) -> np.ndarray:
    """Union of top-k, sink [0,sink) and local window [T-local, T), sorted.

    The set the reference attends to (aq_evaluation.py:210-237); the
    implicit-tail form of :220-222 yields the same set when sink == 0.
    """
    topk_idx = np.asarray(topk_idx)
    R = topk_idx.shape[0]
    sb = min(sink, T_total) if sink > 0 else 0
    start = max(T_total - local, 0) if local > 0 else T_total
    if start <= 0:
        sb = 0
    elif start < sb:
        start = sb
    extra = np.concatenate([np.arange(sb), np.arange(start, T_total)]).astype(np.int32)
    out = [np.unique(np.concatenate([topk_idx[r].astype(np.int32), extra])) for r in range(R)]
    n = max(len(o) for o in out)
    assert all(len(o) == n for o in out)
    return np.stack(out).astype(np.int32)


def encode_greedy(x, codebooks, cb_index=None) -> np.ndarray:
    """Greedy AQ codes (uint8 [N,M]) of fp32 vectors.  quantizer.py:346-355.
    ``d`` must be a multiple of 32 (the fixed 32-lane order of r . c).

    ``codebooks`` is ``[M,K,d]`` or a stack ``[S,M,K,d]`` addressed per vector
    by ``cb_index`` (int32 ``[N]``).
    """
    x = _f32(x)
    cb = _f32(codebooks)
    N, d = x.shape
    M, K = cb.shape[-3], cb.shape[-2]
    out = np.empty((N, M), dtype=np.uint8)
    if N == 0:
        return out
    if d % 32:
        raise ValueError(f"encode_greedy: d={d} is not a multiple of 32")
    idxp = None
    if cb_index is not None:
        cbi = np.ascontiguousarray(np.asarray(cb_index, dtype=np.int32))
        idxp = _p(cbi, _i32p)
    _load().orc_encode_greedy(_p(x, _f32p), _p(cb, _f32p), idxp, N, M, K, d,
                              out.ctypes.data_as(_u8p))
    return out


def encode_icm(x, codebooks, icm_iters: int, cb_index=None, return_sweeps: bool = False):
    """Greedy codes refined by up to ``icm_iters`` ICM sweeps (uint8 [N,M]).
    quantizer.py:346-370: after the greedy pass, each sweep re-chooses code m
    = 0..M-1 of every vector against the reconstruction without it, and a
    sweep that changes no code of the batch ends the refinement.  The batch
    is the set of vectors sharing a codebook set (the reference runs one
    quantizer per codebook group).  With ``return_sweeps`` also the number
    of sweeps each set ran."""
    x = _f32(x)
    cb = _f32(codebooks)
    codes = encode_greedy(x, cb, cb_index)
    N, d = x.shape
    M, K = cb.shape[-3], cb.shape[-2]
    cbi = None
    idxp = None
    if cb_index is not None:
        cbi = np.ascontiguousarray(np.asarray(cb_index, dtype=np.int32))
        idxp = _p(cbi, _i32p)
    nsets = int(cbi.max()) + 1 if cbi is not None and cbi.size else 1
    sweeps = np.zeros(nsets, dtype=np.int32)
    if N and icm_iters > 0:
        _load().orc_encode_icm(_p(x, _f32p), _p(cb, _f32p), idxp, N, M, K, d, int(icm_iters),
                               codes.ctypes.data_as(_u8p), _p(sweeps, _i32p))
    return (codes, sweeps) if return_sweeps else codes


def encode_stage_dists(x_row, codebooks, prefix_codes, m: int) -> np.ndarray:
    """fp64 ||r - C_m[k]||^2 at stage m after the given code prefix."""
    x = _f32(x_row).reshape(-1)
    cb = _f32(codebooks)
    M, K, d = cb.shape
    pre = np.ascontiguousarray(np.asarray(prefix_codes, dtype=np.uint8))
    out = np.empty((K,), dtype=np.float64)
    _load().orc_encode_stage_dists(_p(x, _f32p), _p(cb, _f32p), pre.ctypes.data_as(_u8p),
                                   m, K, d, _p(out, _f64p))
    return out


def _gather_rows(src, head: int, rows) -> np.ndarray:
    """fp32 copy of src[head][rows] for a numpy array or a (CPU) torch tensor."""
    if hasattr(src, "float") and hasattr(src, "numpy"):  # torch tensor, any float dtype
        import torch
        return src[head][torch.from_numpy(np.asarray(rows, dtype=np.int64))].float().numpy()
    return np.asarray(src[head][rows], dtype=np.float32)


def sparse_attention(q, keys, vals, idx, G: int, scale: float | None = None) -> np.ndarray:
    """fp32 softmax(q K[idx]^T * scale) V[idx] per query head.

    aq_evaluation.py:239-253 (gather + SDPA without mask, one query row).
    q [H,D]; keys/vals [Hkv,T,D] (any float dtype, converted per gathered
    row); idx [H,n] absolute positions of the KV head h//G.
    """
    q = _f32(q)
    H, D = q.shape
    idx = np.ascontiguousarray(np.asarray(idx, dtype=np.int32))
    n = idx.shape[1]
    if scale is None:
        scale = 1.0 / float(np.sqrt(D))
    # Gather the used rows only (the full cache may be large) in fp32.
    kg = np.empty((H, n, D), dtype=np.float32)
    vg = np.empty((H, n, D), dtype=np.float32)
    for h in range(H):
        kg[h] = _gather_rows(keys, h // G, idx[h])
        vg[h] = _gather_rows(vals, h // G, idx[h])
    local = np.broadcast_to(np.arange(n, dtype=np.int32), (H, n)).copy()
    out = np.empty((H, D), dtype=np.float32)
    _load().orc_sparse_attention(_p(q, _f32p), _p(kg, _f32p), _p(vg, _f32p),
                                 n * D, D, _p(local, _i32p), H, 1, n, D,
                                 float(scale), _p(out, _f32p))
    return out


# ---------------------------------------------------------------------------
# fp16 arithmetic of the reference CUDA extension (aq_kernels/*.cu)
# ---------------------------------------------------------------------------

def _codes_u8_index(codes) -> np.ndarray:
    """Code bytes read as unsigned 8-bit indices (aq_lut.cu:29-35)."""
    c = np.asarray(codes)
    return (c.astype(np.int64) & 0xFF).astype(np.int64)


def lut_gather_grouped_f16(lut_f16, codes, G: int) -> np.ndarray:
    """fp16 out[h][t] = half(sum_m float(lut[h][m][code])), m in order.

    aq_kernels/aq_lut_gqa.cu:111-149 (and the bit-identical interleaved
    variant :157-212).
    """
    lut32 = np.asarray(lut_f16, dtype=np.float16).astype(np.float32)
    s = score_gqa(lut32, np.asarray(codes), G)
    return s.astype(np.float16)


def lut_gather_gqa_f16(lut_f16, codes, G: int, M_start: int, M_end: int, indices=None) -> np.ndarray:
    """aq_kernels/aq_lut_gqa.cu:20-76: per-head score over m in [M_start, M_end),
    dense or over an index list (indices out of [0,T) give 0)."""
    lut32 = np.asarray(lut_f16, dtype=np.float16).astype(np.float32)
    codes = np.asarray(codes)
    H = lut32.shape[0]
    Hkv, T, _ = codes.shape
    sub = np.ascontiguousarray(lut32[:, M_start:M_end, :])
    csub = codes[:, :, M_start:M_end]
    if indices is None:
        return score_gqa(sub, np.ascontiguousarray(csub), G).astype(np.float16)
    idx = np.asarray(indices).astype(np.int64)
    N = idx.shape[1]
    out = np.zeros((H, N), dtype=np.float32)
    for h in range(H):
        valid = (idx[h] >= 0) & (idx[h] < T)
        rows = csub[h // G][idx[h][valid]].astype(np.int64)  # [n, Mr]
        acc = np.zeros(rows.shape[0], dtype=np.float32)
        for m in range(rows.shape[1]):
            acc = (acc + sub[h, m][rows[:, m]]).astype(np.float32)
        out[h][valid] = acc
    return out.astype(np.float16)


def lut_gather_forward(lut, codes) -> np.ndarray:
    """aq_kernels/aq_lut.cu:581-639: scores[q][n] = sum_{m<min(M,32)} lut[q][m*K +
    clamp(code)] with fp32 (fp16 lut: fp32 accumulate, fp16 result)."""
    lut = np.asarray(lut)
    is_half = lut.dtype == np.float16
    l32 = lut.astype(np.float32)
    c = _codes_u8_index(codes)
    Q, N, M = c.shape
    K = l32.shape[1] // M
    c = np.clip(c, 0, K - 1)
    acc = np.zeros((Q, N), dtype=np.float32)
    for m in range(min(M, 32)):
        acc = (acc + np.take_along_axis(l32, m * K + c[:, :, m], axis=1)).astype(np.float32)
    return acc.astype(np.float16) if is_half else acc


def lut_forward(q, codebooks, codes) -> np.ndarray:
    """aq_kernels/aq_lut.cu:37-149: per token, sum over m of dot(q, C_m[code]).

    fp16: acc(fp32) += float(h.x) + float(h.y) with h = hmul2(q2, c2) rounded
    to fp16 per product pair; fp32/fp64: sequential scalar accumulation.
    Codes outside [0,K) contribute nothing.
    """
    q = np.asarray(q)
    cb = np.asarray(codebooks)
    c = _codes_u8_index(codes)
    Q, N, M = c.shape
    _, K, d = cb.shape
    out = np.zeros((Q, N), dtype=np.float32 if q.dtype == np.float16 else q.dtype)
    for qi in range(Q):
        for n in range(N):
            if q.dtype == np.float16:
                acc = np.float32(0)
                for m in range(M):
                    k = c[qi, n, m]
                    if k >= K:
                        continue
                    prod = (q[qi].astype(np.float32) * cb[m, k].astype(np.float32)).astype(np.float16)
                    pr = prod.astype(np.float32).reshape(-1, 2)
                    for a, b in pr:
                        acc = np.float32(acc + np.float32(a + b))
                out[qi, n] = acc
            else:
                acc = q.dtype.type(0)
                for m in range(M):
                    k = c[qi, n, m]
                    if k >= K:
                        continue
                    for i in range(d):
                        acc = q.dtype.type(acc + q[qi, i] * cb[m, k, i])
                out[qi, n] = acc
    return out.astype(np.float16) if q.dtype == np.float16 else out


# ---------------------------------------------------------------------------
# whole-step restatements
# ---------------------------------------------------------------------------

def scores_per_kv_head(C, q, codes, G: int) -> np.ndarray:
    """Per-query-head fp32 scores with one codebook set per KV head.

    The reference has one shared set per layer; the benchmark configs give
    each KV head its own [M,K,d] set, which the reference handles by scoring
    each KV group with its own manager (aq_kv.py:633 per group).
    C [Hkv,M,K,d]; q [Hq,d]; codes uint8 [Hkv,T,M] -> [Hq,T].
    """
    C = np.asarray(C, dtype=np.float32)
    q = np.asarray(q, dtype=np.float32)
    codes = np.asarray(codes)
    Hkv = codes.shape[0]
    out = [score_gqa(lut(q[h * G:(h + 1) * G], C[h]), codes[h:h + 1], G) for h in range(Hkv)]
    return np.concatenate(out, 0)


def decode_step_group(C, q, codes, keys, vals, k: int, sink: int, local: int, G: int):
    """Sparse decode step with per-KV-head selection on GQA-summed scores.

    Returns (group scores [Hkv,T], top-k [Hkv,k] ascending, keep [Hkv,N],
    attention output fp32 [Hq,D]).
    """
    s = scores_per_kv_head(C, q, codes, G)
    gs = group_sum(s, G)
    T = gs.shape[1]
    lo, hi = candidate_window(T, T, sink, local)
    top = topk_rows(gs, lo, hi, k)
    keep = keep_positions(top, T, sink, local)
    idx_q = np.repeat(keep, G, axis=0)
    out = sparse_attention(np.asarray(q, dtype=np.float32), keys, vals, idx_q, G)
    return gs, top, keep, out


def decode_hook_reference(cb, q, codes, keys, vals, T_total: int, sink: int, local: int,
                          mask_out: float = 0.98, min_remain: int = 20):
    """The reference decode hook (aq_evaluation.py:146-253) for fp32 K/V with a
    shared [M,K,d] codebook: per-query-head scores, per-query-head top-k with
    the mask_out/min_remain size, union with sink and local window, SDPA.
    q [B,Hq,1,D]; codes [B,Hkv,cap,M]; keys/vals [B,Hkv,T,D] -> [B,1,Hq*D].
    """
    q = np.asarray(q, dtype=np.float32)
    B, Hq, _, D = q.shape
    Hkv = codes.shape[1]
    G = Hq // Hkv
    outs = []
    for b in range(B):
        L = lut(q[b, :, 0, :], cb)
        s = score_gqa(L, np.asarray(codes[b, :, :T_total]), G)
        lo, hi = candidate_window(T_total, T_total, sink, local)
        kk = num_keep(hi - lo, mask_out, min_remain)
        top = topk_rows(s, lo, hi, kk)
        keep = keep_positions(top, T_total, sink, local)
        o = sparse_attention(q[b, :, 0, :], np.asarray(keys[b]), np.asarray(vals[b]), keep, G)
        outs.append(o.reshape(1, Hq * D))
    return np.stack(outs)


def topk_overlap(sel, ref, scores, kth, tol: float = 0.0) -> float:
    """Tie-aware overlap of a selected index set with a reference top-k set.

    An index of ``sel`` matches when it is in ``ref`` or its (reference)
    score is within ``tol`` of the k-th value (a tie at the threshold).
    """
    sel = np.asarray(sel).reshape(-1)
    ref_set = set(np.asarray(ref).reshape(-1).tolist())
    hits = 0
    for i in sel.tolist():
        if i in ref_set or abs(float(scores[i]) - float(kth)) <= tol:
            hits += 1
    return hits / max(1, len(sel))
