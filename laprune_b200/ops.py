"""Torch-facing wrappers of the fused sparse-decode hot path.

These functions take CUDA tensors, allocate outputs, and call the C ABI of
``include/laprune_b200.h`` on the current CUDA stream.  They never fall back
to a CPU or PyTorch implementation: a non-CUDA input or a missing library is
an error.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import SparseDecodeArgs

_DTYPE = {torch.float32: _lib.LP_F32, torch.float16: _lib.LP_F16, torch.bfloat16: _lib.LP_BF16}

_ws_lock = threading.Lock()
_ws_cache: dict = {}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device: torch.device) -> int:
    """The current torch stream of ``device`` as a raw handle (the same value
    as ``torch.cuda.current_stream(device).cuda_stream``, read without
    creating a Stream object when torch offers that)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


class _OnDevice:
    """``torch.cuda.device(dev)`` only when ``dev`` is not current already
    (entering the guard costs a few microseconds per call)."""
    __slots__ = ("dev", "guard")

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.guard = None

    def __enter__(self):
        if self.dev.index is not None and self.dev.index != torch.cuda.current_device():
            self.guard = torch.cuda.device(self.dev)
            self.guard.__enter__()
        return self

    def __exit__(self, *exc):
        if self.guard is not None:
            self.guard.__exit__(*exc)
        return False


# Filled argument structs of recent sparse_decode calls, keyed by everything
# but the token counts: a decode loop calls with the same buffers every token,
# so the validation and the struct filling run once per buffer set.  A hit
# hands out a copy (callers on several threads never share one), whose
# T_codes / T_total are then checked and set.
_args_cache: dict = {}
_ARGS_CACHE_MAX = 1024


def _tensor_key(t: Optional[torch.Tensor]):
    if t is None:
        return None
    return (t.data_ptr(), t.dtype, tuple(t.shape), t.stride(), t.device.index, t.is_cuda)


def workspace(nbytes: int, device: torch.device, tag: str = "decode") -> torch.Tensor:
    """A cached, zero-initialised device workspace of at least ``nbytes``.

    One workspace per (device, tag, stream); calls sharing it must be
    stream-ordered (the default for calls issued from one stream).
    """
    dev = torch.device(device)
    key = (dev.index, tag, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
            _ws_cache[key] = ws
        return ws


@dataclass
class SparseDecodeResult:
    out: Optional[torch.Tensor]
    topk: Optional[torch.Tensor]
    head_scores: Optional[torch.Tensor]


def _window(T_codes: int, T_total: int, sink: int, local: int):
    sink_end = min(sink, T_codes) if sink > 0 else 0
    local_start = max(T_total - max(local, 0), 0)
    cand_end = min(T_codes, local_start) if local > 0 else T_codes
    return sink_end, max(sink_end, cand_end)


def num_candidates(T_codes: int, T_total: int, sink: int, local: int) -> int:
    lo, hi = _window(T_codes, T_total, sink, local)
    return hi - lo


def prefetch_regions(codebooks: torch.Tensor, codes: torch.Tensor, T_codes: Optional[int] = None):
    """L2-prefetch regions covering one layer's LUT inputs: its codebooks
    and the valid [0, T_codes) rows of every (batch, KV head) of its code
    cache.  Pass them as ``prefetch`` of the PREVIOUS call so they are
    fetched while that call's selection/attention stages leave HBM idle."""
    c = codes if codes.dim() == 4 else codes.unsqueeze(0)
    T = c.shape[2] if T_codes is None else int(T_codes)
    regs = [(codebooks.data_ptr(), codebooks.numel() * codebooks.element_size(), 1, 0)]
    if c.stride(0) == c.shape[1] * c.stride(1):
        regs.append((c.data_ptr(), T * c.stride(2), c.shape[0] * c.shape[1], c.stride(1)))
    return regs


def build_args(q, codebooks, codes, keys=None, vals=None, *, topk: int, T_codes=None, T_total=None,
               sink: int = 4, local: int = 64, select: str = "kv_group", scale=None,
               out=None, head_scores=None, topk_out=None, prefetch=None) -> SparseDecodeArgs:
    """Validate tensors and fill the C argument struct (no launch)."""
    if q.dim() == 2:
        q = q.unsqueeze(0)
    if codes.dim() == 3:
        codes = codes.unsqueeze(0)
    if keys is not None and keys.dim() == 3:
        keys = keys.unsqueeze(0)
    if vals is not None and vals.dim() == 3:
        vals = vals.unsqueeze(0)
    for name, t in (("q", q), ("codebooks", codebooks), ("codes", codes), ("keys", keys), ("vals", vals)):
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    B, Hq, D = q.shape
    _, Hkv, cap, M = codes.shape
    if codes.dtype != torch.uint8:
        raise RuntimeError("codes must be uint8")
    if Hq % Hkv != 0:
        raise RuntimeError(f"Invalid GQA score heads: Hq={Hq}, Hkv={Hkv}")
    G = Hq // Hkv
    if codebooks.dtype not in (torch.float32, torch.float16, torch.bfloat16) or not codebooks.is_contiguous():
        raise RuntimeError("codebooks must be contiguous fp32 / fp16 / bf16 [Hkv,M,K,D] or [M,K,D]")
    per_kv = codebooks.dim() == 4
    if per_kv and codebooks.shape[0] != Hkv:
        raise RuntimeError("per-KV-head codebooks must have Hkv sets")
    Mc, K, Dc = codebooks.shape[-3:]
    if Mc != M or Dc != D:
        raise RuntimeError(f"AQ shape mismatch: codebook={tuple(codebooks.shape)}, q={tuple(q.shape)}, codes={tuple(codes.shape)}")
    if q.stride(-1) != 1 or codes.stride(-1) != 1:
        raise RuntimeError("q and codes must be contiguous in their last dimension")
    T_codes = cap if T_codes is None else int(T_codes)
    T_total = (keys.shape[2] if keys is not None else T_codes) if T_total is None else int(T_total)
    if not 0 <= T_codes <= cap:
        raise RuntimeError(f"T_codes={T_codes} exceeds the code cache capacity {cap}")
    if keys is not None and (T_total > keys.shape[2] or T_total > vals.shape[2]):
        raise RuntimeError(f"T_total={T_total} exceeds the K/V cache capacity {keys.shape[2]}")
    if keys is not None and (keys.shape[:2] != (B, Hkv) or vals.shape != keys.shape or keys.shape[3] != D):
        raise RuntimeError("expected K/V [B,Hkv,T,D] matching q and codes")
    a = SparseDecodeArgs()
    a.q = q.data_ptr()
    a.q_dtype = _DTYPE[q.dtype]
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
    a.codebooks = codebooks.data_ptr()
    a.cb_per_kv_head = int(per_kv)
    a.cb_dtype = _DTYPE[codebooks.dtype]
    a.codes = codes.data_ptr()
    a.codes_stride_b, a.codes_stride_h, a.codes_stride_t = codes.stride(0), codes.stride(1), codes.stride(2)
    if keys is not None:
        if keys.dtype not in (torch.bfloat16, torch.float16) or vals.dtype != keys.dtype:
            raise RuntimeError("keys/vals must both be bf16 or both fp16")
        if keys.stride(-1) != 1 or vals.stride(-1) != 1:
            raise RuntimeError("K/V head dimension must be contiguous")
        a.keys, a.vals = keys.data_ptr(), vals.data_ptr()
        a.kv_dtype = _DTYPE[keys.dtype]
        a.k_stride_b, a.k_stride_h, a.k_stride_t = keys.stride(0), keys.stride(1), keys.stride(2)
        a.v_stride_b, a.v_stride_h, a.v_stride_t = vals.stride(0), vals.stride(1), vals.stride(2)
    a.B, a.Hkv, a.G, a.D, a.M, a.K = B, Hkv, G, D, M, K
    a.T_codes, a.T_total, a.sink, a.local = T_codes, T_total, int(sink), int(local)
    a.topk = int(topk)
    if select not in ("kv_group", "query_head"):
        raise RuntimeError("select must be 'kv_group' or 'query_head'")
    a.select_mode = _lib.LP_SELECT_KV_GROUP if select == "kv_group" else _lib.LP_SELECT_QUERY_HEAD
    a.scale = float(scale) if scale is not None else 0.0
    if out is not None:
        if out.dim() == 2:
            out = out.unsqueeze(0)
        a.out = out.data_ptr()
        a.out_dtype = _DTYPE[out.dtype]
        a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
    if head_scores is not None:
        a.head_scores = head_scores.data_ptr()
    if topk_out is not None:
        a.topk_out = topk_out.data_ptr()
    for i, reg in enumerate((prefetch or [])[:2]):
        ptr, nbytes, count, stride = reg
        a.prefetch_ptr[i] = int(ptr)
        a.prefetch_bytes[i] = int(nbytes)
        a.prefetch_count[i] = int(count)
        a.prefetch_stride[i] = int(stride)
    return a


def sparse_decode(q: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor,
                  keys: Optional[torch.Tensor] = None, vals: Optional[torch.Tensor] = None, *,
                  topk: int, T_codes: Optional[int] = None, T_total: Optional[int] = None,
                  sink: int = 4, local: int = 64, select: str = "kv_group",
                  scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                  out_dtype: Optional[torch.dtype] = None, return_topk: bool = False,
                  return_head_scores: bool = False, attention: bool = True,
                  ws: Optional[torch.Tensor] = None, stage_events=None,
                  fused: Optional[bool] = None, phase_ns: Optional[torch.Tensor] = None,
                  prefetch=None, exchange_select: bool = False) -> SparseDecodeResult:
    """One sparse decode step of one layer (see lp_sparse_decode).

    q [B,Hq,D] (or [Hq,D]); codebooks [Hkv,M,K,D] or [M,K,D] (fp32, or an fp16 / bf16
    copy: half the bytes, tables built in fp32 from its elements); codes uint8
    [B,Hkv,cap,M]; keys/vals [B,Hkv,cap,D] bf16/fp16.  Returns the attention
    output [B,Hq,D] (``out_dtype``, default the K/V dtype), and optionally the
    selected indices ([B*Hkv, topk] or [B*Hq, topk], ascending int32) and the
    fp32 per-query-head scores [B,Hq,T_codes] (candidate window only).

    ``fused=None`` lets the library run the whole step as one cooperative
    kernel when the geometry allows (KV-group selection with attention);
    ``fused=False`` forces the multi-kernel path; ``exchange_select=True``
    makes the fused kernel settle the top-k through its tie exchange instead
    of the union of published candidates (both are exact).  ``phase_ns`` (int64 [8]
    on the device) receives global-timer stamps of the fused kernel phases.
    ``prefetch`` (see :func:`prefetch_regions`) names up to two regions of
    the NEXT call's inputs to pull into L2 during this call's tail.
    """
    squeeze = q.dim() == 2
    q3 = q.unsqueeze(0) if squeeze else q
    B, Hq, D = q3.shape
    Hkv = codes.shape[-3]
    dev = q.device
    T_codes_v = codes.shape[-2] if T_codes is None else int(T_codes)
    o = None
    if attention:
        if keys is None or vals is None:
            raise RuntimeError("keys and vals are required for the attention stage")
        if out is None:
            out = torch.empty((B, Hq, D), dtype=out_dtype or keys.dtype, device=dev)
        o = out
    units = B * Hkv if select == "kv_group" else B * Hq
    tk = torch.empty((units, max(topk, 1)), dtype=torch.int32, device=dev) if return_topk else None
    hs = torch.zeros((B, Hq, T_codes_v), dtype=torch.float32, device=dev) if return_head_scores else None
    key = (_tensor_key(q3), _tensor_key(codebooks), _tensor_key(codes), _tensor_key(keys), _tensor_key(vals),
           _tensor_key(o), _tensor_key(tk), _tensor_key(hs), int(topk), int(sink), int(local), select,
           None if scale is None else float(scale),
           None if prefetch is None else tuple(tuple(int(x) for x in r) for r in prefetch[:2]))
    base = _args_cache.get(key)
    if base is None:
        a = build_args(q3, codebooks, codes, keys, vals, topk=topk, T_codes=T_codes, T_total=T_total,
                       sink=sink, local=local, select=select, scale=scale, out=o, head_scores=hs,
                       topk_out=tk, prefetch=prefetch)
        if len(_args_cache) >= _ARGS_CACHE_MAX:
            _args_cache.clear()
        _args_cache[key] = SparseDecodeArgs.from_buffer_copy(a)
    else:
        # the same buffers as an earlier call: only the token counts change
        a = SparseDecodeArgs.from_buffer_copy(base)
        cap = codes.shape[-2]
        T_codes_i = cap if T_codes is None else int(T_codes)
        # K/V are [B,Hkv,cap,D] or [Hkv,cap,D]: the token axis is the second to last
        T_total_i = (keys.shape[-2] if keys is not None else T_codes_i) if T_total is None else int(T_total)
        if not 0 <= T_codes_i <= cap:
            raise RuntimeError(f"T_codes={T_codes_i} exceeds the code cache capacity {cap}")
        if keys is not None and (T_total_i > keys.shape[-2] or T_total_i > vals.shape[-2]):
            raise RuntimeError(f"T_total={T_total_i} exceeds the K/V cache capacity {keys.shape[-2]}")
        a.T_codes, a.T_total = T_codes_i, T_total_i
    if fused is False:
        a.flags |= _lib.LP_FLAG_NO_FUSED
    if exchange_select:
        a.flags |= _lib.LP_FLAG_EXCHANGE_SELECT
    if phase_ns is not None:
        a.phase_ns = phase_ns.data_ptr()
    ev_arr = None
    if stage_events is not None:
        ev_arr = event_array(stage_events)
        a.stage_events = ctypes.cast(ev_arr, ctypes.c_void_p)
    lib = _lib.load()
    if ws is None:
        # a caller-given workspace is checked against the geometry by the
        # library itself (LP_ERR_WORKSPACE when it is too small)
        need = lib.lp_sparse_decode_workspace_size(ctypes.byref(a))
        if need == 0:
            _lib.check(_lib.LP_ERR_INVALID)
        ws = workspace(need, dev)
    with _OnDevice(dev):
        _lib.check(lib.lp_sparse_decode(ctypes.byref(a), ws.data_ptr(), ws.numel(), _stream_handle(dev)))
    if o is not None and squeeze:
        o = o[0]
    return SparseDecodeResult(out=o, topk=tk[:, :topk] if tk is not None else None, head_scores=hs)


def _encode_args(x: torch.Tensor, codebooks: torch.Tensor, codes: Optional[torch.Tensor], exact: bool):
    """Validate the encoder's tensors and fill lp_encode_args; allocates
    ``codes`` when omitted.  Returns (args, codes)."""
    flat = x.dim() == 2
    x4 = x.view(1, 1, *x.shape) if flat else x
    if x4.dim() != 4:
        raise RuntimeError("x must be [B,H,T,128] or [N,128]")
    if not x4.is_cuda or not codebooks.is_cuda:
        raise RuntimeError("x and codebooks must be CUDA tensors")
    B, H, T, D = x4.shape
    per_head = codebooks.dim() == 4
    if codebooks.dtype != torch.float32 or not codebooks.is_contiguous():
        raise RuntimeError("codebooks must be contiguous fp32")
    if per_head and codebooks.shape[0] != H:
        raise RuntimeError("per-KV-head codebooks need one set per head of x")
    M, K = codebooks.shape[-3], codebooks.shape[-2]
    if codes is None:
        codes = torch.empty((T, M) if flat else (B, H, T, M), dtype=torch.uint8, device=x.device)
    c4 = codes.view(1, 1, *codes.shape) if codes.dim() == 2 else codes
    if c4.dtype != torch.uint8 or tuple(c4.shape) != (B, H, T, M) or c4.stride(3) != 1:
        raise RuntimeError("codes must be uint8 [B,H,T,M] with contiguous rows")
    dt = {torch.bfloat16: _lib.LP_BF16, torch.float16: _lib.LP_F16, torch.float32: _lib.LP_F32}.get(x4.dtype)
    if dt is None:
        raise RuntimeError("x must be bf16, fp16 or fp32")
    if x4.stride(3) != 1:
        raise RuntimeError("x rows must be contiguous")
    a = _lib.EncodeArgs()
    a.x = x4.data_ptr()
    a.x_dtype = dt
    a.cb_per_kv_head = 1 if per_head else 0
    a.x_stride_b, a.x_stride_h, a.x_stride_t = x4.stride(0), x4.stride(1), x4.stride(2)
    a.codebooks = codebooks.data_ptr()
    a.codes = c4.data_ptr()
    a.codes_stride_b, a.codes_stride_h, a.codes_stride_t = c4.stride(0), c4.stride(1), c4.stride(2)
    a.B, a.H, a.T, a.D, a.M, a.K = B, H, T, D, M, K
    a.flags = _lib.LP_ENCODE_FLAG_EXACT if exact else 0
    return a, codes


def encode_rows_per_cta(x: torch.Tensor, codebooks: torch.Tensor) -> int:
    """Vectors per CTA (128, 64, 32 or 16) that :func:`encode_keys` uses for
    these shapes on x's device (a diagnostic; lp_encode_rows_per_cta)."""
    a, _ = _encode_args(x, codebooks, None, False)
    with torch.cuda.device(x.device):
        return int(_lib.load().lp_encode_rows_per_cta(ctypes.byref(a)))


def encode_keys(x: torch.Tensor, codebooks: torch.Tensor, codes: Optional[torch.Tensor] = None, *,
                icm_iters: int = 0, exact: bool = False, ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy residual additive-quantization codes of vectors (lp_encode_keys).

    x: [B,H,T,128] (bf16/fp16/fp32, any strides) or [N,128]; codebooks fp32
    [H,32,256,128] (vector (b,h,t) uses set h) or [32,256,128] (one set).
    ``codes``: optional uint8 [B,H,T,32] destination (e.g. a slice of a code
    cache, rows of 32 contiguous bytes); allocated when omitted.  Returns it.
    Every distance follows the CPU arithmetic exactly (first minimum on
    ties); ``exact=True`` computes all of them on CUDA cores (testing).
    ``icm_iters`` > 0 refines the greedy codes by up to that many ICM sweeps
    (quantizer.py:356-370; the sweeps stop early for the vectors of a
    codebook set once a sweep changes none of their codes).
    """
    a, codes = _encode_args(x, codebooks, codes, exact)
    if int(icm_iters) < 0:
        raise RuntimeError(f"icm_iters must be non-negative, got {icm_iters}")
    a.icm_iters = int(icm_iters)
    lib = _lib.load()
    need = lib.lp_encode_workspace_size(ctypes.byref(a))
    if need == 0:
        _lib.check(_lib.LP_ERR_INVALID)
    if ws is None:
        ws = workspace(need, x.device, tag="encode")
    with torch.cuda.device(x.device):
        _lib.check(lib.lp_encode_keys(ctypes.byref(a), ws.data_ptr(), ws.numel(), _stream_handle(x.device)))
    return codes


def rope_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                k_cache: torch.Tensor, v_cache: torch.Tensor, pos: int,
                q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode token (lp_rope_append): rotary embedding of its query rows
    (returned, or written to ``q_out``) and key rows, the rotated key and the
    value written to slot ``pos`` of the static caches.

    q ``[B, Hq, 1, D]`` or ``[B, Hq, D]``; k / v ``[B, Hkv, 1, D]`` or
    ``[B, Hkv, D]``; cos / sin ``[B, 1, D]`` or ``[B, D]`` (HF rotary rows of
    the token); k_cache / v_cache ``[B, Hkv, cap, D]``.  All of one dtype
    (bf16 or fp16), rows contiguous.  The rotation rounds like HF
    apply_rotary_pos_emb on these dtypes."""
    def rows(t, name):
        if t.dim() == 4:
            if t.shape[2] != 1:
                raise RuntimeError(f"{name}: one token expected, got {tuple(t.shape)}")
            t = t[:, :, 0]
        if t.dim() != 3 or t.stride(-1) != 1:
            raise RuntimeError(f"{name} must be [B, H, D] with contiguous rows")
        return t
    q3, k3, v3 = rows(q, "q"), rows(k, "k"), rows(v, "v")
    c2 = cos.reshape(cos.shape[0], -1) if cos.dim() == 3 else cos
    s2 = sin.reshape(sin.shape[0], -1) if sin.dim() == 3 else sin
    B, Hq, D = q3.shape
    Hkv = k3.shape[1]
    dt = q3.dtype
    for name, t in (("k", k3), ("v", v3), ("cos", c2), ("sin", s2), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != dt or not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor of the query's dtype {dt}")
    if dt not in (torch.bfloat16, torch.float16):
        raise RuntimeError("rope_append takes bf16 or fp16 tensors")
    if k3.shape != (B, Hkv, D) or v3.shape != (B, Hkv, D) or c2.shape != (B, D) or s2.shape != (B, D):
        raise RuntimeError("shape mismatch between q, k, v, cos and sin")
    if k_cache.dim() != 4 or k_cache.shape[:2] != (B, Hkv) or k_cache.shape[3] != D or v_cache.shape != k_cache.shape:
        raise RuntimeError("k_cache / v_cache must be [B, Hkv, cap, D]")
    if not 0 <= int(pos) < k_cache.shape[2]:
        raise RuntimeError(f"pos={pos} outside the cache capacity {k_cache.shape[2]}")
    if c2.stride(-1) != 1 or s2.stride(-1) != 1 or k_cache.stride(-1) != 1 or v_cache.stride(-1) != 1:
        raise RuntimeError("cos, sin and the caches must have contiguous rows")
    out = torch.empty((B, Hq, D), dtype=dt, device=q3.device) if q_out is None else q_out
    o3 = rows(out, "q_out")
    a = _lib.RopeAppendArgs()
    a.q, a.k, a.v = q3.data_ptr(), k3.data_ptr(), v3.data_ptr()
    a.q_stride_b, a.q_stride_h = q3.stride(0), q3.stride(1)
    a.k_stride_b, a.k_stride_h = k3.stride(0), k3.stride(1)
    a.v_stride_b, a.v_stride_h = v3.stride(0), v3.stride(1)
    a.cos, a.sin, a.cos_stride_b, a.sin_stride_b = c2.data_ptr(), s2.data_ptr(), c2.stride(0), s2.stride(0)
    a.q_out, a.q_out_stride_b, a.q_out_stride_h = o3.data_ptr(), o3.stride(0), o3.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.kc_stride_b, a.kc_stride_h, a.kc_stride_t = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
    a.vc_stride_b, a.vc_stride_h, a.vc_stride_t = v_cache.stride(0), v_cache.stride(1), v_cache.stride(2)
    a.dtype = _DTYPE[dt]
    a.B, a.Hq, a.Hkv, a.D, a.pos = B, Hq, Hkv, D, int(pos)
    with torch.cuda.device(q3.device):
        _lib.check(_lib.load().lp_rope_append(ctypes.byref(a), _stream_handle(q3.device)))
    return out


def event_array(events) -> ctypes.Array:
    """ctypes array of raw cudaEvent_t handles of torch.cuda.Event objects
    (each event is created on the current device if it was not yet)."""
    handles = []
    for e in events:
        if e is None:
            handles.append(None)
            continue
        if not e.cuda_event:
            e.record()  # lazily creates the underlying cudaEvent_t
        handles.append(e.cuda_event)
    return (ctypes.c_void_p * len(handles))(*handles)


def device_errors(ws: Optional[torch.Tensor] = None, device=None) -> int:
    """Read and clear the device-side error bits of a workspace."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if ws is None:
        key = (dev.index, "decode", torch.cuda.current_stream(dev).cuda_stream)
        ws = _ws_cache.get(key)
        if ws is None:
            return 0
    bits = ctypes.c_uint32(0)
    _lib.check(_lib.load().lp_read_device_errors(ws.data_ptr(), ws.numel(), _stream_handle(dev),
                                                 ctypes.byref(bits)))
    return int(bits.value)
