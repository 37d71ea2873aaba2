"""Drop-in for the reference's ``aq_kernels`` package (aq_kernels/__init__.py:1-23).

Same names, argument order, defaults and output shapes/dtypes as the
reference's pybind entry points (aq_kernels/aq_lut.cu:741-745,
aq_kernels/aq_lut_gqa.cu:670-691, aq_kernels/fused_linear_encode.cu:237-242);
bad arguments raise RuntimeError with the reference's check messages.
Outputs are newly allocated torch tensors, inputs are borrowed, launches go
on the current torch stream.  Every op runs the laprune_b200 CUDA library
(there is no CPU fallback); the reference's convention of setting a name to
``None`` when its extension is missing is kept: all names are bound when the
library loads, and importing this module raises if it does not.

Differences, by design:
  * tokens whose index lies outside [0, T) give zero K/V rows in
    gqa_gather_kv(_with_tail) (the reference leaves those rows unwritten);
  * fused_linear_encode_forward computes the exact fp32 greedy codes of the
    reference's CPU path (quantizer.py:346-355) from ``codebooks``;
    ``weight_t`` and ``bias`` (the fp16 transposed codebooks and -||C||^2/2
    the reference's GPU kernel reads) are checked for shape only.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch

from . import _lib
from .ops import _stream_handle, encode_keys

_lib.load()  # raises ImportError when the CUDA library is not built

__all__ = ["aq_lut_forward", "aq_lut_gather_forward", "aq_lut_gather_gqa", "aq_lut_gather_grouped",
           "gqa_gather_kv", "gqa_gather_kv_with_tail", "fused_linear_encode_forward"]


_lut_gather = _lib.load().lp_lut_gather
_lut_build = _lib.load().lp_lut_build
_gqa_gather = _lib.load().lp_gqa_gather_kv
_LutGatherArgs, _LutBuildArgs, _GqaGatherArgs = _lib.LutGatherArgs, _lib.LutBuildArgs, _lib.GqaGatherArgs

_DT = {torch.float16: _lib.LP_F16, torch.float32: _lib.LP_F32, torch.bfloat16: _lib.LP_BF16}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _codes_u8(codes: torch.Tensor) -> torch.Tensor:
    """Code values read as unsigned bytes (aq_lut.cu:29-35)."""
    _check(codes.dtype in (torch.int64, torch.uint8, torch.int8),
           "codes must be int64 (Long) or uint8 (Byte) or int8 (Char)")
    if codes.dtype == torch.uint8:
        return codes.contiguous()
    return (codes.to(torch.int64) & 0xFF).to(torch.uint8).contiguous()


def _gather(lut3: torch.Tensor, codes: torch.Tensor, G: int, m0: int, m1: int, indices: Optional[torch.Tensor],
            out_dtype: torch.dtype, code_mode: int, T: int) -> torch.Tensor:
    Q, M_stride, K = lut3.shape
    N = T if indices is None else indices.shape[1]
    out = torch.empty((Q, N), dtype=out_dtype, device=lut3.device)
    a = _LutGatherArgs()
    a.lut = lut3.data_ptr()
    a.lut_dtype = _DT[lut3.dtype]
    a.code_mode = code_mode
    a.lut_stride_q = lut3.stride(0)
    a.M_stride, a.K, a.m0, a.m1 = M_stride, K, m0, m1
    a.codes = codes.data_ptr()
    a.codes_stride_h, a.codes_stride_t = codes.stride(0), codes.stride(1)
    a.Q, a.G, a.T, a.N = Q, G, T, N
    if indices is not None:
        a.indices = indices.data_ptr()
        a.indices_stride_q = indices.stride(0)
    a.out = out.data_ptr()
    a.out_dtype = _DT[out_dtype]
    a.out_stride_q = out.stride(0)
    with torch.cuda.device(lut3.device):
        _lib.check(_lut_gather(ctypes.byref(a), _stream_handle(lut3.device)))
    return out


def aq_lut_forward(q: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
    """scores[q][n] = sum_m q_q . C_m[codes[q][n][m]] (aq_kernels/aq_lut.cu:445-574).

    q [Q,d] and codebooks [M,K,d] of one dtype (fp16/bf16/fp32), codes
    [Q,N,M]; result [Q,N] in q's dtype (fp32 table and sums inside)."""
    _check(q.is_cuda, "q must be a CUDA tensor")
    _check(codebooks.is_cuda, "codebooks must be a CUDA tensor")
    _check(codes.is_cuda, "codes must be a CUDA tensor")
    _check(q.dim() == 2, "q must be of shape [Q, d]")
    _check(codebooks.dim() == 3, "codebooks must be of shape [M, K, d]")
    _check(codes.dim() == 3, "codes must be of shape [Q, N, M]")
    _check(q.dtype == codebooks.dtype, "q and codebooks must have the same dtype")
    _check(q.dtype in _DT, "q must be fp16, bf16 or fp32")
    Q, d = q.shape
    M, K, _ = codebooks.shape
    c = _codes_u8(codes)
    lut = torch.empty((Q, M, K), dtype=torch.float32, device=q.device)
    b = _LutBuildArgs()
    qc = q.contiguous()
    cb = codebooks.float().contiguous()
    b.q, b.q_dtype, b.q_stride = qc.data_ptr(), _DT[qc.dtype], qc.stride(0)
    b.codebooks, b.Q, b.M, b.K, b.D, b.lut = cb.data_ptr(), Q, M, K, d, lut.data_ptr()
    with torch.cuda.device(q.device):
        _lib.check(_lut_build(ctypes.byref(b), _stream_handle(q.device)))
    # per-query codes: one codes "head" per row (G = 1); codes >= K add nothing
    return _gather(lut, c, 1, 0, M, None, q.dtype if q.dtype != torch.bfloat16 else torch.float32, 1,
                   c.shape[1]).to(q.dtype)


def aq_lut_gather_forward(lut: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
    """scores[q][n] = sum_{m<min(M,32)} lut[q][m*K + clamp(code)] (aq_kernels/aq_lut.cu:641-738)."""
    _check(lut.is_cuda, "lut must be a CUDA tensor")
    _check(codes.is_cuda, "codes must be a CUDA tensor")
    _check(lut.dim() == 2, "lut must be of shape [Q, M*K]")
    _check(codes.dim() == 3, "codes must be of shape [Q, N, M]")
    _check(lut.dtype in (torch.float16, torch.float32), "lut must be fp16 or fp32")
    c = _codes_u8(codes)
    Q, N, M = c.shape
    _check(lut.shape[1] % M == 0, "lut width must be M*K")
    K = lut.shape[1] // M
    l3 = lut.contiguous().view(Q, M, K)
    return _gather(l3, c, 1, 0, min(M, 32), None, lut.dtype, 0, N)


def aq_lut_gather_gqa(lut: torch.Tensor, codes: torch.Tensor, G: int, M_start: int, M_end: int,
                      indices: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GQA-aware LUT gather over codebooks [M_start, M_end), dense or over an
    index list (aq_kernels/aq_lut_gqa.cu:350-422); fp16 out, 0 for indices
    outside [0,T)."""
    _check(lut.is_cuda and codes.is_cuda, "tensors must be on CUDA")
    _check(lut.dtype == torch.float16, "lut must be fp16")
    _check(codes.dtype == torch.uint8, "codes must be uint8")
    _check(lut.dim() == 3 and codes.dim() == 3, "lut and codes must be 3-D")
    _check(codes.stride(2) == 1, "codes last (M) dimension must be contiguous")
    H, M_stride, K = lut.shape
    Hkv, T, _ = codes.shape
    _check(H == Hkv * G, "H must equal Hkv * G")
    _check(M_end <= M_stride and M_start >= 0 and M_end - M_start > 0, "invalid M range")
    idx = None
    if indices is not None:
        _check(indices.size(0) == H, "indices must have one row per head")
        idx = indices.to(torch.int64).contiguous()
    return _gather(lut.contiguous(), codes, G, M_start, M_end, idx, torch.float16, 0, T)


def aq_lut_gather_grouped(lut: torch.Tensor, codes: torch.Tensor, G: int, grid_y_cap: int = 48) -> torch.Tensor:
    """GQA-grouped dense scan: [H,T] fp16 (aq_kernels/aq_lut_gqa.cu:460-534)."""
    _check(lut.is_cuda and codes.is_cuda, "tensors must be CUDA")
    _check(lut.dtype == torch.float16 and codes.dtype == torch.uint8, "lut must be fp16 and codes uint8")
    _check(lut.dim() == 3 and codes.dim() == 3, "lut and codes must be 3-D")
    _check(codes.stride(2) == 1, "codes M dimension must be contiguous")
    H, M, K = lut.shape
    Hkv, T, _ = codes.shape
    _check(H == Hkv * G, "H must equal Hkv*G")
    _check(0 < G <= 4, "grouped kernel supports G<=4")
    _check(grid_y_cap > 0, "grid_y_cap must be positive")
    return _gather(lut.contiguous(), codes, G, 0, M, None, torch.float16, 0, T)


def _gqa(keys, vals, indices, G, tail_start, tail_count) -> List[torch.Tensor]:
    _check(keys.is_cuda and vals.is_cuda and indices.is_cuda, "keys, vals and indices must be CUDA tensors")
    _check(keys.dtype in (torch.float16, torch.bfloat16) and vals.dtype == keys.dtype, "K/V must be fp16 or bf16")
    _check(indices.dtype == torch.int64, "indices must be int64")
    _check(keys.dim() == 4 and vals.dim() == 4 and indices.dim() == 3,
           "expected K/V [B,Hkv,T,D] and indices [B,Hq,N]")
    _check(keys.shape == vals.shape, "K/V shapes must match")
    _check(keys.stride(3) == 1 and vals.stride(3) == 1, "K/V head dimension must be contiguous")
    B, Hkv, T, D = keys.shape
    Hq, Ne = indices.shape[1], indices.shape[2]
    _check(indices.shape[0] == B, "indices batch mismatch")
    _check(Hq == Hkv * G, "Hq must equal Hkv * G")
    _check(tail_count >= 0 and tail_start >= 0 and tail_start + tail_count <= T, "invalid implicit tail range")
    N = Ne + tail_count
    out_k = torch.empty((B, Hq, N, D), dtype=keys.dtype, device=keys.device)
    out_v = torch.empty((B, Hq, N, D), dtype=vals.dtype, device=vals.device)
    idx = indices.contiguous()
    a = _GqaGatherArgs()
    a.keys, a.vals, a.kv_dtype = keys.data_ptr(), vals.data_ptr(), _DT[keys.dtype]
    a.k_stride_b, a.k_stride_h, a.k_stride_t = keys.stride(0), keys.stride(1), keys.stride(2)
    a.v_stride_b, a.v_stride_h, a.v_stride_t = vals.stride(0), vals.stride(1), vals.stride(2)
    a.indices, a.indices_stride_b, a.indices_stride_h = idx.data_ptr(), idx.stride(0), idx.stride(1)
    a.B, a.Hkv, a.G, a.T, a.D = B, Hkv, G, T, D
    a.N_explicit, a.tail_start, a.tail_count = Ne, tail_start, tail_count
    a.out_k, a.out_v = out_k.data_ptr(), out_v.data_ptr()
    with torch.cuda.device(keys.device):
        _lib.check(_gqa_gather(ctypes.byref(a), _stream_handle(keys.device)))
    return [out_k, out_v]


def gqa_gather_kv(keys: torch.Tensor, vals: torch.Tensor, indices: torch.Tensor, G: int,
                  threads: int = 256, vector_width: int = 8) -> List[torch.Tensor]:
    """[K, V] gathered per query head: [B,Hq,N,D] (aq_kernels/aq_lut_gqa.cu:536-598)."""
    _check(vector_width in (2, 8), "vector_width must be 2 or 8 half elements")
    _check(threads in (256, 512, 1024), "threads must be 256/512/1024")
    return _gqa(keys, vals, indices, G, 0, 0)


def gqa_gather_kv_with_tail(keys: torch.Tensor, vals: torch.Tensor, indices: torch.Tensor, G: int,
                            tail_start: int, tail_count: int, threads: int = 256,
                            vector_width: int = 8) -> List[torch.Tensor]:
    """As gqa_gather_kv, then tail_count rows tail_start.. appended
    (aq_kernels/aq_lut_gqa.cu:600-664)."""
    _check(vector_width in (2, 8), "vector_width must be 2 or 8 half elements")
    _check(threads in (256, 512, 1024), "threads must be 256/512/1024")
    return _gqa(keys, vals, indices, G, tail_start, tail_count)


def fused_linear_encode_forward(x: torch.Tensor, weight_t: torch.Tensor, bias: torch.Tensor,
                                codebooks: torch.Tensor, fp32_residual: bool = True,
                                tile_n: int = 0) -> torch.Tensor:
    """Greedy residual codes uint8 [N,M] of x [N,d] (aq_kernels/fused_linear_encode.cu:168-234)."""
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(x.dim() == 2, "x must be [N, d]")
    N, d = x.shape
    M, K = weight_t.shape[0], weight_t.shape[2]
    _check(tuple(weight_t.shape) == (M, d, K), "weight_t must be [M, d, K]")
    _check(tuple(bias.shape) == (M, K), "bias must be [M, K]")
    _check(tuple(codebooks.shape) == (M, K, d), "codebooks must be [M, K, d]")
    xx = x if x.dtype in (torch.float16, torch.bfloat16, torch.float32) else x.float()
    return encode_keys(xx.contiguous(), codebooks.float().contiguous())
