"""Seeded synthetic inputs in the shapes of the LAPrune hot-path benchmarks.

Every generator draws from a CPU ``torch.Generator`` seeded with ``seed`` in a
fixed order, so the same tensors come out on any machine with the same torch
version.  The tests, the golden-vector generator and ``bench.py`` all build
their inputs here.

Shapes (Llama-3.1-8B attention geometry): 32 query heads, 8 KV heads (GQA 4),
head_dim 128; M=32 additive codebooks of K=256 entries.
"""
from __future__ import annotations

import torch

HQ, HKV, D, M, K = 32, 8, 128, 32, 256
ROPE_THETA = 500000.0


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def codebooks_per_kv_head(g: torch.Generator, hkv: int = HKV, m: int = M, k: int = K,
                          d: int = D, std: float = 0.05) -> torch.Tensor:
    """fp32 ``[Hkv, M, K, d]`` ~ N(0, std^2)."""
    return torch.randn((hkv, m, k, d), generator=g, dtype=torch.float32) * std


def uniform_codes(g: torch.Generator, shape) -> torch.Tensor:
    return torch.randint(0, 256, tuple(shape), generator=g, dtype=torch.uint8)


def rope(x: torch.Tensor, positions: torch.Tensor, theta: float = ROPE_THETA) -> torch.Tensor:
    """Llama rotary embedding (rotate-half convention, no scaling), fp32.

    ``x`` is ``[..., T, d]`` and ``positions`` is ``[T]``.
    """
    d = x.shape[-1]
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    freqs = positions.float()[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos(), emb.sin()
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat((-x2, x1), dim=-1)
    return x.float() * cos + rot * sin


def config1(seed: int = 0, T: int = 4096) -> dict:
    """Isolated scoring op, batch 1: C, codes [8,T,32], q bf16 [32,128]."""
    g = _gen(seed)
    C = codebooks_per_kv_head(g)
    codes = uniform_codes(g, (HKV, T, M))
    q = torch.randn((HQ, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return {"C": C, "codes": codes, "q": q, "k": 256, "G": HQ // HKV}


def config2(seed: int = 0, B: int = 4, T_new: int = 64, pos0: int = 32000,
            T_cache: int = 32768) -> dict:
    """Key encode of B x 8 x 64 post-RoPE bf16 keys, then scoring of a seeded
    code cache [B,8,T_cache,32] (new codes land at pos0..pos0+T_new-1) with
    q bf16 [B,32,128]."""
    g = _gen(seed)
    C = codebooks_per_kv_head(g)
    raw = torch.randn((B, HKV, T_new, D), generator=g, dtype=torch.float32)
    positions = torch.arange(pos0, pos0 + T_new, dtype=torch.int64)
    keys = rope(raw, positions).to(torch.bfloat16)
    cache = uniform_codes(g, (B, HKV, T_cache, M))
    q = torch.randn((B, HQ, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return {"C": C, "keys": keys, "code_cache": cache, "q": q, "pos0": pos0, "G": HQ // HKV}


def config3(seed: int = 0, T: int = 131072, k: int = 2048, sink: int = 4,
            local: int = 64, kv_dtype=torch.bfloat16) -> dict:
    """Single-layer sparse decode step, batch 1."""
    g = _gen(seed)
    C = codebooks_per_kv_head(g)
    codes = uniform_codes(g, (HKV, T, M))
    keys = torch.randn((HKV, T, D), generator=g, dtype=torch.float32).to(kv_dtype)
    vals = torch.randn((HKV, T, D), generator=g, dtype=torch.float32).to(kv_dtype)
    q = torch.randn((HQ, D), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return {"C": C, "codes": codes, "keys": keys, "vals": vals, "q": q,
            "k": k, "sink": sink, "local": local, "G": HQ // HKV}


def checksum(t: torch.Tensor) -> float:
    """Order-independent float64 checksum used to detect generator drift."""
    return float(t.double().sum().item()) + float((t.double() ** 2).sum().item()) * 1e-3


def small_shared(seed: int = 7) -> dict:
    """Reference single-group layout: one shared [32,256,128] codebook, a
    ragged strided code prefix (T=77 of capacity 128), 8 query / 2 KV heads,
    and 100 fp32 vectors to encode."""
    g = _gen(seed)
    cb = torch.randn((M, K, D), generator=g) * 0.05
    T, cap = 77, 128
    codes_full = torch.randint(0, 256, (2, cap, M), generator=g, dtype=torch.uint8)
    q = torch.randn((8, D), generator=g).to(torch.bfloat16)
    x = torch.randn((100, D), generator=g)
    return {"cb": cb, "codes_full": codes_full, "T": T, "q": q, "x": x, "G": 4}


def decode_hook_case(seed: int = 11) -> dict:
    """fp32 inputs for the reference decode hook: B=2, Hq=8, Hkv=2, T=3000,
    shared codebook, code cache with 128 spare slots."""
    g = _gen(seed)
    B, Hq, Hk, T = 2, 8, 2, 3000
    cb = torch.randn((M, K, D), generator=g) * 0.05
    codes = torch.randint(0, 256, (B, Hk, T + 128, M), generator=g, dtype=torch.uint8)
    keys = torch.randn((B, Hk, T, D), generator=g)
    vals = torch.randn((B, Hk, T, D), generator=g)
    q = torch.randn((B, Hq, 1, D), generator=g)
    return {"cb": cb, "codes": codes, "keys": keys, "vals": vals, "q": q, "T": T,
            "B": B, "Hq": Hq, "Hkv": Hk}
