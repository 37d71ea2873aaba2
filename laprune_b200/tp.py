"""KV-head tensor parallelism for the sparse-decode path.

GPU ``rank`` of ``world`` owns the KV heads ``[rank*Hkv/world,
(rank+1)*Hkv/world)``, the ``G = Hq/Hkv`` query heads of each, and those
heads' code caches, K/V caches and (per-KV-head layout) codebooks.  LUT
build, scoring, top-k, gather and attention are independent per KV head, so
the decode step needs no exchange: every rank runs ``ops.sparse_decode`` on
its own views and produces the attention output of its query heads.  The
reference runs on one device only (its multi-GPU mode is HF
``device_map="auto"`` layer placement, aq_evaluation.py:42-45, with
codebooks replicated per device, aq_kv.py:702-750); this split is the
layout of a tensor-parallel Llama, whose o_proj and MLP all-reduces belong
to the model around this path.

``gather_heads`` reassembles the full ``[B, Hq, D]`` output (an all-gather
over the process group) for callers that want it on every rank.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch

__all__ = ["kv_head_range", "query_head_range", "shard_decode_inputs", "gather_heads",
           "init_process_group"]


def kv_head_range(n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """KV heads ``[h0, h1)`` owned by ``rank``: contiguous, equal blocks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def query_head_range(n_q_heads: int, n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Query heads ``[q0, q1)`` of the KV heads ``rank`` owns (head h serves
    query heads ``[h*G, (h+1)*G)``, the GQA grouping of the reference's
    ``repeat_kv``)."""
    if n_q_heads % n_kv_heads:
        raise ValueError(f"{n_q_heads} query heads are not a multiple of {n_kv_heads} KV heads")
    g = n_q_heads // n_kv_heads
    h0, h1 = kv_head_range(n_kv_heads, world, rank)
    return h0 * g, h1 * g


def _kv_axis(t: torch.Tensor) -> int:
    # [Hkv, T, x] or [B, Hkv, T, x]
    if t.dim() == 3:
        return 0
    if t.dim() == 4:
        return 1
    raise ValueError(f"expected a [Hkv,T,*] or [B,Hkv,T,*] cache, got shape {tuple(t.shape)}")


def shard_decode_inputs(q: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor,
                        keys: Optional[torch.Tensor], vals: Optional[torch.Tensor],
                        world: int, rank: int) -> dict:
    """This rank's views of one layer's decode inputs (no copies).

    q ``[Hq, D]`` or ``[B, Hq, D]``; codebooks ``[Hkv, M, K, D]`` (per KV head,
    sliced) or ``[M, K, D]`` (shared, replicated); codes ``[(B,) Hkv, T, M]``;
    keys / vals ``[(B,) Hkv, T, D]`` or None.  Returns a dict with the same
    keys plus ``kv_heads`` and ``q_heads`` (the owned ranges).
    """
    hkv = codes.shape[_kv_axis(codes)]
    hq = q.shape[-2]
    h0, h1 = kv_head_range(hkv, world, rank)
    q0, q1 = query_head_range(hq, hkv, world, rank)
    out = {"q": q.narrow(q.dim() - 2, q0, q1 - q0),
           "codes": codes.narrow(_kv_axis(codes), h0, h1 - h0),
           "keys": None if keys is None else keys.narrow(_kv_axis(keys), h0, h1 - h0),
           "vals": None if vals is None else vals.narrow(_kv_axis(vals), h0, h1 - h0),
           "kv_heads": (h0, h1), "q_heads": (q0, q1)}
    if codebooks.dim() == 4:
        if codebooks.shape[0] != hkv:
            raise ValueError(f"per-KV-head codebooks {tuple(codebooks.shape)} do not match {hkv} KV heads")
        out["codebooks"] = codebooks.narrow(0, h0, h1 - h0)
    elif codebooks.dim() == 3:
        out["codebooks"] = codebooks
    else:
        raise ValueError(f"codebooks must be [M,K,D] or [Hkv,M,K,D], got {tuple(codebooks.shape)}")
    return out


def gather_heads(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's ``[..., Hq/world, D]`` attention output into
    ``[..., Hq, D]`` (rank order = head order)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts = [torch.empty_like(out_local) for _ in range(world)]
    dist.all_gather(parts, out_local.contiguous(), group=group)
    return torch.cat(parts, dim=out_local.dim() - 2)


def init_process_group(backend: str = "nccl", timeout_s: float = 60.0) -> tuple[int, int, int]:
    """``torch.distributed`` from the launcher's environment (RANK,
    WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT) with a short timeout, so that a
    missing or failed rank ends the others' next collective with an error.
    Returns (world, rank, local_rank); world 1 initialises nothing."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, init_method="env://",
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local
