"""Drop-in for the reference's AQ codebook manager on the decode path.

Mirrors ``AQLayerConfig`` / ``AQLayerCodebookManager`` of
laprune/llm/aq_kv.py:79-699: the on-disk codebook format
(``layer_{L}_group_{G}.pt`` holding ``{"M", "K", "d", "codebooks" [M,K,d]}``,
aq_kv.py:251-342), greedy key encoding (``encode_keys`` /
``encode_keys_batch``, greedy with optional ICM refinement,
aq_kv.py:348-429) and LUT
scoring (``approx_inner_product*``, aq_kv.py:459-699), with every compute
call on this package's sm_100a kernels:

* encoding  -> ``ops.encode_keys`` (tcgen05 contraction + exact refinement;
  codes equal the CPU arithmetic's);
* scoring   -> ``ops.sparse_decode`` with ``attention=False`` (LUT build and
  int32 fixed-point gather-sum; scores within 1e-3 relative of fp32).

Codebooks are held in fp32 on the manager's device whatever ``dtype`` says
(``dtype`` is the dtype of returned scores, as the reference's manager dtype).
There is no CPU fallback: a missing CUDA device or extension raises.
Codebook training is outside the decode path and is not provided.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from . import ops

__all__ = ["AQLayerConfig", "AQLayerCodebookManager", "ShardedAQLayerCodebookManager"]


@dataclass
class AQLayerConfig:
    """One layer's AQ geometry (aq_kv.py:79-93): M sub-codebooks of K entries
    of dimension d; ``heads_per_group`` heads share one codebook."""
    M: int
    K: int
    d: int
    heads_per_group: int = 2
    num_heads: Optional[int] = None


class AQLayerCodebookManager:
    """Per-(layer, head-group) codebooks and LUT scoring (aq_kv.py:96-699)."""

    def __init__(self, layer_cfgs: Dict[int, AQLayerConfig], device: Optional[torch.device] = None,
                 dtype: torch.dtype = torch.float32) -> None:
        self.layer_cfgs = layer_cfgs
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self._cb: Dict[Tuple[int, int], torch.Tensor] = {}
        self._stacks: Dict[Tuple[int, int], torch.Tensor] = {}

    # ---- codebooks -------------------------------------------------------
    def set_codebooks(self, layer_idx: int, group_idx: int, codebooks: torch.Tensor) -> None:
        """Install the ``[M,K,d]`` codebooks of one (layer, group)."""
        if codebooks.dim() != 3:
            raise ValueError(f"codebooks must be [M,K,d], got {tuple(codebooks.shape)}")
        self._cb[(layer_idx, group_idx)] = codebooks.detach().to(device=self.device, dtype=torch.float32).contiguous()
        self._stacks = {k: v for k, v in self._stacks.items() if k[0] != layer_idx}

    def codebooks(self, layer_idx: int, group_idx: int = 0) -> torch.Tensor:
        try:
            return self._cb[(layer_idx, group_idx)]
        except KeyError:
            raise KeyError(f"no codebooks loaded for layer {layer_idx}, group {group_idx}") from None

    def _group(self, layer_idx: int, head_idx: int) -> int:
        # head_idx // heads_per_group; heads_per_group <= 0 means one shared group
        hpg = self.layer_cfgs[layer_idx].heads_per_group
        return head_idx // hpg if hpg > 0 else 0

    def group_codebooks(self, layer_idx: int, groups) -> torch.Tensor:
        """``[len(groups), M, K, d]``: the codebooks of the listed groups in
        order (a per-KV-head stack for the kernels), built once per layer."""
        key = (layer_idx, tuple(int(g) for g in groups))
        st = self._stacks.get(key)
        if st is None:
            st = torch.stack([self.codebooks(layer_idx, g) for g in key[1]]).contiguous()
            self._stacks[key] = st
        return st

    def save(self, save_dir: str) -> None:
        """``{save_dir}/layer_{L}_group_{G}.pt`` = ``{"M", "K", "d", "codebooks"}`` (aq_kv.py:251-275)."""
        os.makedirs(save_dir, exist_ok=True)
        for (layer_idx, group_idx), cb in self._cb.items():
            M, K, d = cb.shape
            torch.save({"M": M, "K": K, "d": d, "codebooks": cb.to("cpu")},
                       os.path.join(save_dir, f"layer_{layer_idx}_group_{group_idx}.pt"))

    def load(self, save_dir: str) -> None:
        """Load every ``layer_{L}_group_{G}.pt`` whose layer is configured,
        skipping groups beyond ``num_heads // heads_per_group`` and updating
        the layer's M/K/d to the file's (aq_kv.py:277-342)."""
        if not os.path.isdir(save_dir):
            raise FileNotFoundError(save_dir)
        for fname in os.listdir(save_dir):
            if not fname.startswith("layer_") or "_group_" not in fname:
                continue
            try:
                core, _ = os.path.splitext(fname)
                _, layer_str, _, group_str = core.split("_")
                layer_idx, group_idx = int(layer_str), int(group_str)
            except ValueError:
                continue
            if layer_idx not in self.layer_cfgs:
                continue
            cfg = self.layer_cfgs[layer_idx]
            if cfg.num_heads is not None and cfg.heads_per_group > 0:
                expected = int(cfg.num_heads) // int(cfg.heads_per_group)
                if expected > 0 and group_idx >= expected:
                    continue
            ckpt = torch.load(os.path.join(save_dir, fname), map_location="cpu", weights_only=True)
            M, K, d = int(ckpt["M"]), int(ckpt["K"]), int(ckpt["d"])
            if (cfg.M, cfg.K, cfg.d) != (M, K, d):
                self.layer_cfgs[layer_idx] = AQLayerConfig(M=M, K=K, d=d, heads_per_group=int(cfg.heads_per_group),
                                                           num_heads=cfg.num_heads)
            self.set_codebooks(layer_idx, group_idx, ckpt["codebooks"])

    # ---- encoding -------------------------------------------------------
    @torch.no_grad()
    def encode_keys(self, layer_idx: int, head_idx: int, keys: torch.Tensor, batch_size: int = 3_000_000,
                    icm_iters: int = 2) -> torch.Tensor:
        """Codes ``[N, M]`` (uint8) of ``keys [N, d]`` with the codebook of
        ``head_idx``'s group: greedy, then ``icm_iters`` ICM sweeps
        (aq_kv.py:348-388)."""
        group_idx = self._group(layer_idx, head_idx)
        return self.encode_keys_batch(layer_idx, group_idx, keys, batch_size=batch_size, icm_iters=icm_iters)

    @torch.no_grad()
    def encode_keys_batch(self, layer_idx: int, group_idx: int, keys: torch.Tensor, batch_size: int = 3_000_000,
                          icm_iters: int = 2) -> torch.Tensor:
        """Codes ``[N_all, M]`` (uint8) of ``keys [N_all, d]`` with one group's
        codebook: greedy, then ``icm_iters`` ICM sweeps (aq_kv.py:390-429,
        quantizer.py:346-370).  fp32, fp16 and bf16 keys are read as they are
        (the reference casts to the manager dtype first)."""
        x = keys.to(device=self.device)
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            x = x.to(self.dtype)
        return ops.encode_keys(x.contiguous() if x.stride(-1) != 1 else x, self.codebooks(layer_idx, group_idx),
                               icm_iters=icm_iters)

    @torch.no_grad()
    def reconstruct(self, layer_idx: int, head_idx: int, codes: torch.Tensor) -> torch.Tensor:
        """``sum_m C_m[codes[:, m]]`` ``[N, d]`` (aq_kv.py:431-457)."""
        cb = self.codebooks(layer_idx, self._group(layer_idx, head_idx))
        idx = codes.to(device=cb.device, dtype=torch.long)
        out = torch.zeros((idx.shape[0], cb.shape[2]), device=cb.device, dtype=cb.dtype)
        for m in range(cb.shape[0]):
            out += cb[m][idx[:, m]]
        return out.to(self.dtype)

    # ---- scoring -------------------------------------------------------
    def _scores(self, q3: torch.Tensor, codes4: torch.Tensor, cb: torch.Tensor) -> torch.Tensor:
        # q3 [B, Hq, d], codes4 [B, Hkv, N, M]: every score of [0, N)
        r = ops.sparse_decode(q3, cb, codes4, topk=0, sink=0, local=0, attention=False,
                              return_head_scores=True)
        return r.head_scores

    @torch.no_grad()
    def approx_inner_product(self, layer_idx: int, head_idx: int, q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        """Scores ``[N]`` of one query ``[d]`` (or ``[1, d]``) against codes
        ``[N, M]`` (aq_kv.py:459-520)."""
        if q.dim() == 2:
            if q.shape[0] != 1:
                raise ValueError(f"q must be [d] or [1, d], got {tuple(q.shape)}")
            q = q[0]
        cb = self.codebooks(layer_idx, self._group(layer_idx, head_idx))
        q3 = q.to(self.device).reshape(1, 1, -1)
        s = self._scores(q3, codes.to(self.device).reshape(1, 1, *codes.shape), cb)
        return s.reshape(-1).to(self.dtype)

    @torch.no_grad()
    def approx_inner_product_multihead(self, layer_idx: int, q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        """Scores ``[Q, N]`` of queries ``[Q, d]`` against their own codes
        ``[Q, N, M]`` with the layer's group-0 codebook (aq_kv.py:522-630)."""
        if q.dim() == 1:
            q = q[None, :]
        cb = self.codebooks(layer_idx, 0)
        Q, N, M = codes.shape
        if M != cb.shape[0] or q.shape[-1] != cb.shape[2] or q.shape[0] != Q:
            raise ValueError(f"AQ shape mismatch: codebook={tuple(cb.shape)}, q={tuple(q.shape)}, codes={tuple(codes.shape)}")
        s = self._scores(q.to(self.device).reshape(Q, 1, -1), codes.to(self.device).reshape(Q, 1, N, M), cb)
        return s.reshape(Q, N).to(self.dtype)

    @torch.no_grad()
    def approx_inner_product_multihead_gqa(self, layer_idx: int, q: torch.Tensor, codes: torch.Tensor,
                                           num_kv_group: int, scoring_m: int = 32) -> torch.Tensor:
        """GQA scores ``[B*Hq, N]`` for queries ``[B*Hq, d]`` and KV-head codes
        ``[B*Hkv, N, M]`` without expanding the codes (aq_kv.py:633-699)."""
        if q.dim() == 1:
            q = q[None, :]
        q = q.to(self.device)
        codes = codes.to(self.device)
        q_heads = q.shape[0]
        kv_heads, n_tokens, m_codes = codes.shape
        group = int(num_kv_group)
        if q_heads != kv_heads * group:
            raise ValueError(f"Invalid GQA score heads: Hq={q_heads}, Hkv={kv_heads}, G={group}")
        if int(scoring_m) != 32:
            raise ValueError(f"aq_scoring_m must be 32, got {scoring_m}")
        cb = self.codebooks(layer_idx, 0)
        if cb.shape[0] != m_codes or cb.shape[2] != q.shape[-1]:
            raise ValueError(f"AQ shape mismatch: codebook={tuple(cb.shape)}, q={tuple(q.shape)}, codes={tuple(codes.shape)}")
        s = self._scores(q.reshape(kv_heads, group, -1), codes.reshape(kv_heads, 1, n_tokens, m_codes), cb)
        return s.reshape(q_heads, n_tokens).to(self.dtype)


class ShardedAQLayerCodebookManager:
    """One ``AQLayerCodebookManager`` per device, each loading the same
    codebook directory (aq_kv.py:702-803).  For a model spread over several
    GPUs layer by layer: every call runs on the device of its input tensor,
    so no codebook crosses devices.  The first device's manager is created
    at once, the others on first use."""

    def __init__(self, layer_cfgs: Dict[int, AQLayerConfig], aq_codebook_dir: str, devices=None,
                 dtype: torch.dtype = torch.float16) -> None:
        self.layer_cfgs = layer_cfgs
        self.aq_codebook_dir = aq_codebook_dir
        self.dtype = dtype
        if not devices:
            devices = [torch.device("cuda", torch.cuda.current_device())]
        self.devices = sorted({torch.device(d) for d in devices}, key=str)
        self._mgr_by_device: Dict[str, AQLayerCodebookManager] = {}
        self._default_device = self.devices[0]
        self._default_mgr = self.for_device(self._default_device)

    def for_device(self, device) -> AQLayerCodebookManager:
        """The manager holding the codebooks on ``device`` (loaded on first use)."""
        key = str(torch.device(device))
        mgr = self._mgr_by_device.get(key)
        if mgr is None:
            mgr = AQLayerCodebookManager(self.layer_cfgs, device=torch.device(device), dtype=self.dtype)
            mgr.load(self.aq_codebook_dir)
            self._mgr_by_device[key] = mgr
        return mgr

    def _on(self, t) -> AQLayerCodebookManager:
        return self.for_device(t.device if isinstance(t, torch.Tensor) else self._default_device)

    def codebooks(self, layer_idx: int, group_idx: int = 0) -> torch.Tensor:
        return self._default_mgr.codebooks(layer_idx, group_idx)

    def encode_keys(self, layer_idx: int, head_idx: int, keys: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._on(keys).encode_keys(layer_idx, head_idx, keys, **kwargs)

    def encode_keys_batch(self, layer_idx: int, group_idx: int, keys: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._on(keys).encode_keys_batch(layer_idx, group_idx, keys, **kwargs)

    def reconstruct(self, layer_idx: int, head_idx: int, codes: torch.Tensor) -> torch.Tensor:
        return self._on(codes).reconstruct(layer_idx, head_idx, codes)

    def approx_inner_product(self, layer_idx: int, head_idx: int, q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        return self._on(q).approx_inner_product(layer_idx, head_idx, q, codes)

    def approx_inner_product_multihead(self, layer_idx: int, q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        return self._on(q).approx_inner_product_multihead(layer_idx, q, codes)

    def approx_inner_product_multihead_gqa(self, layer_idx: int, q: torch.Tensor, codes: torch.Tensor,
                                           num_kv_group: int, scoring_m: int = 32) -> torch.Tensor:
        return self._on(q).approx_inner_product_multihead_gqa(layer_idx, q, codes, num_kv_group,
                                                               scoring_m=scoring_m)
