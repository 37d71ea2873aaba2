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

Codebooks are held in fp32 on the manager's device (the encoder reads these);
with a half-precision manager dtype the scoring kernels read an fp16 / bf16
copy, persisted beside the codebook file (``write_codebook_copies``).
``dtype`` is also the dtype of returned scores, as the reference's manager
dtype.
There is no CPU fallback: a missing CUDA device or extension raises.
Codebook training is outside the decode path and is not provided.
"""
from __future__ import annotations

import hashlib
import os
import re
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from . import ops

__all__ = ["AQLayerConfig", "AQLayerCodebookManager", "ShardedAQLayerCodebookManager", "codebook_copies",
           "codebook_file_index"]


@dataclass
class AQLayerConfig:
    """One layer's AQ geometry (aq_kv.py:79-93): M sub-codebooks of K entries
    of dimension d; ``heads_per_group`` heads share one codebook."""
    M: int
    K: int
    d: int
    heads_per_group: int = 2
    num_heads: Optional[int] = None


_CODEBOOK_FILE = re.compile(r"^layer_(\d+)_group_(\d+)\.pt$")
_COPIES_SUFFIX = ".lpcopies.pt"
_COPIES_FORMAT = "laprune_b200 codebook copies v1"
_HALF = (torch.float16, torch.bfloat16)


def codebook_file_index(fname: str) -> Optional[Tuple[int, int]]:
    """``(layer, group)`` of a codebook file name ``layer_{L}_group_{G}.pt``
    (aq_kv.py:251-342), None for any other name (derived-copy files
    ``layer_{L}_group_{G}.lpcopies.pt`` included; the reference's loader
    skips those too, as their group field is not an integer)."""
    m = _CODEBOOK_FILE.match(fname)
    return (int(m.group(1)), int(m.group(2))) if m else None


def _digest(cb: torch.Tensor) -> str:
    return hashlib.sha256(cb.detach().to("cpu", torch.float32).contiguous().numpy().tobytes()).hexdigest()


def codebook_copies(cb: torch.Tensor) -> Dict[str, object]:
    """The derived tensors of one fp32 ``[M,K,d]`` codebook set, as
    persisted beside its file: fp16 and bf16 copies (the scoring kernels read
    these when the manager's dtype is half precision: half the bytes of the
    table build), and the reference's per-process fp16 encode operands
    (aq_kv.py:61-72: the transposed codebooks ``weight_t [M,d,K]`` and
    ``bias = -||C||^2 / 2 [M,K]`` computed from the fp16 copy), with the
    digest of the fp32 source they were made from."""
    c = cb.detach().to("cpu", torch.float32).contiguous()
    half = c.to(torch.float16)
    return {"format": _COPIES_FORMAT, "source_sha256": _digest(c), "shape": tuple(c.shape),
            "codebooks_fp16": half, "codebooks_bf16": c.to(torch.bfloat16),
            "weight_t_fp16": half.transpose(1, 2).contiguous(),
            "bias_fp16": (-0.5 * half.float().pow(2).sum(dim=-1)).to(torch.float16)}


class AQLayerCodebookManager:
    """Per-(layer, head-group) codebooks and LUT scoring (aq_kv.py:96-699).

    Storage: the fp32 ``[M,K,d]`` set of each (layer, group) -- what the
    encoder reads, so codes stay those of the CPU arithmetic -- and, for a
    half-precision manager dtype, a copy in that dtype that the scoring
    kernels read (the reference's fp16 manager scores from fp16 codebooks,
    aq_kv.py:61-72, 671-687).  The copies come from the derived-copy file
    beside the codebook file when its source digest matches, else they are
    converted on first use; ``write_codebook_copies`` persists them."""

    def __init__(self, layer_cfgs: Dict[int, AQLayerConfig], device: Optional[torch.device] = None,
                 dtype: torch.dtype = torch.float32) -> None:
        self.layer_cfgs = layer_cfgs
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self._cb: Dict[Tuple[int, int], torch.Tensor] = {}
        self._copies: Dict[Tuple[int, int, torch.dtype], torch.Tensor] = {}
        self._stacks: Dict[Tuple[int, Tuple[int, ...], torch.dtype], torch.Tensor] = {}

    # ---- codebooks -------------------------------------------------------
    def set_codebooks(self, layer_idx: int, group_idx: int, codebooks: torch.Tensor,
                      copies: Optional[Dict[torch.dtype, torch.Tensor]] = None) -> None:
        """Install the ``[M,K,d]`` codebooks of one (layer, group), and
        optionally ready-made half-precision copies of them."""
        if codebooks.dim() != 3:
            raise ValueError(f"codebooks must be [M,K,d], got {tuple(codebooks.shape)}")
        key = (layer_idx, group_idx)
        self._cb[key] = codebooks.detach().to(device=self.device, dtype=torch.float32).contiguous()
        self._copies = {k: v for k, v in self._copies.items() if k[:2] != key}
        for dt, t in (copies or {}).items():
            self._copies[key + (dt,)] = t.to(self.device).contiguous()
        self._stacks = {k: v for k, v in self._stacks.items() if k[0] != layer_idx}

    def codebooks(self, layer_idx: int, group_idx: int = 0, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """The set of one (layer, group): fp32, or its fp16 / bf16 copy."""
        key = (layer_idx, group_idx)
        if key not in self._cb:
            raise KeyError(f"no codebooks loaded for layer {layer_idx}, group {group_idx}")
        if dtype == torch.float32:
            return self._cb[key]
        if dtype not in _HALF:
            raise ValueError(f"codebook copies are fp16 or bf16, not {dtype}")
        copy = self._copies.get(key + (dtype,))
        if copy is None:
            copy = self._cb[key].to(dtype).contiguous()
            self._copies[key + (dtype,)] = copy
        return copy

    @property
    def scoring_dtype(self) -> torch.dtype:
        """Codebook dtype the scoring kernels read: the manager's dtype when
        it is half precision, else fp32."""
        return self.dtype if self.dtype in _HALF else torch.float32

    def _group(self, layer_idx: int, head_idx: int) -> int:
        # head_idx // heads_per_group; heads_per_group <= 0 means one shared group
        hpg = self.layer_cfgs[layer_idx].heads_per_group
        return head_idx // hpg if hpg > 0 else 0

    def group_codebooks(self, layer_idx: int, groups, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """``[len(groups), M, K, d]``: the codebooks of the listed groups in
        order (a per-KV-head stack for the kernels), built once per layer."""
        key = (layer_idx, tuple(int(g) for g in groups), dtype)
        st = self._stacks.get(key)
        if st is None:
            st = torch.stack([self.codebooks(layer_idx, g, dtype) for g in key[1]]).contiguous()
            self._stacks[key] = st
        return st

    # ---- codebook files ----------------------------------------------------
    def save(self, save_dir: str) -> None:
        """``{save_dir}/layer_{L}_group_{G}.pt`` = ``{"M", "K", "d", "codebooks"}`` (aq_kv.py:251-275)."""
        os.makedirs(save_dir, exist_ok=True)
        for (layer_idx, group_idx), cb in self._cb.items():
            M, K, d = cb.shape
            torch.save({"M": M, "K": K, "d": d, "codebooks": cb.to("cpu")},
                       os.path.join(save_dir, f"layer_{layer_idx}_group_{group_idx}.pt"))

    def write_codebook_copies(self, save_dir: str) -> int:
        """Persist ``layer_{L}_group_{G}.lpcopies.pt`` (see
        :func:`codebook_copies`) beside every loaded set; returns the count."""
        os.makedirs(save_dir, exist_ok=True)
        for (layer_idx, group_idx), cb in self._cb.items():
            torch.save(codebook_copies(cb),
                       os.path.join(save_dir, f"layer_{layer_idx}_group_{group_idx}{_COPIES_SUFFIX}"))
        return len(self._cb)

    def _usable_group(self, layer_idx: int, group_idx: int) -> bool:
        # groups past num_heads // heads_per_group are leftovers of another
        # grouping and are skipped (aq_kv.py:301-309)
        cfg = self.layer_cfgs.get(layer_idx)
        if cfg is None:
            return False
        if cfg.num_heads is None or cfg.heads_per_group <= 0:
            return True
        n_groups = int(cfg.num_heads) // int(cfg.heads_per_group)
        return n_groups <= 0 or group_idx < n_groups

    def _read_copies(self, path: str, cb: torch.Tensor) -> Dict[torch.dtype, torch.Tensor]:
        # the derived copies of `cb` from `path`, if that file was made from it
        if not os.path.exists(path):
            return {}
        blob = torch.load(path, map_location="cpu", weights_only=True)
        if blob.get("format") != _COPIES_FORMAT or blob.get("source_sha256") != _digest(cb):
            return {}
        return {torch.float16: blob["codebooks_fp16"], torch.bfloat16: blob["codebooks_bf16"]}

    def load(self, save_dir: str, use_copies: bool = True) -> None:
        """Load the codebook files of ``save_dir`` (aq_kv.py:277-342): every
        ``layer_{L}_group_{G}.pt`` of a configured layer and a usable group; a
        file whose M/K/d differ from the layer's config updates the config
        (grouping kept).  Derived copies beside a file are used when their
        source digest matches it (``use_copies``)."""
        if not os.path.isdir(save_dir):
            raise FileNotFoundError(save_dir)
        for fname in sorted(os.listdir(save_dir)):
            idx = codebook_file_index(fname)
            if idx is None or not self._usable_group(*idx):
                continue
            layer_idx, group_idx = idx
            blob = torch.load(os.path.join(save_dir, fname), map_location="cpu", weights_only=True)
            shape = (int(blob["M"]), int(blob["K"]), int(blob["d"]))
            cfg = self.layer_cfgs[layer_idx]
            if (cfg.M, cfg.K, cfg.d) != shape:
                self.layer_cfgs[layer_idx] = AQLayerConfig(*shape, heads_per_group=int(cfg.heads_per_group),
                                                           num_heads=cfg.num_heads)
            cb = blob["codebooks"].to(torch.float32)
            copies = {}
            if use_copies:
                copies = self._read_copies(os.path.join(save_dir, fname[:-3] + _COPIES_SUFFIX), cb)
            self.set_codebooks(layer_idx, group_idx, cb, copies)

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
        cb = self.codebooks(layer_idx, self._group(layer_idx, head_idx), self.scoring_dtype)
        q3 = q.to(self.device).reshape(1, 1, -1)
        s = self._scores(q3, codes.to(self.device).reshape(1, 1, *codes.shape), cb)
        return s.reshape(-1).to(self.dtype)

    @torch.no_grad()
    def approx_inner_product_multihead(self, layer_idx: int, q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        """Scores ``[Q, N]`` of queries ``[Q, d]`` against their own codes
        ``[Q, N, M]`` with the layer's group-0 codebook (aq_kv.py:522-630)."""
        if q.dim() == 1:
            q = q[None, :]
        cb = self.codebooks(layer_idx, 0, self.scoring_dtype)
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
        cb = self.codebooks(layer_idx, 0, self.scoring_dtype)
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

    def codebooks(self, layer_idx: int, group_idx: int = 0, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return self._default_mgr.codebooks(layer_idx, group_idx, dtype)

    def write_codebook_copies(self, save_dir: str) -> int:
        return self._default_mgr.write_codebook_copies(save_dir)

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
