"""Drop-in for the reference's decode hook (laprune/llm/modifiers/aq_evaluation.py).

``self_attn_forward`` (aq_evaluation.py:279-322), ``_decode_attention``
(:146-253), ``_prepare_aq_cache`` (:324-494), ``_kv_cache_append``
(:65-112), ``_cached_position_ids`` (:56-63) and ``do_sdpa_attn``
(laprune/attention.py:21-73) with the reference's signatures, config keys
and cache dictionaries, the sparse path on this package's kernels:

* one decode token (Tq == 1): per-query-head LUT scores over the candidate
  window, top-k of the reference's size (``mask_out`` / ``min_remain``), the
  union with the sink and local-window tokens, the GQA K/V gather and the
  attention -- all in one ``ops.sparse_decode(select="query_head")`` call;
  then ``self_attn.o_proj``.  With ``aq_use_pruned_attn`` off the reference
  attends the same token set through a mask (:255-278), so both settings run
  the same kernel;
* new keys are encoded greedily straight into the code cache slice
  (``ops.encode_keys(..., codes=cache[:, :, t0:t1])``), every
  ``aq_decode_group_size`` tokens as the reference does.

Dense attention (prefill, dense layers) stays the reference's torch SDPA
call.  fp16 / bf16 K/V caches only (the reference's CUDA kernels take fp16; its
fp32 path is its torch fallback).  Multi-token decode (Tq > 1) and key
reconstruction are outside the decode path and raise.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .aq_kv import AQLayerCodebookManager

__all__ = ["self_attn_forward", "_decode_attention", "_prepare_aq_cache", "_kv_cache_append", "_cached_position_ids",
           "do_sdpa_attn", "decode_keep_size"]


def decode_keep_size(num_candidate: int, mask_out: float = 0.98, min_remain: int = 20) -> int:
    """Top-k size of the decode hook (aq_evaluation.py:193-197)."""
    if num_candidate <= 0:
        return 0
    k = num_candidate - int(num_candidate * mask_out)
    k = max(min(num_candidate, min_remain), k)
    return max(1, min(k, num_candidate))


def _scoring_codebooks(manager: AQLayerCodebookManager, layer_idx: int, Hq: int, Hkv: int) -> torch.Tensor:
    """The decode hook's codebooks, in the manager's scoring dtype (a
    half-precision copy for an fp16 / bf16 manager, as the reference scores
    from its manager-dtype codebooks): one for every head when
    heads_per_group covers the Hq query heads (aq_evaluation.py:161-167),
    else query head h uses group h // heads_per_group (:169-176) -- stacked
    per KV head, which needs the G query heads of a KV head in one group."""
    cfg = manager.layer_cfgs.get(layer_idx)
    dt = manager.scoring_dtype
    if cfg is None or cfg.heads_per_group <= 0 or cfg.heads_per_group >= Hq:
        return manager.codebooks(layer_idx, 0, dt)
    G, hpg = Hq // Hkv, cfg.heads_per_group
    groups = [(kv * G) // hpg for kv in range(Hkv)]
    if any((kv * G + G - 1) // hpg != groups[kv] for kv in range(Hkv)):
        raise NotImplementedError(f"heads_per_group={hpg} splits the {G} query heads of a KV head over codebooks")
    return manager.group_codebooks(layer_idx, groups, dt)


def _encoding_codebooks(manager: AQLayerCodebookManager, layer_idx: int, Hkv: int) -> torch.Tensor:
    """The code cache's codebooks: one for all when heads_per_group covers
    the Hkv cached heads, else KV head h uses group h // heads_per_group
    (aq_evaluation.py:384-401)."""
    cfg = manager.layer_cfgs.get(layer_idx)
    if cfg is None or cfg.heads_per_group <= 0 or cfg.heads_per_group >= Hkv:
        return manager.codebooks(layer_idx, 0)
    return manager.group_codebooks(layer_idx, [h // cfg.heads_per_group for h in range(Hkv)])


def _on_device(manager, device) -> AQLayerCodebookManager:
    # a per-device manager (ShardedAQLayerCodebookManager) resolves to the
    # one holding the codebooks on the tensors' device
    return manager.for_device(device) if hasattr(manager, "for_device") else manager


def _decode_attention(self_attn, manager: AQLayerCodebookManager, layer_idx: int, Q_rope: torch.Tensor,
                      K_rope: torch.Tensor, vals_full: torch.Tensor, aq_cache: dict, conf: dict) -> torch.Tensor:
    """Sparse attention of the last query token over the AQ-selected keys,
    then ``self_attn.o_proj`` (aq_evaluation.py:146-253).

    Q_rope ``[B, H, 1, D]``; K_rope / vals_full ``[B, Hkv, Tk_total, D]``;
    ``aq_cache["codes"]`` ``[B, Hkv, cap, M]`` uint8 with ``seq_len`` valid.
    """
    B, H, Tq, D = Q_rope.shape
    manager = _on_device(manager, Q_rope.device)
    scoring_m = int(conf.get("aq_scoring_m", 32))
    if scoring_m != 32:
        raise ValueError(f"aq_scoring_m must be 32, got {scoring_m}")
    if Tq != 1:
        raise NotImplementedError(f"decode of {Tq} query tokens at once is outside the single-token decode path")
    codes = aq_cache["codes"]
    seq_len_codes = int(aq_cache.get("seq_len", codes.shape[2]))
    seq_len_codes = max(0, min(seq_len_codes, codes.shape[2]))
    Hkv = int(codes.shape[1])
    if H % Hkv != 0 or K_rope.shape[1] != Hkv:
        raise ValueError(f"Invalid GQA code heads: Hq={H}, Hkv={Hkv}, K heads={K_rope.shape[1]}")
    Tk_total = int(getattr(self_attn, "total_seq_len", seq_len_codes))
    if K_rope.dtype not in (torch.float16, torch.bfloat16) or vals_full.dtype != K_rope.dtype:
        raise RuntimeError(f"K/V caches must be fp16 or bf16 (got {K_rope.dtype}, {vals_full.dtype})")

    sink = int(conf.get("sink_size", 4))
    local = int(conf.get("local_window", 64))
    n_cand = ops.num_candidates(seq_len_codes, Tk_total, sink, local)
    k = decode_keep_size(n_cand, float(conf.get("mask_out", 0.98)), int(conf.get("min_remain", 20)))
    cb = _scoring_codebooks(manager, layer_idx, H, Hkv)
    r = ops.sparse_decode(Q_rope[:, :, -1, :], cb, codes, K_rope, vals_full, topk=k, T_codes=seq_len_codes,
                          T_total=Tk_total, sink=sink, local=local, select="query_head")
    attn_output = r.out.reshape(B, 1, H * D)
    return self_attn.o_proj(attn_output)


# ---- the layer's K/V cache --------------------------------------------------
# Observable contract (aq_evaluation.py:65-112): buffers self_attn.k_cache /
# v_cache [B, Hkv, cap, D] of which k_cache_len tokens are valid and
# k_cache_capacity slots exist; callers get [B, Hkv, total, D] views of them.
# Capacity policy (it fixes the views' strides): the first buffers hold
# total + aq_kv_extra_capacity slots (at least 16), or max(total, 2 max(16, L))
# when they start from an input cache of L tokens; a full buffer doubles (at
# least to total).  Decode tokens land in place: with the slots reserved,
# the fused rotary + append kernel writes each token's rotated key and value
# straight into its slot, so the buffers are static between doublings.


def _kv_slots(total_len: int, have: int, prefix_len: Optional[int], extra: int) -> int:
    """Slots the buffers need for ``total_len`` tokens when they hold ``have``
    (0: not allocated yet; ``prefix_len`` is the input cache's length then)."""
    if have > 0:
        return have if total_len <= have else max(total_len, 2 * have)
    if prefix_len is not None:
        return max(total_len, 2 * max(16, prefix_len))
    return max(total_len + extra, 16)


def _kv_reserve(self_attn, like_k: torch.Tensor, like_v: torch.Tensor, total_len: int, input_kv_cache=None):
    """Buffers on ``self_attn`` with room for ``total_len`` tokens, allocated
    or grown as the policy above says; returns ``(k_buf, v_buf, valid)``."""
    k_buf, v_buf = getattr(self_attn, "k_cache", None), getattr(self_attn, "v_cache", None)
    have = int(getattr(self_attn, "k_cache_capacity", 0)) if k_buf is not None and v_buf is not None else 0
    valid = int(getattr(self_attn, "k_cache_len", 0)) if have > 0 else 0
    conf = getattr(self_attn, "draft_kwargs", {}) or {}
    extra = max(0, int(conf.get("aq_kv_extra_capacity", 0)))
    B, H, _, D = like_k.shape
    prefix = None
    if have == 0 and input_kv_cache is not None:
        prefix = input_kv_cache
        valid = int(prefix[0].shape[-2])
    need = _kv_slots(total_len, have, None if prefix is None else valid, extra)
    if need != have:
        src_k, src_v = (prefix if prefix is not None else (k_buf, v_buf))
        proto_k = src_k if src_k is not None else like_k
        proto_v = src_v if src_v is not None else like_v
        new_k = proto_k.new_empty((B, H, need, D))
        new_v = proto_v.new_empty((B, H, need, D))
        if valid > 0:
            new_k[:, :, :valid].copy_(src_k[:, :, :valid])
            new_v[:, :, :valid].copy_(src_v[:, :, :valid])
        k_buf, v_buf = new_k, new_v
        self_attn.k_cache, self_attn.v_cache, self_attn.k_cache_capacity = k_buf, v_buf, need
    return k_buf, v_buf, valid


def _kv_publish(self_attn, end: int):
    """Record ``end`` valid tokens; the [B, Hkv, end, D] views and their data."""
    self_attn.k_cache_len = end
    k_view, v_view = self_attn.k_cache[:, :, :end], self_attn.v_cache[:, :, :end]
    return k_view, v_view, (k_view.data, v_view.data)


def _kv_cache_append(self_attn, k_new: torch.Tensor, v_new: torch.Tensor, total_len: int, input_kv_cache=None):
    """Append ``k_new`` / ``v_new`` ``[B, H, Tn, D]`` (post-RoPE keys) to the
    layer's K/V buffers (aq_evaluation.py:65-112).  Returns the
    ``[B, H, total, D]`` views and ``(K_view.data, V_view.data)``."""
    k_buf, v_buf, valid = _kv_reserve(self_attn, k_new, v_new, total_len, input_kv_cache)
    end = valid + int(k_new.shape[2])
    k_buf[:, :, valid:end].copy_(k_new)
    v_buf[:, :, valid:end].copy_(v_new)
    return _kv_publish(self_attn, end)


def _rope_append_decode(self_attn, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor,
                        sin: torch.Tensor, total_len: int, input_kv_cache=None):
    """One decode token: rotary embedding of q and k fused with the append of
    the rotated key and the value into their reserved slot (ops.rope_append),
    replacing apply_rotary_pos_emb + _kv_cache_append (aq_evaluation.py:
    296-308).  Returns ``(Q_rope, K_view, V_view, (K_view.data, V_view.data))``."""
    k_buf, v_buf, valid = _kv_reserve(self_attn, k, v, total_len, input_kv_cache)
    q_rot = ops.rope_append(q, k, v, cos, sin, k_buf, v_buf, valid)
    k_view, v_view, data = _kv_publish(self_attn, valid + 1)
    return q_rot.unsqueeze(2), k_view, v_view, data


def _encode_into(manager: AQLayerCodebookManager, layer_idx: int, keys: torch.Tensor, codes_dst: torch.Tensor,
                 icm_iters: int = 0) -> None:
    # keys [B, H, t, d] -> codes_dst [B, H, t, M] (a slice of the cache)
    if keys.shape[2] == 0:
        return
    ops.encode_keys(keys, _encoding_codebooks(manager, layer_idx, keys.shape[1]), codes=codes_dst,
                    icm_iters=icm_iters)


def _prepare_aq_cache(self, manager: AQLayerCodebookManager, layer_idx: int, keys: torch.Tensor, need_recon: bool,
                      decode_group_size: int = 1, is_prefill: bool = False) -> dict:
    """The layer's code cache ``self._aq_cache`` = ``{"seq_len",
    "encoded_len", "batch_size", "codes" [B, H, cap, M] uint8, "approx"}``
    kept in step with ``keys [B, H, T, d]`` (aq_evaluation.py:324-494):
    capacity doubling, new keys encoded once ``decode_group_size`` of them
    are pending (prefill: at once), ``aq_code_extra_capacity`` spare slots
    after prefill."""
    if need_recon:
        raise NotImplementedError("key reconstruction (aq_use_exact_true_score=False) is not on the decode path")
    manager = _on_device(manager, keys.device)
    conf = getattr(self, "draft_kwargs", {}) or {}
    B, H, T, d = keys.shape
    cfg = manager.layer_cfgs.get(layer_idx)
    M = cfg.M if cfg is not None else manager.codebooks(layer_idx, 0).shape[0]
    cache: Optional[dict] = getattr(self, "_aq_cache", None)
    if cache is not None and cache.get("batch_size") == B:
        cached_seq = int(cache.get("seq_len", 0))
        encoded = int(cache.get("encoded_len", cached_seq))
        if cached_seq == T:
            return cache
        if T > cached_seq:
            codes = cache["codes"]
            cap = codes.shape[2]
            if T > cap:
                new_cap = max(cap * 2 if cap > 0 else T, T)
                grown = codes.new_empty((B, H, new_cap, codes.shape[3]))
                if encoded > 0:
                    grown[:, :, :encoded] = codes[:, :, :encoded]
                codes = grown
                cache["codes"] = codes
            pending = T - encoded
            if not is_prefill and decode_group_size > 1 and pending < decode_group_size:
                cache["seq_len"], cache["encoded_len"] = T, encoded
                self._aq_cache = cache
                return cache
            if pending > 0:
                icm = int(conf.get("aq_encode_icm_iters_decode", 0))
                _encode_into(manager, layer_idx, keys[:, :, encoded:T], codes[:, :, encoded:T], icm)
            cache["seq_len"], cache["encoded_len"], cache["codes"] = T, T, codes
            self._aq_cache = cache
            return cache
    icm = int(conf.get("aq_encode_icm_iters_prefill", 0 if is_prefill else 2))
    extra = max(0, int(conf.get("aq_code_extra_capacity", 0))) if is_prefill else 0
    codes = torch.empty((B, H, T + extra, M), dtype=torch.uint8, device=keys.device)
    group = int(conf.get("aq_prefill_group_size", 0))
    group = T if group <= 0 else group
    for t0 in range(0, T, group):
        t1 = min(T, t0 + group)
        _encode_into(manager, layer_idx, keys[:, :, t0:t1], codes[:, :, t0:t1], icm)
    cache = {"seq_len": T, "encoded_len": T, "batch_size": B, "codes": codes, "approx": None}
    self._aq_cache = cache
    return cache


def _cached_position_ids(owner, device: torch.device, end: int) -> torch.Tensor:
    """A shared ``arange`` on ``device``, grown only when needed (aq_evaluation.py:56-63)."""
    cache = getattr(owner, "_laprune_position_ids", None)
    if cache is None or cache.device != device or int(cache.numel()) < int(end):
        cache = torch.arange(max(int(end), 1024), device=device, dtype=torch.long)
        owner._laprune_position_ids = cache
    return cache


def do_sdpa_attn(query, key, value, cos=None, sin=None, out_proj=None, query_down_proj=None, key_down_proj=None,
                 mask=None, already_rope: bool = False):
    """Dense attention of post-RoPE q over a native GQA cache (laprune/attention.py:21-73): the
    reference's path for dense layers and prefill, kept as its torch SDPA call (not part of the
    sparse decode path)."""
    if not already_rope:
        raise ValueError("LAPrune attention expects post-RoPE query and key tensors")
    q, k, v = query, key, value
    hq, nq = int(q.shape[1]), int(q.shape[-2])
    if query_down_proj is not None:
        q = (q.transpose(1, 2).flatten(2) @ query_down_proj).unflatten(-1, (hq, -1)).transpose(1, 2)
    if key_down_proj is not None:
        k = (k.transpose(1, 2).flatten(2) @ key_down_proj).unflatten(-1, (hq, -1)).transpose(1, 2)
    gqa = hq != int(k.shape[1])
    if gqa and hq % int(k.shape[1]):
        raise ValueError(f"invalid GQA head counts: Hq={hq}, Hkv={k.shape[1]}")
    sdpa = torch.nn.functional.scaled_dot_product_attention
    nk = int(k.shape[-2])
    if mask is not None:
        o = sdpa(q, k, v, attn_mask=mask, is_causal=False, enable_gqa=gqa)
    elif nk == nq:
        o = sdpa(q, k, v, is_causal=True, enable_gqa=gqa)
    elif nq == 1:
        o = sdpa(q, k, v, is_causal=False, enable_gqa=gqa)
    else:  # queries at the end of the cache
        m = torch.full((1, 1, nq, nk), torch.finfo(q.dtype).min, dtype=torch.float32, device=q.device)
        m[..., -nq:].triu_(diagonal=1)
        m[..., :nk - nq].fill_(0)
        o = sdpa(q, k, v, attn_mask=m.to(q.dtype), is_causal=False, enable_gqa=gqa)
    o = o.transpose(1, 2).flatten(2)
    return out_proj(o) if out_proj is not None else o


def _rope_rows(self, manager, q: torch.Tensor, past: int, n_new: int):
    """HF rotary rows (cos, sin) ``[B, n_new, D]`` of positions past .. past +
    n_new - 1, computed once per step and shared by the layers: they depend
    only on the positions, the batch size, the device and the dtype, which
    together key the copy kept on the manager."""
    key = (q.device, q.dtype, int(past), int(n_new), int(q.shape[0]))
    held = getattr(manager, "_lp_rope_rows", None)
    if held is None or held[0] != key:
        pos = _cached_position_ids(manager, q.device, past + n_new)[past:past + n_new]
        cos, sin = self.rotary_emb(q, pos.unsqueeze(0).expand(q.shape[0], -1))
        held = (key, cos, sin)
        manager._lp_rope_rows = held
    return held[1], held[2]


def _sparse_layer(self, manager, conf: dict, is_prefill: bool) -> bool:
    """Whether the layer runs the AQ path (aq_evaluation.py:310-314): AQ on
    and encoding on, not a fixed / dense (full-KV) layer, a configured layer,
    and not a prefill with aq_disable_prefill."""
    if not conf.get("enable", True) or conf.get("aq_disable_encode", False):
        return False
    if self.is_fix_layer or getattr(self, "full_kv_layer", False) or self.layer_idx not in manager.layer_cfgs:
        return False
    return not (is_prefill and conf.get("aq_disable_prefill", False))


def self_attn_forward(self, hidden_states: torch.Tensor, kv_cache=None):
    """The reference's replacement Llama attention forward (aq_evaluation.py:279-322), bound to a
    ``LlamaAttention`` that carries ``aq_manager``, ``layer_idx``, ``draft_kwargs``,
    ``is_fix_layer``, ``rotary_emb`` and ``config``.  Returns ``(attn_output, kv_cache_out, None,
    None)``.

    A decode token (one new position) goes through one fused kernel for the rotary embedding of
    its query and key and the append of its key and value to the layer's static cache
    (``_rope_append_decode``); longer inputs take HF ``apply_rotary_pos_emb`` and
    ``_kv_cache_append``.  Prefill and dense layers attend densely (torch SDPA); a sparse
    layer's decode token goes through ``_decode_attention`` after ``_prepare_aq_cache`` has
    brought its code cache up to date."""
    manager, conf = self.aq_manager, self.draft_kwargs
    n_q, n_kv = self.config.num_attention_heads, self.config.num_key_value_heads
    d = self.config.hidden_size // n_q
    n_new = hidden_states.shape[-2]
    is_prefill = n_new > 1 and kv_cache is None

    def heads(proj, n):  # [B, T, n*d] -> [B, n, T, d]
        return proj(hidden_states).unflatten(-1, (n, d)).transpose(1, 2)

    q, k, v = heads(self.q_proj, n_q), heads(self.k_proj, n_kv), heads(self.v_proj, n_kv)
    past = int(getattr(self, "total_seq_len", 0))
    total = past + n_new
    cos, sin = _rope_rows(self, manager, q, past, n_new)
    if n_new == 1 and q.is_cuda and q.dtype in (torch.float16, torch.bfloat16) and d % 2 == 0:
        q_rope, k_all, v_all, kv_out = _rope_append_decode(self, q, k, v, cos, sin, total, kv_cache)
    else:
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        q_rope, k_rope = apply_rotary_pos_emb(q, k, cos, sin)
        k_all, v_all, kv_out = _kv_cache_append(self, k_rope, v, total, kv_cache)
    self.total_seq_len = total

    if not _sparse_layer(self, manager, conf, is_prefill):
        return do_sdpa_attn(q_rope, k_all, v_all, out_proj=self.o_proj, already_rope=True), kv_out, None, None
    aq_cache = _prepare_aq_cache(self, manager, self.layer_idx, k_all,
                                 need_recon=not conf.get("aq_use_exact_true_score", True),
                                 decode_group_size=int(conf.get("aq_decode_group_size", 1)),
                                 is_prefill=is_prefill)
    if is_prefill:
        return do_sdpa_attn(q_rope, k_all, v_all, out_proj=self.o_proj, already_rope=True), kv_out, None, None
    out = _decode_attention(self, manager, self.layer_idx, q_rope, k_all, v_all, aq_cache, conf)
    return out, kv_out, None, None
