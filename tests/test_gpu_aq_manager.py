"""The reference-facing manager and decode hook on the GPU, against the
reference's own outputs (golden fixtures made by running the reference's
AQLayerCodebookManager and _decode_attention) and the oracle."""
import types

import numpy as np
import pytest
import torch

import oracle
from laprune_b200 import aq_evaluation as aqe
from laprune_b200 import synthetic as syn
from laprune_b200.aq_kv import AQLayerCodebookManager, AQLayerConfig

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _mgr(cb, num_heads, hpg=None, layer=0):
    m = AQLayerCodebookManager({layer: AQLayerConfig(M=32, K=256, d=128, heads_per_group=hpg or num_heads,
                                                     num_heads=num_heads)}, device=_dev())
    if cb.dim() == 3:
        m.set_codebooks(layer, 0, cb)
    else:
        for g in range(cb.shape[0]):
            m.set_codebooks(layer, g, cb[g])
    return m


def test_gqa_scores_and_batch_encode_match_the_reference(golden_dir):
    fix = np.load(golden_dir / "small_shared.npz")
    sm = syn.small_shared(7)
    m = _mgr(sm["cb"], 8)
    codes = sm["codes_full"][:, :sm["T"]].to(_dev())  # strided prefix, as the decode cache
    s = m.approx_inner_product_multihead_gqa(0, sm["q"].to(_dev()), codes, sm["G"])
    torch.cuda.synchronize()
    ref = fix["scores"]
    assert s.shape == (8, sm["T"]) and s.dtype == torch.float32
    assert np.abs(s.cpu().numpy() - ref).max() <= 1e-3 * np.abs(ref).max()
    enc = m.encode_keys_batch(0, 0, sm["x"].to(_dev()), icm_iters=0).cpu().numpy()
    assert np.array_equal(enc, oracle.encode_greedy(sm["x"].numpy(), sm["cb"].numpy()))
    assert (enc == fix["codes_enc"]).all(1).mean() >= 0.99


def test_single_and_multihead_scores_match_the_oracle():
    g = torch.Generator().manual_seed(2)
    cb = torch.randn((32, 256, 128), generator=g) * 0.05
    q = torch.randn((5, 128), generator=g)
    codes = torch.randint(0, 256, (5, 300, 32), generator=g, dtype=torch.uint8)
    m = _mgr(cb, 8)
    multi = m.approx_inner_product_multihead(0, q.to(_dev()), codes.to(_dev())).cpu().numpy()
    one = m.approx_inner_product(0, 3, q[2].to(_dev()), codes[2].to(_dev())).cpu().numpy()
    L = oracle.lut(q.numpy(), cb.numpy())
    want = np.stack([oracle.score_gqa(L[i:i + 1], codes[i:i + 1].numpy(), 1)[0] for i in range(5)])
    assert np.abs(multi - want).max() <= 1e-3 * np.abs(want).max()
    assert np.abs(one - want[2]).max() <= 1e-3 * np.abs(want[2]).max()


@pytest.mark.parametrize("sink", [0, 4])
def test_decode_hook_matches_the_reference(golden_dir, sink):
    fix = np.load(golden_dir / "decode_hook.npz")
    dh = syn.decode_hook_case(11)
    m = _mgr(dh["cb"], dh["Hq"])
    dev = _dev()
    conf = {"mask_out": 0.98, "min_remain": 20, "sink_size": sink, "local_window": 64,
            "aq_use_pruned_attn": True, "aq_scoring_m": 32}
    self_attn = types.SimpleNamespace(total_seq_len=dh["T"], o_proj=torch.nn.Identity())
    aq_cache = {"codes": dh["codes"].to(dev), "seq_len": dh["T"]}
    # the reference ran this case on fp32 K/V (its torch fallback); the
    # kernels take fp16 caches, so the bar is the bf16 tolerance
    out = aqe._decode_attention(self_attn, m, 0, dh["q"].to(dev).half(), dh["keys"].to(dev).half(),
                                dh["vals"].to(dev).half(), aq_cache, conf)
    torch.cuda.synchronize()
    ref = fix[f"out_sink{sink}"]
    assert out.shape == ref.shape
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 2e-2


def test_decode_hook_rejects_fp32_caches_and_bad_scoring_m():
    dh = syn.decode_hook_case(11)
    m = _mgr(dh["cb"], dh["Hq"])
    self_attn = types.SimpleNamespace(total_seq_len=dh["T"], o_proj=torch.nn.Identity())
    aq_cache = {"codes": dh["codes"].to(_dev()), "seq_len": dh["T"]}
    args = (dh["q"].to(_dev()), dh["keys"].to(_dev()), dh["vals"].to(_dev()), aq_cache)
    with pytest.raises(RuntimeError):
        aqe._decode_attention(self_attn, m, 0, *args[:3], args[3], {})
    with pytest.raises(ValueError):
        aqe._decode_attention(self_attn, m, 0, *args[:3], args[3], {"aq_scoring_m": 16})


def test_code_cache_follows_prefill_and_grouped_decode():
    g = torch.Generator().manual_seed(4)
    Hkv, D = 2, 128
    cb = torch.randn((Hkv, 32, 256, D), generator=g) * 0.05
    m = _mgr(cb, Hkv, hpg=1)  # one codebook per KV head
    dev = _dev()
    keys = (torch.randn((1, Hkv, 300, D), generator=g) * 0.5).to(torch.bfloat16)
    attn = types.SimpleNamespace(draft_kwargs={"aq_code_extra_capacity": 8})
    c = aqe._prepare_aq_cache(attn, m, 0, keys[:, :, :250].to(dev), need_recon=False, decode_group_size=16,
                              is_prefill=True)
    assert c["seq_len"] == c["encoded_len"] == 250 and c["codes"].shape == (1, Hkv, 258, 32)
    enc = 250
    for T in range(251, 300):
        c = aqe._prepare_aq_cache(attn, m, 0, keys[:, :, :T].to(dev), need_recon=False, decode_group_size=16)
        if T - enc >= 16:  # a full encode group is pending: encoded at once
            enc = T
        assert c["seq_len"] == T and c["encoded_len"] == enc and c["codes"].shape[2] >= T
    torch.cuda.synchronize()
    n = c["encoded_len"]
    assert n == 298
    got = c["codes"][0, :, :n].cpu().numpy()
    for h in range(Hkv):
        want = oracle.encode_greedy(keys[0, h, :n].float().numpy(), cb[h].numpy())
        assert np.array_equal(got[h], want)


@pytest.mark.parametrize("mgr_dtype,tol", [(torch.float32, 2e-2), (torch.float16, 5e-2)])
def test_sharded_manager_drives_the_decode_hook(golden_dir, tmp_path, mgr_dtype, tol):
    """The per-device manager through the decode hook against the
    reference's own hook output (made with an fp32 manager).  An fp16
    manager scores from the fp16 codebook copy, as the reference's fp16
    manager does: the rounded codebooks move scores by about 1e-3 of their
    range, which can swap tokens at the selection threshold, so its bound is
    the looser 5e-2 (the kernels themselves are exact on the rounded values:
    test_half_precision_codebooks_select_like_their_fp32_values)."""
    from laprune_b200.aq_kv import ShardedAQLayerCodebookManager
    fix = np.load(golden_dir / "decode_hook.npz")
    dh = syn.decode_hook_case(11)
    _mgr(dh["cb"], dh["Hq"]).save(str(tmp_path))
    sh = ShardedAQLayerCodebookManager({0: AQLayerConfig(M=32, K=256, d=128, heads_per_group=dh["Hq"],
                                                         num_heads=dh["Hq"])}, str(tmp_path), devices=[_dev()],
                                       dtype=mgr_dtype)
    dev = _dev()
    conf = {"mask_out": 0.98, "min_remain": 20, "sink_size": 4, "local_window": 64, "aq_scoring_m": 32}
    self_attn = types.SimpleNamespace(total_seq_len=dh["T"], o_proj=torch.nn.Identity())
    out = aqe._decode_attention(self_attn, sh, 0, dh["q"].to(dev).half(), dh["keys"].to(dev).half(),
                                dh["vals"].to(dev).half(), {"codes": dh["codes"].to(dev), "seq_len": dh["T"]}, conf)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - fix["out_sink4"]).max() <= tol


@torch.no_grad()
def test_attention_forward_prefill_then_sparse_decode():
    # the reference's attention forward on a small Llama layer (head_dim 128,
    # GQA 4): a dense prefill that fills the code cache, then decode tokens
    # through the sparse path, each checked against the oracle's decode hook
    # on the same cache
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention, LlamaRotaryEmbedding, apply_rotary_pos_emb
    dev = _dev()
    cfg = LlamaConfig(hidden_size=512, num_attention_heads=4, num_key_value_heads=1, num_hidden_layers=4,
                      intermediate_size=1024, rope_theta=500000.0, max_position_embeddings=4096)
    g = torch.Generator().manual_seed(12)
    attn = LlamaAttention(cfg, layer_idx=2)
    for prm in attn.parameters():
        prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
    attn = attn.to(dev, torch.float16)
    attn.rotary_emb = LlamaRotaryEmbedding(cfg, device=dev)
    cb = torch.randn((32, 256, 128), generator=g) * 0.05
    attn.aq_manager = _mgr(cb, 4, layer=2)
    attn.draft_kwargs = {"sink_size": 0, "local_window": 64, "mask_out": 0.98, "min_remain": 20,
                         "aq_decode_group_size": 16, "aq_use_pruned_attn": True,
                         "aq_encode_icm_iters_prefill": 0, "aq_encode_icm_iters_decode": 0}
    attn.is_fix_layer = False
    fwd = types.MethodType(aqe.self_attn_forward, attn)
    T0 = 700
    _, kv, _, _ = fwd((torch.randn((1, T0, 512), generator=g) * 0.5).to(dev, torch.float16))
    for step in range(3):
        h1 = (torch.randn((1, 1, 512), generator=g) * 0.5).to(dev, torch.float16)
        out, kv, _, _ = fwd(h1, kv_cache=kv)
        torch.cuda.synchronize()
        total = T0 + step + 1
        q = attn.q_proj(h1).unflatten(-1, (4, 128)).transpose(1, 2)
        cos, sin = attn.rotary_emb(q, torch.tensor([[total - 1]], device=dev))
        q_rope, _ = apply_rotary_pos_emb(q, q[:, :1], cos, sin)
        c = attn._aq_cache
        ref = oracle.decode_hook_reference(cb.numpy(), q_rope.float().cpu().numpy(), c["codes"].cpu().numpy(),
                                           attn.k_cache[:, :, :total].float().cpu().numpy(),
                                           attn.v_cache[:, :, :total].float().cpu().numpy(), total, 0, 64)
        ref = ref @ attn.o_proj.weight.float().cpu().numpy().T
        got = out.float().cpu().numpy()
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()


def test_quantizer_encode_matches_the_oracle_and_its_loss():
    from laprune_b200.quantizer import AdditiveQuantizer
    g = torch.Generator().manual_seed(13)
    cb = torch.randn((32, 256, 128), generator=g) * 0.05
    x = torch.randn((333, 128), generator=g) * 0.5
    aq = AdditiveQuantizer(M=32, K=256, d=128, device=_dev(), codebooks=cb)
    codes, loss, extra = aq.encode(x.to(_dev()), icm_iters=0)
    want = oracle.encode_greedy(x.numpy(), cb.numpy()).astype(np.int64)
    assert codes.dtype == torch.int64 and extra is None
    assert np.array_equal(codes.cpu().numpy(), want)
    recon = cb.numpy()[np.arange(32)[None, :], want].sum(1)
    ref = np.sqrt(((x.numpy() - recon) ** 2).sum(1)).mean()
    assert abs(loss - ref) <= 1e-4 * ref
    codes2, loss2, _ = aq.encode(x.to(_dev()), icm_iters=0, return_loss=False)
    assert torch.equal(codes2, codes) and loss2 == 0.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_token_rope_append_equals_hf_rotation_and_slice_copy(dtype):
    """lp_rope_append against HF apply_rotary_pos_emb + the slice copies of
    the reference's _kv_cache_append (aq_evaluation.py:296-308, 65-112):
    rotated query, rotated key and value in slot `pos`, bit for bit, with
    Llama-3.1's rope scaling; every other cache slot untouched."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, apply_rotary_pos_emb
    from laprune_b200 import ops
    dev = _dev()
    cfg = LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8, rope_theta=500000.0,
                      max_position_embeddings=131072,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    rot = LlamaRotaryEmbedding(cfg, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    B, Hq, Hkv, D, cap, pos = 2, 32, 8, 128, 300, 257
    q = torch.randn((B, Hq, 1, D), generator=g, device=dev).to(dtype)
    k = torch.randn((B, Hkv, 1, D), generator=g, device=dev).to(dtype)
    v = torch.randn((B, Hkv, 1, D), generator=g, device=dev).to(dtype)
    kc = torch.randn((B, Hkv, cap, D), generator=g, device=dev).to(dtype)
    vc = torch.randn((B, Hkv, cap, D), generator=g, device=dev).to(dtype)
    kc0, vc0 = kc.clone(), vc.clone()
    cos, sin = rot(q, torch.full((B, 1), 100000, device=dev))
    q_rot = ops.rope_append(q, k, v, cos, sin, kc, vc, pos)
    q_ref, k_ref = apply_rotary_pos_emb(q, k, cos, sin)
    torch.cuda.synchronize()
    assert torch.equal(q_rot, q_ref[:, :, 0])
    assert torch.equal(kc[:, :, pos], k_ref[:, :, 0]) and torch.equal(vc[:, :, pos], v[:, :, 0])
    keep = torch.ones(cap, dtype=torch.bool)
    keep[pos] = False
    assert torch.equal(kc[:, :, keep], kc0[:, :, keep]) and torch.equal(vc[:, :, keep], vc0[:, :, keep])


@torch.no_grad()
def test_attention_forward_keeps_the_cache_contract():
    """The rewritten attention forward against the reference's contract: the
    cache views it returns, the buffers' capacity policy (first buffers
    total + aq_kv_extra_capacity, doubling when full) and the rotated keys
    in the cache (HF rotation) through prefill and decode tokens."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention, LlamaRotaryEmbedding, apply_rotary_pos_emb
    dev = _dev()
    cfg = LlamaConfig(hidden_size=512, num_attention_heads=4, num_key_value_heads=1, num_hidden_layers=4,
                      intermediate_size=1024, rope_theta=500000.0, max_position_embeddings=4096)
    g = torch.Generator().manual_seed(31)
    attn = LlamaAttention(cfg, layer_idx=0)
    for prm in attn.parameters():
        prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
    attn = attn.to(dev, torch.bfloat16)
    attn.rotary_emb = LlamaRotaryEmbedding(cfg, device=dev)
    attn.aq_manager = _mgr(torch.randn((32, 256, 128), generator=g) * 0.05, 4, layer=0)
    attn.draft_kwargs = {"aq_kv_extra_capacity": 3, "enable": False}
    attn.is_fix_layer = False
    fwd = types.MethodType(aqe.self_attn_forward, attn)
    T0 = 20
    hs = (torch.randn((1, T0, 512), generator=g) * 0.5).to(dev, torch.bfloat16)
    _, kv, _, _ = fwd(hs)
    assert attn.k_cache_capacity == T0 + 3 and attn.k_cache_len == T0
    for step in range(6):  # 3 tokens fill the extra slots, the 4th doubles the buffers
        h1 = (torch.randn((1, 1, 512), generator=g) * 0.5).to(dev, torch.bfloat16)
        _, kv, _, _ = fwd(h1, kv_cache=kv)
        total = T0 + step + 1
        assert attn.k_cache_len == total and kv[0].shape[2] == total
        assert attn.k_cache_capacity == (T0 + 3 if total <= T0 + 3 else 2 * (T0 + 3))
        assert kv[0].data_ptr() == attn.k_cache.data_ptr() and kv[0].stride(1) == attn.k_cache_capacity * 128
        k = attn.k_proj(h1).unflatten(-1, (1, 128)).transpose(1, 2)
        q = attn.q_proj(h1).unflatten(-1, (4, 128)).transpose(1, 2)
        cos, sin = attn.rotary_emb(q, torch.tensor([[total - 1]], device=dev))
        _, k_ref = apply_rotary_pos_emb(q, k, cos, sin)
        assert torch.equal(attn.k_cache[:, :, total - 1], k_ref[:, :, 0])
        assert torch.equal(attn.v_cache[:, :, total - 1], attn.v_proj(h1).unflatten(-1, (1, 128)).transpose(1, 2)[:, :, 0])
