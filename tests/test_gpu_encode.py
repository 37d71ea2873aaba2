"""Parity of the tcgen05 key encoder (lp_encode_keys) with the oracle / reference.

The encoder follows the CPU arithmetic exactly (sequential fp32 fused
multiply-adds, first minimum on ties), so its codes must equal the oracle's
bit for bit; the oracle itself is pinned to the reference's codes (golden
fixture: rows may differ only where the reference's own fp32 distances tie
within 1e-4, north-star bar "codes bit-exact except at documented fp
near-ties").
"""
import numpy as np
import pytest
import torch

import oracle
from laprune_b200 import ops
from laprune_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _oracle_codes(keys, C):
    """oracle codes [B,H,T,32] for keys [B,H,T,128] and codebooks [H,32,256,128] or [32,256,128]."""
    B, H, T, D = keys.shape
    x = keys.permute(1, 0, 2, 3).reshape(H * B * T, D).float().numpy()
    if C.dim() == 4:
        cbi = np.repeat(np.arange(H, dtype=np.int32), B * T)
        codes = oracle.encode_greedy(x, C.numpy(), cbi)
    else:
        codes = oracle.encode_greedy(x, C.numpy())
    return codes.reshape(H, B, T, 32).transpose(1, 0, 2, 3)


def test_cfg2_codes_equal_the_oracle_and_agree_with_the_reference(golden_dir):
    fix = np.load(golden_dir / "cfg2_encode.npz")
    c = syn.config2(0)
    dev = _dev()
    codes = ops.encode_keys(c["keys"].to(dev), c["C"].to(dev))
    torch.cuda.synchronize()
    got = codes.cpu().numpy()
    want = _oracle_codes(c["keys"], c["C"])
    assert np.array_equal(got, want)
    # agreement with the reference's own codes (the oracle's near-tie rule)
    ref = fix["codes"]
    rows_equal = (got == ref).all(-1)
    assert rows_equal.mean() >= 0.99, f"row agreement {rows_equal.mean():.4f}"


def test_tensor_core_filter_matches_all_exact_distances():
    c = syn.config2(1)
    dev = _dev()
    keys, C = c["keys"].to(dev), c["C"].to(dev)
    a = ops.encode_keys(keys, C)
    b = ops.encode_keys(keys, C, exact=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_shared_codebook_ragged_count(dtype):
    g = torch.Generator().manual_seed(3)
    C = torch.randn((32, 256, 128), generator=g) * 0.05
    x = (torch.randn((300, 128), generator=g) * 0.7).to(dtype)
    dev = _dev()
    got = ops.encode_keys(x.to(dev), C.to(dev))
    torch.cuda.synchronize()
    want = oracle.encode_greedy(x.float().numpy(), C.numpy())
    assert np.array_equal(got.cpu().numpy(), want)


def test_equal_distances_take_the_first_codeword():
    # duplicated codewords tie exactly: the first index must win every stage
    g = torch.Generator().manual_seed(4)
    C = torch.randn((32, 256, 128), generator=g) * 0.05
    C[:, 128:] = C[:, :128]
    x = torch.randn((64, 128), generator=g) * 0.5
    dev = _dev()
    got = ops.encode_keys(x.to(dev), C.to(dev)).cpu().numpy()
    want = oracle.encode_greedy(x.numpy(), C.numpy())
    assert np.array_equal(got, want)
    assert (got < 128).all()


def test_codes_written_into_a_cache_slice_score_like_the_reference(golden_dir):
    fix = np.load(golden_dir / "cfg2_encode.npz")
    c = syn.config2(0)
    dev = _dev()
    cache = c["code_cache"].to(dev)
    p0 = c["pos0"]
    before = cache.clone()
    ops.encode_keys(c["keys"].to(dev), c["C"].to(dev), codes=cache[:, :, p0:p0 + 64])
    torch.cuda.synchronize()
    # untouched outside the slice
    assert torch.equal(cache[:, :, :p0], before[:, :, :p0])
    assert torch.equal(cache[:, :, p0 + 64:], before[:, :, p0 + 64:])
    r = ops.sparse_decode(c["q"].to(dev), c["C"].to(dev), cache, topk=0, sink=0, local=0,
                          attention=False, return_head_scores=True)
    torch.cuda.synchronize()
    hs = r.head_scores.cpu().numpy()[:, :, fix["sample"]]
    ref = fix["scores"]
    assert np.abs(hs - ref).max() <= 1e-3 * np.abs(ref).max()


@pytest.mark.parametrize("B,H,T,per_head,rows", [
    (1, 8, 4096, True, 128),    # prefill chunk: 1 x 8 KV heads x 4096 keys, 256 CTAs of 128 vectors
    (1, 1, 12288, False, 128),  # 12k vectors on one shared codebook, 96 CTAs of 128
    (1, 8, 1024, True, 64),     # 8 x 1024: 128 CTAs of 64 vectors (2 copies of the rows in the MMA tile)
    (1, 8, 512, True, 32),      # 8 x 512: 128 CTAs of 32 vectors (4 copies)
    (1, 8, 256, True, 16),      # 8 x 256: 128 CTAs of 16 vectors (8 copies)
])
def test_large_tiles_equal_the_oracle(B, H, T, per_head, rows):
    """Every CTA tile (128, 64, 32 and 16 vectors), each checked to be the
    tile the library picks and bit-exact with the oracle."""
    g = torch.Generator().manual_seed(20 + rows + H)
    C = torch.randn((H, 32, 256, 128) if per_head else (32, 256, 128), generator=g) * 0.05
    keys = torch.randn((B, H, T, 128), generator=g).to(torch.bfloat16)
    dev = _dev()
    kd, cd = keys.to(dev), C.to(dev)
    assert ops.encode_rows_per_cta(kd, cd) == rows
    got = ops.encode_keys(kd, cd)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), _oracle_codes(keys, C))


def test_icm_codes_equal_the_oracle_and_the_reference(golden_dir):
    """ICM refinement with the reference's default two sweeps
    (quantizer.py:356-370): config 2 on per-KV-head codebooks and the small
    shared-codebook case, bit-exact with the oracle and agreeing with the
    reference's own codes (golden fixture)."""
    fix = np.load(golden_dir / "icm_encode.npz")
    c = syn.config2(0)
    dev = _dev()
    got = ops.encode_keys(c["keys"].to(dev), c["C"].to(dev), icm_iters=2).cpu().numpy()
    B, H, T, D = c["keys"].shape
    x = c["keys"].permute(1, 0, 2, 3).reshape(H * B * T, D).float().numpy()
    cbi = np.repeat(np.arange(H, dtype=np.int32), B * T)
    want = oracle.encode_icm(x, c["C"].numpy(), 2, cbi).reshape(H, B, T, 32).transpose(1, 0, 2, 3)
    assert np.array_equal(got, want)
    assert (got == fix["codes_cfg2"]).all(-1).mean() >= 0.99
    sm = syn.small_shared(7)
    got_s = ops.encode_keys(sm["x"].to(dev), sm["cb"].to(dev), icm_iters=2).cpu().numpy()
    assert np.array_equal(got_s, oracle.encode_icm(sm["x"].float().numpy(), sm["cb"].numpy(), 2))
    assert (got_s == fix["codes_small"]).all(-1).mean() >= 0.99


def test_icm_sets_stop_at_their_own_sweep():
    """Many sweeps: each codebook set stops after its first sweep without a
    change (the sets converge after different numbers of sweeps), exactly as
    the oracle's per-set early exit."""
    g = torch.Generator().manual_seed(61)
    H = 3
    C = torch.randn((H, 32, 256, 128), generator=g) * 0.05
    keys = torch.randn((1, H, 50, 128), generator=g) * torch.tensor([0.3, 1.0, 2.0]).view(1, H, 1, 1)
    dev = _dev()
    got = ops.encode_keys(keys.to(dev), C.to(dev), icm_iters=40).cpu().numpy()
    x = keys[0].reshape(H * 50, 128).numpy()
    cbi = np.repeat(np.arange(H, dtype=np.int32), 50)
    want, sweeps = oracle.encode_icm(x, C.numpy(), 40, cbi, return_sweeps=True)
    assert np.array_equal(got[0].reshape(H * 50, 32), want)
    assert (sweeps < 40).all() and len(set(sweeps.tolist())) > 1, sweeps


def test_reference_default_arguments_refine_with_icm():
    """The manager's encode_keys(_batch) and AdditiveQuantizer.encode default
    to icm_iters=2 (aq_kv.py:354, 396; quantizer.py:319): called with the
    reference's defaults they now return the ICM-refined codes."""
    from laprune_b200.aq_kv import AQLayerCodebookManager, AQLayerConfig
    from laprune_b200.quantizer import AdditiveQuantizer
    g = torch.Generator().manual_seed(62)
    C = torch.randn((32, 256, 128), generator=g) * 0.05
    x = torch.randn((300, 128), generator=g)
    dev = _dev()
    want = oracle.encode_icm(x.numpy(), C.numpy(), 2)
    m = AQLayerCodebookManager({0: AQLayerConfig(M=32, K=256, d=128, heads_per_group=8, num_heads=8)}, device=dev)
    m.set_codebooks(0, 0, C)
    assert np.array_equal(m.encode_keys(0, 3, x).cpu().numpy(), want)
    assert np.array_equal(m.encode_keys_batch(0, 0, x).cpu().numpy(), want)
    aq = AdditiveQuantizer(M=32, K=256, d=128, device=dev, codebooks=C)
    codes, loss, _ = aq.encode(x)
    assert codes.dtype == torch.int64 and np.array_equal(codes.cpu().numpy(), want.astype(np.int64))
    recon = sum(C[m_][torch.from_numpy(want[:, m_]).long()] for m_ in range(32))
    assert abs(loss - float(torch.sqrt(((x - recon) ** 2).sum(1)).mean())) <= 1e-4
