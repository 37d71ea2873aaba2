"""The aq_kernels-named drop-in surface against the oracle's restatements of
the reference entry points (aq_kernels/aq_lut.cu, aq_lut_gqa.cu,
fused_linear_encode.cu)."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def aqk():
    from laprune_b200 import aq_kernels
    return aq_kernels


def _lut_codes(seed, H=32, Hkv=8, T=300, cap=320):
    g = torch.Generator().manual_seed(seed)
    lut = (torch.randn((H, 32, 256), generator=g)).to(torch.float16)
    full = torch.randint(0, 256, (Hkv, cap, 32), generator=g, dtype=torch.uint8)
    return lut, full[:, :T]  # strided codes view, as the reference's code cache


def test_exports_match_the_reference_package(aqk):
    for name in ("aq_lut_forward", "aq_lut_gather_forward", "aq_lut_gather_gqa", "aq_lut_gather_grouped",
                 "gqa_gather_kv", "gqa_gather_kv_with_tail", "fused_linear_encode_forward"):
        assert callable(getattr(aqk, name))


def test_lut_gather_grouped(aqk):
    lut, codes = _lut_codes(1)
    dev = _dev()
    got = aqk.aq_lut_gather_grouped(lut.to(dev), codes.to(dev), 4)
    torch.cuda.synchronize()
    want = oracle.lut_gather_grouped_f16(lut.numpy(), codes.numpy(), 4)
    assert got.dtype == torch.float16 and tuple(got.shape) == (32, 300)
    assert np.array_equal(got.cpu().numpy(), want)


def test_lut_gather_gqa_range_and_indices(aqk):
    lut, codes = _lut_codes(2, T=200)
    dev = _dev()
    dense = aqk.aq_lut_gather_gqa(lut.to(dev), codes.to(dev), 4, 4, 20)
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(-3, 205, (32, 57), generator=g, dtype=torch.int64)  # some out of [0, T)
    sparse = aqk.aq_lut_gather_gqa(lut.to(dev), codes.to(dev), 4, 0, 32, idx.to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(dense.cpu().numpy(), oracle.lut_gather_gqa_f16(lut.numpy(), codes.numpy(), 4, 4, 20))
    assert np.array_equal(sparse.cpu().numpy(),
                          oracle.lut_gather_gqa_f16(lut.numpy(), codes.numpy(), 4, 0, 32, idx.numpy()))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_lut_gather_forward(aqk, dtype):
    g = torch.Generator().manual_seed(3)
    Q, N, M, K = 6, 90, 32, 256
    lut = torch.randn((Q, M * K), generator=g).to(dtype)
    codes = torch.randint(0, 300, (Q, N, M), generator=g, dtype=torch.int64)  # read as bytes
    dev = _dev()
    got = aqk.aq_lut_gather_forward(lut.to(dev), codes.to(dev))
    torch.cuda.synchronize()
    want = oracle.lut_gather_forward(lut.numpy(), codes.numpy())
    assert got.dtype == dtype
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("dtype,rtol", [(torch.float32, 1e-4), (torch.float16, 1e-2)])
def test_lut_forward(aqk, dtype, rtol):
    g = torch.Generator().manual_seed(4)
    Q, N, M, K, d = 3, 40, 32, 256, 128
    q = torch.randn((Q, d), generator=g).to(dtype)
    cb = (torch.randn((M, K, d), generator=g) * 0.05).to(dtype)
    codes = torch.randint(0, 256, (Q, N, M), generator=g, dtype=torch.uint8)
    dev = _dev()
    got = aqk.aq_lut_forward(q.to(dev), cb.to(dev), codes.to(dev))
    torch.cuda.synchronize()
    want = oracle.lut_forward(q.numpy(), cb.numpy(), codes.numpy()).astype(np.float32)
    assert got.dtype == dtype
    assert np.abs(got.float().cpu().numpy() - want).max() <= rtol * np.abs(want).max()


def _gather_ref(keys, vals, idx, G, tail_start=0, tail_count=0):
    B, Hkv, T, D = keys.shape
    Hq, Ne = idx.shape[1], idx.shape[2]
    ok = torch.zeros((B, Hq, Ne + tail_count, D), dtype=keys.dtype)
    ov = torch.zeros_like(ok)
    for b in range(B):
        for h in range(Hq):
            toks = list(idx[b, h].tolist()) + list(range(tail_start, tail_start + tail_count))
            for n, t in enumerate(toks):
                if 0 <= t < T:
                    ok[b, h, n] = keys[b, h // G, t]
                    ov[b, h, n] = vals[b, h // G, t]
    return ok, ov


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gqa_gather_kv_and_tail(aqk, dtype):
    g = torch.Generator().manual_seed(6)
    B, Hkv, G, cap, T, D = 2, 2, 4, 64, 50, 128
    kf = torch.randn((B, Hkv, cap, D), generator=g).to(dtype)
    vf = torch.randn((B, Hkv, cap, D), generator=g).to(dtype)
    keys, vals = kf[:, :, :T], vf[:, :, :T]  # strided cache views
    idx = torch.randint(-2, T + 3, (B, Hkv * G, 11), generator=g, dtype=torch.int64)
    dev = _dev()
    k1, v1 = aqk.gqa_gather_kv(keys.to(dev), vals.to(dev), idx.to(dev), G)
    k2, v2 = aqk.gqa_gather_kv_with_tail(keys.to(dev), vals.to(dev), idx.to(dev), G, T - 7, 7)
    torch.cuda.synchronize()
    rk, rv = _gather_ref(keys, vals, idx, G)
    assert torch.equal(k1.cpu(), rk) and torch.equal(v1.cpu(), rv)
    rk, rv = _gather_ref(keys, vals, idx, G, T - 7, 7)
    assert torch.equal(k2.cpu(), rk) and torch.equal(v2.cpu(), rv)


def test_fused_linear_encode_forward(aqk):
    g = torch.Generator().manual_seed(8)
    M, K, d, N = 32, 256, 128, 100
    cb = torch.randn((M, K, d), generator=g) * 0.05
    x = (torch.randn((N, d), generator=g) * 0.5).to(torch.float16)
    weight_t = cb.permute(0, 2, 1).contiguous().to(torch.float16)
    bias = (-0.5 * (cb * cb).sum(-1)).to(torch.float16)
    dev = _dev()
    got = aqk.fused_linear_encode_forward(x.to(dev), weight_t.to(dev), bias.to(dev), cb.to(torch.float16).to(dev))
    torch.cuda.synchronize()
    want = oracle.encode_greedy(x.float().numpy(), cb.to(torch.float16).float().numpy())
    assert got.dtype == torch.uint8 and tuple(got.shape) == (N, M)
    assert np.array_equal(got.cpu().numpy(), want)
