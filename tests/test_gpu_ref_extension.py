"""The ``aq_kernels`` drop-ins against the reference's OWN CUDA extension.

``oracle/build_ref.py`` compiles the reference's three extension sources
(aq_kernels/aq_lut.cu, aq_lut_gqa.cu, fused_linear_encode.cu) unchanged for
sm_100a into ``oracle/_ref``; here both run on the same GPU on the same
seeded inputs.  The LUT gathers and the K/V gathers must agree bit for bit
(both sum fp16 table entries in fp32 in codebook order and round once);
``aq_lut_forward`` (the reference dots every codeword with q per token, this
package builds an fp32 table first) within fp16 rounding; the encoder
(the reference keeps an fp16 residual, this package the exact fp32 greedy
arithmetic of the reference's CPU path) by its agreement rate and its
reconstruction error.
"""
import numpy as np
import pytest
import torch

from oracle import build_ref

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not all(build_ref.available(n) for n in build_ref.NAMES),
                       reason="reference extension not built (python -m oracle.build_ref)"),
]


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ref():
    return {n: build_ref.load(n) for n in build_ref.NAMES}


@pytest.fixture(scope="module")
def aqk():
    from laprune_b200 import aq_kernels
    return aq_kernels


def _inputs(seed, H=32, Hkv=8, T=4000, cap=4160):
    g = torch.Generator().manual_seed(seed)
    lut = torch.randn((H, 32, 256), generator=g).to(torch.float16)
    full = torch.randint(0, 256, (Hkv, cap, 32), generator=g, dtype=torch.uint8)
    dev = _dev()
    return lut.to(dev), full.to(dev)[:, :T]  # strided prefix of a code cache, as the decode hook's


@pytest.mark.parametrize("G", [4, 2, 1])
def test_grouped_scan_equals_the_reference(ref, aqk, G):
    lut, codes = _inputs(11, H=8 * G)
    got = aqk.aq_lut_gather_grouped(lut, codes, G)
    want = ref["aq_lut_gqa"].aq_lut_gather_grouped(lut, codes, G)
    torch.cuda.synchronize()
    assert got.dtype == want.dtype and got.shape == want.shape
    assert torch.equal(got, want)


def test_range_and_index_gather_equal_the_reference(ref, aqk):
    lut, codes = _inputs(12)
    T = codes.shape[1]
    g = torch.Generator().manual_seed(13)
    idx = torch.randint(-5, T + 5, (32, 777), generator=g, dtype=torch.int64).to(_dev())
    for m0, m1, ix in ((0, 32, None), (4, 20, None), (0, 32, idx), (7, 9, idx)):
        got = aqk.aq_lut_gather_gqa(lut, codes, 4, m0, m1, ix)
        want = ref["aq_lut_gqa"].aq_lut_gather(lut, codes, 4, m0, m1, ix)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (m0, m1, ix is not None)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_flat_gather_forward_equals_the_reference(ref, aqk, dtype):
    g = torch.Generator().manual_seed(14)
    Q, N, M, K = 16, 3000, 32, 256
    lut = torch.randn((Q, M * K), generator=g).to(dtype).to(_dev())
    for cdt in (torch.uint8, torch.int64):
        hi = 400 if cdt == torch.int64 else 256  # int64 codes are read by their low byte
        codes = torch.randint(0, hi, (Q, N, M), generator=g, dtype=torch.int64).to(cdt).to(_dev())
        got = aqk.aq_lut_gather_forward(lut, codes)
        want = ref["aq_lut"].aq_lut_gather_forward(lut, codes)
        torch.cuda.synchronize()
        assert got.dtype == want.dtype
        assert torch.equal(got, want), cdt


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_lut_forward_matches_the_reference(ref, aqk, dtype):
    g = torch.Generator().manual_seed(15)
    Q, N, M, K, d = 8, 500, 32, 256, 128
    q = torch.randn((Q, d), generator=g).to(dtype).to(_dev())
    cb = (torch.randn((M, K, d), generator=g) * 0.05).to(dtype).to(_dev())
    codes = torch.randint(0, 256, (Q, N, M), generator=g, dtype=torch.uint8).to(_dev())
    got = aqk.aq_lut_forward(q, cb, codes)
    want = ref["aq_lut"].aq_lut_forward(q, cb, codes)
    torch.cuda.synchronize()
    assert got.dtype == want.dtype
    # fp32: both exact sums in different orders; fp16: one fp16 rounding of the output
    tol = 1e-5 if dtype == torch.float32 else 2e-3
    err = (got.float() - want.float()).abs().max().item()
    assert err <= tol * want.float().abs().max().item(), err


@pytest.mark.parametrize("with_tail", [False, True])
def test_kv_gather_equals_the_reference(ref, aqk, with_tail):
    g = torch.Generator().manual_seed(16)
    B, Hkv, G, cap, T, D = 2, 8, 4, 2300, 2200, 128
    kf = torch.randn((B, Hkv, cap, D), generator=g).to(torch.float16).to(_dev())
    vf = torch.randn((B, Hkv, cap, D), generator=g).to(torch.float16).to(_dev())
    keys, vals = kf[:, :, :T], vf[:, :, :T]  # strided cache prefixes
    # in-range indices only: the reference leaves rows of out-of-range indices unwritten
    idx = torch.randint(0, T - 64, (B, Hkv * G, 437), generator=g, dtype=torch.int64).to(_dev())
    if with_tail:
        got = aqk.gqa_gather_kv_with_tail(keys, vals, idx, G, T - 64, 64)
        want = ref["aq_lut_gqa"].gqa_gather_kv_with_tail(keys, vals, idx, G, T - 64, 64)
    else:
        got = aqk.gqa_gather_kv(keys, vals, idx, G)
        want = ref["aq_lut_gqa"].gqa_gather_kv(keys, vals, idx, G)
    torch.cuda.synchronize()
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])


@pytest.mark.parametrize("N", [512, 2048])
def test_encode_agrees_with_the_reference_kernel(ref, aqk, N):
    """N = 512 runs the reference's single fused kernel, N = 2048 its
    cuBLAS-tiled path.  The reference's fp16 residual drifts from exact
    arithmetic stage by stage, so full rows need not agree; the first stage
    (no residual yet) agrees except at fp16 near-ties, and the exact greedy
    codes reconstruct the keys at least as well on average."""
    g = torch.Generator().manual_seed(17)
    M, K, d = 32, 256, 128
    cb = (torch.randn((M, K, d), generator=g) * 0.05).to(torch.float16)
    x = torch.randn((N, d), generator=g).to(torch.float16)
    weight_t = cb.permute(0, 2, 1).contiguous()
    bias = (-0.5 * cb.float().pow(2).sum(-1)).to(torch.float16)
    dev = _dev()
    args = (x.to(dev), weight_t.to(dev), bias.to(dev), cb.to(dev), True, 0)
    got = aqk.fused_linear_encode_forward(*args)
    want = ref["fused_linear_encode"].fused_linear_encode_forward(*args)
    torch.cuda.synchronize()
    assert got.dtype == want.dtype == torch.uint8 and got.shape == want.shape == (N, M)
    stage0 = (got[:, 0] == want[:, 0]).float().mean().item()
    assert stage0 >= 0.99, stage0

    C = cb.float().to(dev)

    def recon_err(codes):
        r = x.float().to(dev).clone()
        for m in range(M):
            r -= C[m][codes[:, m].long()]
        return r.norm(dim=1).mean().item()

    assert recon_err(got) <= recon_err(want) * 1.001
