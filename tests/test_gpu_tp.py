"""KV-head shards through the CUDA path: each rank's views (strided slices of
the full caches) run through ops.sparse_decode on one GPU, one rank after the
other.  The selected token sets must equal the unsharded call's rows for the
same heads (selection is exact, independent of how many units a launch
holds), and the attention outputs must agree within the bf16 tolerance of
the north-star bar (the split-K partition of a unit depends on the launch's
unit count, so the last bits may differ)."""
import pytest
import torch

from laprune_b200 import ops, tp

pytestmark = pytest.mark.gpu

B, HKV, G, T, D, M, K = 2, 8, 4, 8192, 128, 32, 256
TOPK, SINK, LOCAL = 256, 4, 64


def _problem(dev):
    g = torch.Generator(device=dev).manual_seed(5)
    C = torch.randn((HKV, M, K, D), generator=g, device=dev) * 0.05
    codes = torch.randint(0, 256, (B, HKV, T, M), generator=g, device=dev, dtype=torch.uint8)
    keys = torch.randn((B, HKV, T, D), generator=g, device=dev).to(torch.bfloat16)
    vals = torch.randn((B, HKV, T, D), generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((B, HKV * G, D), generator=g, device=dev).to(torch.bfloat16)
    return q, C, codes, keys, vals


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_match_the_unsharded_step(world):
    dev = torch.device("cuda", 0)
    q, C, codes, keys, vals = _problem(dev)
    full = ops.sparse_decode(q, C, codes, keys, vals, topk=TOPK, sink=SINK, local=LOCAL, return_topk=True)
    outs = []
    for r in range(world):
        sh = tp.shard_decode_inputs(q, C, codes, keys, vals, world, r)
        res = ops.sparse_decode(sh["q"], sh["codebooks"], sh["codes"], sh["keys"], sh["vals"], topk=TOPK,
                                sink=SINK, local=LOCAL, return_topk=True)
        h0, h1 = sh["kv_heads"]
        want = full.topk.view(B, HKV, TOPK)[:, h0:h1].reshape(-1, TOPK)
        assert torch.equal(res.topk, want), f"rank {r}: selected sets differ"
        outs.append(res.out)
    torch.cuda.synchronize()
    got = torch.cat(outs, dim=1).float()
    assert (got - full.out.float()).abs().max().item() <= 2e-2
