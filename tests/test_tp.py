"""KV-head tensor parallelism (laprune_b200.tp) on CPU ranks (gloo).

The shard math is checked with the oracle as the per-rank compute: every
rank decodes only its KV heads, the outputs are all-gathered over gloo, and
the result must equal the unsharded decode bit for bit (the heads are
independent, so the split changes no arithmetic).  A rank that fails before
the collective must surface as an error on the other rank, not a hang.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from laprune_b200 import tp

B, HKV, G, T, D, M, K = 2, 4, 4, 600, 128, 32, 256
TOPK, SINK, LOCAL = 64, 4, 16


def _problem():
    g = torch.Generator().manual_seed(21)
    C = torch.randn((HKV, M, K, D), generator=g) * 0.05
    codes = torch.randint(0, 256, (B, HKV, T, M), generator=g, dtype=torch.uint8)
    keys = torch.randn((B, HKV, T, D), generator=g).to(torch.bfloat16)
    vals = torch.randn((B, HKV, T, D), generator=g).to(torch.bfloat16)
    q = torch.randn((B, HKV * G, D), generator=g).to(torch.bfloat16)
    return q, C, codes, keys, vals


def _decode_oracle(q, C, codes, keys, vals):
    import oracle
    outs, tops = [], []
    for b in range(q.shape[0]):
        _, top, _, out = oracle.decode_step_group(
            np.ascontiguousarray(C.numpy()), np.ascontiguousarray(q[b].float().numpy()),
            np.ascontiguousarray(codes[b].numpy()), np.ascontiguousarray(keys[b].float().numpy()),
            np.ascontiguousarray(vals[b].float().numpy()), TOPK, SINK, LOCAL, G)
        outs.append(out)
        tops.append(top)
    return torch.from_numpy(np.stack(outs)), np.stack(tops)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, results):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", init_method="env://", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        q, C, codes, keys, vals = _problem()
        sh = tp.shard_decode_inputs(q, C, codes, keys, vals, world, rank)
        out_local, _ = _decode_oracle(sh["q"], sh["codebooks"], sh["codes"], sh["keys"], sh["vals"])
        full = tp.gather_heads(out_local)
        if rank == 0:
            want, _ = _decode_oracle(q, C, codes, keys, vals)
            results.put(("equal", bool(torch.equal(full, want)), tuple(full.shape)))
        dist.barrier()
    except Exception as e:  # reported to the parent, never swallowed silently
        results.put(("error", rank, f"{type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not results.empty():
        out.append(results.get())
    return out, alive


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_kv_head_ranges_partition_the_heads(world):
    seen = []
    for r in range(world):
        h0, h1 = tp.kv_head_range(8, world, r)
        q0, q1 = tp.query_head_range(32, 8, world, r)
        assert (h1 - h0) == 8 // world and (q0, q1) == (4 * h0, 4 * h1)
        seen.extend(range(h0, h1))
    assert seen == list(range(8))


def test_uneven_split_and_bad_rank_are_rejected():
    with pytest.raises(ValueError):
        tp.kv_head_range(8, 3, 0)
    with pytest.raises(ValueError):
        tp.kv_head_range(8, 2, 2)
    with pytest.raises(ValueError):
        tp.query_head_range(30, 8, 2, 0)


def test_shards_are_views_of_the_owned_heads():
    q, C, codes, keys, vals = _problem()
    sh = tp.shard_decode_inputs(q, C, codes, keys, vals, 2, 1)
    assert sh["kv_heads"] == (2, 4) and sh["q_heads"] == (8, 16)
    assert sh["codes"].data_ptr() == codes[:, 2].data_ptr()
    assert torch.equal(sh["keys"], keys[:, 2:4]) and torch.equal(sh["q"], q[:, 8:16])
    assert torch.equal(sh["codebooks"], C[2:4])
    shared = tp.shard_decode_inputs(q, C[0], codes, keys, vals, 2, 1)
    assert shared["codebooks"].shape == (M, K, D)


def test_two_gloo_ranks_reproduce_the_unsharded_decode():
    out, alive = _run(2)
    assert not alive, "a rank did not finish"
    assert out == [("equal", True, (B, HKV * G, D))], out


def test_failed_rank_surfaces_as_an_error_on_the_other():
    out, alive = _run(2, fail_rank=1, timeout=90)
    assert not alive, "a rank hung after its peer failed"
    errs = {r: msg for kind, r, msg in (o for o in out if o[0] == "error")}
    assert "injected rank failure" in errs.get(1, "")
    assert 0 in errs, f"rank 0 did not see the failure: {out}"
