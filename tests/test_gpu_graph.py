"""A multi-layer sparse decode step captured in a CUDA graph and replayed.

The decode loop of a serving runtime calls the fused step once per sparse
layer; capturing those calls in one CUDA graph removes the per-call host cost
(argument packing, the ctypes call, the launch).  The reference's decode hook
runs eagerly (aq_evaluation.py:146-253); a captured step must give the same
bits as eager calls on the same inputs, every replay, with the inputs read
live from their static buffers.
"""
import ctypes

import pytest
import torch

from laprune_b200 import _lib, ops

LAYERS = 3


def _layers(dev, T=20000, Hkv=8, G=4, seed=40):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(LAYERS):
        C = (torch.randn((Hkv, 32, 256, 128), generator=g) * 0.05).to(dev)
        codes = torch.randint(0, 256, (1, Hkv, T, 32), generator=g, dtype=torch.uint8).to(dev)
        K = torch.randn((1, Hkv, T, 128), generator=g).to(torch.bfloat16).to(dev)
        V = torch.randn((1, Hkv, T, 128), generator=g).to(torch.bfloat16).to(dev)
        out.append((C, codes, K, V))
    return out


def _q(seed, dev, Hq=32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((1, Hq, 128), generator=g).to(torch.bfloat16).to(dev)


@pytest.mark.gpu
def test_graph_replay_of_a_multi_layer_step_matches_eager_calls():
    dev = torch.device("cuda", 0)
    k, sink, local = 400, 4, 64
    layers = _layers(dev)
    q_static = [torch.empty((1, 32, 128), dtype=torch.bfloat16, device=dev) for _ in range(LAYERS)]
    out_static = [torch.empty((1, 32, 128), dtype=torch.bfloat16, device=dev) for _ in range(LAYERS)]
    top_static = [torch.empty((8, k), dtype=torch.int32, device=dev) for _ in range(LAYERS)]

    # one caller-owned workspace shared by every layer call, eager and captured:
    # its persistent words (launch counter, barriers) must survive the capture
    lib = _lib.load()

    def args(l, outs, tops):
        C, codes, K, V = layers[l]
        return ops.build_args(q_static[l], C, codes, K, V, topk=k, sink=sink, local=local,
                              out=outs[l], topk_out=tops[l])

    need = max(lib.lp_sparse_decode_workspace_size(ctypes.byref(args(l, out_static, top_static)))
               for l in range(LAYERS))
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)

    def step(outs, tops):
        for l in range(LAYERS):
            a = args(l, outs, tops)
            _lib.check(lib.lp_sparse_decode(ctypes.byref(a), ws.data_ptr(), ws.numel(),
                                            ops._stream_handle(dev)))

    def eager(seed):
        for l in range(LAYERS):
            q_static[l].copy_(_q(seed + l, dev))
        outs = [torch.empty_like(o) for o in out_static]
        tops = [torch.empty_like(t) for t in top_static]
        step(outs, tops)
        torch.cuda.synchronize(dev)
        return outs, tops

    with torch.cuda.device(dev):
        eager(100)  # first calls on this device: attribute set-up happens outside the capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(out_static, top_static)
        torch.cuda.synchronize(dev)
        for seed in (200, 300, 200):
            ref_out, ref_top = eager(seed)
            for l in range(LAYERS):
                q_static[l].copy_(_q(seed + l, dev))
            out_static[0].fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize(dev)
            for l in range(LAYERS):
                assert torch.equal(top_static[l], ref_top[l]), f"layer {l}, seed {seed}: top-k differs"
                assert torch.equal(out_static[l], ref_out[l]), f"layer {l}, seed {seed}: output differs"
        assert ops.device_errors(ws, dev) == 0
        del graph
