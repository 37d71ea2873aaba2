"""The allocation-free entry point, lp_sparse_decode_noalloc.

Some callers cannot allocate device memory at decode time: a serving runtime
that has given all of HBM to its own memory pool (a cudaMalloc there fails or
fragments the pool), or a latency-critical decode loop in which cudaMalloc and
cudaFree would synchronise the device.  lp_sparse_decode_noalloc serves them
from a scratch array the library keeps in device memory.  These tests call it
through the C ABI and check it against lp_sparse_decode with a caller-owned
workspace.  The file is collected last on purpose, so that a run that stops at
the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from laprune_b200 import _lib, ops

ATTN_ATOL = 2e-2  # the attention tolerance of the other parity tests


def _case(seed, T=20000, Hkv=8, G=4):
    g = torch.Generator().manual_seed(seed)
    C = torch.randn((Hkv, 32, 256, 128), generator=g) * 0.05
    codes = torch.randint(0, 256, (1, Hkv, T, 32), generator=g, dtype=torch.uint8)
    K = torch.randn((1, Hkv, T, 128), generator=g).to(torch.bfloat16)
    V = torch.randn((1, Hkv, T, 128), generator=g).to(torch.bfloat16)
    q = torch.randn((1, Hkv * G, 128), generator=g).to(torch.bfloat16)
    return q, C, codes, K, V


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    dev = torch.device("cuda", 0)
    q, C, codes, K, V = (t.to(dev) for t in _case(21))
    k, sink, local = 400, 4, 64
    ref = ops.sparse_decode(q, C, codes, K, V, topk=k, sink=sink, local=local, return_topk=True)
    lib = _lib.load()
    stream = ops._stream_handle(dev)
    # every output exists before the first call, so that device memory in use
    # can only change through the entry point itself
    outs = [(torch.empty_like(ref.out), torch.empty((8, k), dtype=torch.int32, device=dev)) for _ in range(2)]
    torch.cuda.synchronize(dev)
    free = []
    for out, top in outs:  # the second call runs on the scratch the first one left behind
        a = ops.build_args(q, C, codes, K, V, topk=k, T_codes=None, T_total=None, sink=sink, local=local,
                           select="kv_group", scale=None, out=out, head_scores=None, topk_out=top,
                           prefetch=None)
        bits = ctypes.c_uint32(0xFFFFFFFF)
        with torch.cuda.device(dev):
            _lib.check(lib.lp_sparse_decode_noalloc(ctypes.byref(a), stream, ctypes.byref(bits)))
        torch.cuda.synchronize(dev)
        free.append(torch.cuda.mem_get_info(dev)[0])
        assert bits.value & _lib.LP_DEVERR_WAIT_TIMEOUT == 0
        assert torch.equal(top, ref.topk)
        assert (out.float() - ref.out.float()).abs().max().item() <= ATTN_ATOL
    # no device memory was taken by the second call (the first may have loaded
    # the library's device code into the context)
    assert free[1] == free[0]


def test_noalloc_rejects_a_geometry_beyond_its_scratch():
    # batch 8 at 128k tokens needs ~59 MiB of workspace; the check runs on
    # the host before any device work
    lib = _lib.load()
    a = _lib.SparseDecodeArgs()
    a.B, a.Hkv, a.G, a.D, a.M, a.K = 8, 8, 4, 128, 32, 256
    a.T_codes = a.T_total = 131072
    a.sink, a.local, a.topk = 4, 64, 2048
    a.select_mode = _lib.LP_SELECT_KV_GROUP
    a.q_dtype = a.kv_dtype = a.out_dtype = _lib.LP_BF16
    a.out = 1  # attention requested (never dereferenced: the call is rejected first)
    assert lib.lp_sparse_decode_workspace_size(ctypes.byref(a)) > _lib.LP_NOALLOC_SCRATCH_BYTES
    rc = lib.lp_sparse_decode_noalloc(ctypes.byref(a), None, None)
    assert rc == _lib.LP_ERR_WORKSPACE
    msg = lib.lp_last_error().decode()
    assert "built-in scratch" in msg and str(_lib.LP_NOALLOC_SCRATCH_BYTES) in msg
