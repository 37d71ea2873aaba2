"""Parity of the fused CUDA sparse-decode pipeline with the oracle / reference.

Bars (from the north-star definition of correctness):
  * scores within 1e-3 relative (fp32), here max|a-b| <= 1e-3 * max|ref|;
  * top-k index sets >= 99.9% overlap (ties at the k-th value count);
  * attention outputs within bf16 tolerance: max abs err <= 2e-2.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from laprune_b200 import _lib, ops
from laprune_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

SCORE_RTOL = 1e-3
ATTN_ATOL = 2e-2


def _dev():
    return torch.device("cuda", 0)


def _overlap(sel, ref, scores_ref, kth, tol):
    return oracle.topk_overlap(sel, ref, scores_ref, kth, tol=tol)


def _check_errors():
    assert ops.device_errors(device=_dev()) & 1 == 0, "a bounded device wait timed out"


def test_cfg1_scoring_op(golden_dir):
    fix = np.load(golden_dir / "cfg1_scoring.npz")
    c = syn.config1(0)
    dev = _dev()
    C, codes, q = c["C"].to(dev), c["codes"].to(dev), c["q"].to(dev)
    T = codes.shape[1]
    # per-head scores (HEADS tables) + per-KV-head top-k on summed scores
    r = ops.sparse_decode(q, C, codes, topk=c["k"], sink=0, local=0, attention=False,
                          return_topk=True, return_head_scores=True)
    hs = r.head_scores[0].cpu().numpy()
    ref = fix["scores"]
    assert np.abs(hs - ref).max() <= SCORE_RTOL * np.abs(ref).max()
    gs_ref = ref.reshape(8, 4, T).sum(1)
    top = r.topk.cpu().numpy()
    for h in range(8):
        assert _overlap(top[h], fix["topk"][h], gs_ref[h], fix["kth"][h], 1e-3) >= 0.999
    # GROUP tables (summed query) give the same selection
    r2 = ops.sparse_decode(q, C, codes, topk=c["k"], sink=0, local=0, attention=False, return_topk=True)
    top2 = r2.topk.cpu().numpy()
    for h in range(8):
        assert _overlap(top2[h], fix["topk"][h], gs_ref[h], fix["kth"][h], 1e-3) >= 0.999
    _check_errors()


MODES = {"auto": dict(fused=None), "exchange": dict(fused=None, exchange_select=True), "multi": dict(fused=False)}


@pytest.mark.parametrize("mode", list(MODES))
def test_cfg3_sparse_decode_step(golden_dir, mode):
    fix = np.load(golden_dir / "cfg3_decode.npz")
    c = syn.config3(0)
    dev = _dev()
    C, codes, K, V, q = (c[n].to(dev) for n in ("C", "codes", "keys", "vals", "q"))
    r = ops.sparse_decode(q, C, codes, K, V, topk=c["k"], sink=c["sink"], local=c["local"],
                          return_topk=True, **MODES[mode])
    torch.cuda.synchronize()
    top = r.topk.cpu().numpy()
    T = codes.shape[1]
    gs_ref = oracle.group_sum(oracle.scores_per_kv_head(c["C"].numpy(), c["q"].float().numpy(),
                                                        c["codes"].numpy(), 4), 4)
    for h in range(8):
        assert len(np.unique(top[h])) == c["k"]
        assert top[h].min() >= c["sink"] and top[h].max() < T - c["local"]
        assert _overlap(top[h], fix["topk"][h], gs_ref[h], fix["kth"][h], 1e-3) >= 0.999
    out = r.out.float().cpu().numpy()
    # against fp32 attention over the SAME kept set
    keep = oracle.keep_positions(top, T, c["sink"], c["local"])
    ref_same = oracle.sparse_attention(c["q"].float().numpy(), c["keys"], c["vals"],
                                       np.repeat(keep, 4, axis=0), 4)
    assert np.abs(out - ref_same).max() <= ATTN_ATOL
    # and against the reference's own output (its top-k set)
    assert np.abs(out - fix["out"]).max() <= ATTN_ATOL
    _check_errors()


def _rand_case(seed, B, Hkv, G, T, cap=None, per_kv=True, kv_dtype=torch.bfloat16, q_dtype=torch.bfloat16,
               equal_codes=False):
    g = torch.Generator().manual_seed(seed)
    cap = cap or T
    C = torch.randn((Hkv, 32, 256, 128) if per_kv else (32, 256, 128), generator=g) * 0.05
    codes = torch.randint(0, 256, (B, Hkv, cap, 32), generator=g, dtype=torch.uint8)
    if equal_codes:
        codes[:] = 7
    K = torch.randn((B, Hkv, cap, 128), generator=g).to(kv_dtype)
    V = torch.randn((B, Hkv, cap, 128), generator=g).to(kv_dtype)
    q = torch.randn((B, Hkv * G, 128), generator=g).to(q_dtype)
    return C, codes, K, V, q


def _oracle_step(C, codes, K, V, q, T_codes, T_total, k, sink, local, per_kv, select):
    B, Hq, D = q.shape
    Hkv = codes.shape[1]
    G = Hq // Hkv
    tops, outs, scores = [], [], []
    for b in range(B):
        cb = C.numpy() if per_kv else np.broadcast_to(C.numpy(), (Hkv,) + tuple(C.shape)).copy()
        s = oracle.scores_per_kv_head(cb, q[b].float().numpy(), codes[b, :, :T_codes].numpy(), G)
        s_sel = oracle.group_sum(s, G) if select == "kv_group" else s
        lo, hi = oracle.candidate_window(T_codes, T_total, sink, local)
        top = oracle.topk_rows(s_sel, lo, hi, k)
        keep = oracle.keep_positions(top, T_total, sink, local)
        idx_q = np.repeat(keep, G, axis=0) if select == "kv_group" else keep
        o = oracle.sparse_attention(q[b].float().numpy(), K[b].float().numpy(), V[b].float().numpy(), idx_q, G)
        tops.append(top)
        outs.append(o)
        scores.append(s_sel)
    return np.concatenate(tops), np.stack(outs), np.concatenate(scores)


CASES = [
    # B, Hkv, G, T_codes, T_total, cap, k, sink, local, per_kv, select, kv, q
    (1, 8, 4, 4096, 4096, 4096, 64, 4, 64, True, "kv_group", torch.bfloat16, torch.bfloat16),
    (1, 2, 4, 77, 77, 128, 5, 4, 16, False, "kv_group", torch.bfloat16, torch.bfloat16),
    (2, 2, 4, 3000, 3000, 3128, 59, 0, 64, False, "query_head", torch.float16, torch.float32),
    (2, 3, 2, 1000, 1030, 1100, 100, 4, 64, True, "kv_group", torch.float16, torch.float16),
    (1, 4, 1, 513, 513, 513, 1, 0, 0, True, "kv_group", torch.bfloat16, torch.bfloat16),
    (1, 2, 8, 700, 700, 700, 636, 0, 64, True, "kv_group", torch.bfloat16, torch.bfloat16),  # k = all
    (1, 2, 4, 5000, 5000, 5000, 300, 4, 64, True, "query_head", torch.bfloat16, torch.bfloat16),
    (3, 1, 4, 9000, 9000, 9100, 180, 4, 64, True, "kv_group", torch.bfloat16, torch.bfloat16),
]


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_pipeline_vs_oracle(case, mode):
    B, Hkv, G, Tc, Tt, cap, k, sink, local, per_kv, select, kvd, qd = case
    C, codes, K, V, q = _rand_case(1000 + Tc, B, Hkv, G, Tt, cap=cap, per_kv=per_kv, kv_dtype=kvd, q_dtype=qd)
    dev = _dev()
    r = ops.sparse_decode(q.to(dev), C.to(dev), codes.to(dev), K.to(dev), V.to(dev), topk=k,
                          T_codes=Tc, T_total=Tt, sink=sink, local=local, select=select,
                          return_topk=True, out_dtype=torch.float32, **MODES[mode])
    torch.cuda.synchronize()
    top_ref, out_ref, s_ref = _oracle_step(C, codes, K, V, q, Tc, Tt, k, sink, local, per_kv, select)
    top = r.topk.cpu().numpy()
    for u in range(top.shape[0]):
        kth = np.sort(s_ref[u][top_ref[u]])[0] if k > 0 else 0.0
        assert _overlap(top[u], top_ref[u], s_ref[u], kth, 1e-4) >= 0.999
    # attention against fp32 attention over the set the kernel selected
    G_ = G
    outs = []
    for b in range(B):
        nu = top.shape[0] // B
        keep = oracle.keep_positions(top[b * nu:(b + 1) * nu], Tt, sink, local)
        idx_q = np.repeat(keep, G_, axis=0) if select == "kv_group" else keep
        outs.append(oracle.sparse_attention(q[b].float().numpy(), K[b].float().numpy(),
                                            V[b].float().numpy(), idx_q, G_))
    out = r.out.cpu().numpy()
    assert np.abs(out - np.stack(outs)).max() <= 2e-3
    assert np.abs(out - out_ref).max() <= ATTN_ATOL
    _check_errors()


@pytest.mark.parametrize("mode", list(MODES))
def test_ties_take_lowest_index(mode):
    # every code equal -> every candidate score equal -> exact slow path; the
    # first k candidates (lowest indices) must be chosen
    C, codes, K, V, q = _rand_case(5, 1, 2, 4, 6000, equal_codes=True)
    dev = _dev()
    k, sink, local = 100, 4, 64
    r = ops.sparse_decode(q.to(dev), C.to(dev), codes.to(dev), K.to(dev), V.to(dev), topk=k,
                          sink=sink, local=local, return_topk=True, **MODES[mode])
    torch.cuda.synchronize()
    top = r.topk.cpu().numpy()
    for u in range(2):
        assert (top[u] == np.arange(sink, sink + k)).all()
    bits = ops.device_errors(device=dev)
    assert bits & 1 == 0 and bits & 2 == 2  # slow exact path ran, no timeout


@pytest.mark.parametrize("mode", list(MODES))
def test_repeat_calls_deterministic(mode):
    C, codes, K, V, q = _rand_case(9, 1, 8, 4, 20000)
    dev = _dev()
    args = [t.to(dev) for t in (q, C, codes, K, V)]
    outs = [ops.sparse_decode(*args, topk=400, sink=4, local=64, return_topk=True, **MODES[mode])
            for _ in range(3)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o.topk, outs[0].topk)
        assert torch.equal(o.out, outs[0].out)
    _check_errors()


def test_calls_on_the_same_buffers_follow_the_token_counts():
    # a decode loop calls sparse_decode on the same caches with growing token
    # counts: calls that reuse an earlier call's argument struct (same
    # buffers) must equal calls on fresh copies of the buffers, whatever
    # T_codes / T_total they pass, for [Hkv,T,.] and [B,Hkv,T,.] tensors
    C, codes, K, V, q = _rand_case(13, 1, 8, 4, 12000)
    dev = _dev()
    q, C, codes, K, V = (t.to(dev) for t in (q, C, codes, K, V))
    for T_codes, T_total in ((9000, 9100), (11936, 12000), (9000, 9100)):
        for dims in (4, 3):
            cd, kk, vv, qq = (codes, K, V, q) if dims == 4 else (codes[0], K[0], V[0], q[0])
            same = ops.sparse_decode(qq, C, cd, kk, vv, topk=300, T_codes=T_codes, T_total=T_total, sink=4,
                                     local=64, return_topk=True)
            fresh = ops.sparse_decode(qq.clone(), C.clone(), cd.clone(), kk.clone(), vv.clone(), topk=300,
                                      T_codes=T_codes, T_total=T_total, sink=4, local=64, return_topk=True)
            torch.cuda.synchronize()
            assert torch.equal(same.topk, fresh.topk)
            assert torch.equal(same.out, fresh.out)
    with pytest.raises(RuntimeError, match="T_total"):
        ops.sparse_decode(q, C, codes, K, V, topk=300, T_codes=9000, T_total=12001, sink=4, local=64)
    _check_errors()


def test_candidate_union_and_tie_exchange_select_the_same_set():
    # both fused selection paths are exact: identical index sets, and the
    # attention outputs agree to accumulation-order rounding
    C, codes, K, V, q = _rand_case(11, 1, 8, 4, 40000)
    dev = _dev()
    args = [t.to(dev) for t in (q, C, codes, K, V)]
    a = ops.sparse_decode(*args, topk=1024, sink=4, local=64, return_topk=True)
    b = ops.sparse_decode(*args, topk=1024, sink=4, local=64, return_topk=True, exchange_select=True)
    torch.cuda.synchronize()
    assert torch.equal(a.topk, b.topk)
    assert (a.out.float() - b.out.float()).abs().max().item() <= 1e-2
    _check_errors()


def test_fused_path_is_taken_for_cfg3_geometry():
    # the fused kernel stamps its phases; the multi-kernel path does not
    c = syn.config3(0, T=32768)
    dev = _dev()
    args = [c[n].to(dev) for n in ("q", "C", "codes", "keys", "vals")]
    ns = torch.zeros(8, dtype=torch.int64, device=dev)
    ops.sparse_decode(*args, topk=512, sink=4, local=64, phase_ns=ns)
    torch.cuda.synchronize()
    t = ns.cpu().numpy()
    assert (t > 0).all() and (np.diff(t) >= 0).all()
    ns.zero_()
    ops.sparse_decode(*args, topk=512, sink=4, local=64, phase_ns=ns, fused=False)
    torch.cuda.synchronize()
    assert (ns.cpu().numpy() == 0).all()


def test_workspace_shared_across_geometries():
    # one workspace, alternating shapes: the persistent state (error word,
    # grid-barrier word) must sit at geometry-independent offsets
    dev = _dev()
    ws = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
    outs = {}
    for rep in range(2):
        for T, Hkv in ((4096, 8), (20000, 2), (777, 4)):
            C, codes, K, V, q = _rand_case(T, 1, Hkv, 4, T)
            r = ops.sparse_decode(q.to(dev), C.to(dev), codes.to(dev), K.to(dev), V.to(dev),
                                  topk=32, sink=4, local=64, return_topk=True, ws=ws)
            torch.cuda.synchronize()
            if rep == 0:
                outs[T] = (r.topk.clone(), r.out.clone())
            else:
                assert torch.equal(outs[T][0], r.topk) and torch.equal(outs[T][1], r.out)
    assert ops.device_errors(ws, dev) & 1 == 0


def test_prefetch_of_next_inputs_does_not_change_results():
    dev = _dev()
    C, codes, K, V, q = [t.to(dev) for t in _rand_case(21, 1, 8, 4, 30000)]
    C2, codes2, _, _, _ = [t.to(dev) for t in _rand_case(22, 1, 8, 4, 30000)]
    r0 = ops.sparse_decode(q, C, codes, K, V, topk=600, sink=4, local=64, return_topk=True)
    r1 = ops.sparse_decode(q, C, codes, K, V, topk=600, sink=4, local=64, return_topk=True,
                           prefetch=ops.prefetch_regions(C2, codes2))
    torch.cuda.synchronize()
    assert torch.equal(r0.topk, r1.topk) and torch.equal(r0.out, r1.out)
    assert ops.device_errors(device=dev) & 1 == 0


def test_fused_calls_after_other_paths_on_a_fresh_shared_workspace():
    # a fresh workspace gives the fused kernel small launch numbers (1, 2, 3
    # ...) as exchange tags; the calls before them -- the multi-kernel path,
    # per-query-head selection, other geometries -- write small integers
    # (histogram counts, bitmap words) into their scratch.  None of that may
    # reach the fused kernel's exchange arena: every result must equal the
    # one computed on a workspace of its own.
    dev = _dev()
    cases = [dict(T=20000, Hkv=2, B=1, fused=False, select="kv_group"),
             dict(T=3000, Hkv=2, B=2, fused=None, select="query_head"),
             dict(T=8192, Hkv=2, B=2, fused=None, select="kv_group"),
             dict(T=20000, Hkv=8, B=1, fused=None, select="kv_group"),
             dict(T=4096, Hkv=1, B=4, fused=False, select="kv_group"),
             dict(T=8192, Hkv=4, B=1, fused=None, select="kv_group")]
    inputs, refs = [], []
    for i, c in enumerate(cases):
        C, codes, K, V, q = [t.to(dev) for t in _rand_case(300 + i, c["B"], c["Hkv"], 4, c["T"])]
        kw = dict(topk=64, sink=4, local=64, return_topk=True, fused=c["fused"], select=c["select"])
        a = ops.build_args(q, C, codes, K, V, topk=64, sink=4, local=64, select=c["select"],
                           out=torch.empty((c["B"], c["Hkv"] * 4, 128), dtype=K.dtype, device=dev))
        own = torch.zeros(_lib.load().lp_sparse_decode_workspace_size(ctypes.byref(a)), dtype=torch.uint8,
                          device=dev)
        refs.append(ops.sparse_decode(q, C, codes, K, V, ws=own, **kw))
        inputs.append((q, C, codes, K, V, kw))
    torch.cuda.synchronize()
    shared = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
    for rep in range(3):
        for (q, C, codes, K, V, kw), ref in zip(inputs, refs):
            r = ops.sparse_decode(q, C, codes, K, V, ws=shared, **kw)
            torch.cuda.synchronize()
            assert torch.equal(r.topk, ref.topk) and torch.equal(r.out, ref.out)
    assert ops.device_errors(shared, dev) & 1 == 0


def test_wait_timeout_is_reported_and_the_next_call_recovers():
    # failure detection without a fault: with LP_FLAG_TEST_WAIT_TIMEOUT one
    # CTA withholds its share of its unit's table, the unit's bounded waits
    # give up, the error bit is read back on the host, and the next call on
    # the same workspace gives the result of a clean workspace
    dev = _dev()
    C, codes, K, V, q = [t.to(dev) for t in _rand_case(77, 1, 8, 4, 8192)]
    kw = dict(topk=256, sink=4, local=64)
    ref = ops.sparse_decode(q, C, codes, K, V, return_topk=True, **kw)
    out = torch.empty_like(ref.out)
    a = ops.build_args(q, C, codes, K, V, out=out, **kw)
    lib = _lib.load()
    ws = torch.zeros(lib.lp_sparse_decode_workspace_size(ctypes.byref(a)), dtype=torch.uint8, device=dev)
    a.flags |= _lib.LP_FLAG_TEST_WAIT_TIMEOUT
    with torch.cuda.device(dev):
        _lib.check(lib.lp_sparse_decode(ctypes.byref(a), ws.data_ptr(), ws.numel(), ops._stream_handle(dev)))
    assert ops.device_errors(ws, dev) & _lib.LP_DEVERR_WAIT_TIMEOUT
    again = ops.sparse_decode(q, C, codes, K, V, return_topk=True, ws=ws, **kw)
    torch.cuda.synchronize()
    assert ops.device_errors(ws, dev) == 0
    assert torch.equal(again.topk, ref.topk) and torch.equal(again.out, ref.out)


@pytest.mark.parametrize("select,mode", [("kv_group", "auto"), ("kv_group", "exchange"), ("kv_group", "multi"),
                                         ("query_head", "auto")])
def test_batched_long_context_at_the_config5_unit_count(select, mode):
    """B = 8 sequences x 8 KV heads = 64 selection units (256 per query
    head) at T = 32768, the unit count of batched decode; checked against
    the oracle whichever path the library takes for it."""
    B, Hkv, G, T = 8, 8, 4, 32768
    sink, local = 4, 64
    k = ops.num_candidates(T, T, sink, local) // 50
    C, codes, K, V, q = _rand_case(4242, B, Hkv, G, T)
    dev = _dev()
    r = ops.sparse_decode(q.to(dev), C.to(dev), codes.to(dev), K.to(dev), V.to(dev), topk=k, sink=sink,
                          local=local, select=select, return_topk=True, out_dtype=torch.float32, **MODES[mode])
    torch.cuda.synchronize()
    top = r.topk.cpu().numpy()
    top_ref, out_ref, s_ref = _oracle_step(C, codes, K, V, q, T, T, k, sink, local, True, select)
    for u in range(top.shape[0]):
        kth = np.sort(s_ref[u][top_ref[u]])[0]
        assert _overlap(top[u], top_ref[u], s_ref[u], kth, 1e-4) >= 0.999, u
    nu = top.shape[0] // B
    for b in range(B):
        keep = oracle.keep_positions(top[b * nu:(b + 1) * nu], T, sink, local)
        idx_q = np.repeat(keep, G, axis=0) if select == "kv_group" else keep
        want = oracle.sparse_attention(q[b].float().numpy(), K[b].float().numpy(), V[b].float().numpy(), idx_q, G)
        assert np.abs(r.out[b].cpu().numpy() - want).max() <= 2e-3
    assert np.abs(r.out.cpu().numpy() - out_ref).max() <= ATTN_ATOL
    _check_errors()


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float16])
def test_query_head_selection_is_a_top_k_of_the_cache_dtype_scores(kv_dtype):
    """The reference's decode hook casts its scores to the K/V cache dtype
    before torch.topk (aq_evaluation.py:166, :199), so many tokens tie at the
    k-th value and torch picks among them in an unspecified order.  This
    package selects on the unrounded scores (exact fixed-point sums, ties by
    lower index).  Rounding is monotone, so that choice is always one of the
    reference's valid outcomes: every token whose rounded score lies strictly
    above the k-th rounded score is selected, and every selected token rounds
    to at least that value.  Keep-set tolerance: none (100 % of the tokens
    above the tie value, and only tokens at or above it)."""
    Hkv, G, T, sink, local = 8, 4, 131072, 0, 64
    k = 2621  # the decode hook's keep size at 128k (mask_out 0.98)
    C, codes, _, _, q = _rand_case(515, 1, Hkv, G, 8, cap=8)  # codebooks and queries only
    g = torch.Generator().manual_seed(516)
    codes = torch.randint(0, 256, (1, Hkv, T, 32), generator=g, dtype=torch.uint8)
    dev = _dev()
    r = ops.sparse_decode(q.to(dev), C[0].to(dev), codes.to(dev), topk=k, sink=sink, local=local,
                          select="query_head", attention=False, return_topk=True, return_head_scores=True)
    torch.cuda.synchronize()
    lo, hi = ops._window(T, T, sink, local)
    rounded = r.head_scores[0, :, lo:hi].to(torch.float16).to(kv_dtype).float()
    sel = r.topk.long() - lo
    ties_at_kth = 0
    for h in range(Hkv * G):
        kth = torch.topk(rounded[h], k).values.min()
        mine = rounded[h][sel[h]]
        assert (mine >= kth).all(), h
        above = rounded[h] > kth
        assert int(above.sum()) == int((mine > kth).sum()), h
        ties_at_kth += int((rounded[h] == kth).sum()) - int((mine == kth).sum())
    assert ties_at_kth > 0  # the rounded scores do tie at the threshold (the case this covers)
    _check_errors()


@pytest.mark.parametrize("mode", ["auto", "exchange"])
def test_query_head_units_on_the_fused_path_at_the_decode_hook_settings(mode):
    """The reference decode hook's shipped settings: one codebook for every
    head, fp16 K/V, T = 131072, top-2621 per QUERY head, sink 0, local 64.
    The fused kernel runs one unit per query head (4.6 CTAs each, so their
    scores spill to the L2-resident buffer); its selection must equal the
    multi-kernel path's exactly and match the oracle."""
    B, Hkv, G, T = 1, 8, 4, 131072
    k, sink, local = 2621, 0, 64
    C, codes, K, V, q = _rand_case(777, B, Hkv, G, T, per_kv=False, kv_dtype=torch.float16,
                                   q_dtype=torch.float16)
    dev = _dev()
    args = [t.to(dev) for t in (q, C, codes, K, V)]
    kw = dict(topk=k, sink=sink, local=local, select="query_head", return_topk=True, out_dtype=torch.float32)
    ns = torch.zeros(8, dtype=torch.int64, device=dev)
    r = ops.sparse_decode(*args, phase_ns=ns, **kw, **MODES[mode])
    m = ops.sparse_decode(*args, fused=False, **kw)
    torch.cuda.synchronize()
    assert (ns.cpu().numpy() > 0).all(), "the fused kernel did not run"
    assert torch.equal(r.topk, m.topk)
    assert (r.out - m.out).abs().max().item() <= 2e-3
    top_ref, out_ref, s_ref = _oracle_step(C, codes, K, V, q, T, T, k, sink, local, False, "query_head")
    top = r.topk.cpu().numpy()
    for u in range(top.shape[0]):
        kth = np.sort(s_ref[u][top_ref[u]])[0]
        assert _overlap(top[u], top_ref[u], s_ref[u], kth, 1e-4) >= 0.999, u
    keep = oracle.keep_positions(top, T, sink, local)
    want = oracle.sparse_attention(q[0].float().numpy(), K[0].float().numpy(), V[0].float().numpy(), keep, G)
    assert np.abs(r.out[0].cpu().numpy() - want).max() <= 2e-3
    assert np.abs(r.out.cpu().numpy() - out_ref).max() <= ATTN_ATOL
    _check_errors()


@pytest.mark.parametrize("B,Hkv,T,k", [(8, 8, 32768, 640), (2, 8, 131072, 2048), (4, 8, 65536, 1300)])
def test_spilled_scores_select_like_the_multi_kernel_path(B, Hkv, T, k):
    """KV-group selection with more tokens per CTA than its shared-memory
    score buffer holds (B*Hkv units over 148 CTAs): the fused kernel keeps
    its scores in the global buffer; selection equal to the multi-kernel
    path's, attention within accumulation-order rounding."""
    C, codes, K, V, q = _rand_case(900 + B, B, Hkv, 4, T)
    dev = _dev()
    args = [t.to(dev) for t in (q, C, codes, K, V)]
    ns = torch.zeros(8, dtype=torch.int64, device=dev)
    r = ops.sparse_decode(*args, topk=k, sink=4, local=64, return_topk=True, phase_ns=ns)
    m = ops.sparse_decode(*args, topk=k, sink=4, local=64, return_topk=True, fused=False)
    torch.cuda.synchronize()
    assert (ns.cpu().numpy() > 0).all(), "the fused kernel did not run"
    assert torch.equal(r.topk, m.topk)
    assert (r.out.float() - m.out.float()).abs().max().item() <= 1e-2
    _check_errors()


@pytest.mark.parametrize("cbdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("select,mode", [("kv_group", "auto"), ("kv_group", "multi"), ("query_head", "auto"),
                                         ("query_head", "multi")])
def test_half_precision_codebooks_select_like_their_fp32_values(cbdt, select, mode):
    """Scoring from an fp16 / bf16 codebook copy (half the bytes of the
    table build): its elements widen to fp32 exactly, so the tables, the
    selection and the attention equal those of the fp32 tensor holding the
    same values, bit for bit, on every path."""
    C, codes, K, V, q = _rand_case(1313, 1, 8, 4, 20000, per_kv=(select == "kv_group"))
    dev = _dev()
    Ch = C.to(cbdt).to(dev)
    args = [t.to(dev) for t in (codes, K, V)]
    kw = dict(topk=400, sink=4, local=64, select=select, return_topk=True, **MODES[mode])
    r = ops.sparse_decode(q.to(dev), Ch, *args, **kw)
    w = ops.sparse_decode(q.to(dev), Ch.float(), *args, **kw)
    torch.cuda.synchronize()
    assert torch.equal(r.topk, w.topk) and torch.equal(r.out, w.out)
    if mode == "multi":
        hs = ops.sparse_decode(q.to(dev), Ch, *args, topk=400, sink=4, local=64, select=select,
                               return_head_scores=True, attention=False).head_scores
        hw = ops.sparse_decode(q.to(dev), Ch.float(), *args, topk=400, sink=4, local=64, select=select,
                               return_head_scores=True, attention=False).head_scores
        torch.cuda.synchronize()
        assert torch.equal(hs, hw)
    _check_errors()
