"""Host logic of the reference-facing manager and decode-hook mirror (no GPU):
the codebook file format, the top-k size rule, the K/V buffer growth and the
refusal of work outside the decode path."""
import numpy as np
import pytest
import torch

import oracle
from laprune_b200 import aq_evaluation as aqe
from laprune_b200.aq_kv import AQLayerCodebookManager, AQLayerConfig


def _mgr(layers=(0, 3), hpg=4, num_heads=8):
    return AQLayerCodebookManager({L: AQLayerConfig(M=32, K=256, d=128, heads_per_group=hpg, num_heads=num_heads)
                                   for L in layers}, device="cpu")


def test_codebook_files_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    a = _mgr()
    cbs = {(L, G): torch.randn((32, 256, 128), generator=g) for L in (0, 3) for G in (0, 1)}
    for (L, G), cb in cbs.items():
        a.set_codebooks(L, G, cb)
    a.save(str(tmp_path))
    names = sorted(p.name for p in tmp_path.iterdir())
    assert names == ["layer_0_group_0.pt", "layer_0_group_1.pt", "layer_3_group_0.pt", "layer_3_group_1.pt"]
    b = _mgr()
    b.load(str(tmp_path))
    for (L, G), cb in cbs.items():
        assert torch.equal(b.codebooks(L, G), cb)


def test_load_skips_stale_groups_and_unknown_layers_and_adopts_file_shapes(tmp_path):
    torch.save({"M": 16, "K": 256, "d": 128, "codebooks": torch.zeros(16, 256, 128)}, tmp_path / "layer_0_group_0.pt")
    torch.save({"M": 16, "K": 256, "d": 128, "codebooks": torch.zeros(16, 256, 128)}, tmp_path / "layer_0_group_5.pt")
    torch.save({"M": 16, "K": 256, "d": 128, "codebooks": torch.zeros(16, 256, 128)}, tmp_path / "layer_9_group_0.pt")
    (tmp_path / "notes.txt").write_text("not a codebook")
    m = _mgr(layers=(0,), hpg=4, num_heads=8)  # 2 groups expected: group 5 is stale
    m.load(str(tmp_path))
    assert m.layer_cfgs[0].M == 16 and m.layer_cfgs[0].heads_per_group == 4
    assert m.codebooks(0, 0).shape == (16, 256, 128)
    with pytest.raises(KeyError):
        m.codebooks(0, 5)
    with pytest.raises(KeyError):
        m.codebooks(9, 0)
    with pytest.raises(FileNotFoundError):
        m.load(str(tmp_path / "missing"))


def test_encoding_has_no_cpu_fallback():
    # greedy or with the reference's default ICM sweeps, the codes come from
    # the CUDA kernels only: host tensors are an error, not a slow path
    m = _mgr()
    m.set_codebooks(0, 0, torch.zeros(32, 256, 128))
    for icm in (0, 2):
        with pytest.raises(RuntimeError, match="CUDA"):
            m.encode_keys(0, 0, torch.zeros(4, 128), icm_iters=icm)
        with pytest.raises(RuntimeError, match="CUDA"):
            m.encode_keys_batch(0, 0, torch.zeros(4, 128), icm_iters=icm)


def test_group_stacks_follow_heads_per_group():
    m = _mgr(layers=(0,), hpg=2, num_heads=8)
    for G in range(4):
        m.set_codebooks(0, G, torch.full((32, 256, 128), float(G)))
    st = m.group_codebooks(0, [h // 2 for h in range(8)])
    assert [int(st[h, 0, 0, 0]) for h in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]
    # the decode hook's grouping: query heads (G=4 per KV head) over hpg=2 split a KV head
    with pytest.raises(NotImplementedError):
        aqe._scoring_codebooks(m, 0, 8, 2)
    m.layer_cfgs[0].heads_per_group = 4
    m._stacks.clear()
    st = aqe._scoring_codebooks(m, 0, 8, 2)
    assert st.shape[0] == 2 and int(st[1, 0, 0, 0]) == 1


@pytest.mark.parametrize("n", [0, 1, 5, 19, 20, 21, 999, 1000, 1001, 131004])
def test_decode_keep_size_matches_the_oracle(n):
    assert aqe.decode_keep_size(n) == oracle.num_keep(n)


def test_kv_cache_append_grows_and_keeps_the_prefix():
    class Attn:
        pass
    a = Attn()
    g = torch.Generator().manual_seed(1)
    ks, vs = [], []
    total = 0
    for step, tn in enumerate([20, 1, 1, 30, 1]):
        k = torch.randn((2, 2, tn, 8), generator=g)
        v = torch.randn((2, 2, tn, 8), generator=g)
        ks.append(k)
        vs.append(v)
        total += tn
        kv, vv, (kd, vd) = aqe._kv_cache_append(a, k, v, total)
        assert kv.shape == (2, 2, total, 8) and a.k_cache_len == total and a.k_cache_capacity >= total
        assert torch.equal(kv, torch.cat(ks, 2)) and torch.equal(vv, torch.cat(vs, 2))
    assert a.k_cache_capacity == 80  # 20 -> 20 (first: max(total, 16)), 21 -> 40, 52 -> 80


def test_sharded_manager_loads_one_copy_per_device_on_first_use(tmp_path):
    from laprune_b200.aq_kv import ShardedAQLayerCodebookManager
    src = _mgr(layers=(0,), hpg=8, num_heads=8)
    cb = torch.randn((32, 256, 128), generator=torch.Generator().manual_seed(5))
    src.set_codebooks(0, 0, cb)
    src.save(str(tmp_path))
    sh = ShardedAQLayerCodebookManager({0: AQLayerConfig(M=32, K=256, d=128, heads_per_group=8, num_heads=8)},
                                       str(tmp_path), devices=["cpu"])
    assert list(sh._mgr_by_device) == ["cpu"]
    assert sh.for_device("cpu") is sh.for_device(torch.device("cpu"))
    assert torch.equal(sh.codebooks(0, 0), cb)
    assert sh._on(torch.zeros(1)) is sh.for_device("cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        sh.encode_keys(0, 0, torch.zeros(4, 128), icm_iters=2)


def test_quantizer_encode_surface_refuses_training_and_host_tensors():
    from laprune_b200.quantizer import AdditiveQuantizer
    with pytest.raises(NotImplementedError):
        AdditiveQuantizer(M=32, K=256, d=128, init="random", device="cpu")
    with pytest.raises(ValueError):
        AdditiveQuantizer(M=32, K=256, d=128, device="cpu", codebooks=torch.zeros(16, 256, 128))
    aq = AdditiveQuantizer(M=32, K=256, d=128, device="cpu", codebooks=torch.zeros(32, 256, 128))
    with pytest.raises(RuntimeError, match="CUDA"):
        aq.encode(torch.zeros(4, 128), icm_iters=2)
    with pytest.raises(NotImplementedError):
        aq.encode(torch.zeros(4, 128), method="beam", icm_iters=0)


def test_codebook_copies_round_trip_and_stale_copies_are_ignored(tmp_path):
    from laprune_b200.aq_kv import codebook_file_index
    src = _mgr(layers=(0, 1), hpg=8, num_heads=8)
    g = torch.Generator().manual_seed(8)
    cbs = {(l, 0): torch.randn((32, 256, 128), generator=g) * 0.05 for l in (0, 1)}
    for (l, gr), cb in cbs.items():
        src.set_codebooks(l, gr, cb)
    src.save(str(tmp_path))
    assert src.write_codebook_copies(str(tmp_path)) == 2
    names = sorted(p.name for p in tmp_path.iterdir())
    assert names == ["layer_0_group_0.lpcopies.pt", "layer_0_group_0.pt",
                     "layer_1_group_0.lpcopies.pt", "layer_1_group_0.pt"]
    # only the codebook files themselves name a (layer, group), as for the
    # reference's loader (its group field must parse as an integer)
    assert codebook_file_index("layer_1_group_0.pt") == (1, 0)
    assert codebook_file_index("layer_1_group_0.lpcopies.pt") is None
    blob = torch.load(tmp_path / "layer_1_group_0.lpcopies.pt", weights_only=True)
    c16 = cbs[(1, 0)].to(torch.float16)
    assert torch.equal(blob["codebooks_fp16"], c16)
    assert torch.equal(blob["weight_t_fp16"], c16.transpose(1, 2))
    assert torch.equal(blob["bias_fp16"], (-0.5 * c16.float().pow(2).sum(-1)).to(torch.float16))
    # loaded copies are the persisted tensors
    blob["codebooks_fp16"][0, 0, 0] = 1.0  # marker: a copy from the file, not a fresh conversion
    torch.save(blob, tmp_path / "layer_1_group_0.lpcopies.pt")
    m = _mgr(layers=(0, 1), hpg=8, num_heads=8)
    m.dtype = torch.float16
    m.load(str(tmp_path))
    assert m.scoring_dtype == torch.float16
    assert m.codebooks(1, 0, torch.float16)[0, 0, 0].item() == 1.0
    assert torch.equal(m.codebooks(1, 0), cbs[(1, 0)])
    # a copy file made from other codebooks is ignored: converted afresh
    torch.save(src._cb[(0, 0)] * 2, tmp_path / "unused.pt")
    other = dict(blob, source_sha256="0" * 64)
    torch.save(other, tmp_path / "layer_1_group_0.lpcopies.pt")
    m2 = _mgr(layers=(0, 1), hpg=8, num_heads=8)
    m2.load(str(tmp_path))
    assert torch.equal(m2.codebooks(1, 0, torch.float16), c16)
    m3 = _mgr(layers=(0, 1), hpg=8, num_heads=8)
    m3.load(str(tmp_path), use_copies=False)
    assert torch.equal(m3.codebooks(0, 0, torch.bfloat16), cbs[(0, 0)].to(torch.bfloat16))
