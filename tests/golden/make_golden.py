"""Generate the golden fixtures of tests/golden by running the REFERENCE code.

Usage (needs a checkout of the reference LAPrune repository; runs on CPU):

    python tests/golden/make_golden.py --reference <path-to-LAPrune-checkout>

The reference is imported from that checkout and driven through its own
public functions on its CPU/PyTorch path:

* scoring   -- AQLayerCodebookManager.approx_inner_product_multihead_gqa
               (laprune/llm/aq_kv.py:633), one manager per KV head for the
               per-KV-head codebooks of the benchmark configs;
* encoding  -- AQLayerCodebookManager.encode_keys_batch(icm_iters=0)
               (laprune/llm/aq_kv.py:390 -> laprune/quantizer.py:346), and
               with the reference's default icm_iters=2 (quantizer.py:346-370);
* selection -- torch.topk over the candidate window (as
               laprune/llm/modifiers/aq_evaluation.py:185-201);
* attention -- torch SDPA over the kept rows (aq_evaluation.py:251);
* decode hook -- the reference's own _decode_attention
               (aq_evaluation.py:146) on fp32 inputs.

Inputs come from laprune_b200.synthetic (seeded, reproducible); each fixture
stores checksums of its inputs so a test fails loudly if the generator drifts.
"""
from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from laprune_b200 import synthetic as syn  # noqa: E402

OUT = Path(__file__).resolve().parent


def ref_manager(AQLayerCodebookManager, AQLayerConfig, AdditiveQuantizer, cb_mkd, num_heads):
    """A reference manager on CPU/fp32 holding one [M,K,d] codebook set."""
    M, K, d = cb_mkd.shape
    cfg = {0: AQLayerConfig(M=M, K=K, d=d, heads_per_group=num_heads, num_heads=num_heads)}
    mgr = AQLayerCodebookManager(cfg, device=torch.device("cpu"), dtype=torch.float32)
    aq = AdditiveQuantizer(M=M, K=K, d=d, init="pretrained", device=torch.device("cpu"),
                           dtype=torch.float32, codebooks=cb_mkd.clone())
    aq._precompute_icm_lut()
    mgr._aq_per_group[(0, 0)] = aq
    return mgr


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference LAPrune checkout")
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--only", default="", help="comma-separated fixtures to (re)generate: "
                    "cfg1,cfg2,cfg3,small,hook,icm (default: all)")
    args = ap.parse_args()
    only = set(x for x in args.only.split(",") if x)

    def want(name):
        return not only or name in only
    if args.threads:
        torch.set_num_threads(args.threads)
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from laprune.llm.aq_kv import AQLayerCodebookManager, AQLayerConfig
    from laprune.quantizer import AdditiveQuantizer
    from laprune.llm.modifiers import aq_evaluation as aqe

    def mgr_for(cb, nh):
        return ref_manager(AQLayerCodebookManager, AQLayerConfig, AdditiveQuantizer, cb, nh)

    def per_kv_scores(C, q, codes, G):
        Hkv = codes.shape[0]
        outs = []
        for h in range(Hkv):
            mgr = mgr_for(C[h], G)
            s = mgr.approx_inner_product_multihead_gqa(0, q[h * G:(h + 1) * G], codes[h:h + 1], G)
            outs.append(s.float())
        return torch.cat(outs, 0)

    # ---------------- config 1: scoring op (T=4096) ----------------
    if want("cfg1"):
        cfg1(per_kv_scores)
    if want("cfg2"):
        cfg2(mgr_for, per_kv_scores)
    if want("cfg3"):
        cfg3(per_kv_scores)
    if want("small"):
        small(mgr_for)
    if want("hook"):
        hook(mgr_for, aqe)
    if want("icm"):
        icm(mgr_for)


def cfg1(per_kv_scores):
    c1 = syn.config1(0)
    s1 = per_kv_scores(c1["C"], c1["q"], c1["codes"], c1["G"])          # [32,4096] fp32
    gs1 = s1.reshape(8, 4, -1).sum(1)
    top1 = torch.topk(gs1, k=c1["k"], dim=-1, sorted=False).indices.sort(-1).values
    kth1 = torch.topk(gs1, k=c1["k"], dim=-1).values[:, -1]
    np.savez_compressed(
        OUT / "cfg1_scoring.npz",
        checksums=np.array([syn.checksum(c1["C"]), syn.checksum(c1["codes"]), syn.checksum(c1["q"])]),
        scores=s1.numpy(), topk=top1.numpy().astype(np.int32), kth=kth1.numpy())
    print("cfg1 done", s1.shape)


def cfg2(mgr_for, per_kv_scores):
    # ---------------- config 2: encode + scoring (B=4) ----------------
    c2 = syn.config2(0)
    B, Hkv, Tn, D = c2["keys"].shape
    codes2 = torch.empty((B, Hkv, Tn, 32), dtype=torch.uint8)
    for h in range(Hkv):
        mgr = mgr_for(c2["C"][h], 4)
        x = c2["keys"][:, h].reshape(B * Tn, D).float()
        cc = mgr.encode_keys_batch(0, 0, x, icm_iters=0)
        codes2[:, h] = cc.reshape(B, Tn, 32).to(torch.uint8)
    cache = c2["code_cache"].clone()
    p0 = c2["pos0"]
    cache[:, :, p0:p0 + Tn] = codes2
    sample = torch.arange(p0 - 64, p0 + Tn)
    s2 = torch.empty((B, 32, sample.numel()), dtype=torch.float32)
    for b in range(B):
        sb = per_kv_scores(c2["C"], c2["q"][b], cache[b][:, sample], 4)
        s2[b] = sb
    np.savez_compressed(
        OUT / "cfg2_encode.npz",
        checksums=np.array([syn.checksum(c2["C"]), syn.checksum(c2["keys"]),
                            syn.checksum(c2["code_cache"]), syn.checksum(c2["q"])]),
        codes=codes2.numpy(), sample=sample.numpy().astype(np.int32), scores=s2.numpy())
    print("cfg2 done")


def cfg3(per_kv_scores):
    # ---------------- config 3: sparse decode step (T=131072) ----------------
    c3 = syn.config3(0)
    T = c3["codes"].shape[1]
    s3 = per_kv_scores(c3["C"], c3["q"], c3["codes"], 4)
    gs3 = s3.reshape(8, 4, -1).sum(1)
    lo, hi = c3["sink"], T - c3["local"]
    top3 = torch.topk(gs3[:, lo:hi], k=c3["k"], dim=-1, sorted=False).indices + lo
    top3 = top3.sort(-1).values
    kth3 = torch.topk(gs3[:, lo:hi], k=c3["k"], dim=-1).values[:, -1]
    keep = torch.cat([torch.arange(c3["sink"]).expand(8, -1), top3,
                      torch.arange(hi, T).expand(8, -1)], dim=-1)
    idx = keep[:, None, :, None].expand(8, 1, keep.shape[1], 128)
    kk = torch.take_along_dim(c3["keys"].float()[:, None], idx, dim=2)    # [8,1,N,128]
    vv = torch.take_along_dim(c3["vals"].float()[:, None], idx, dim=2)
    qq = c3["q"].float().reshape(8, 4, 1, 128)
    out3 = torch.nn.functional.scaled_dot_product_attention(qq, kk.expand(8, 4, -1, -1),
                                                            vv.expand(8, 4, -1, -1))
    np.savez_compressed(
        OUT / "cfg3_decode.npz",
        checksums=np.array([syn.checksum(c3["C"]), syn.checksum(c3["codes"]),
                            syn.checksum(c3["keys"]), syn.checksum(c3["vals"]),
                            syn.checksum(c3["q"])]),
        topk=top3.numpy().astype(np.int32), kth=kth3.numpy(),
        out=out3.reshape(32, 128).numpy())
    print("cfg3 done")


def small(mgr_for):
    # ---------------- small cases: shared codebook, ragged, strided ----------------
    sm = syn.small_shared(7)
    codes_s = sm["codes_full"][:, :sm["T"]]          # strided prefix like the decode cache
    mgr = mgr_for(sm["cb"], 8)
    s_small = mgr.approx_inner_product_multihead_gqa(0, sm["q"], codes_s, sm["G"]).float()
    codes_enc = mgr.encode_keys_batch(0, 0, sm["x"], icm_iters=0).to(torch.uint8)
    np.savez_compressed(
        OUT / "small_shared.npz",
        checksums=np.array([syn.checksum(sm["cb"]), syn.checksum(sm["codes_full"]),
                            syn.checksum(sm["q"]), syn.checksum(sm["x"])]),
        scores=s_small.numpy(), codes_enc=codes_enc.numpy())
    print("small done")


def hook(mgr_for, aqe):
    # ---------------- the reference decode hook on fp32 inputs ----------------
    dh = syn.decode_hook_case(11)
    mgr = mgr_for(dh["cb"], dh["Hq"])
    conf = {"mask_out": 0.98, "min_remain": 20, "sink_size": 0, "local_window": 64,
            "aq_use_pruned_attn": True, "aq_scoring_m": 32}
    outs = {}
    for sink in (0, 4):
        self_attn = types.SimpleNamespace(total_seq_len=dh["T"], o_proj=torch.nn.Identity())
        aq_cache = {"codes": dh["codes"], "seq_len": dh["T"]}
        out = aqe._decode_attention(self_attn, mgr, 0, dh["q"], dh["keys"], dh["vals"],
                                    aq_cache, dict(conf, sink_size=sink))
        outs[f"out_sink{sink}"] = out.float().numpy()
    np.savez_compressed(
        OUT / "decode_hook.npz",
        checksums=np.array([syn.checksum(dh["cb"]), syn.checksum(dh["codes"]),
                            syn.checksum(dh["keys"]), syn.checksum(dh["vals"]),
                            syn.checksum(dh["q"])]),
        **outs)
    print("decode hook done")


def icm(mgr_for):
    # ---------------- encoding with the reference's default ICM refinement ----------------
    # config 2's keys per KV head (one quantizer per head, as the reference
    # would run per-KV-head codebooks) and the small shared-codebook case
    c2 = syn.config2(0)
    B, Hkv, Tn, D = c2["keys"].shape
    codes = torch.empty((B, Hkv, Tn, 32), dtype=torch.uint8)
    for h in range(Hkv):
        mgr = mgr_for(c2["C"][h], 4)
        x = c2["keys"][:, h].reshape(B * Tn, D).float()
        codes[:, h] = mgr.encode_keys_batch(0, 0, x, icm_iters=2).reshape(B, Tn, 32).to(torch.uint8)
    sm = syn.small_shared(7)
    mgr = mgr_for(sm["cb"], 8)
    codes_small = mgr.encode_keys_batch(0, 0, sm["x"], icm_iters=2).to(torch.uint8)
    np.savez_compressed(
        OUT / "icm_encode.npz",
        checksums=np.array([syn.checksum(c2["C"]), syn.checksum(c2["keys"]),
                            syn.checksum(sm["cb"]), syn.checksum(sm["x"])]),
        codes_cfg2=codes.numpy(), codes_small=codes_small.numpy())
    print("icm done")


if __name__ == "__main__":
    main()
