"""Generate golden vectors from the reference implementation (bitxwolf/kitty-kv).

Run once in a container that has the reference checked out (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/kitty-kv

The reference package is imported under the alias ``kitty_ref`` (both it and
this repository's drop-in are named ``kitty``), only its CPU PyTorch path is
run, and the results are written next to this script:

* ``golden_small.npz``  - small cases stored in full (inputs and outputs);
* ``golden_manifest.json`` - seeds, shapes, SHA-256 of generated inputs and of
  every reference output for the 128-channel cases, plus the reference's
  attention outputs for those cases.

The GPU tests regenerate the 128-channel inputs from the recorded seeds with
``synthetic`` (numpy PCG64, identical bytes everywhere), run the CUDA
kernels and compare against these hashes/outputs; the CPU tests check that the
numpy oracle reproduces every recorded reference output.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "kitty-kv_b200"))
sys.path.insert(0, str(REPO))
import synthetic  # noqa: E402  (numpy-only input generator at the repository root)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_reference(root: Path):
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    spec = importlib.util.spec_from_file_location(
        "kitty_ref", root / "kitty" / "__init__.py",
        submodule_search_locations=[str(root / "kitty")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["kitty_ref"] = mod
    spec.loader.exec_module(mod)
    import kitty_ref.kernels as kk  # noqa: F401
    return mod


# ---------------------------------------------------------------------------
# small, fully-stored cases
# ---------------------------------------------------------------------------

def small_key_cases(rng):
    """(name, key (D,G) f16, boost_idx (D,), d_boost, sentinel)."""
    cases = []
    D, G, K = 16, 8, 4
    sent = K + 1
    base_bidx = np.full(D, sent, np.uint8); base_bidx[:K] = np.arange(K)
    for i in range(4):
        cases.append((f"rand{i}", rng.standard_normal((D, G)).astype(np.float16), base_bidx, K, sent))
    k = rng.standard_normal((D, G)).astype(np.float16); k[3] = 1.5; k[7] = 0.0; k[K] = -2.25
    cases.append(("constant_channels", k, base_bidx, K, sent))
    cases.append(("all_zero", np.zeros((D, G), np.float16), base_bidx, K, sent))
    k = (rng.standard_normal((D, G)) * rng.uniform(0.01, 50.0, size=(D, 1))).astype(np.float16)
    cases.append(("wide_ranges", k, base_bidx, K, sent))
    perm = rng.permutation(D)
    b = np.full(D, sent, np.uint8); b[perm[:K]] = np.arange(K)
    cases.append(("permuted_boost", rng.standard_normal((D, G)).astype(np.float16), b, K, sent))
    # duplicate rows: two channels map to the same high-plane row (bits are OR-ed)
    b = base_bidx.copy(); b[9] = 1
    cases.append(("duplicate_rows", rng.standard_normal((D, G)).astype(np.float16), b, K, sent))
    # boost_idx == d_boost: INT4 range (< sentinel) but high bits not stored (< d_boost fails)
    b = base_bidx.copy(); b[10] = K; sent2 = 255
    cases.append(("boost_eq_k", rng.standard_normal((D, G)).astype(np.float16), b, K, sent2))
    # no boosted channels at all, sentinel 255 (reference known-answer test layout)
    kk = np.tile(np.array([0.0, 1.0, 2.0, 3.0], np.float16), (4, 1))
    cases.append(("known_answer_0123", kk, np.full(4, 255, np.uint8), 0, 255))
    # half-way values: x/scale lands on .5 for some elements (round-half-to-even)
    k = np.zeros((D, G), np.float16)
    k[:, :] = (np.arange(G)[None, :] * 0.5 - 1.0).astype(np.float16)
    k[:, -1] = 2.5
    cases.append(("halfway", k, base_bidx, K, sent))
    # D=128 layout with G=128: one outlier-distributed page
    k, _ = synthetic.make_kv(rng, 1, 128, 128)
    b = np.full(128, 17, np.uint8); b[rng.permutation(128)[:16]] = np.arange(16)
    cases.append(("d128_page", np.ascontiguousarray(k[0].T), b, 16, 17))
    return cases


def small_value_cases(rng):
    cases = []
    G, D = 8, 16
    for i in range(3):
        cases.append((f"rand{i}", rng.standard_normal((G, D)).astype(np.float16)))
    cases.append(("constant_3", np.full((G, D), 3.0, np.float16)))
    cases.append(("all_zero", np.zeros((G, D), np.float16)))
    v = rng.standard_normal((G, D)).astype(np.float16); v[2] = -7.0; v[5] = 0.25
    cases.append(("constant_rows", v))
    v = (rng.standard_normal((G, D)) * rng.uniform(0.01, 50.0, size=(G, 1))).astype(np.float16)
    cases.append(("wide_ranges", v))
    v = np.zeros((G, D), np.float16); v[:, :] = (np.arange(D)[None, :] * 0.5 - 2.0).astype(np.float16)
    cases.append(("halfway", v))
    _, vv = synthetic.make_kv(rng, 1, 128, 128)
    cases.append(("d128_page", vv[0]))
    return cases


def run_small(ref, rng, store):
    from kitty_ref.kernels import (quantize_key_page_torch, quantize_value_page_torch,
                                   dequantize_key_page_torch, dequantize_value_page_torch)
    names = []
    for name, key, bidx, K, sent in small_key_cases(rng):
        t2b, thi, sc, zp = quantize_key_page_torch(torch.from_numpy(key), torch.from_numpy(bidx), K, sent)
        rec = dequantize_key_page_torch(t2b, thi, sc, zp, torch.from_numpy(bidx), K)
        p = f"key/{name}/"
        store[p + "key"] = key
        store[p + "boost_idx"] = bidx
        store[p + "params"] = np.array([K, sent], np.int64)
        store[p + "low"] = t2b.numpy(); store[p + "high"] = thi.numpy()
        store[p + "scale"] = sc.numpy(); store[p + "zero"] = zp.numpy()
        store[p + "dequant"] = rec.numpy()
        names.append(("key", name))
    for name, val in small_value_cases(rng):
        pk, sc, zp = quantize_value_page_torch(torch.from_numpy(val))
        rec = dequantize_value_page_torch(pk, sc, zp)
        p = f"value/{name}/"
        store[p + "value"] = val
        store[p + "codes"] = pk.numpy(); store[p + "scale"] = sc.numpy(); store[p + "zero"] = zp.numpy()
        store[p + "dequant"] = rec.numpy()
        names.append(("value", name))
    return names


def nonfinite_cases():
    """Key and value pages holding +-inf and NaN, small and D = G = 128 (their own
    generator, so every other set keeps its bytes).  A channel (key) or token (value)
    that holds one becomes a non-finite range and scale in the reference."""
    rng = np.random.default_rng(2026)
    keys = []
    k = rng.standard_normal((16, 8)).astype(np.float16)
    k[1, 2] = np.inf; k[5, 0] = -np.inf; k[6, 3] = np.nan; k[12, :] = np.inf
    b = np.full(16, 5, np.uint8); b[[1, 6, 9, 13]] = np.arange(4)
    keys.append(("nonfinite", k, b, 4, 5))
    k = rng.standard_normal((128, 128)).astype(np.float16)
    k[3, 5] = np.inf; k[10, 7] = -np.inf; k[20, 9] = np.nan; k[30, :] = np.inf; k[40, 11] = 60000.0
    k[50, 3] = np.nan; k[50, 4] = np.inf
    boosted = [3, 20, 50] + [c for c in rng.permutation(128).tolist() if c not in (3, 20, 50)][:13]
    b = np.full(128, 17, np.uint8); b[boosted] = np.arange(16)
    keys.append(("nonfinite_d128", k, b, 16, 17))
    values = []
    v = rng.standard_normal((8, 16)).astype(np.float16)
    v[1, 2] = np.inf; v[3, 0] = np.nan; v[6, :] = -np.inf
    values.append(("nonfinite", v))
    v = rng.standard_normal((128, 128)).astype(np.float16)
    v[2, 5] = np.inf; v[9, :] = -np.inf; v[17, 3] = np.nan; v[33, 0] = 65504.0; v[60, 1] = -np.inf
    values.append(("nonfinite_d128", v))
    return keys, values


def run_nonfinite_sets(ref, store, manifest):
    from kitty_ref.kernels import (quantize_key_page_torch, quantize_value_page_torch,
                                   dequantize_key_page_torch, dequantize_value_page_torch)
    keys, values = nonfinite_cases()
    for name, key, bidx, K, sent in keys:
        t2b, thi, sc, zp = quantize_key_page_torch(torch.from_numpy(key), torch.from_numpy(bidx), K, sent)
        rec = dequantize_key_page_torch(t2b, thi, sc, zp, torch.from_numpy(bidx), K)
        p = f"key/{name}/"
        store[p + "key"] = key
        store[p + "boost_idx"] = bidx
        store[p + "params"] = np.array([K, sent], np.int64)
        store[p + "low"] = t2b.numpy(); store[p + "high"] = thi.numpy()
        store[p + "scale"] = sc.numpy(); store[p + "zero"] = zp.numpy()
        store[p + "dequant"] = rec.numpy()
        if ["key", name] not in manifest["small"]:
            manifest["small"].append(["key", name])
    for name, val in values:
        pk, sc, zp = quantize_value_page_torch(torch.from_numpy(val))
        rec = dequantize_value_page_torch(pk, sc, zp)
        p = f"value/{name}/"
        store[p + "value"] = val
        store[p + "codes"] = pk.numpy(); store[p + "scale"] = sc.numpy(); store[p + "zero"] = zp.numpy()
        store[p + "dequant"] = rec.numpy()
        if ["value", name] not in manifest["small"]:
            manifest["small"].append(["value", name])


def build_pools_ref(ref, case: synthetic.DecodeCase, phys_of, n_phys):
    """Quantise every page-head of ``case`` with the reference into pools of
    ``n_phys`` pages; sequence b's page i goes to physical page phys_of[b][i]."""
    from kitty_ref.kernels import quantize_key_page_torch, quantize_value_page_torch
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    kl = torch.zeros(n_phys, H, D, G // 4, dtype=torch.uint8)
    kh = torch.zeros(n_phys, H, K, G // 4, dtype=torch.uint8)
    km = torch.zeros(n_phys, H, 2, D, dtype=torch.float16)
    vc = torch.zeros(n_phys, H, G, D // 4, dtype=torch.uint8)
    vm = torch.zeros(n_phys, H, G, 2, dtype=torch.float16)
    bidx = torch.from_numpy(case.boost_idx)
    for b, sq in enumerate(case.seqs):
        pk = sq.page_keys(); pv = sq.page_values()
        for i in range(sq.n_pages):
            p = int(phys_of[b][i])
            for h in range(H):
                a, hh, s, z = quantize_key_page_torch(torch.from_numpy(pk[i, h]), bidx[h], K, case.sentinel)
                kl[p, h] = a; kh[p, h] = hh; km[p, h, 0] = s; km[p, h, 1] = z
                c, s2, z2 = quantize_value_page_torch(torch.from_numpy(pv[i, h]))
                vc[p, h] = c; vm[p, h, :, 0] = s2; vm[p, h, :, 1] = z2
    return kl, kh, km, vc, vm


def run_attention_case(ref, case, phys_of, n_phys):
    from kitty_ref.kernels import paged_attention_reference
    pools = build_pools_ref(ref, case, phys_of, n_phys)
    H, D = case.num_kv_heads, case.head_dim
    outs = []
    for b, sq in enumerate(case.seqs):
        sk, sv = sq.sink_kv(); tk, tv = sq.tail_kv()
        o = paged_attention_reference(
            q=torch.from_numpy(case.q[b]), page_list=[int(x) for x in phys_of[b][:sq.n_pages]],
            key_baseline=pools[0], key_boost=pools[1], key_meta=pools[2],
            value_pool=pools[3], value_meta=pools[4], boost_idx=torch.from_numpy(case.boost_idx),
            D_boost=case.d_boost, sink_k=torch.from_numpy(sk), sink_v=torch.from_numpy(sv),
            qbuf_k=torch.from_numpy(tk), qbuf_v=torch.from_numpy(tv),
            num_q_heads=case.num_q_heads, num_kv_heads=H, head_dim=D)
        outs.append(o.numpy())
    return pools, np.stack(outs)


def phys_layout(case, seed, spare=3):
    """Scatter every sequence's pages over a shared pool with a seeded permutation."""
    total = sum(s.n_pages for s in case.seqs)
    n_phys = total + spare
    perm = np.random.default_rng(seed).permutation(n_phys)[:total]
    phys_of, at = [], 0
    for s in case.seqs:
        phys_of.append(perm[at:at + s.n_pages].astype(np.int32)); at += s.n_pages
    return phys_of, n_phys


SMALL_ATTN = [
    # name, seed, B, Hq, H, D, contexts, sink, group, boost_rate, tails
    ("tiny_mixed", 11, 3, 4, 2, 16, [4 + 3 * 8 + 5, 4 + 8, 4 + 2 * 8 + 7], 4, 8, 0.25, None),
    ("tiny_sink_only", 12, 1, 4, 2, 16, [4], 4, 8, 0.25, None),
    ("tiny_no_sink", 13, 2, 4, 2, 16, [2 * 8 + 3, 8], 0, 8, 0.25, None),
    ("tiny_tail_only", 14, 1, 4, 2, 16, [6], 0, 8, 0.25, None),
    ("tiny_gqa8", 15, 2, 16, 2, 16, [4 + 4 * 8 + 1, 4 + 8 + 7], 4, 8, 0.25, None),
    ("d128_short", 16, 2, 8, 2, 128, [32 + 2 * 128 + 17, 32 + 128], 32, 128, 0.125, None),
]

BIG_ATTN = [
    # config 1 of the benchmark: B=1, 32q/8kv, T=4096 -> 31 pages + 96-token tail, K=16
    ("config1", 1, 1, 32, 8, 128, [4096], 32, 128, 0.125, None),
    # a short batched mixed-length case with Kitty-Pro boost (K=32) and random tails
    ("batched_pro", 21, 3, 32, 8, 128, [32 + 5 * 128 + 40, 32 + 9 * 128 + 127, 32 + 2 * 128],
     32, 128, 0.25, [40, 127, 0]),
]


def run_attention_sets(ref, store, manifest):
    for name, seed, B, Hq, H, D, ctx, S, G, rate, tails in SMALL_ATTN + BIG_ATTN:
        t0 = time.time()
        case = synthetic.make_decode_case(seed, B, Hq, H, D, ctx, sink=S, group=G,
                                          boost_rate=rate, tails=tails)
        phys_of, n_phys = phys_layout(case, seed + 1000)
        pools, out = run_attention_case(ref, case, phys_of, n_phys)
        entry = {"seed": seed, "batch": B, "num_q_heads": Hq, "num_kv_heads": H, "head_dim": D,
                 "contexts": ctx, "sink": S, "group": G, "boost_rate": rate, "tails": tails,
                 "phys_seed": seed + 1000, "n_phys": n_phys,
                 "d_boost": case.d_boost, "sentinel": case.sentinel,
                 "inputs_sha": {"q": sha(case.q), "boost_idx": sha(case.boost_idx),
                                "k": [sha(s.k) for s in case.seqs], "v": [sha(s.v) for s in case.seqs]},
                 "pools_sha": {n: sha(p.numpy()) for n, p in
                               zip(["key_low", "key_high", "key_meta", "val_codes", "val_meta"], pools)}}
        # by-value metadata hashes (+0/-0 folded), since the reference's zero-point sign is lane dependent
        entry["pools_sha"]["key_meta_value"] = sha(pools[2].numpy().astype(np.float32) + 0.0)
        entry["pools_sha"]["val_meta_value"] = sha(pools[4].numpy().astype(np.float32) + 0.0)
        store[f"attn/{name}/out"] = out
        if D <= 16:
            for n, p in zip(["key_low", "key_high", "key_meta", "val_codes", "val_meta"], pools):
                store[f"attn/{name}/{n}"] = p.numpy()
        manifest["attention"][name] = entry
        print(f"  attention {name}: {time.time() - t0:.1f}s", flush=True)


def run_pipeline_compat(ref, store, manifest):
    """Drive the reference state machine (num_layers=1) and record pool bytes, buffers
    and attention outputs at the steps where the reference is well defined."""
    from kitty_ref.config import KittyConfig
    from kitty_ref.layout import PageCentricKVLayoutManager
    from kitty_ref.pipeline import KittyInferencePipeline
    from kitty_ref.kernels.attention import paged_attention_reference
    specs = [
        ("tiny", 31, dict(num_layers=1, num_kv_heads=2, head_dim=16, q_buffer_size=8, sink_size=4,
                          local_value_window=8, boost_rate=0.25, max_seq_len=64, device="cpu"), 4, 4 + 3 * 8 + 5),
        ("d128", 32, dict(num_layers=1, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32,
                          local_value_window=128, boost_rate=0.125, max_seq_len=600, device="cpu"), 4, 32 + 2 * 128 + 9),
    ]
    for name, seed, cfgd, hq, steps in specs:
        cfg = KittyConfig(**cfgd)
        rng = np.random.default_rng(seed)
        H, D = cfg.num_kv_heads, cfg.head_dim
        k, v = synthetic.make_kv(rng, H, steps, D)
        bidx = synthetic.boost_idx_from_scores(synthetic.channel_scores([k]), cfg.d_boost, cfg.sentinel)[None]
        qs = synthetic.make_q(rng, (steps, hq, D))
        layout = PageCentricKVLayoutManager(cfg, torch.from_numpy(bidx))
        pipe = KittyInferencePipeline(cfg, layout, torch.from_numpy(bidx))
        outs, valid_steps = [], []
        for t in range(steps):
            pipe.push_token(0, torch.from_numpy(k[:, t]), torch.from_numpy(v[:, t]))
            ctx = pipe.get_attention_context(0, 0)
            qlen, rlen = ctx["key_qbuf"].shape[1], ctx["val_local"].shape[1]
            if qlen == 0 or qlen == rlen:
                o = paged_attention_reference(
                    q=torch.from_numpy(qs[t]), page_list=ctx["page_list"],
                    key_baseline=layout.key_baseline, key_boost=layout.key_boost,
                    key_meta=layout.key_metadata, value_pool=layout.value_pool,
                    value_meta=layout.value_metadata, boost_idx=torch.from_numpy(bidx[0]),
                    D_boost=cfg.d_boost, sink_k=ctx["sink_k"], sink_v=ctx["sink_v"],
                    qbuf_k=ctx["key_qbuf"], qbuf_v=ctx["val_local"],
                    num_q_heads=hq, num_kv_heads=H, head_dim=D)
                outs.append(o.numpy()); valid_steps.append(t)
        pools = [layout.key_baseline, layout.key_boost, layout.key_metadata, layout.value_pool,
                 layout.value_metadata]
        entry = {"seed": seed, "config": cfgd, "num_q_heads": hq, "steps": steps,
                 "valid_steps": valid_steps, "page_list": layout.get_page_list(0, 0),
                 "state": {"sink_fill": pipe.sink_fill, "key_qbuf_len": pipe.key_qbuf_len,
                           "val_local_len": pipe.val_local_len, "val_qbuf_len": pipe.val_qbuf_len},
                 "pools_sha": {n: sha(p.numpy()) for n, p in
                               zip(["key_low", "key_high", "key_meta", "val_codes", "val_meta"], pools)},
                 "buffers_sha": {"sink_k": sha(pipe.sink_k.numpy()), "key_qbuf": sha(pipe.key_qbuf.numpy()),
                                 "val_local": sha(pipe.val_local.numpy()), "val_qbuf": sha(pipe.val_qbuf.numpy())}}
        entry["pools_sha"]["key_meta_value"] = sha(pools[2].numpy().astype(np.float32) + 0.0)
        entry["pools_sha"]["val_meta_value"] = sha(pools[4].numpy().astype(np.float32) + 0.0)
        store[f"pipeline/{name}/outs"] = np.stack(outs)
        if D <= 16:
            for n, p in zip(["key_low", "key_high", "key_meta", "val_codes", "val_meta"], pools):
                store[f"pipeline/{name}/{n}"] = p.numpy()
        manifest["pipeline"][name] = entry
        print(f"  pipeline {name}: {len(valid_steps)} attention checkpoints", flush=True)


def run_quant_sets(ref, manifest, store):
    """Config-3-shaped page quantisation (K=32) on a sample of sequences: hash of every
    reference output, per sequence, in (page, head) order."""
    from kitty_ref.kernels import quantize_key_page_torch, quantize_value_page_torch
    name, seed, H, D, G, T, K = "config3_sample", 3, 8, 128, 128, 32768, 32
    n_seq = 2
    sent = K + 1
    rng = np.random.default_rng(seed)
    seqs = [synthetic.make_kv(rng, H, T, D) for _ in range(n_seq)]
    bidx = synthetic.boost_idx_from_scores(synthetic.channel_scores([s[0] for s in seqs]), K, sent)
    S = 32
    n = (T - S) // G
    entry = {"seed": seed, "num_kv_heads": H, "head_dim": D, "group": G, "tokens": T, "d_boost": K,
             "sentinel": sent, "sink": S, "n_pages": n, "n_seq": n_seq,
             "inputs_sha": {"k": [sha(s[0]) for s in seqs], "v": [sha(s[1]) for s in seqs],
                            "boost_idx": sha(bidx)}, "outputs_sha": []}
    t0 = time.time()
    for si, (k, v) in enumerate(seqs):
        sq = synthetic.SequenceKV(k=k, v=v, sink=S, n_pages=n, tail=(T - S) - n * G, group=G)
        pk, pv = sq.page_keys(), sq.page_values()
        low = np.zeros((n, H, D, G // 4), np.uint8); high = np.zeros((n, H, K, G // 4), np.uint8)
        ks = np.zeros((n, H, D), np.float16); kz = np.zeros((n, H, D), np.float16)
        vc = np.zeros((n, H, G, D // 4), np.uint8)
        vs = np.zeros((n, H, G), np.float16); vz = np.zeros((n, H, G), np.float16)
        bt = torch.from_numpy(bidx)
        for i in range(n):
            for h in range(H):
                a, b, c, d = quantize_key_page_torch(torch.from_numpy(pk[i, h]), bt[h], K, sent)
                low[i, h] = a.numpy(); high[i, h] = b.numpy(); ks[i, h] = c.numpy(); kz[i, h] = d.numpy()
                e, f, g_ = quantize_value_page_torch(torch.from_numpy(pv[i, h]))
                vc[i, h] = e.numpy(); vs[i, h] = f.numpy(); vz[i, h] = g_.numpy()
        entry["outputs_sha"].append({
            "key_low": sha(low), "key_high": sha(high),
            "key_scale": sha(ks), "key_zero_value": sha(kz.astype(np.float32) + 0.0),
            "val_codes": sha(vc), "val_scale": sha(vs), "val_zero_value": sha(vz.astype(np.float32) + 0.0)})
        if si == 0:
            store["quant/config3_sample/first_key_low"] = low[0]
            store["quant/config3_sample/first_key_high"] = high[0]
            store["quant/config3_sample/first_val_codes"] = vc[0]
        print(f"  quant seq {si}: {time.time() - t0:.1f}s", flush=True)
    manifest["quant"][name] = entry


def check_profiler(ref, manifest):
    """The reference profiler's boost index equals synthetic.boost_idx_from_scores."""
    from kitty_ref.config import KittyConfig
    from kitty_ref.sensitivity import KittySensitivityProfiler, _ChannelAccumulator
    cfg = KittyConfig(num_layers=2, num_kv_heads=4, head_dim=128, device="cpu", boost_rate=0.125)
    rng = np.random.default_rng(41)
    prof = KittySensitivityProfiler(cfg)
    keys = []
    for layer in range(2):
        k, _ = synthetic.make_kv(rng, 4, 256, 128)
        acc = _ChannelAccumulator(4, 128, "cpu")
        # fill the accumulator directly: the reference's update() reshapes (B,H,T,D)
        # to (-1,H,D) without moving H next to D, which mixes heads when T > 1
        acc.sum_abs = torch.from_numpy(np.abs(k.astype(np.float32)).sum(axis=1))
        acc.token_count = k.shape[1]
        prof._accumulators[layer] = acc
        keys.append(k)
    prof.compute()
    mine = np.stack([synthetic.boost_idx_from_scores(synthetic.channel_scores([k]), cfg.d_boost, cfg.sentinel)
                     for k in keys])
    manifest["profiler"] = {"seed": 41, "equal": bool((prof.boost_idx_uint8.numpy() == mine).all()),
                            "boost_idx_sha": sha(prof.boost_idx_uint8.numpy())}


BF16_ATTN = [
    # bfloat16 cache: same generator, values rounded to bf16 (name, seed, B, Hq, H, D, contexts, sink, group, rate)
    ("bf16_tiny", 51, 2, 4, 2, 16, [4 + 3 * 8 + 5, 4 + 8 + 2], 4, 8, 0.25),
    ("bf16_d128", 52, 2, 8, 2, 128, [32 + 2 * 128 + 17, 32 + 128 + 96], 32, 128, 0.125),
]


def run_bf16_sets(ref, rng, store, manifest):
    """A bfloat16 cache (KittyConfig(dtype="bfloat16")): the reference launchers write
    into bf16 pool views through their CPU branch (quantize_key.py:261-269,
    quantize_value.py:223-227), so the stored scale / zero-point are the fp16 results
    converted to bf16; dequantisation and attention read everything with .float()."""
    from kitty_ref.kernels import (quantize_key_page, quantize_value_page, dequantize_key_page_torch,
                                   dequantize_value_page_torch, paged_attention_reference)
    bf = torch.bfloat16
    names = []
    for name, key, bidx, K, sent in small_key_cases(rng):
        kb = torch.from_numpy(key.astype(np.float32)).to(bf)
        D, G = key.shape
        low = torch.zeros(D, G // 4, dtype=torch.uint8); high = torch.zeros(K, G // 4, dtype=torch.uint8)
        meta = torch.zeros(2, D, dtype=bf)
        quantize_key_page(kb, torch.from_numpy(bidx), K, sent, low, high, meta[0], meta[1])
        rec = dequantize_key_page_torch(low, high, meta[0], meta[1], torch.from_numpy(bidx), K)
        p = f"bf16key/{name}/"
        store[p + "key"] = kb.float().numpy()
        store[p + "boost_idx"] = bidx
        store[p + "params"] = np.array([K, sent], np.int64)
        store[p + "low"] = low.numpy(); store[p + "high"] = high.numpy()
        store[p + "scale"] = meta[0].float().numpy(); store[p + "zero"] = meta[1].float().numpy()
        store[p + "dequant"] = rec.numpy()
        names.append(("bf16key", name))
    for name, val in small_value_cases(rng):
        vb = torch.from_numpy(val.astype(np.float32)).to(bf)
        G, D = val.shape
        packed = torch.zeros(G, D // 4, dtype=torch.uint8)
        vmeta = torch.zeros(G, 2, dtype=bf)
        quantize_value_page(vb, packed, vmeta[:, 0], vmeta[:, 1])
        rec = dequantize_value_page_torch(packed, vmeta[:, 0], vmeta[:, 1])
        p = f"bf16value/{name}/"
        store[p + "value"] = vb.float().numpy()
        store[p + "codes"] = packed.numpy()
        store[p + "scale"] = vmeta[:, 0].float().numpy(); store[p + "zero"] = vmeta[:, 1].float().numpy()
        store[p + "dequant"] = rec.numpy()
        names.append(("bf16value", name))
    manifest["bf16_small"] = names
    manifest["bf16_attention"] = {}
    for name, seed, B, Hq, H, D, ctx, S, G, rate in BF16_ATTN:
        case = synthetic.make_decode_case(seed, B, Hq, H, D, ctx, sink=S, group=G, boost_rate=rate)
        phys_of, n_phys = phys_layout(case, seed + 1000)
        K = case.d_boost
        kl = torch.zeros(n_phys, H, D, G // 4, dtype=torch.uint8)
        kh = torch.zeros(n_phys, H, K, G // 4, dtype=torch.uint8)
        km = torch.zeros(n_phys, H, 2, D, dtype=bf)
        vc = torch.zeros(n_phys, H, G, D // 4, dtype=torch.uint8)
        vm = torch.zeros(n_phys, H, G, 2, dtype=bf)
        bidx = torch.from_numpy(case.boost_idx)
        outs = []
        for b, sq in enumerate(case.seqs):
            pk = sq.page_keys(); pv = sq.page_values()
            for i in range(sq.n_pages):
                pg = int(phys_of[b][i])
                for h in range(H):
                    quantize_key_page(torch.from_numpy(pk[i, h].astype(np.float32)).to(bf), bidx[h], K, case.sentinel,
                                      kl[pg, h], kh[pg, h], km[pg, h, 0], km[pg, h, 1])
                    quantize_value_page(torch.from_numpy(pv[i, h].astype(np.float32)).to(bf), vc[pg, h],
                                        vm[pg, h, :, 0], vm[pg, h, :, 1])
        for b, sq in enumerate(case.seqs):
            sk, sv = sq.sink_kv(); tk, tv = sq.tail_kv()
            cv = lambda a: torch.from_numpy(a.astype(np.float32)).to(bf)
            o = paged_attention_reference(
                q=cv(case.q[b]), page_list=[int(x) for x in phys_of[b][:sq.n_pages]],
                key_baseline=kl, key_boost=kh, key_meta=km, value_pool=vc, value_meta=vm, boost_idx=bidx,
                D_boost=K, sink_k=cv(sk), sink_v=cv(sv), qbuf_k=cv(tk), qbuf_v=cv(tv),
                num_q_heads=case.num_q_heads, num_kv_heads=H, head_dim=D)
            outs.append(o.numpy())
        entry = {"seed": seed, "batch": B, "num_q_heads": Hq, "num_kv_heads": H, "head_dim": D, "contexts": ctx,
                 "sink": S, "group": G, "boost_rate": rate, "phys_seed": seed + 1000, "n_phys": n_phys,
                 "d_boost": K, "sentinel": case.sentinel,
                 "pools_sha": {"key_low": sha(kl.numpy()), "key_high": sha(kh.numpy()), "val_codes": sha(vc.numpy()),
                               "key_meta_value": sha(km.float().numpy() + 0.0),
                               "val_meta_value": sha(vm.float().numpy() + 0.0)}}
        store[f"bf16attn/{name}/out"] = np.stack(outs)
        manifest["bf16_attention"][name] = entry
        print(f"  bf16 attention {name}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("KITTY_REFERENCE"),
                    help="checkout of the reference project (default: $KITTY_REFERENCE)")
    ap.add_argument("--skip-quant", action="store_true")
    ap.add_argument("--bf16-only", action="store_true",
                    help="add the bfloat16 sets to the existing golden files and keep everything else")
    ap.add_argument("--nonfinite-only", action="store_true",
                    help="add the non-finite key / value pages to the existing golden files")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set KITTY_REFERENCE")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = load_reference(Path(args.reference))
    if args.nonfinite_only:
        with np.load(HERE / "golden_small.npz") as z:
            store = {k: z[k] for k in z.files}
        manifest = json.loads((HERE / "golden_manifest.json").read_text())
        run_nonfinite_sets(ref, store, manifest)
        np.savez_compressed(HERE / "golden_small.npz", **store)
        (HERE / "golden_manifest.json").write_text(json.dumps(manifest, indent=1, default=int))
        return
    if args.bf16_only:
        with np.load(HERE / "golden_small.npz") as z:
            store = {k: z[k] for k in z.files}
        manifest = json.loads((HERE / "golden_manifest.json").read_text())
        run_bf16_sets(ref, np.random.default_rng(2025), store, manifest)
        np.savez_compressed(HERE / "golden_small.npz", **store)
        (HERE / "golden_manifest.json").write_text(json.dumps(manifest, indent=1, default=int))
        return
    rng = np.random.default_rng(2024)
    store = {}
    manifest = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                "numpy": np.__version__, "attention": {}, "pipeline": {}, "quant": {}}
    manifest["small"] = [list(x) for x in run_small(ref, rng, store)]
    run_nonfinite_sets(ref, store, manifest)
    run_attention_sets(ref, store, manifest)
    run_pipeline_compat(ref, store, manifest)
    check_profiler(ref, manifest)
    run_bf16_sets(ref, np.random.default_rng(2025), store, manifest)
    if not args.skip_quant:
        run_quant_sets(ref, manifest, store)
    np.savez_compressed(HERE / "golden_small.npz", **store)
    (HERE / "golden_manifest.json").write_text(json.dumps(manifest, indent=1, default=int))
    print("wrote", HERE / "golden_small.npz", (HERE / "golden_small.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
