"""Host-side logic of bench.py: workload layouts, algorithmic byte counts, sharding,
and the reference (CPU) arm on the small configuration."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_config2_bytes_match_the_specification():
    spec = bench.WORKLOADS["config2"]
    lay = bench.sequence_layout(spec)
    assert lay == [(255, 96)] * 32
    assert bench.decode_bytes(lay, 32, 8, 128, 128, 16) == 652_377_984


def test_config3_and_config4_bytes():
    lay3 = bench.sequence_layout(bench.WORKLOADS["config3"])
    assert lay3 == [(255, 96)] * 8
    # fp16 K and V in (2 x 534.8 MB) + packed planes and metadata out (167.1 MB)
    assert bench.quantize_bytes(lay3, 8, 128, 128, 32) == 8 * 255 * 8 * (2 * 128 * 128 * 2 + 10240)
    lay4 = bench.sequence_layout(bench.WORKLOADS["config4"])
    assert lay4 == [(1023, 96)] * 64
    assert abs(bench.decode_bytes(lay4, 64, 8, 128, 128, 16) - 5.131e9) < 0.01e9


def test_config5_layout_is_seeded_and_in_range():
    spec = bench.WORKLOADS["config5"]
    a, b = bench.sequence_layout(spec), bench.sequence_layout(spec)
    assert a == b and len(a) == 256
    for n, t in a:
        T = bench.SINK + n * bench.GROUP + t
        assert 0 <= t < bench.GROUP and 1024 - bench.GROUP <= T <= 65536
    total = bench.decode_bytes(a, 32, 8, 128, 128, 32)
    assert 4.5e9 < total < 6.5e9          # ~5.5 GB at a mean context of ~33K


@pytest.mark.parametrize("name,world", [("config4", 2), ("config4", 8), ("config5", 2), ("config5", 8),
                                        ("config2", 4)])
def test_shards_cover_the_workload(name, world):
    spec = bench.WORKLOADS[name]
    parts = [bench.shard(spec, world, r) for r in range(world)]
    if spec["shard"] == "kv_head":
        heads = sorted(h for _, (h0, h1) in parts for h in range(h0, h1))
        assert heads == list(range(spec["num_kv_heads"]))
        assert all(seqs == list(range(spec["batch"])) for seqs, _ in parts)
    elif spec["shard"] == "sequence":
        seqs = sorted(s for ss, _ in parts for s in ss)
        assert seqs == list(range(spec["batch"]))
        lay = bench.sequence_layout(spec)
        loads = [bench.decode_bytes([lay[s] for s in ss], 32, 8, 128, 128, 32) for ss, _ in parts]
        assert max(loads) <= 1.02 * sum(loads) / world + 1e8     # LPT keeps ranks within a few percent
    else:   # replicas: every rank builds the full per-GPU workload
        assert all(ss == list(range(spec["batch"])) and hh == (0, 8) for ss, hh in parts)


def test_reference_arm_runs_on_cpu():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "config1",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def _cpu_workload():
    """A small decode workload in the shape bench.build_decode_workload returns, on CPU
    tensors, with pools quantised by the oracle (permuted physical pages, ragged tails)."""
    import numpy as np
    import torch
    import synthetic
    from oracle import kitty_oracle as O
    case = synthetic.make_decode_case(3, 3, 16, 4, 128, [32 + 5 * 128 + 7, 32 + 2 * 128, 32 + 3 * 128 + 100],
                                      tails=[7, 0, 100])
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    total = sum(s.n_pages for s in case.seqs)
    perm = np.random.default_rng(5).permutation(total + 2)[:total]
    pools = [np.zeros((total + 2, H, D, G // 4), np.uint8), np.zeros((total + 2, H, K, G // 4), np.uint8),
             np.zeros((total + 2, H, 2, D), np.float16), np.zeros((total + 2, H, G, D // 4), np.uint8),
             np.zeros((total + 2, H, G, 2), np.float16)]
    bt = np.zeros((3, 5), np.int32)
    at = 0
    for b, s in enumerate(case.seqs):
        low, high, sc, zp = O.quantize_key_pages(s.page_keys(), case.boost_idx, K, case.sentinel)
        codes, vs, vz = O.quantize_value_pages(s.page_values())
        ids = perm[at:at + s.n_pages]
        pools[0][ids], pools[1][ids] = low, high
        pools[2][ids] = np.stack([sc, zp], axis=2)
        pools[3][ids], pools[4][ids] = codes, np.stack([vs, vz], axis=3)
        bt[b, :s.n_pages] = ids
        at += s.n_pages
    sk = np.stack([s.sink_kv()[0] for s in case.seqs]); sv = np.stack([s.sink_kv()[1] for s in case.seqs])
    tk = np.zeros((3, H, 100, D), np.float16); tv = np.zeros_like(tk)
    for b, s in enumerate(case.seqs):
        a, c = s.tail_kv(); tk[b, :, :s.tail] = a; tv[b, :, :s.tail] = c
    T = torch.from_numpy
    w = dict(q=T(case.q), bt=T(bt), pools=[T(p) for p in pools], bidx=T(case.boost_idx), K=K, sink_k=T(sk),
             sink_v=T(sv), tail_k=T(tk), tail_v=T(tv), tail_len=T(np.array([7, 0, 100], np.int32)),
             layout=[(s.n_pages, s.tail) for s in case.seqs], H=H, Hq=case.num_q_heads, D=D)
    sl = np.full(3, 32, np.int32)
    exp = O.paged_attention_batched(case.q, bt, np.array([s.n_pages for s in case.seqs]), tuple(pools),
                                    case.boost_idx, K, sk, sv, sl, tk, tv, np.array([7, 0, 100]))
    return w, exp


def test_oracle_check_accepts_the_oracle_and_flags_an_error():
    import numpy as np
    import torch
    w, exp = _cpu_workload()
    assert bench.oracle_sample(w["layout"]) == [0, 1]     # first = most pages, fewest pages
    rows = [0, 1, 2]
    ratio, abs_err = bench.oracle_check(w, torch.from_numpy(exp), rows)
    assert ratio == 0.0 and abs_err == 0.0
    bad = exp.copy()
    bad[2, 13, 77] += np.float16(0.05)          # one element of the last KV head of row 2
    ratio, abs_err = bench.oracle_check(w, torch.from_numpy(bad), rows)
    assert ratio > 1.0 and abs_err > 0.04
    assert bench.oracle_sample([(255, 96)] * 32) == [0, 31]
