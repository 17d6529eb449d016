"""Time the reference's own CPU decode against the numpy restatement (config 1).

Run in a container that has the reference checked out (read-only is fine):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/time_reference.py --reference /path/to/kitty-kv

The reference cannot travel to the GPU box (it is not installed there), so the
CPU baseline that ``bench.py`` times on the box's host cores is the numpy
restatement in ``oracle/``.  This script measures, on one host, both the
reference's ``paged_attention_reference`` (``kitty/kernels/attention.py:46-189``)
and the restatement on the same config-1 step (batch 1, 32 q / 8 KV heads, 4096
tokens: 31 quantised pages, 32 sinks, a 96-token tail), and writes the factor to
``reference_timing.json`` beside this script; ``bench.py`` reports it next to its
own CPU numbers so the port's speed relative to the reference is on record.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

import make_golden as MG  # noqa: E402
import synthetic  # noqa: E402
from oracle import kitty_oracle as O  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    ref = MG.load_reference(args.reference)
    from kitty_ref.kernels import paged_attention_reference
    case = synthetic.make_decode_case(1, 1, 32, 8, 128, [4096], sink=32, group=128, boost_rate=0.125)
    phys_of, n_phys = MG.phys_layout(case, 1001)
    pools = MG.build_pools_ref(ref, case, phys_of, n_phys)
    sq = case.seqs[0]
    sk, sv = sq.sink_kv(); tk, tv = sq.tail_kv()
    pages = [int(x) for x in phys_of[0][:sq.n_pages]]
    H, D = case.num_kv_heads, case.head_dim

    def run_ref():
        return paged_attention_reference(
            q=torch.from_numpy(case.q[0]), page_list=pages, key_baseline=pools[0], key_boost=pools[1],
            key_meta=pools[2], value_pool=pools[3], value_meta=pools[4],
            boost_idx=torch.from_numpy(case.boost_idx), D_boost=case.d_boost, sink_k=torch.from_numpy(sk),
            sink_v=torch.from_numpy(sv), qbuf_k=torch.from_numpy(tk), qbuf_v=torch.from_numpy(tv),
            num_q_heads=case.num_q_heads, num_kv_heads=H, head_dim=D).numpy()

    np_pools = [p.numpy() for p in pools]

    def run_port():
        return O.paged_attention(case.q[0], pages, *np_pools, case.boost_idx, case.d_boost, sk, sv, tk, tv,
                                 case.num_q_heads, H, D)

    a, b = run_ref(), run_port()           # warm-up, and the two must agree
    np.testing.assert_allclose(a.astype(np.float32), b.astype(np.float32), atol=2e-3, rtol=1e-2)
    t_ref, t_port = [], []
    for _ in range(args.reps):
        t0 = time.perf_counter(); run_ref(); t_ref.append(time.perf_counter() - t0)
        t0 = time.perf_counter(); run_port(); t_port.append(time.perf_counter() - t0)
    rec = {"what": "config 1 decode step (batch 1, 32 q / 8 KV heads, 31 pages, 32 sinks, 96-token tail), "
                   "one Python thread issuing; torch / numpy use their default intra-op threads",
           "reference": "kitty/kernels/attention.py:46-189 paged_attention_reference (reference's CPU torch path)",
           "port": "oracle/kitty_oracle.py paged_attention (numpy restatement)",
           "host_cpus": os.cpu_count(), "torch_threads": torch.get_num_threads(),
           "reference_s_per_step": round(min(t_ref), 4), "port_s_per_step": round(min(t_port), 4),
           "port_speedup_over_reference": round(min(t_ref) / min(t_port), 2), "reps": args.reps,
           "measured_in": "the build container (no GPU), not the GPU box"}
    (HERE / "reference_timing.json").write_text(json.dumps(rec, indent=1) + "\n")
    print(json.dumps(rec))


if __name__ == "__main__":
    main()
