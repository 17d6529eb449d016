"""Decode parity at the benchmark shapes (configs 2, 4 and 5), against the oracle.

The workloads are built exactly as ``bench.py`` builds them (same seeded synthetic
inputs, the CUDA page quantiser filling the resident pools, the library's automatic
split plan), decoded once through ``paged_attention_batched``, and sampled rows are
compared with the numpy oracle (the restatement of the reference's
``paged_attention_reference``, ``kitty/kernels/attention.py:46-189``) over every
query head at the fp16 tolerance atol 2e-3 / rtol 1e-2:

* config 2: batch 32 x 32768 tokens (255 pages), 32 q / 8 KV heads, K = 16;
* config 4: batch 64 x 131072 tokens (1023 pages), 64 q / 8 KV heads (GQA 8:1);
* config 5: 256 sequences of 1024-65536 tokens with random tails, the block table a
  seeded permutation of a shared pool, K = 32.

These are the shapes where the integer kernel's fixed-point folding (23-bit key
digits, 16-bit P' digits) meets the longest softmax ranges, so the error budget is
checked where the benchmark runs it.
"""

from __future__ import annotations

import pytest
import torch

import bench as BN

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _decode(workload, batch=0):
    spec = dict(BN.WORKLOADS[workload])
    if batch:
        spec["batch"] = batch
    seqs, heads = BN.shard(spec, 1, 0)
    w = BN.build_decode_workload(spec, seqs, heads, DEV, seed=1234)
    out = BN.decode_call(w)
    torch.cuda.synchronize()
    return w, out


@pytest.mark.parametrize("workload", ["config2", "config4", "config5"])
def test_benchmark_shape_vs_oracle(workload):
    w, out = _decode(workload)
    assert torch.isfinite(out).all()
    rows = BN.oracle_sample(w["layout"])
    assert len(rows) >= 2
    ratio, abs_err = BN.oracle_check(w, out, rows)
    assert ratio <= 1.0, f"{workload}: rows {rows}: max |err| / tol = {ratio:.3f} (max |err| {abs_err:.2e})"
    del w, out
    torch.cuda.empty_cache()


def test_config5_every_tail_length_class():
    """Config 5's random tails: rows with an empty tail, a nearly full one and a short
    sequence, each against the oracle."""
    w, out = _decode("config5")
    lay = w["layout"]
    pick = {min(range(len(lay)), key=lambda i: lay[i][1]),           # shortest tail (0 if drawn)
            max(range(len(lay)), key=lambda i: lay[i][1]),           # longest tail
            min(range(len(lay)), key=lambda i: lay[i][0])}           # fewest pages
    ratio, abs_err = BN.oracle_check(w, out, sorted(pick))
    assert ratio <= 1.0, f"rows {sorted(pick)}: max |err| / tol = {ratio:.3f} (max |err| {abs_err:.2e})"
    del w, out
    torch.cuda.empty_cache()
