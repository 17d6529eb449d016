"""Rebuild the golden decode / quantisation cases from their recorded seeds.

The manifest written by ``tests/golden/make_golden.py`` stores only seeds and
shapes for the 128-channel cases; these helpers regenerate the exact inputs
with ``synthetic`` (and check their hashes) so both the numpy oracle
(CPU tests) and the CUDA kernels (GPU tests) can be compared against the
reference's recorded outputs.
"""

from __future__ import annotations

import numpy as np

import synthetic

from conftest import sha


def decode_case_from_manifest(entry) -> synthetic.DecodeCase:
    case = synthetic.make_decode_case(entry["seed"], entry["batch"], entry["num_q_heads"],
                                      entry["num_kv_heads"], entry["head_dim"], entry["contexts"],
                                      sink=entry["sink"], group=entry["group"],
                                      boost_rate=entry["boost_rate"], tails=entry["tails"])
    ins = entry["inputs_sha"]
    assert sha(case.q) == ins["q"], "synthetic generator drifted (q)"
    assert sha(case.boost_idx) == ins["boost_idx"], "synthetic generator drifted (boost_idx)"
    assert [sha(s.k) for s in case.seqs] == ins["k"], "synthetic generator drifted (k)"
    assert [sha(s.v) for s in case.seqs] == ins["v"], "synthetic generator drifted (v)"
    return case


def phys_layout(case, seed, n_phys):
    total = sum(s.n_pages for s in case.seqs)
    perm = np.random.default_rng(seed).permutation(n_phys)[:total]
    phys_of, at = [], 0
    for s in case.seqs:
        phys_of.append(perm[at:at + s.n_pages].astype(np.int32))
        at += s.n_pages
    return phys_of


def padded_regions(case, dtype=np.float16):
    """(B, H, S, D) sinks, (B, H, Q, D) tails (zero padded) and their lengths
    (float32 arrays of bf16 values for a bfloat16 case)."""
    B, H, D = len(case.seqs), case.num_kv_heads, case.head_dim
    S = max([s.sink for s in case.seqs] + [1])
    Q = max([s.tail for s in case.seqs] + [1])
    sk = np.zeros((B, H, S, D), dtype); sv = np.zeros_like(sk)
    tk = np.zeros((B, H, Q, D), dtype); tv = np.zeros_like(tk)
    for b, s in enumerate(case.seqs):
        a, c = s.sink_kv(); sk[b, :, :s.sink] = a; sv[b, :, :s.sink] = c
        a, c = s.tail_kv(); tk[b, :, :s.tail] = a; tv[b, :, :s.tail] = c
    sl = np.array([s.sink for s in case.seqs], np.int32)
    tl = np.array([s.tail for s in case.seqs], np.int32)
    return sk, sv, sl, tk, tv, tl


def block_table(case, phys_of):
    B = len(case.seqs)
    W = max([s.n_pages for s in case.seqs] + [1])
    bt = np.zeros((B, W), np.int32)
    for b, p in enumerate(phys_of):
        bt[b, :len(p)] = p
    return bt, np.array([len(p) for p in phys_of], np.int32)


def bf16_case_from_manifest(entry, bf16_round) -> synthetic.DecodeCase:
    """A recorded bfloat16 decode case: the fp16 generator's keys, values and queries
    rounded to bf16 (float32 arrays); boost_idx as generated."""
    case = synthetic.make_decode_case(entry["seed"], entry["batch"], entry["num_q_heads"],
                                      entry["num_kv_heads"], entry["head_dim"], entry["contexts"],
                                      sink=entry["sink"], group=entry["group"], boost_rate=entry["boost_rate"])
    for s in case.seqs:
        s.k = bf16_round(s.k.astype(np.float32))
        s.v = bf16_round(s.v.astype(np.float32))
    case.q = bf16_round(case.q.astype(np.float32))
    return case
