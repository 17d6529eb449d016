"""Seeded synthetic KV workloads with the shapes and value distributions of the
benchmark configurations.

There is no public dataset behind the benchmarks: keys/values are float16
N(0, 1) with, per KV head, 16 of the ``head_dim`` channels multiplied by
U(4, 10) (outlier channels, applied independently to K and to V), and queries
are float16 N(0, 1).  The boost index follows the sensitivity profiler's rule
(``kitty/sensitivity.py:164-207`` in the reference): channels ranked by mean
|K| over the same tensor, the top ``d_boost`` get ranks 0..K-1, all others the
sentinel.

Everything here is generated with ``numpy.random.default_rng`` (PCG64), so the
bytes are identical on every machine with the same numpy, which is what lets
committed hashes of reference outputs pin the GPU results.  ``torch_*``
helpers generate the same *distribution* directly on a CUDA device for
benchmark-sized inputs (bit-reproducibility is not needed there).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

NUM_OUTLIER_CHANNELS = 16
OUTLIER_LOW, OUTLIER_HIGH = 4.0, 10.0


def make_kv(rng: np.random.Generator, num_heads: int, num_tokens: int, head_dim: int,
            n_outlier: int = NUM_OUTLIER_CHANNELS):
    """K and V as (H, T, D) float16 with per-head outlier channels."""
    out = []
    for _ in range(2):
        x = rng.standard_normal((num_heads, num_tokens, head_dim), dtype=np.float32)
        for h in range(num_heads):
            ch = rng.permutation(head_dim)[:n_outlier]
            mult = rng.uniform(OUTLIER_LOW, OUTLIER_HIGH, size=n_outlier).astype(np.float32)
            x[h][:, ch] *= mult
        out.append(x.astype(np.float16))
    return out[0], out[1]


def make_q(rng: np.random.Generator, shape) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16)


def channel_scores(keys: Sequence[np.ndarray]) -> np.ndarray:
    """Mean |K| per (head, channel) over all tokens of all given (H, T, D) tensors."""
    total = None
    count = 0
    for k in keys:
        s = np.abs(k.astype(np.float32)).sum(axis=1, dtype=np.float64)
        total = s if total is None else total + s
        count += k.shape[1]
    return (total / max(count, 1)).astype(np.float32)


def boost_idx_from_scores(scores: np.ndarray, d_boost: int, sentinel: int) -> np.ndarray:
    """Rank r < d_boost -> index r; other channels -> sentinel (uint8)."""
    order = np.argsort(-np.asarray(scores, dtype=np.float32), axis=-1, kind="stable")
    out = np.full(scores.shape, sentinel, dtype=np.uint8)
    for rank in range(d_boost):
        np.put_along_axis(out, order[..., rank:rank + 1], np.uint8(rank), axis=-1)
    return out


@dataclass
class SequenceKV:
    """One sequence's float16 cache contents, split into the Kitty regions.

    Tokens [0, sink) are the attention sinks, then ``n_pages`` groups of
    ``group`` tokens that become quantised pages, then ``tail`` tokens that
    stay float16 (the Key Q-buffer and, aligned with it, the value tail).
    """
    k: np.ndarray          # (H, T, D) float16
    v: np.ndarray          # (H, T, D) float16
    sink: int
    n_pages: int
    tail: int
    group: int

    def page_keys(self) -> np.ndarray:
        """(n_pages, H, D, G) float16: the (D, G) transposed key block per page-head."""
        s, G, n = self.sink, self.group, self.n_pages
        H, D = self.k.shape[0], self.k.shape[2]
        blk = self.k[:, s:s + n * G].reshape(H, n, G, D)   # (H, n, G, D)
        return np.ascontiguousarray(blk.transpose(1, 0, 3, 2))

    def page_values(self) -> np.ndarray:
        """(n_pages, H, G, D) float16."""
        s, G, n = self.sink, self.group, self.n_pages
        H, D = self.v.shape[0], self.v.shape[2]
        blk = self.v[:, s:s + n * G].reshape(H, n, G, D)
        return np.ascontiguousarray(blk.transpose(1, 0, 2, 3))

    def sink_kv(self):
        return self.k[:, :self.sink], self.v[:, :self.sink]

    def tail_kv(self):
        a = self.sink + self.n_pages * self.group
        return self.k[:, a:a + self.tail], self.v[:, a:a + self.tail]


@dataclass
class DecodeCase:
    """A seeded batched decode problem."""
    seqs: List[SequenceKV]
    q: np.ndarray                      # (B, Hq, D) float16
    boost_idx: np.ndarray              # (H, D) uint8
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    group: int
    d_boost: int
    sentinel: int
    seed: int = 0
    meta: dict = field(default_factory=dict)


def split_context(total: int, sink: int, group: int):
    """T = sink + n*G + tail with tail = (T - sink) % G (the reference's fill order)."""
    if total <= sink:
        return total, 0, 0
    n = (total - sink) // group
    return sink, n, (total - sink) - n * group


def make_decode_case(seed: int, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                     contexts: Sequence[int], sink: int = 32, group: int = 128,
                     boost_rate: float = 0.125, tails: Optional[Sequence[int]] = None) -> DecodeCase:
    """Generate a batched decode case.  ``contexts[b]`` is sequence b's token count;
    if ``tails`` is given it overrides the tail length (n_pages then follows)."""
    rng = np.random.default_rng(seed)
    d_boost = round(boost_rate * head_dim)
    sentinel = min(d_boost + 1, 255)
    seqs = []
    for b in range(batch):
        T = int(contexts[b])
        if tails is not None:
            tail = int(tails[b])
            s = min(sink, T)
            n = max(0, (T - s - tail) // group)
            tail = T - s - n * group
        else:
            s, n, tail = split_context(T, sink, group)
        k, v = make_kv(rng, num_kv_heads, T, head_dim)
        seqs.append(SequenceKV(k=k, v=v, sink=s, n_pages=n, tail=tail, group=group))
    q = make_q(rng, (batch, num_q_heads, head_dim))
    scores = channel_scores([sq.k for sq in seqs])
    bidx = boost_idx_from_scores(scores, d_boost, sentinel)
    return DecodeCase(seqs=seqs, q=q, boost_idx=bidx, num_q_heads=num_q_heads,
                      num_kv_heads=num_kv_heads, head_dim=head_dim, group=group,
                      d_boost=d_boost, sentinel=sentinel, seed=seed)


def config1_case(seed: int = 1) -> DecodeCase:
    """Benchmark config 1: B=1, 32 q / 8 kv heads, D=128, T=4096 (32 sinks + 31 pages
    + a 96-token tail), INT4 ratio 12.5%."""
    return make_decode_case(seed, 1, 32, 8, 128, [4096])


# ---------------------------------------------------------------------------
# device-side generation for benchmark-sized inputs
# ---------------------------------------------------------------------------

def torch_make_kv(gen, num_heads: int, num_tokens: int, head_dim: int, device,
                  n_outlier: int = NUM_OUTLIER_CHANNELS):
    """Same distribution as :func:`make_kv`, generated on ``device`` with torch."""
    import torch
    out = []
    for _ in range(2):
        x = torch.randn(num_heads, num_tokens, head_dim, generator=gen, device=device,
                        dtype=torch.float32)
        mult = torch.ones(num_heads, head_dim, device=device)
        for h in range(num_heads):
            ch = torch.randperm(head_dim, generator=gen, device=device)[:n_outlier]
            mult[h, ch] = torch.empty(n_outlier, device=device).uniform_(
                OUTLIER_LOW, OUTLIER_HIGH, generator=gen)
        out.append((x * mult[:, None, :]).to(torch.float16))
    return out[0], out[1]
