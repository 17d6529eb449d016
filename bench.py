"""Benchmark: fused quantized paged decode attention (and page quantisation) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kitty|reference]
                    [--workload config1..config5] [--variant auto|simt|int8|tc]

One step = one decode step of one layer for the whole batch (every sequence,
every query head) over the quantised KV pools resident in HBM; for config3 one
step = quantising every page-head of the prefill (keys and values).  Workloads
(the benchmark configurations; synthetic data with the specified shapes and
distribution: fp16 N(0,1) K/V with 16 outlier channels per KV head scaled by
U(4,10), fp16 N(0,1) queries, boost indices from mean |K|):

  config1  batch 1, 32 q / 8 kv heads, 4096 tokens (31 pages)          weak
  config2  batch 32, 32 / 8, 32768 tokens (255 pages) - the default      weak: every rank its own 32 sequences
  config3  quantise a 32768-token prefill, batch 8, 8 kv heads, K = 32   weak
  config4  batch 64, 64 / 8 (GQA 8:1), 131072 tokens (1023 pages)        strong: KV heads sharded over ranks,
                                                                          NCCL all-gather of the outputs
  config5  256 sequences, lengths U[1024, 65536], tails U{0..127},       strong: sequences assigned to ranks by
           permuted shared pool, K = 32                                    longest-processing-time on their bytes

Reported (one JSON line from rank 0):
  value      algorithmic HBM GB/s of the whole job (bytes every step must read
             and write: each page-head once, fp16 sinks and tails, q, out,
             block table) / device time, max over ranks;
  e2e        the same metric through the public API with host buffers (q and
             block table copied H2D from pinned memory and the output copied
             D2H inside the timed region, every step; config3: keys and values
             H2D, packed pools D2H);
  roofline   achieved GB/s of the dominant launch vs the measured HBM copy
             bandwidth, with the DRAM traffic of one ncu capture where one exists;
  cpu_baseline  the numpy oracle (CPU restatement of the reference's path) on
             a bounded sample, N=1 rank 0 only.
Inputs (>= 650 MB per GPU, except config1) exceed the 126 MB L2, so no flush is
needed; config1 (3 MB) is timed back to back and says so.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kitty-kv_b200"))

METRIC = "quantized paged decode-attn HBM GB/s (% of peak) & tokens/s at 1/2/4/8 B200"
# DRAM bytes (read + write) of one decode launch per algorithmic byte, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of this script on the same
# workload and kernel: (captured traffic, algorithmic bytes of the captured launch).
# Every page-head is read once, so the ratio carries over to other batch sizes and to
# each rank's share.  Config 2 was captured at full size, config 4 at `--batch 8`,
# config 5 at `--batch 32` (its first 32 sequences).
MEASURED_TRAFFIC = {
    ("config2", "decode_i8_kernel"): (652_503_552 + 4_320_256, 652_377_984),
    ("config4", "decode_i8_kernel"): (642_340_352 + 8_742_912, 641_400_800),
    ("config5", "decode_i8_kernel"): (624_861_952 + 4_979_200, 624_760_012),
}


def measured_traffic(workload, kernel, nbytes, pages_only=False):
    """DRAM bytes of one decode launch on this rank moving `nbytes` algorithmic bytes,
    scaled from the capture; None where no capture of this workload and kernel exists
    (and for the pages-only form, which the captures do not cover)."""
    t = MEASURED_TRAFFIC.get((workload, kernel))
    if t is None or pages_only:
        return None
    return int(round(t[0] / t[1] * nbytes))


WORKLOADS = {
    "config1": dict(kind="decode", batch=1, num_q_heads=32, num_kv_heads=8, head_dim=128, context=4096,
                    boost_rate=0.125, shard="replica"),
    "config2": dict(kind="decode", batch=32, num_q_heads=32, num_kv_heads=8, head_dim=128, context=32768,
                    boost_rate=0.125, shard="replica"),
    "config3": dict(kind="quantize", batch=8, num_q_heads=8, num_kv_heads=8, head_dim=128, context=32768,
                    boost_rate=0.25, shard="replica"),
    "config4": dict(kind="decode", batch=64, num_q_heads=64, num_kv_heads=8, head_dim=128, context=131072,
                    boost_rate=0.125, shard="kv_head"),
    "config5": dict(kind="decode", batch=256, num_q_heads=32, num_kv_heads=8, head_dim=128,
                    context=[1024, 65536], boost_rate=0.25, shard="sequence", random_tails=True,
                    permuted_pool=True),
}
SINK, GROUP = 32, 128


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def page_head_bytes(D, G, K):
    return D * G // 4 + K * G // 4 + 2 * D * 2 + G * D // 4 + G * 2 * 2


def sequence_layout(spec):
    """(n_pages, tail) of every sequence: T = sinks + n * G + tail.  Config 5 draws
    T ~ U[1024, 65536] and tail ~ U{0..G-1} independently (seeded)."""
    import numpy as np
    B = spec["batch"]
    if isinstance(spec["context"], list):
        lo, hi = spec["context"]
        rng = np.random.default_rng(20250105)
        T = rng.integers(lo, hi + 1, size=B)
        tails = rng.integers(0, GROUP, size=B) if spec.get("random_tails") else (T - SINK) % GROUP
        n = np.maximum((T - SINK - tails) // GROUP, 0)
        return [(int(a), int(b)) for a, b in zip(n, tails)]
    T = spec["context"]
    n = (T - SINK) // GROUP
    return [(n, T - SINK - n * GROUP)] * B


def decode_bytes(layout, Hq, H, D, G, K, fp16_regions=True):
    """Bytes one decode step must move for these sequences (each page-head once, fp16
    sinks and tails for keys and values unless the step skips them, q and out,
    block-table entries)."""
    f = 1 if fp16_regions else 0
    return sum(H * (n * page_head_bytes(D, G, K) + f * (SINK + t) * D * 2 * 2) + 2 * Hq * D * 2 + 4 * n
               for n, t in layout)


def quantize_bytes(layout, H, D, G, K):
    """Bytes one prefill quantisation moves: fp16 keys and values in, packed planes and
    metadata out."""
    pages = sum(n for n, _ in layout)
    return pages * H * (2 * G * D * 2 + page_head_bytes(D, G, K))


def shard(spec, world, rank):
    """(sequence ids, KV-head range) built by ``rank``."""
    layout = sequence_layout(spec)
    H = spec["num_kv_heads"]
    if spec["shard"] == "kv_head" and world > 1:
        from kitty.distributed import kv_head_range
        return list(range(spec["batch"])), kv_head_range(H, world, rank)
    if spec["shard"] == "sequence" and world > 1:
        from kitty.distributed import lpt_assign, sequence_costs
        costs = sequence_costs([n for n, _ in layout], [SINK] * len(layout), [t for _, t in layout], H,
                               page_head_bytes(spec["head_dim"], GROUP, round(spec["boost_rate"] * spec["head_dim"])),
                               spec["head_dim"])
        return lpt_assign(costs, world)[rank], (0, H)
    return list(range(spec["batch"])), (0, H)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 5 ms while the timed
    region runs (a decode step is well under a millisecond, so nvidia-smi's 200 ms
    polling would see nothing)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self.error = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(visible.split(",")[self.idx]) if visible and visible.split(",")[0].isdigit() else self.idx
            h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML unavailable: report it instead of clocks
            self.error = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception:
                    pass
                time.sleep(0.005)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        return False

    def summary(self):
        if self.error:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error], "samples": 0}
        sm = [c for c, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm)}


# ---------------------------------------------------------------------------
# workload construction on the GPU
# ---------------------------------------------------------------------------

def _kv(spec, b, T, heads, device, seed):
    """fp16 keys and values (H_local, T, D) of sequence ``b``: one generator per
    (sequence, KV head), so a shard builds exactly its part of the full workload."""
    import torch
    import synthetic
    ks, vs = [], []
    for h in range(*heads):
        gen = torch.Generator(device=device)
        gen.manual_seed(seed * 1_000_003 + b * 1009 + h)
        k, v = synthetic.torch_make_kv(gen, 1, T, spec["head_dim"], device)
        ks.append(k[0]); vs.append(v[0])
    return torch.stack(ks), torch.stack(vs)


def _boost_idx(spec, seq_ids, layout, heads, device, seed):
    """boost_idx (H_local, D) from mean |K| over the built sequences (the profiler's rule:
    the channel with the r-th largest score gets index r < K, the others the sentinel)."""
    import torch
    D = spec["head_dim"]
    K = round(spec["boost_rate"] * D)
    sentinel = min(K + 1, 255)
    H = heads[1] - heads[0]
    score = torch.zeros(H, D, dtype=torch.float64, device=device)
    for b in seq_ids:
        n, t = layout[b]
        k, _ = _kv(spec, b, SINK + n * GROUP + t, heads, device, seed)
        score += k.float().abs().sum(dim=1, dtype=torch.float64)
    order = torch.argsort(-score, dim=-1, stable=True)
    bidx = torch.full((H, D), sentinel, dtype=torch.uint8, device=device)
    bidx.scatter_(1, order[:, :K], torch.arange(K, dtype=torch.uint8, device=device).expand(H, K).contiguous())
    return bidx, K, sentinel


def build_decode_workload(spec, seq_ids, heads, device, seed):
    """Quantise the shard's sequences (all their pages, its KV heads) into resident pools
    with the CUDA page quantiser; keep the fp16 sinks and tails."""
    import torch
    from kitty import kernels as KK
    layout_all = sequence_layout(spec)
    D, G, S = spec["head_dim"], GROUP, SINK
    g = spec["num_q_heads"] // spec["num_kv_heads"]
    h0, h1 = heads
    H, Hq = h1 - h0, (h1 - h0) * g
    lay = [layout_all[b] for b in seq_ids]
    B = len(lay)
    bidx, K, sentinel = _boost_idx(spec, seq_ids, layout_all, heads, device, seed)
    P = max(1, sum(n for n, _ in lay))
    pools = [torch.zeros(P, H, D, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, K, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, 2, D, dtype=torch.float16, device=device),
             torch.zeros(P, H, G, D // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, G, 2, dtype=torch.float16, device=device)]
    if spec.get("permuted_pool"):
        cpu_gen = torch.Generator().manual_seed(seed + 77)
        page_ids = torch.randperm(P, generator=cpu_gen).to(torch.int32).to(device)
    else:
        page_ids = torch.arange(P, dtype=torch.int32, device=device)
    maxn = max([n for n, _ in lay] + [0])
    maxt = max([t for _, t in lay] + [0])
    bt = torch.zeros(B, max(maxn, 1), dtype=torch.int32, device=device)
    sink_k = torch.empty(B, H, S, D, dtype=torch.float16, device=device)
    sink_v = torch.empty_like(sink_k)
    tail_k = torch.zeros(B, H, max(maxt, 1), D, dtype=torch.float16, device=device)
    tail_v = torch.zeros_like(tail_k)
    q = torch.empty(B, Hq, D, dtype=torch.float16, device=device)
    start = 0
    for i, (b, (n, t)) in enumerate(zip(seq_ids, lay)):
        T = S + n * G + t
        k, v = _kv(spec, b, T, heads, device, seed)
        if n:
            dst = page_ids[start:start + n]
            offs = ((S + torch.arange(n, device=device) * G) * D).to(torch.int64)
            KK.quantize_key_pages(k, offs, (T * D, D, 1), bidx, K, sentinel, dst, *pools[:3], H, D, G)
            KK.quantize_value_pages(v, offs, (T * D, D, 1), dst, pools[3], pools[4], H, D, G)
            bt[i, :n] = dst
        sink_k[i] = k[:, :S]; sink_v[i] = v[:, :S]
        if t:
            tail_k[i, :, :t] = k[:, S + n * G:]; tail_v[i, :, :t] = v[:, S + n * G:]
        start += n
        gq = torch.Generator(device=device)
        gq.manual_seed(seed * 1_000_003 + b * 1009 + 997)
        q[i] = torch.randn(spec["num_q_heads"], D, generator=gq, device=device)[h0 * g:h1 * g].to(torch.float16)
    npg = torch.tensor([n for n, _ in lay], dtype=torch.int32, device=device)
    tails = [t for _, t in lay]
    tail_len = tails[0] if len(set(tails)) <= 1 else torch.tensor(tails, dtype=torch.int32, device=device)
    torch.cuda.empty_cache()
    torch.cuda.synchronize(device)
    return dict(q=q, bt=bt, npg=npg, pools=pools, bidx=bidx, K=K, sink_k=sink_k, sink_v=sink_v, tail_k=tail_k,
                tail_v=tail_v, tail_len=tail_len, n_pages=maxn, layout=lay, B=B, Hq=Hq, H=H, D=D, G=G)


def decode_call(w, q=None, bt=None, npg=None, out=None):
    from kitty import kernels as KK
    if w.get("pages_only"):   # the quantised pages alone (no fp16 sink / tail tokens)
        return KK.paged_attention_batched(
            w["q"] if q is None else q, w["bt"] if bt is None else bt, w["npg"] if npg is None else npg,
            *w["pools"], w["bidx"], w["K"], sink_len=0, tail_len=0, out=out, max_pages_per_seq=w["n_pages"])
    return KK.paged_attention_batched(
        w["q"] if q is None else q, w["bt"] if bt is None else bt, w["npg"] if npg is None else npg, *w["pools"],
        w["bidx"], w["K"], sink_k=w["sink_k"], sink_v=w["sink_v"], sink_len=SINK, tail_k=w["tail_k"],
        tail_v=w["tail_v"], tail_len=w["tail_len"], out=out, max_pages_per_seq=w["n_pages"])


ATOL, RTOL = 2e-3, 1e-2   # fp16 output tolerance for attention (atol 2e-3 / rtol 1e-2)


def oracle_sample(layout, k=2):
    """Rows of a decode batch whose outputs are checked against the oracle: the first
    row and the row with the most pages (the last row when all are equal), plus the
    shortest row for mixed-length batches."""
    if not layout:
        return []
    rows = [0, max(range(len(layout)), key=lambda i: (layout[i][0], i))]
    if len({n for n, _ in layout}) > 1:
        rows.append(min(range(len(layout)), key=lambda i: (layout[i][0], i)))
    return sorted(set(rows))[:max(k, 1) + 1]


def oracle_check(w, out, rows):
    """Compare rows of a decode output (B, Hq, D) with the numpy oracle (the CPU
    restatement of the reference's paged_attention_reference,
    kitty/kernels/attention.py:46-189) on the same pools, every query head.  The
    row's pages are read back from the resident pools in block-table order.  Returns
    the worst |got - exp| / (atol + rtol |exp|) over the rows (<= 1 passes) and the
    worst absolute error.  The KV heads of a row are independent (query head qh reads
    KV head qh // g), so the oracle runs one KV head per host thread."""
    import concurrent.futures as cf
    import numpy as np
    from oracle import kitty_oracle as O
    bidx = w["bidx"].cpu().numpy()
    tails = w["tail_len"]
    H, Hq, D = w["H"], w["Hq"], w["D"]
    pages_only = bool(w.get("pages_only"))
    g = Hq // H
    jobs = []
    for i in rows:
        n, t = w["layout"][i]
        assert isinstance(tails, int) or int(tails[i].item()) == t
        idx = w["bt"][i, :n].long()
        pools = [p.index_select(0, idx).cpu().numpy() for p in w["pools"]]
        q = w["q"][i].cpu().numpy()
        reg = [w["sink_k"][i].cpu().numpy(), w["sink_v"][i].cpu().numpy(),
               w["tail_k"][i, :, :t].cpu().numpy(), w["tail_v"][i, :, :t].cpu().numpy()]
        if pages_only:
            reg = [r[:, :0] for r in reg]
        got = out[i].float().cpu().numpy()
        for h in range(H):
            jobs.append((q[h * g:(h + 1) * g], [np.ascontiguousarray(p[:, h:h + 1]) for p in pools],
                         bidx[h:h + 1], [r[h:h + 1] for r in reg], got[h * g:(h + 1) * g]))

    def one(job):
        q, pools, b, reg, got = job
        exp = O.paged_attention(q, list(range(pools[0].shape[0])), *pools, b, w["K"], *reg, g, 1, D)
        err = np.abs(got - exp.astype(np.float32))
        ratio = err / (ATOL + RTOL * np.abs(exp.astype(np.float32)))
        return float(np.nan_to_num(ratio, nan=np.inf).max()), float(np.nan_to_num(err, nan=np.inf).max())

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        res = list(ex.map(one, jobs))
    return max((r for r, _ in res), default=0.0), max((a for _, a in res), default=0.0)


def build_quantize_workload(spec, device, seed):
    """fp16 prefill keys and values (B, H, T, D) and empty pools for every page-head."""
    import torch
    layout = sequence_layout(spec)
    D, G, S, H = spec["head_dim"], GROUP, SINK, spec["num_kv_heads"]
    B = spec["batch"]
    n, t = layout[0]
    T = S + n * G + t
    seqs = list(range(B))
    bidx, K, sentinel = _boost_idx(spec, seqs, layout, (0, H), device, seed)
    k_all = torch.empty(B, H, T, D, dtype=torch.float16, device=device)
    v_all = torch.empty_like(k_all)
    for b in seqs:
        k, v = _kv(spec, b, T, (0, H), device, seed)
        k_all[b].copy_(k); v_all[b].copy_(v)
    P = B * n
    pools = [torch.zeros(P, H, D, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, K, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, 2, D, dtype=torch.float16, device=device),
             torch.zeros(P, H, G, D // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, G, 2, dtype=torch.float16, device=device)]
    bb = torch.arange(B, device=device).repeat_interleave(n)
    pp = torch.arange(n, device=device).repeat(B)
    offs = (bb * (H * T * D) + (S + pp * G) * D).to(torch.int64)
    dst = torch.arange(P, dtype=torch.int32, device=device)
    torch.cuda.synchronize(device)
    return dict(k=k_all, v=v_all, offs=offs, dst=dst, pools=pools, bidx=bidx, K=K, sentinel=sentinel, layout=layout,
                B=B, H=H, D=D, G=G, T=T, n=n)


def quantize_call(w, k=None, v=None):
    from kitty import kernels as KK
    k = w["k"] if k is None else k
    v = w["v"] if v is None else v
    T, D, G, H = w["T"], w["D"], w["G"], w["H"]
    KK.quantize_key_pages(k, w["offs"], (T * D, D, 1), w["bidx"], w["K"], w["sentinel"], w["dst"], *w["pools"][:3],
                          H, D, G)
    KK.quantize_value_pages(v, w["offs"], (T * D, D, 1), w["dst"], w["pools"][3], w["pools"][4], H, D, G)


# ---------------------------------------------------------------------------
# CPU restatement timing (numpy oracle) - the reference's path on host cores
# ---------------------------------------------------------------------------

def _cpu_unit(u):
    """One unit of oracle work on a host thread: a (sequence, KV head) decode stream
    (the reference's algorithm for the g query heads that share the KV head), or the
    quantisation of one (sequence, KV head)'s pages."""
    from oracle import kitty_oracle as O
    if u[0] == "decode":
        _, q, pages, pools, bidx, K, sk, sv, tk, tv, g, D = u
        return O.paged_attention(q, pages, *pools, bidx, K, sk, sv, tk, tv, g, 1, D)
    _, keys, vals, bidx, K, sentinel = u
    O.quantize_key_pages(keys, bidx, K, sentinel)
    O.quantize_value_pages(vals)


def cpu_sample(spec, n_seq, seed=11):
    """A bounded CPU sample of the workload built with the numpy quantiser, split into
    independent (sequence, KV head) units; returns (units, algorithmic bytes, label)."""
    import numpy as np
    sys.path.insert(0, str(ROOT))
    import synthetic
    from oracle import kitty_oracle as O
    lay = sequence_layout(spec)[:n_seq]
    n_seq = len(lay)
    contexts = [SINK + n * GROUP + t for n, t in lay]
    case = synthetic.make_decode_case(seed, n_seq, spec["num_q_heads"], spec["num_kv_heads"], spec["head_dim"],
                                      contexts, boost_rate=spec["boost_rate"], tails=[t for _, t in lay])
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    g = case.num_q_heads // H
    units = []
    if spec["kind"] == "quantize":
        for s in case.seqs:
            pk, pv = s.page_keys(), s.page_values()
            for h in range(H):
                units.append(("quantize", np.ascontiguousarray(pk[:, h]), np.ascontiguousarray(pv[:, h]),
                              case.boost_idx[h], K, case.sentinel))
        nbytes = quantize_bytes([(s.n_pages, s.tail) for s in case.seqs], H, D, G, K)
        label = (f"{n_seq} sequence(s) of {spec['batch']} ({H} KV heads x {case.seqs[0].n_pages} pages), numpy "
                 "restatement of the reference's quantize_key_page_torch / quantize_value_page_torch")
        return units, nbytes, label
    for b, s in enumerate(case.seqs):
        low, high, sc, zp = O.quantize_key_pages(s.page_keys(), case.boost_idx, K, case.sentinel)
        codes, vs, vz = O.quantize_value_pages(s.page_values())
        km = np.stack([sc, zp], axis=2); vm = np.stack([vs, vz], axis=3)
        sk, sv = s.sink_kv(); tk, tv = s.tail_kv()
        for h in range(H):
            pools = tuple(np.ascontiguousarray(p[:, h:h + 1]) for p in (low, high, km, codes, vm))
            units.append(("decode", case.q[b, h * g:(h + 1) * g], list(range(s.n_pages)), pools,
                          case.boost_idx[h:h + 1], K, sk[h:h + 1], sv[h:h + 1], tk[h:h + 1], tv[h:h + 1], g, D))
    nbytes = decode_bytes([(s.n_pages, s.tail) for s in case.seqs], case.num_q_heads, H, D, G, K)
    label = (f"{n_seq} of {spec['batch']} sequence(s) ({H} KV heads, "
             f"{'/'.join(str(s.n_pages) for s in case.seqs)} pages), numpy restatement of the reference's "
             "paged_attention_reference")
    return units, nbytes, label


class CpuRunner:
    """Runs the units on a persistent pool of host threads (numpy releases the
    GIL inside its array kernels); BLAS is limited to one thread per worker."""

    def __init__(self, workers):
        import concurrent.futures as cf
        self.workers = workers
        self.ex = cf.ThreadPoolExecutor(max_workers=workers)
        try:
            from threadpoolctl import threadpool_limits
            self._limit = threadpool_limits(limits=1)
        except Exception:
            self._limit = None

    def run(self, units):
        t0 = time.perf_counter()
        list(self.ex.map(_cpu_unit, units))
        return time.perf_counter() - t0

    def close(self):
        self.ex.shutdown()
        if self._limit is not None:
            self._limit.unregister() if hasattr(self._limit, "unregister") else None


def reference_arm(args, spec):
    """--impl reference: the reference path's CPU restatement on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n_seq = min(spec["batch"], 1 if spec["kind"] == "quantize" or spec["context"] == 131072 else 2)
    units, nbytes, label = cpu_sample(spec, n_seq)
    workers = max(1, min(os.cpu_count() or 1, len(units)))
    runner = CpuRunner(workers)
    for _ in range(args.warmup):
        runner.run(units)
    times = [runner.run(units) for _ in range(args.steps)]
    runner.close()
    sec = sum(times) / len(times)
    value = nbytes / sec / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak" if spec["shard"] == "replica" else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, **spec, "sample_sequences": n_seq},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": workers, "kind": "port",
                             "sample": f"{label}, (sequence, KV head) units on a host thread pool",
                             **host_cores(), "reference_own_path": reference_timing()},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if spec["kind"] == "decode":
        line["tokens_per_s"] = round(n_seq / sec, 3)
    print(json.dumps(line), flush=True)


def cpu_baseline(spec, workload):
    n_seq = 1
    units, cbytes, label = cpu_sample(spec, n_seq)
    workers = max(1, min(os.cpu_count() or 1, len(units)))
    runner = CpuRunner(workers)
    runner.run(units)
    reps = 3
    sec = sum(runner.run(units) for _ in range(reps)) / reps
    runner.close()
    return {"value": round(cbytes / sec / 1e9, 4), "unit": "GB/s", "cores": workers, "kind": "port",
            "sample": f"{label}, mean of {reps} runs", **host_cores(), "reference_own_path": reference_timing()}


def host_cores():
    """The host's logical CPUs and torch's intra-op thread count, beside the worker
    threads the CPU leg used (``cores``)."""
    import torch
    return {"host_cpus": os.cpu_count(), "torch_threads": torch.get_num_threads()}


def reference_timing():
    """The reference's own CPU decode (paged_attention_reference) against this numpy
    restatement on one config-1 step, as recorded by tests/golden/time_reference.py
    where the reference is importable (it is not installed on the GPU box)."""
    p = ROOT / "tests" / "golden" / "reference_timing.json"
    return json.loads(p.read_text()) if p.exists() else None


# ---------------------------------------------------------------------------
# GPU arms
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self, torch, dist, device):
        self.torch, self.dist, self.device = torch, dist, device
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def reduce(self, x, op):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed(stream, steps, fn, torch, device, d):
    """Device time of ``steps`` calls (CUDA events on the launch stream), max over ranks,
    and the mean per-call event time of this rank."""
    d.barrier()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    e0 = torch.cuda.Event(enable_timing=True); e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    e1.record(stream)
    torch.cuda.synchronize(device)
    d.barrier()
    torch.cuda.synchronize(device)
    total = d.reduce(e0.elapsed_time(e1), d.dist.ReduceOp.MAX) if d.world > 1 else e0.elapsed_time(e1)
    return total / steps, statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))


def kitty_arm(args, spec):
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    d = Dist(torch, dist, device)
    from kitty.kernels import _lib
    _lib.force_decode_variant(args.variant)
    if spec["kind"] == "quantize":
        line = quantize_arm(args, spec, d, device, local)
    else:
        line = decode_arm(args, spec, d, device, local)
    if d.rank == 0:
        print(json.dumps(line), flush=True)
    d.close()


def decode_arm(args, spec, d, device, local):
    import torch
    world, rank = d.world, d.rank
    replica = spec["shard"] == "replica"
    seq_ids, heads = shard(spec, world, rank)
    seed = 1234 + rank if replica else 1234
    w = build_decode_workload(spec, seq_ids, heads, device, seed)
    w["pages_only"] = bool(spec.get("pages_only"))
    B, Hq, H, D, G, K = w["B"], w["Hq"], w["H"], w["D"], w["G"], w["K"]
    kernel = decode_kernel_name(args.variant, Hq // max(H, 1), D, G, fp16_regions=not w["pages_only"])
    nbytes_local = decode_bytes(w["layout"], Hq, H, D, G, K, fp16_regions=not w["pages_only"])
    nbytes_total = nbytes_local * world if replica else d.reduce(nbytes_local, d.dist.ReduceOp.SUM)
    stream = torch.cuda.current_stream(device)
    gather = spec["shard"] == "kv_head" and world > 1
    if gather:
        # the decode writes this rank's heads head-major, (Hq_local, B, D), through the
        # output strides, straight into the buffer the all-gather sends; the gathered
        # (Hq, B, D) buffer needs no reordering either
        from kitty.distributed import PeerGather, gather_head_outputs
        out_hm = torch.empty(Hq, B, D, dtype=torch.float16, device=device)
        out = out_hm.permute(1, 0, 2)
        full = torch.empty(world * Hq, B, D, dtype=torch.float16, device=device)
        peer_gather = None
        if args.gather == "p2p":   # direct NVLink stores into every rank's exchange region
            try:
                peer_gather = PeerGather(Hq, B, D, device=device)
            except RuntimeError as e:   # raised on every rank alike: all fall back to NCCL
                print(f"[bench] {e}; using the NCCL all-gather", file=sys.stderr)
                args.gather = "nccl"
        if peer_gather is not None:
            gather_fn = lambda src, dst: peer_gather(src, full=dst)
        else:                      # NCCL all_gather_into_tensor
            gather_fn = lambda src, dst: gather_head_outputs(src, full=dst)
    else:
        out = torch.empty(B, Hq, D, dtype=torch.float16, device=device)

    def eager_step():
        decode_call(w, out=out)
        if gather:
            gather_fn(out_hm, full)

    for _ in range(args.warmup):
        eager_step()
    torch.cuda.synchronize(device)
    # device-resident steps replay the step from CUDA graphs (no host work between
    # steps): the decode launches, and for the tensor-parallel configuration the NCCL
    # all-gather captured in the same graph
    def capture(fn):
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            fn()                             # first call on this stream sets up its workspace
            torch.cuda.synchronize(device)
            with torch.cuda.graph(g, stream=cap):
                fn()
        stream.wait_stream(cap)
        torch.cuda.synchronize(device)
        return g

    graphs = []
    g_decode = g_step = None
    launch_mode = "cuda graph replay" + (" (decode + all-gather in one graph)" if gather else "")
    try:
        g_decode = capture(lambda: decode_call(w, out=out))
        graphs.append(g_decode)
        run_decode = g_decode.replay
    except Exception as e:   # capture unavailable: eager launches
        launch_mode = f"eager ({type(e).__name__})"
        run_decode = lambda: decode_call(w, out=out)
    step = run_decode
    if gather:
        try:
            g_step = capture(eager_step)
            graphs.append(g_step)
            step = g_step.replay
        except Exception as e:
            launch_mode += f"; all-gather eager ({type(e).__name__})"
            step = lambda: (run_decode(), gather_fn(out_hm, full))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        ms, _ = timed(stream, args.steps, step, torch, device, d)
    decode_ms, launch_ms = timed(stream, args.steps, run_decode, torch, device, d)
    gather_ms = None
    if gather:
        gather_ms, _ = timed(stream, args.steps, lambda: gather_fn(out_hm, full), torch, device, d)
    step_out = full if gather else out      # the step's result: the gathered heads under TP

    # ---- end to end through the public API with host buffers: a step's inputs (q, block
    # table, page counts) sit in one pinned staging buffer and cross to the device in one
    # copy (as a serving loop would stage them); the output comes back in another (under
    # tensor parallelism the gathered output of all heads, head-major)
    def pack(ts):
        parts = [t.cpu().contiguous().view(torch.uint8).reshape(-1) for t in ts]
        host = torch.empty(sum(p.numel() for p in parts), dtype=torch.uint8).pin_memory()
        views, at = [], 0
        for t, p in zip(ts, parts):
            host[at:at + p.numel()].copy_(p)
            views.append((at, p.numel(), t.dtype, t.shape))
            at += p.numel()   # q (fp16) first, then the int32 tables: 4-byte aligned
        return host, views
    in_host, in_views = pack([w["q"], w["bt"], w["npg"]])
    in_dev = torch.empty_like(in_host, device=device)
    out_host = torch.empty(tuple(step_out.shape), dtype=torch.float16).pin_memory()
    h2d = in_host.numel()
    d2h = out_host.numel() * 2
    if gather:
        e2e_hm = torch.empty(Hq, B, D, dtype=torch.float16, device=device)
        e2e_full = torch.empty_like(full)

    def e2e_step():
        in_dev.copy_(in_host, non_blocking=True)
        q, bt, npg = (in_dev[at:at + n].view(dt).view(shape) for at, n, dt, shape in in_views)
        if gather:
            decode_call(w, q=q, bt=bt, npg=npg, out=e2e_hm.permute(1, 0, 2))
            gather_fn(e2e_hm, e2e_full)
            out_host.copy_(e2e_full, non_blocking=True)
        else:
            out_host.copy_(decode_call(w, q=q, bt=bt, npg=npg), non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize(device)
    e2e_ms, _ = timed(stream, args.steps, e2e_step, torch, device, d)
    same = bool(torch.equal(step_out.cpu(), out_host))
    gather_exact = None
    if gather:
        # the exchanged output against an NCCL all-gather of the same per-rank slices
        ref_full = torch.empty_like(full)
        d.dist.all_gather_into_tensor(ref_full, out_hm)
        ok = torch.tensor([1 if torch.equal(ref_full, full) else 0], device=device)
        d.dist.all_reduce(ok, op=d.dist.ReduceOp.MIN)
        gather_exact = bool(ok.item())
        same = same and gather_exact
    # graphs holding NCCL calls are released before the process group is destroyed
    step = run_decode = g_decode = g_step = None
    graphs.clear()
    if gather and peer_gather is not None:
        peer_gather.close()
    # the timed output against the oracle on sampled rows of this rank's batch
    check = None
    if rank == 0:
        rows = oracle_sample(w["layout"])
        t0 = time.perf_counter()
        ratio, abs_err = oracle_check(w, out, rows)
        check = {"vs": "numpy oracle (restatement of the reference's paged_attention_reference)",
                 "rows": rows, "query_heads": Hq, "atol": ATOL, "rtol": RTOL,
                 "max_abs_err": round(abs_err, 6), "max_err_over_tol": round(ratio, 4),
                 "pass": bool(ratio <= 1.0) and same, "e2e_equals_device_resident": same,
                 "check_s": round(time.perf_counter() - t0, 2)}
        if gather_exact is not None:
            check["gathered_equals_nccl_all_gather"] = gather_exact

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(spec, args.workload)
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    value = nbytes_total / (ms * 1e-3) / 1e9
    achieved = nbytes_local / (launch_ms * 1e-3) / 1e9
    lay = sequence_layout(spec)
    cfg = {"workload": args.workload, **{k: v for k, v in spec.items() if k not in ("kind",)},
           "global_batch": len(lay) if not replica else spec["batch"] * world, "sink": SINK, "group": GROUP,
           "pages_per_seq": w["n_pages"] if len(set(n for n, _ in lay)) == 1 else
           [min(n for n, _ in lay), max(n for n, _ in lay)],
           "tail": w["tail_len"] if isinstance(w["tail_len"], int) else "per sequence", "d_boost": K,
           "parallelism": ("single GPU" if world == 1 else
                           {"replica": f"sequence-sharded x{world} (own sequences per rank)",
                            "kv_head": f"KV-head tensor parallel x{world} + " + (
                                "peer-memory all-gather of outputs (NVLink stores, kitty_tp_allgather)"
                                if args.gather == "p2p" else "NCCL all-gather of outputs"),
                            "sequence": f"sequences over {world} ranks by longest-processing-time"}[spec["shard"]]),
           "decode_kernel": kernel, "launch": launch_mode,
           "l2": "inputs larger than L2 (no flush)" if nbytes_local > 126e6 else
                 "inputs smaller than L2, steps back to back"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak" if replica else "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "hbm_frac_of_peak": round(value / (peak * world), 4),
        "tokens_per_s": round(cfg["global_batch"] / (ms * 1e-3), 1),
        "config": cfg,
        "e2e": {"value": round(nbytes_total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": measured_traffic(args.workload, kernel, nbytes_local, w["pages_only"]),
                     "peak_source": f"{peak_kind} copy bandwidth", "kernel": f"{kernel} (+ split merge)",
                     "algorithmic_bytes_per_launch": nbytes_local},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": 2 * args.steps,
        "output_check": check,
    }
    if gather:
        line["decode_only_ms_per_step"] = round(decode_ms, 4)
        line["all_gather_ms_per_step"] = round(gather_ms, 4)
    return line


def quantize_arm(args, spec, d, device, local):
    """Config 3: quantise every page-head of the prefill (one key and one value launch
    per step); the packed pools are checked bit for bit against the numpy oracle on a
    sample of sequences."""
    import numpy as np
    import torch
    world, rank = d.world, d.rank
    w = build_quantize_workload(spec, device, seed=1234 + rank)
    H, D, G, K = w["H"], w["D"], w["G"], w["K"]
    nbytes_local = quantize_bytes(w["layout"], H, D, G, K)
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        quantize_call(w)
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        ms, launch_ms = timed(stream, args.steps, lambda: quantize_call(w), torch, device, d)

    # ---- end to end: keys and values from pinned host memory, packed pools back to the host
    k_host = w["k"].cpu().pin_memory()
    v_host = w["v"].cpu().pin_memory()
    pools_host = [p.cpu().pin_memory() for p in w["pools"]]
    h2d = (k_host.numel() + v_host.numel()) * 2
    d2h = sum(p.numel() * p.element_size() for p in pools_host)
    kd, vd = torch.empty_like(w["k"]), torch.empty_like(w["v"])

    def e2e_step():
        kd.copy_(k_host, non_blocking=True)
        vd.copy_(v_host, non_blocking=True)
        quantize_call(w, k=kd, v=vd)
        for ph, p in zip(pools_host, w["pools"]):
            ph.copy_(p, non_blocking=True)

    e2e_steps = min(args.steps, 5)
    e2e_step()
    torch.cuda.synchronize(device)
    e2e_ms, _ = timed(stream, e2e_steps, e2e_step, torch, device, d)

    # ---- bit-exactness on a sample (2 sequences, all heads) against the numpy oracle
    check = None
    if rank == 0:
        from oracle import kitty_oracle as O
        n, S = w["n"], SINK
        bidx = w["bidx"].cpu().numpy()
        mism, checked = 0, 0
        for b in range(min(2, w["B"])):
            k = w["k"][b, :, S:S + n * G].cpu().numpy().reshape(H, n, G, D)
            v = w["v"][b, :, S:S + n * G].cpu().numpy().reshape(H, n, G, D)
            low, high, sc, zp = O.quantize_key_pages(np.ascontiguousarray(k.transpose(1, 0, 3, 2)), bidx[None], K,
                                                     w["sentinel"])
            codes, vs, vz = O.quantize_value_pages(np.ascontiguousarray(v.transpose(1, 0, 2, 3)))
            sl = slice(b * n, (b + 1) * n)
            got = [p[sl].numpy() for p in pools_host]
            mism += int((got[0] != low).any(axis=(2, 3)).sum() + (got[1] != high).any(axis=(2, 3)).sum())
            mism += int((got[2][:, :, 0].astype(np.float32) != sc.astype(np.float32)).any(axis=2).sum())
            mism += int((got[2][:, :, 1].astype(np.float32) != zp.astype(np.float32)).any(axis=2).sum())
            mism += int((got[3] != codes).any(axis=(2, 3)).sum())
            mism += int((got[4][..., 0].astype(np.float32) != vs.astype(np.float32)).any(axis=2).sum())
            mism += int((got[4][..., 1].astype(np.float32) != vz.astype(np.float32)).any(axis=2).sum())
            checked += 2 * n * H
        check = {"page_heads_checked": checked, "mismatching_page_heads": mism}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(spec, args.workload)
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    value = nbytes_local * world / (ms * 1e-3) / 1e9
    return {
        "metric": "page-quantize/pack HBM GB/s (fp16 K/V in + packed planes out)", "value": round(value, 2),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "hbm_frac_of_peak": round(value / (peak * world), 4),
        "config": {"workload": args.workload, **{k: v for k, v in spec.items() if k != "kind"},
                   "page_heads": 2 * w["B"] * w["n"] * H, "d_boost": K,
                   "parallelism": "single GPU" if world == 1 else f"replicas x{world}",
                   "l2": "inputs larger than L2 (no flush)"},
        "e2e": {"value": round(nbytes_local * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": round(nbytes_local / (launch_ms * 1e-3) / 1e9, 2), "peak": peak,
                     "unit": "GB/s", "frac": round(nbytes_local / (launch_ms * 1e-3) / 1e9 / peak, 4),
                     "traffic": None, "peak_source": f"{peak_kind} copy bandwidth",
                     "kernel": "quantize_key_d128_kernel + quantize_value_d128_kernel",
                     "algorithmic_bytes_per_launch": nbytes_local},
        "bit_exact": check,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": 2 * args.steps,
    }


def decode_kernel_name(variant, g, D, G, fp16_regions=True):
    """Kernel family a decode call runs (the library's choice for "auto"; the tcgen05
    family takes pages-only calls and falls back to the library's choice otherwise)."""
    i8 = D == 128 and G == 128 and g <= 16   # above 8 query heads per KV head: in passes of 8
    if variant == "tc" and i8 and not fp16_regions:
        return "decode_tc_kernel"
    if variant in ("auto", "tc", "int8"):
        variant = "int8" if i8 else "simt"
    return {"int8": "decode_i8_kernel", "simt": "decode_simt_kernel"}[variant]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["kitty", "reference"], default="kitty")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--variant", choices=["auto", "simt", "int8", "tc"], default="auto",
                    help="decode kernel family (auto: integer tensor-core kernel for head_dim = group = 128, "
                         "CUDA-core kernel otherwise)")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="tensor-parallel output exchange (config 4 on several GPUs): direct NVLink stores "
                         "into every rank's exchange region, or an NCCL all-gather")
    ap.add_argument("--pages-only", action="store_true",
                    help="decode the quantised pages alone (no fp16 sink / tail tokens; the bytes count "
                         "the pages only): isolates the page path, and the only calls the tcgen05 family takes")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's batch of sequences (smaller cases for profiler captures); the JSON "
                         "line's config then records the reduced batch")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    spec = dict(WORKLOADS[args.workload])
    if args.batch > 0:
        if "batch" not in spec:
            raise SystemExit("--batch applies to the workloads with a fixed batch")
        spec["batch"] = args.batch
    if args.pages_only:
        if spec["kind"] != "decode":
            raise SystemExit("--pages-only applies to the decode workloads")
        spec["pages_only"] = True
    if args.impl == "reference":
        reference_arm(args, spec)
    else:
        kitty_arm(args, spec)


if __name__ == "__main__":
    main()
