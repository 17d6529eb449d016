"""Benchmark: fused quantized paged decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kitty|reference] [--workload config2]

One step = one decode step of one layer for the whole batch (every sequence,
every query head) over the quantised KV pools resident in HBM.  Default
workload = benchmark config 2 per GPU (Llama-3-8B-shaped layer: batch 32,
32 q / 8 kv heads, head_dim 128, 32768 tokens per sequence = 32 fp16 sinks +
255 quantised 128-token pages + 96-token fp16 tail, INT4 ratio 12.5%).
Multi-GPU runs (torchrun, one process per GPU) shard by sequence: every rank
owns its own 32 sequences (weak scaling, no data-path collective).

Reported (one JSON line from rank 0):
  value      algorithmic HBM GB/s of the whole job (bytes every step must read
             and write: each page-head once, fp16 sinks and tails, q, out,
             block table) / device time, max over ranks;
  e2e        the same metric through the public API with host buffers (q and
             block table copied H2D from pinned memory and the output copied
             D2H inside the timed region, every step);
  roofline   achieved GB/s of the decode launch (decode + split merge) vs the
             measured HBM copy bandwidth;
  cpu_baseline  the numpy oracle (CPU restatement of the reference's path) on
             a bounded sample, N=1 rank 0 only.
Inputs (~650 MB per GPU) exceed the 126 MB L2, so no flush is needed.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kitty-kv_b200"))

METRIC = "quantized paged decode-attn HBM GB/s (% of peak) & tokens/s at 1/2/4/8 B200"
# DRAM bytes (read + write) of one decode launch, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of this script on the same workload
# and kernel; None where no capture exists.
MEASURED_TRAFFIC = {
    ("config2", "decode_i8_kernel"): 652_401_408 + 5_087_744,
    ("config2", "decode_mma_kernel"): 652_734_720 + 5_091_328,
}

WORKLOADS = {
    # name: batch, q heads, kv heads, head_dim, context, boost_rate
    "config2": dict(batch=32, num_q_heads=32, num_kv_heads=8, head_dim=128, context=32768, boost_rate=0.125),
    "config1": dict(batch=1, num_q_heads=32, num_kv_heads=8, head_dim=128, context=4096, boost_rate=0.125),
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


def algorithmic_bytes(batch, Hq, H, D, G, K, n_pages, sink, tail):
    """Bytes one decode step must move (each page-head once + fp16 regions + q/out + table)."""
    per_head = n_pages * page_head_bytes(D, G, K) + sink * D * 2 * 2 + tail * D * 2 * 2
    per_seq = H * per_head + 2 * Hq * D * 2 + 4 * n_pages
    return batch * per_seq


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

def build_workload(spec, device, seed):
    """Quantise a synthetic batch into resident pools with the CUDA page quantiser."""
    import torch
    from kitty import kernels as KK
    from kitty import synthetic

    B, Hq, H, D, T, rate = (spec[k] for k in ("batch", "num_q_heads", "num_kv_heads", "head_dim", "context",
                                               "boost_rate"))
    G, S = GROUP, SINK
    K = round(rate * D)
    sentinel = min(K + 1, 255)
    n_pages = (T - S) // G
    tail = T - S - n_pages * G
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    k_all = torch.empty(B, H, T, D, dtype=torch.float16, device=device)
    v_all = torch.empty(B, H, T, D, dtype=torch.float16, device=device)
    score = torch.zeros(H, D, dtype=torch.float64, device=device)
    for b in range(B):
        k, v = synthetic.torch_make_kv(gen, H, T, D, device)
        k_all[b].copy_(k); v_all[b].copy_(v)
        score += k.float().abs().sum(dim=1, dtype=torch.float64)
    order = torch.argsort(-score, dim=-1, stable=True)
    bidx = torch.full((H, D), sentinel, dtype=torch.uint8, device=device)
    bidx.scatter_(1, order[:, :K], torch.arange(K, dtype=torch.uint8, device=device).expand(H, K).contiguous())
    P = B * n_pages
    pools = [torch.zeros(P, H, D, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, K, G // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, 2, D, dtype=torch.float16, device=device),
             torch.zeros(P, H, G, D // 4, dtype=torch.uint8, device=device),
             torch.zeros(P, H, G, 2, dtype=torch.float16, device=device)]
    if n_pages:
        bb = torch.arange(B, device=device).repeat_interleave(n_pages)
        pp = torch.arange(n_pages, device=device).repeat(B)
        offs = (bb * (H * T * D) + (S + pp * G) * D).to(torch.int64)
        dst = torch.arange(P, dtype=torch.int32, device=device)   # contiguous block tables
        KK.quantize_key_pages(k_all, offs, (T * D, D, 1), bidx, K, sentinel, dst, *pools[:3], H, D, G)
        KK.quantize_value_pages(v_all, offs, (T * D, D, 1), dst, pools[3], pools[4], H, D, G)
    sink_k = k_all[:, :, :S].contiguous(); sink_v = v_all[:, :, :S].contiguous()
    a = S + n_pages * G
    tail_k = k_all[:, :, a:].contiguous(); tail_v = v_all[:, :, a:].contiguous()
    del k_all, v_all
    torch.cuda.empty_cache()
    q = torch.randn(B, Hq, D, generator=gen, device=device, dtype=torch.float32).to(torch.float16)
    bt = torch.arange(P, dtype=torch.int32, device=device).view(B, max(n_pages, 1)) if n_pages else \
        torch.zeros(B, 1, dtype=torch.int32, device=device)
    npg = torch.full((B,), n_pages, dtype=torch.int32, device=device)
    torch.cuda.synchronize(device)
    return dict(q=q, bt=bt, npg=npg, pools=pools, bidx=bidx, K=K, sink_k=sink_k, sink_v=sink_v, tail_k=tail_k,
                tail_v=tail_v, n_pages=n_pages, tail=tail, B=B, Hq=Hq, H=H, D=D, G=G)


def decode_call(w, q=None, bt=None, npg=None, out=None):
    from kitty import kernels as KK
    return KK.paged_attention_batched(
        w["q"] if q is None else q, w["bt"] if bt is None else bt, w["npg"] if npg is None else npg, *w["pools"],
        w["bidx"], w["K"], sink_k=w["sink_k"], sink_v=w["sink_v"], sink_len=SINK, tail_k=w["tail_k"],
        tail_v=w["tail_v"], tail_len=w["tail"], out=out, max_pages_per_seq=w["n_pages"])


# ---------------------------------------------------------------------------
# CPU restatement timing (numpy oracle) - the reference's path on host cores
# ---------------------------------------------------------------------------

def _cpu_unit(u):
    """One (sequence, KV head) stream of oracle decode work: the reference's
    algorithm for the g query heads that share the KV head."""
    from oracle import kitty_oracle as O
    q, pages, pools, bidx, K, sk, sv, tk, tv, g, D = u
    return O.paged_attention(q, pages, *pools, bidx, K, sk, sv, tk, tv, g, 1, D)


def cpu_sample(spec, n_seq, seed=11):
    """Build a bounded CPU sample of the workload with the oracle quantiser (numpy),
    split into independent (sequence, KV head) units."""
    import numpy as np
    sys.path.insert(0, str(ROOT))
    from kitty import synthetic
    from oracle import kitty_oracle as O
    case = synthetic.make_decode_case(seed, n_seq, spec["num_q_heads"], spec["num_kv_heads"], spec["head_dim"],
                                      [spec["context"]] * n_seq, boost_rate=spec["boost_rate"])
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    g = case.num_q_heads // H
    units = []
    for b, s in enumerate(case.seqs):
        low, high, sc, zp = O.quantize_key_pages(s.page_keys(), case.boost_idx, K, case.sentinel)
        codes, vs, vz = O.quantize_value_pages(s.page_values())
        km = np.stack([sc, zp], axis=2); vm = np.stack([vs, vz], axis=3)
        sk, sv = s.sink_kv(); tk, tv = s.tail_kv()
        for h in range(H):
            pools = tuple(np.ascontiguousarray(p[:, h:h + 1]) for p in (low, high, km, codes, vm))
            units.append((case.q[b, h * g:(h + 1) * g], list(range(s.n_pages)), pools, case.boost_idx[h:h + 1],
                          K, sk[h:h + 1], sv[h:h + 1], tk[h:h + 1], tv[h:h + 1], g, D))
    n_pages = case.seqs[0].n_pages
    nbytes = algorithmic_bytes(n_seq, case.num_q_heads, H, D, G, K, n_pages, case.seqs[0].sink, case.seqs[0].tail)
    return units, nbytes


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
    n_seq = 2
    units, nbytes = cpu_sample(spec, n_seq)
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
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "tokens_per_s": round(n_seq / sec, 3),
            "config": {"workload": args.workload, **spec, "sample_sequences": n_seq},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": workers, "kind": "port",
                             "sample": f"{n_seq} sequences of {args.workload} ({n_seq} x {spec['num_kv_heads']} "
                                       "(sequence, KV head) streams on a host thread pool), numpy restatement "
                                       "of the reference's paged_attention_reference"},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def kitty_arm(args, spec):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from kitty.kernels import _lib
    _lib.force_decode_variant(args.variant)
    w = build_workload(spec, device, seed=1234 + rank)
    B, Hq, H, D, G, K = w["B"], w["Hq"], w["H"], w["D"], w["G"], w["K"]
    kernel = decode_kernel_name(args.variant, Hq // H, D, G)
    nbytes = algorithmic_bytes(B, Hq, H, D, G, K, w["n_pages"], SINK, w["tail"])
    stream = torch.cuda.current_stream(device)
    out = torch.empty(B, Hq, D, dtype=torch.float16, device=device)

    # ---- device-resident steady state (value + roofline)
    for _ in range(args.warmup):
        decode_call(w, out=out)
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        e0 = torch.cuda.Event(enable_timing=True); e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            decode_call(w, out=out)
            ends[i].record(stream)
        e1.record(stream)
        torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    total_ms = max_over_ranks(e0.elapsed_time(e1))
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    ms = total_ms / args.steps

    # ---- end to end through the public API with host buffers
    q_host = w["q"].cpu().pin_memory()
    bt_host = w["bt"].cpu().pin_memory()
    npg_host = w["npg"].cpu().pin_memory()
    out_host = torch.empty(B, Hq, D, dtype=torch.float16).pin_memory()
    h2d = q_host.numel() * 2 + bt_host.numel() * 4 + npg_host.numel() * 4
    d2h = out_host.numel() * 2

    def e2e_step():
        q = q_host.to(device, non_blocking=True)
        bt = bt_host.to(device, non_blocking=True)
        npg = npg_host.to(device, non_blocking=True)
        o = decode_call(w, q=q, bt=bt, npg=npg)
        out_host.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    f0 = torch.cuda.Event(enable_timing=True); f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / args.steps

    # ---- correctness spot check of the timed output (finite, identical to the e2e output)
    ok = bool(torch.isfinite(out).all().item()) and bool(torch.equal(out.cpu(), out_host))

    # ---- launches per decode call
    from kitty.kernels import _lib
    a_bytes = _lib.c_size(0); a_splits = _lib.c_i32(0)
    launches_per_step = 1
    try:
        import ctypes
        lib = _lib.load()
        args_struct = _decode_args_for_plan(w)
        _lib.check(lib.kitty_paged_decode_workspace_size(args_struct, a_bytes, ctypes.byref(a_splits)), "plan")
        launches_per_step = 2 if a_splits.value > 1 else 1
    except Exception:  # plan query is informational
        pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_seq = 1
        units, cbytes = cpu_sample(spec, n_seq)
        workers = max(1, min(os.cpu_count() or 1, len(units)))
        runner = CpuRunner(workers)
        runner.run(units)
        reps = 3
        sec = sum(runner.run(units) for _ in range(reps)) / reps
        runner.close()
        cpu = {"value": round(cbytes / sec / 1e9, 4), "unit": "GB/s", "cores": workers, "kind": "port",
               "sample": f"{n_seq} sequence of {args.workload} ({spec['num_kv_heads']} KV heads x "
                         f"{(spec['context'] - SINK) // GROUP} pages), numpy restatement of the reference's "
                         f"paged_attention_reference, mean of {reps} runs"}

    if rank == 0:
        peak, peak_kind = measured_peaks()
        value = nbytes * world / (ms * 1e-3) / 1e9
        achieved = nbytes / (launch_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "hbm_frac_of_peak": round(value / (peak * world), 4),
            "tokens_per_s": round(B * world / (ms * 1e-3), 1),
            "config": {"workload": args.workload, **spec, "global_batch": B * world, "sink": SINK, "group": GROUP,
                       "pages_per_seq": w["n_pages"], "tail": w["tail"], "d_boost": K,
                       "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (no flush)"},
            "e2e": {"value": round(nbytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": MEASURED_TRAFFIC.get((args.workload, kernel)),
                         "peak_source": f"{peak_kind} copy bandwidth", "kernel": f"{kernel} (+ split merge)",
                         "algorithmic_bytes_per_launch": nbytes},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "output_check": "finite and identical between device-resident and e2e runs" if ok else "FAILED",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def decode_kernel_name(variant, g, D, G):
    """Kernel family a decode call runs (the library's choice for "auto")."""
    if variant == "auto":
        variant = "int8" if (D == 128 and G == 128 and g <= 4) else ("mma" if (D == 128 and G == 128 and g <= 8)
                                                                      else "simt")
    return {"int8": "decode_i8_kernel", "mma": "decode_mma_kernel", "simt": "decode_simt_kernel"}[variant]


def _decode_args_for_plan(w):
    from kitty.kernels import _lib
    a = _lib.DecodeArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.group, a.d_boost = w["B"], w["Hq"], w["H"], w["D"], \
        w["G"], w["K"]
    a.q = a.out = a.num_pages = a.boost_idx = 1
    a.block_table = a.key_low = a.key_high = a.key_meta = a.val_codes = a.val_meta = 1
    a.sink_k = a.sink_v = a.tail_k = a.tail_v = 1
    a.sink_len_all, a.tail_len_all = SINK, w["tail"]
    a.max_pages_per_seq = w["n_pages"]
    a.pool_pages = w["pools"][0].shape[0]
    return a


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["kitty", "reference"], default="kitty")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--variant", choices=["auto", "simt", "mma", "int8"], default="auto",
                    help="decode kernel family (auto: integer tensor-core kernel for <= 4 query heads per "
                         "KV head, fp16 tensor-core kernel up to 8, CUDA-core kernel otherwise)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    spec = WORKLOADS[args.workload]
    if args.impl == "reference":
        reference_arm(args, spec)
    else:
        kitty_arm(args, spec)


if __name__ == "__main__":
    main()
