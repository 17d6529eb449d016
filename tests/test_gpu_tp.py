"""GPU tests of the tensor-parallel output exchange over peer memory
(``kitty.distributed.PeerGather`` -> ``kitty_tp_allgather``).

One process (a one-rank group): every call must return the slice it was given, call
after call (the device-side epoch and the alternating buffers) and when the two kernels
are captured in a CUDA graph and replayed with new slice contents.  With two or more
visible GPUs, two ranks (spawned processes, NCCL) must assemble exactly what an NCCL
all-gather of the same slices assembles, eagerly and from a graph; skipped on one GPU.
No test makes a rank stop or wait forever: every rank makes the same calls."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_single_rank_exchange_calls_and_graph_replays():
    from kitty.distributed import PeerGather
    from kitty.kernels import _lib
    own_group = not dist.is_initialized()
    if own_group:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", world_size=1, rank=0)
    try:
        hq, B, D = 4, 3, 128
        pg = PeerGather(hq, B, D, device=DEV)
        full = torch.empty(hq, B, D, dtype=torch.float16, device=DEV)
        gen = torch.Generator(device=DEV).manual_seed(3)
        for _ in range(5):   # epochs 1..5: both buffers, twice over
            x = torch.randn(hq, B, D, generator=gen, device=DEV).half()
            got = pg(x, full=full)
            torch.cuda.synchronize()
            assert torch.equal(full, x)
            assert tuple(got.shape) == (B, hq, D) and torch.equal(got, x.permute(1, 0, 2))
        xs = torch.empty(hq, B, D, dtype=torch.float16, device=DEV)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(DEV)
        s.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                pg(xs, full=full)
        torch.cuda.current_stream(DEV).wait_stream(s)
        for _ in range(3):
            xs.copy_(torch.randn(hq, B, D, generator=gen, device=DEV).half())
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(full, xs)
        del g
        assert _lib.device_error_flags() == 0
        with pytest.raises(RuntimeError):
            pg(torch.empty(hq + 1, B, D, dtype=torch.float16, device=DEV), full=full)
        pg.close()
    finally:
        if own_group:
            dist.destroy_process_group()


def _two_rank_child(rank: int, world: int, port: int, result_dir: str) -> None:
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank,
                            device_id=dev)
    ok = False
    try:
        from kitty.distributed import PeerGather
        hq, B, D = 8, 5, 128
        pg = PeerGather(hq, B, D, device=dev)
        full = torch.empty(world * hq, B, D, dtype=torch.float16, device=dev)
        ref = torch.empty_like(full)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        good = True
        for _ in range(6):
            x = torch.randn(hq, B, D, generator=gen, device=dev).half()
            pg(x, full=full)
            dist.all_gather_into_tensor(ref, x)
            torch.cuda.synchronize(dev)
            good &= bool(torch.equal(full, ref))
        xs = torch.empty(hq, B, D, dtype=torch.float16, device=dev)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                pg(xs, full=full)
        torch.cuda.current_stream(dev).wait_stream(s)
        for _ in range(4):
            xs.copy_(torch.randn(hq, B, D, generator=gen, device=dev).half())
            g.replay()
            dist.all_gather_into_tensor(ref, xs)
            torch.cuda.synchronize(dev)
            good &= bool(torch.equal(full, ref))
        del g
        from kitty.kernels import _lib
        good &= _lib.device_error_flags() == 0
        pg.close()
        ok = good
    finally:
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "fail")
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_match_nccl_all_gather(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_two_rank_child, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", f"rank {r}"
