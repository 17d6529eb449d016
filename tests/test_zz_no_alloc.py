"""GPU test of kitty_paged_decode_noalloc, the decode entry point for callers that
cannot allocate device memory (for example an engine whose memory arena forbids
allocation on the decode path, or a host driving the library through a plain FFI
with no device allocator).  It keeps its split partial results in a static device
array inside the library instead of a caller-provided workspace.

Both entry points are called directly through the C ABI with the same argument
struct; the allocation-free one must agree with kitty_paged_decode (fp16
tolerance: atol 2e-3, rtol 1e-2) on two calls in a row, the second with other
queries, so stale contents of the shared static array cannot leak into a result,
and with the numpy oracle on the same pools.  A batch whose partials at the
library's default split count exceed the static array checks that the split count
is lowered to fit.  This file is collected last on purpose."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

import synthetic
from kitty.kernels import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case_tensors(seed, contexts=(32 + 40 * 128 + 77, 32 + 9 * 128 + 5, 32 + 23 * 128)):
    case = synthetic.make_decode_case(seed, len(contexts), 32, 8, 128, list(contexts))
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    n_phys = sum(s.n_pages for s in case.seqs)
    pools = [torch.zeros(n_phys, H, D, G // 4, dtype=torch.uint8, device=DEV),
             torch.zeros(n_phys, H, K, G // 4, dtype=torch.uint8, device=DEV),
             torch.zeros(n_phys, H, 2, D, dtype=torch.float16, device=DEV),
             torch.zeros(n_phys, H, G, D // 4, dtype=torch.uint8, device=DEV),
             torch.zeros(n_phys, H, G, 2, dtype=torch.float16, device=DEV)]
    from kitty import kernels as KK
    bidx = torch.from_numpy(case.boost_idx).to(DEV)
    B = len(case.seqs)
    W = max(s.n_pages for s in case.seqs)
    assert B <= 64
    bt = torch.zeros(B, W, dtype=torch.int32, device=DEV)
    at = 0
    S, Q = 32, max(max(s.tail for s in case.seqs), 1)
    sk = torch.zeros(B, H, S, D, dtype=torch.float16, device=DEV); sv = torch.zeros_like(sk)
    tk = torch.zeros(B, H, Q, D, dtype=torch.float16, device=DEV); tv = torch.zeros_like(tk)
    for b, s in enumerate(case.seqs):
        k = torch.from_numpy(s.k).to(DEV); v = torch.from_numpy(s.v).to(DEV)
        offs = torch.tensor([(s.sink + i * G) * D for i in range(s.n_pages)], dtype=torch.int64, device=DEV)
        dst = torch.arange(at, at + s.n_pages, dtype=torch.int32, device=DEV)
        KK.quantize_key_pages(k, offs, tuple(k.stride()), bidx, K, case.sentinel, dst, *pools[:3], H, D, G)
        KK.quantize_value_pages(v, offs, tuple(v.stride()), dst, pools[3], pools[4], H, D, G)
        bt[b, :s.n_pages] = dst
        at += s.n_pages
        sk[b] = k[:, :S]; sv[b] = v[:, :S]
        a = S + s.n_pages * G
        tk[b, :, :s.tail] = k[:, a:a + s.tail]; tv[b, :, :s.tail] = v[:, a:a + s.tail]
    npg = torch.tensor([s.n_pages for s in case.seqs], dtype=torch.int32, device=DEV)
    tl = torch.tensor([s.tail for s in case.seqs], dtype=torch.int32, device=DEV)
    return case, pools, bidx, bt, npg, sk, sv, tk, tv, tl


def _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, out):
    a = _lib.DecodeArgs()
    B, Hq, D = q.shape
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim, a.group, a.d_boost = B, Hq, case.num_kv_heads, D, \
        case.group, case.d_boost
    a.sm_scale = 1.0 / math.sqrt(D)
    a.q, a.q_s_seq, a.q_s_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.out, a.out_s_seq, a.out_s_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.block_table, a.bt_s_seq, a.num_pages = bt.data_ptr(), bt.stride(0), npg.data_ptr()
    a.pool_pages = pools[0].shape[0]
    a.key_low, a.key_high, a.key_meta = pools[0].data_ptr(), pools[1].data_ptr(), pools[2].data_ptr()
    a.val_codes, a.val_meta = pools[3].data_ptr(), pools[4].data_ptr()
    a.boost_idx, a.bidx_s_head = bidx.data_ptr(), bidx.stride(0)
    a.sink_k, (a.sk_s_seq, a.sk_s_head, a.sk_s_tok) = sk.data_ptr(), sk.stride()[:3]
    a.sink_v, (a.sv_s_seq, a.sv_s_head, a.sv_s_tok) = sv.data_ptr(), sv.stride()[:3]
    a.sink_len, a.sink_len_all = 0, sk.shape[2]
    a.tail_k, (a.tk_s_seq, a.tk_s_head, a.tk_s_tok) = tk.data_ptr(), tk.stride()[:3]
    a.tail_v, (a.tv_s_seq, a.tv_s_head, a.tv_s_tok) = tv.data_ptr(), tv.stride()[:3]
    a.tail_len, a.tail_len_all = tl.data_ptr(), 0
    a.max_pages_per_seq, a.num_splits = bt.shape[1], 0
    return a


def test_noalloc_decode_matches_workspace_decode_twice():
    lib = _lib.load()
    stream = torch.cuda.current_stream(torch.device(DEV)).cuda_stream
    case, pools, bidx, bt, npg, sk, sv, tk, tv, tl = _case_tensors(17)
    rng = np.random.default_rng(99)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((3, 32, 128)).astype(np.float16)).to(DEV)
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        a = _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, ref)
        need = _lib.c_size(0)
        _lib.check(lib.kitty_paged_decode_workspace_size(a, need, None), "workspace_size")
        assert need.value > 0, "the case must exercise the split partials (scratch memory)"
        ws = torch.empty(need.value, dtype=torch.uint8, device=DEV)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.kitty_paged_decode(a, stream), "kitty_paged_decode")
        b = _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, got)
        b.workspace, b.workspace_bytes = 0, 0           # ignored by the allocation-free entry point
        _lib.check(lib.kitty_paged_decode_noalloc(b, stream), "kitty_paged_decode_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {call}: output not fully written"
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), atol=2e-3, rtol=1e-2)
        _assert_oracle(case, pools, bt, q, got, rows=range(3))


def _assert_oracle(case, pools, bt, q, got, rows):
    """The allocation-free output against the numpy oracle on the same pools."""
    from oracle import kitty_oracle as O
    np_pools = [p.cpu().numpy() for p in pools]
    H, D = case.num_kv_heads, case.head_dim
    for b in rows:
        s = case.seqs[b]
        sk, sv = s.sink_kv()
        tk, tv = s.tail_kv()
        exp = O.paged_attention(q[b].cpu().numpy(), bt[b, :s.n_pages].cpu().numpy(), *np_pools, case.boost_idx,
                                case.d_boost, sk, sv, tk, tv, case.num_q_heads, H, D)
        np.testing.assert_allclose(got[b].float().cpu().numpy(), exp.astype(np.float32), atol=2e-3, rtol=1e-2)


def test_noalloc_lowers_the_split_count_to_fit():
    """64 sequences x 8 KV heads with 2 pages each: at the library's default split
    count the partials need more than the 8 MiB static array, so the entry point must
    pick a smaller split count itself and still produce the right output."""
    lib = _lib.load()
    stream = torch.cuda.current_stream(torch.device(DEV)).cuda_stream
    ctx = [32 + 2 * 128 + (i * 37) % 128 for i in range(64)]
    case, pools, bidx, bt, npg, sk, sv, tk, tv, tl = _case_tensors(19, ctx)
    q = torch.from_numpy(np.random.default_rng(5).standard_normal((64, 32, 128)).astype(np.float16)).to(DEV)
    ref = torch.empty_like(q)
    got = torch.full_like(q, float("nan"))
    a = _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, ref)
    need = _lib.c_size(0)
    _lib.check(lib.kitty_paged_decode_workspace_size(a, need, None), "workspace_size")
    assert need.value > 8 << 20, f"the case must overflow the static array at the default split count ({need.value})"
    ws = torch.empty(need.value, dtype=torch.uint8, device=DEV)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.kitty_paged_decode(a, stream), "kitty_paged_decode")
    b = _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, got)
    _lib.check(lib.kitty_paged_decode_noalloc(b, stream), "kitty_paged_decode_noalloc")
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), atol=2e-3, rtol=1e-2)
    _assert_oracle(case, pools, bt, q, got, rows=[0, 31, 63])


def test_noalloc_rejects_explicit_splits_beyond_the_scratch():
    lib = _lib.load()
    stream = torch.cuda.current_stream(torch.device(DEV)).cuda_stream
    case, pools, bidx, bt, npg, sk, sv, tk, tv, tl = _case_tensors(18)
    q = torch.zeros(3, 32, 128, dtype=torch.float16, device=DEV)
    out = torch.empty_like(q)
    a = _args(case, pools, bidx, bt, npg, sk, sv, tk, tv, tl, q, out)
    # the plan clamps the request to 1023 split slots (plus one), whose partials for
    # 3 sequences x 32 query heads x 130 floats (about 50 MB) are far beyond 8 MiB
    a.num_splits = 1 << 20
    a.max_pages_per_seq = 1 << 20
    rc = lib.kitty_paged_decode_noalloc(a, stream)
    assert rc == 4 and b"static scratch" in lib.kitty_last_error()
