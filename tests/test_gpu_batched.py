"""GPU parity of the device-resident batched cache (kitty_cache_append / _release /
_reset through the C ABI, driven by ``kitty.BatchedKVCache``).

After a schedule of decode steps over a changing subset of sequences (random
order, every layer), each sequence's cache must equal the oracle's state after
the same token history: counters, fp16 sinks and tail bit-exact, every page's
key and value planes bit-exact (metadata by value), and decode attention over
the cache within the fp16 tolerance of the oracle (atol 2e-3, rtol 1e-2).
Allocator failures (pool exhausted, block table full, repeated ids) are made on
the host side of the interface and checked through the sticky error flags.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kitty import BatchedKVCache, KittyConfig
import synthetic
from kitty.kernels import _lib
from oracle import kitty_oracle as O

from conftest import meta_by_value

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-3, 1e-2

CONFIGS = {
    # D = G = 128 (fast quantisers, integer decode), two layers
    "d128": dict(num_layers=2, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32, boost_rate=0.125,
                 max_seq_len=512),
    # small pages (generic quantisers, fp16 tensor-core decode), no sinks
    "g16": dict(num_layers=1, num_kv_heads=2, head_dim=64, q_buffer_size=16, sink_size=0, boost_rate=0.25,
                max_seq_len=128),
    "tiny": dict(num_layers=1, num_kv_heads=2, head_dim=16, q_buffer_size=8, sink_size=4, boost_rate=0.25,
                 max_seq_len=64),
}


def make_cache(name, max_seqs, seed, **kw):
    cfg = KittyConfig(device=DEV, local_value_window=0, **CONFIGS[name])
    rng = np.random.default_rng(seed)
    L, H, D = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    scores = rng.random((L, H, D), dtype=np.float32)
    bidx = O.boost_idx_from_scores(scores, cfg.d_boost, cfg.sentinel)
    cache = BatchedKVCache(cfg, torch.from_numpy(bidx), max_seqs=max_seqs, **kw)
    return cfg, cache, bidx, rng


def check_sequence(cache, cfg, bidx, l, s, keys, values):
    """Cache slot s of layer l vs the oracle state of the token history keys / values (T, H, D)."""
    exp = O.sequence_state(keys, values, cfg.sink_size, cfg.q_buffer_size, bidx[l], cfg.d_boost, cfg.sentinel)
    sl, npg, tl = O.cache_regions(keys.shape[0], cfg.sink_size, cfg.q_buffer_size)
    got = cache.lengths(l)
    assert (int(got["sink_len"][s]), int(got["num_pages"][s]), int(got["tail_len"][s])) == (sl, npg, tl)
    np.testing.assert_array_equal(cache.sink_k[l, s, :, :sl].cpu().numpy(), exp["sink_k"])
    np.testing.assert_array_equal(cache.sink_v[l, s, :, :sl].cpu().numpy(), exp["sink_v"])
    np.testing.assert_array_equal(cache.tail_k[l, s, :, :tl].cpu().numpy(), exp["tail_k"])
    np.testing.assert_array_equal(cache.tail_v[l, s, :, :tl].cpu().numpy(), exp["tail_v"])
    pages = cache.block_table[l, s, :npg].cpu().numpy()
    for j, page in enumerate(pages):
        e = exp["pages"][j]
        np.testing.assert_array_equal(cache.key_baseline[page].cpu().numpy(), e["key_low"])
        np.testing.assert_array_equal(cache.key_boost[page].cpu().numpy(), e["key_high"])
        km = cache.key_metadata[page].cpu().numpy()
        np.testing.assert_array_equal(meta_by_value(km[:, 0]), meta_by_value(e["key_scale"]))
        np.testing.assert_array_equal(meta_by_value(km[:, 1]), meta_by_value(e["key_zero"]))
        np.testing.assert_array_equal(cache.value_pool[page].cpu().numpy(), e["val_codes"])
        vm = cache.value_metadata[page].cpu().numpy()
        np.testing.assert_array_equal(meta_by_value(vm[..., 0]), meta_by_value(e["val_scale"]))
        np.testing.assert_array_equal(meta_by_value(vm[..., 1]), meta_by_value(e["val_zero"]))
    return pages


def oracle_decode(cache, cfg, l, s, q_row):
    lens = cache.lengths(l)
    sl, npg, tl = int(lens["sink_len"][s]), int(lens["num_pages"][s]), int(lens["tail_len"][s])
    pools = [t.cpu().numpy() for t in (cache.key_baseline, cache.key_boost, cache.key_metadata,
                                       cache.value_pool, cache.value_metadata)]
    return O.paged_attention(q_row, cache.block_table[l, s, :npg].cpu().numpy(), *pools,
                             cache.boost_idx[l].cpu().numpy(), cfg.d_boost,
                             cache.sink_k[l, s, :, :sl].cpu().numpy(), cache.sink_v[l, s, :, :sl].cpu().numpy(),
                             cache.tail_k[l, s, :, :tl].cpu().numpy(), cache.tail_v[l, s, :, :tl].cpu().numpy(),
                             q_row.shape[0], cfg.num_kv_heads, cfg.head_dim)


def run_schedule(cache, cfg, rng, max_seqs, steps, p_active=0.7):
    """Random steps over subsets of slots; returns per-(layer, slot) histories (T, H, D)."""
    L, H, D = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    T = steps
    kv = [[synthetic.make_kv(rng, H, T, D) for _ in range(max_seqs)] for _ in range(L)]
    K_all = torch.from_numpy(np.stack([[k.transpose(1, 0, 2) for k, _ in row] for row in kv])).to(DEV)
    V_all = torch.from_numpy(np.stack([[v.transpose(1, 0, 2) for _, v in row] for row in kv])).to(DEV)
    count = np.zeros((L, max_seqs), np.int64)
    for _ in range(steps):
        active = [s for s in range(max_seqs) if rng.random() < p_active]
        if not active:
            continue
        ids = np.array(rng.permutation(active), dtype=np.int32)
        ids_t = torch.from_numpy(ids).to(DEV)
        for l in range(L):
            pos = torch.from_numpy(count[l, ids]).to(DEV)
            cache.append(l, ids_t, K_all[l, ids_t.long(), pos].contiguous(), V_all[l, ids_t.long(), pos].contiguous())
            count[l, ids] += 1
    torch.cuda.synchronize()
    hist = {(l, s): (kv[l][s][0].transpose(1, 0, 2)[:count[l, s]], kv[l][s][1].transpose(1, 0, 2)[:count[l, s]])
            for l in range(L) for s in range(max_seqs)}
    return hist


@pytest.mark.parametrize("name,steps", [("d128", 420), ("g16", 90), ("tiny", 40)])
def test_append_schedule_matches_oracle(name, steps):
    max_seqs = 5
    cfg, cache, bidx, rng = make_cache(name, max_seqs, seed=11)
    hist = run_schedule(cache, cfg, rng, max_seqs, steps)
    cache.check_errors()
    used = 0
    for (l, s), (k, v) in hist.items():
        used += len(check_sequence(cache, cfg, bidx, l, s, k, v))
    assert cache.free_page_count() == cache.num_pages - used
    # every allocated page is distinct
    all_pages = np.concatenate([cache.block_table[l, s, :int(cache.page_count[l, s])].cpu().numpy()
                                for l in range(cfg.num_layers) for s in range(max_seqs)])
    assert len(set(all_pages.tolist())) == len(all_pages) == used
    # decode over a permuted subset of slots (seq_map) vs the oracle
    Hq = 2 * cfg.num_kv_heads
    for l in range(cfg.num_layers):
        ids = np.array(rng.permutation(max_seqs)[:3], dtype=np.int32)
        q = synthetic.make_q(rng, (len(ids), Hq, cfg.head_dim))
        out = cache.decode(l, torch.from_numpy(q).to(DEV), torch.from_numpy(ids).to(DEV))
        torch.cuda.synchronize()
        for i, s in enumerate(ids):
            exp = oracle_decode(cache, cfg, l, int(s), q[i])
            np.testing.assert_allclose(out[i].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)


def test_release_returns_pages_and_slots_restart():
    cfg, cache, bidx, rng = make_cache("tiny", 3, seed=5)
    hist = run_schedule(cache, cfg, rng, 3, 30, p_active=1.0)
    cache.check_errors()
    before = cache.free_page_count()
    n1 = int(cache.page_count[0, 1])
    assert n1 > 0
    cache.release([1, 1])                 # a repeated id releases once
    torch.cuda.synchronize()
    cache.check_errors()
    assert cache.free_page_count() == before + n1
    assert [int(x[1]) for x in cache.lengths(0).values()] == [0, 0, 0]
    # slot 1 restarts from an empty history; the others are untouched
    k2, v2 = synthetic.make_kv(rng, cfg.num_kv_heads, 20, cfg.head_dim)
    k2, v2 = k2.transpose(1, 0, 2), v2.transpose(1, 0, 2)
    for t in range(20):
        cache.append(0, [1], torch.from_numpy(k2[t:t + 1]).to(DEV), torch.from_numpy(v2[t:t + 1]).to(DEV))
    torch.cuda.synchronize()
    cache.check_errors()
    check_sequence(cache, cfg, bidx, 0, 1, k2, v2)
    for s in (0, 2):
        check_sequence(cache, cfg, bidx, 0, s, *hist[(0, s)])


def test_pool_exhaustion_drops_token_and_recovers():
    # 2 pages in the pool: the third flush has no page
    cfg, cache, bidx, rng = make_cache("tiny", 3, seed=7, num_pages=2)
    H, D, S, G = cfg.num_kv_heads, cfg.head_dim, cfg.sink_size, cfg.q_buffer_size
    T = S + G
    k, v = synthetic.make_kv(rng, H, T, D)
    keys = torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).to(DEV)
    vals = torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).to(DEV)
    ids = torch.tensor([0, 1, 2], dtype=torch.int32, device=DEV)
    for t in range(T):
        cache.append(0, ids, keys[t].expand(3, H, D).contiguous(), vals[t].expand(3, H, D).contiguous())
    torch.cuda.synchronize()
    bits = _lib.device_error_flags(clear=True)
    assert bits & (1 << 1), bits
    lens = cache.lengths(0)
    # slots 0 and 1 got the two pages (token order); slot 2's last token was dropped
    assert lens["num_pages"].tolist() == [1, 1, 0]
    assert lens["tail_len"].tolist() == [0, 0, G - 1]
    assert cache.free_page_count() == 0
    kh, vh = k.transpose(1, 0, 2), v.transpose(1, 0, 2)
    check_sequence(cache, cfg, bidx, 0, 0, kh, vh)
    check_sequence(cache, cfg, bidx, 0, 2, kh[:T - 1], vh[:T - 1])
    # releasing slot 0 frees its page; slot 2's retried token then flushes into it
    cache.release([0])
    cache.append(0, [2], keys[T - 1:T].contiguous(), vals[T - 1:T].contiguous())
    torch.cuda.synchronize()
    cache.check_errors()
    check_sequence(cache, cfg, bidx, 0, 2, kh, vh)
    assert cache.free_page_count() == 0


def test_block_table_full_and_bad_ids():
    cfg, cache, bidx, rng = make_cache("tiny", 2, seed=9, max_pages_per_seq=1)
    H, D, S, G = cfg.num_kv_heads, cfg.head_dim, cfg.sink_size, cfg.q_buffer_size
    T = S + 2 * G
    k, v = synthetic.make_kv(rng, H, T, D)
    kh, vh = k.transpose(1, 0, 2), v.transpose(1, 0, 2)
    for t in range(T):
        cache.append(0, [0], torch.from_numpy(kh[t:t + 1]).to(DEV), torch.from_numpy(vh[t:t + 1]).to(DEV))
    torch.cuda.synchronize()
    bits = _lib.device_error_flags(clear=True)
    assert bits == 1 << 2, bits
    check_sequence(cache, cfg, bidx, 0, 0, kh[:T - 1], vh[:T - 1])
    # a repeated id appends once and flags; an id out of range flags and appends nothing
    one = torch.from_numpy(np.ascontiguousarray(np.stack([kh[0], kh[1]]))).to(DEV)
    onev = torch.from_numpy(np.ascontiguousarray(np.stack([vh[0], vh[1]]))).to(DEV)
    cache.append(0, [1, 1], one, onev)
    torch.cuda.synchronize()
    assert _lib.device_error_flags(clear=True) == 1 << 3
    assert int(cache.lengths(0)["sink_len"][1]) == 1
    cache.append(0, [7], one[:1].contiguous(), onev[:1].contiguous())
    torch.cuda.synchronize()
    assert _lib.device_error_flags(clear=True) == 1 << 3
    assert int(cache.lengths(0)["sink_len"][1]) == 1
    # the claims were cleared: the slot accepts the next step normally
    cache.append(0, [1], one[1:].contiguous(), onev[1:].contiguous())
    torch.cuda.synchronize()
    cache.check_errors()
    assert int(cache.lengths(0)["sink_len"][1]) == 2


def test_decode_step_in_cuda_graph():
    """One decode step (append + attention) captured once and replayed: the replays
    must leave the same cache and outputs as the oracle for the same history."""
    cfg, cache, bidx, rng = make_cache("d128", 4, seed=13)
    cfg_h, D = cfg.num_kv_heads, cfg.head_dim
    Hq = 4 * cfg_h
    ids = torch.tensor([3, 0, 2], dtype=torch.int32, device=DEV)
    n = ids.numel()
    steps = 200            # crosses the sinks and one flush (S = 32, G = 128)
    k = np.stack([synthetic.make_kv(rng, cfg_h, steps, D)[0].transpose(1, 0, 2) for _ in range(n)], axis=1)
    v = np.stack([synthetic.make_kv(rng, cfg_h, steps, D)[1].transpose(1, 0, 2) for _ in range(n)], axis=1)
    q = synthetic.make_q(rng, (steps, n, Hq, D))
    kd, vd, qd = (torch.from_numpy(np.ascontiguousarray(x)).to(DEV) for x in (k, v, q))
    sk = torch.empty(n, cfg_h, D, dtype=torch.float16, device=DEV)
    sv, sq = torch.empty_like(sk), torch.empty(n, Hq, D, dtype=torch.float16, device=DEV)
    out = torch.empty(n, Hq, D, dtype=torch.float16, device=DEV)
    # warm-up outside the capture on a scratch cache, then capture on the real one
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        scratch = BatchedKVCache(cfg, cache.boost_idx, max_seqs=4)
        for l in range(cfg.num_layers):
            scratch.append(l, ids, sk, sv)
            scratch.decode(l, sq, ids, out=out)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for l in range(cfg.num_layers):
            cache.append(l, ids, sk, sv)
            cache.decode(l, sq, ids, out=out)
    cache.reset()
    torch.cuda.synchronize()
    outs = []
    for t in range(steps):
        sk.copy_(kd[t]); sv.copy_(vd[t]); sq.copy_(qd[t])
        g.replay()
        if t in (31, 127, 159, steps - 1):
            outs.append((t, out.clone()))
    torch.cuda.synchronize()
    cache.check_errors()
    for l in range(cfg.num_layers):
        for i, s in enumerate(ids.tolist()):
            check_sequence(cache, cfg, bidx, l, s, k[:, i], v[:, i])
    t, o = outs[-1]
    l = cfg.num_layers - 1
    for i, s in enumerate(ids.tolist()):
        exp = oracle_decode(cache, cfg, l, s, q[t, i])
        np.testing.assert_allclose(o[i].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)
    del g


@pytest.mark.parametrize("name", ["d128", "g16", "tiny"])
def test_prefill_matches_token_by_token_oracle(name):
    """Bulk append (prefill) on top of existing states - empty slots, slots inside
    their sinks, slots with a partly filled buffer - in two chunks, then a decode
    step: every slot must equal the oracle state of its whole token history."""
    max_seqs = 6
    cfg, cache, bidx, rng = make_cache(name, max_seqs, seed=21)
    L, H, D, S, G = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.sink_size, cfg.q_buffer_size
    pre_len = [0, max(S // 2, 1), S + 3, S + G - 1, S + G + 5, 0]           # tokens appended first
    chunk1 = [2 * G + 3, G, G + 1, 1, 3 * G, 0]                             # first prefill chunk
    chunk2 = [G - 1, 0, 2 * G, G + 2, 5, S + G + 7]                          # second chunk
    total = [a + b + c + 1 for a, b, c in zip(pre_len, chunk1, chunk2)]
    hist = {(l, s): [x.transpose(1, 0, 2) for x in synthetic.make_kv(rng, H, total[s], D)]
            for l in range(L) for s in range(max_seqs)}
    for l in range(L):
        for t in range(max(pre_len)):
            ids = [s for s in range(max_seqs) if t < pre_len[s]]
            k = np.stack([hist[(l, s)][0][t] for s in ids]); v = np.stack([hist[(l, s)][1][t] for s in ids])
            cache.append(l, ids, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
    pos = list(pre_len)
    for chunk in (chunk1, chunk2):
        order = [int(s) for s in rng.permutation(max_seqs)]
        for l in range(L):
            k = np.concatenate([hist[(l, s)][0][pos[s]:pos[s] + chunk[s]] for s in order])
            v = np.concatenate([hist[(l, s)][1][pos[s]:pos[s] + chunk[s]] for s in order])
            cache.prefill(l, order, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV),
                          [chunk[s] for s in order])
        for s in range(max_seqs):
            pos[s] += chunk[s]
    # one more decode-step append, then compare everything
    for l in range(L):
        k = np.stack([hist[(l, s)][0][pos[s]] for s in range(max_seqs)])
        v = np.stack([hist[(l, s)][1][pos[s]] for s in range(max_seqs)])
        cache.append(l, list(range(max_seqs)), torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
    torch.cuda.synchronize()
    cache.check_errors()
    for (l, s), (k, v) in hist.items():
        check_sequence(cache, cfg, bidx, l, s, k, v)
    Hq = 2 * H
    ids = np.array([5, 0, 3], dtype=np.int32)
    q = synthetic.make_q(rng, (3, Hq, D))
    out = cache.decode(L - 1, torch.from_numpy(q).to(DEV), torch.from_numpy(ids).to(DEV))
    torch.cuda.synchronize()
    for i, s in enumerate(ids):
        exp = oracle_decode(cache, cfg, L - 1, int(s), q[i])
        np.testing.assert_allclose(out[i].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)


def test_prefill_out_of_pages_serves_sequences_in_order():
    cfg, cache, bidx, rng = make_cache("tiny", 4, seed=23, num_pages=5)
    H, D, S, G = cfg.num_kv_heads, cfg.head_dim, cfg.sink_size, cfg.q_buffer_size
    lens = [S + 2 * G, S + 2 * G + 1, S + 3 * G, S + G - 2]     # pages needed: 2, 2, 3, 0
    kv = [[x.transpose(1, 0, 2) for x in synthetic.make_kv(rng, H, n, D)] for n in lens]
    k = np.concatenate([x[0] for x in kv]); v = np.concatenate([x[1] for x in kv])
    cache.prefill(0, [0, 1, 2, 3], torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), lens)
    torch.cuda.synchronize()
    assert _lib.device_error_flags(clear=True) == 1 << 1
    # sequences 0 and 1 took 4 of the 5 pages; sequence 2 needed 3 and is unchanged;
    # sequence 3 needs no page and is served
    for s in (0, 1, 3):
        check_sequence(cache, cfg, bidx, 0, s, kv[s][0], kv[s][1])
    assert [int(x) for x in cache.lengths(0)["sink_len"]] == [S, S, 0, S]
    assert cache.free_page_count() == 1
    # with pages released, sequence 2's prefill goes through
    cache.release([0])
    cache.prefill(0, [2], torch.from_numpy(kv[2][0]).to(DEV), torch.from_numpy(kv[2][1]).to(DEV), [lens[2]])
    torch.cuda.synchronize()
    cache.check_errors()
    check_sequence(cache, cfg, bidx, 0, 2, kv[2][0], kv[2][1])
    assert cache.free_page_count() == 0
