"""GPU parity for a bfloat16 cache (KittyConfig(dtype="bfloat16")), through the C ABI.

Against the reference's own recorded bfloat16 outputs (tests/golden, produced by
its CPU path writing into bf16 pool views): packed planes bit-exact, scale and
zero-point equal by value (fp16 rounding, then bf16), dequantised keys exact,
decode outputs within atol 2e-3 / rtol 1e-2 (float16 outputs, as the reference
returns).  The functional ``*_torch`` forms return fp16 metadata for a bf16
input, as the reference's do.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kitty import BatchedKVCache, KittyConfig
from kitty import kernels as KK
import synthetic
from oracle import kitty_oracle as O

from conftest import meta_by_value, sha
import golden_cases as GC

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-3, 1e-2
BF = torch.bfloat16

KEYS = ["rand0", "rand1", "rand2", "rand3", "constant_channels", "all_zero", "wide_ranges", "permuted_boost",
        "duplicate_rows", "boost_eq_k", "known_answer_0123", "halfway", "d128_page"]
VALUES = ["rand0", "rand1", "rand2", "constant_3", "all_zero", "constant_rows", "wide_ranges", "halfway", "d128_page"]


def bf(a):
    """float32 array of bf16 values -> CUDA bfloat16 tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV).to(BF)


def f32(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("name", KEYS)
def test_key_launcher_into_bf16_pool_views(golden_npz, name):
    p = f"bf16key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    key = golden_npz[p + "key"]
    D, G = key.shape
    kl = torch.full((3, 2, D, G // 4), 0xAA, dtype=torch.uint8, device=DEV)
    kh = torch.full((3, 2, K, G // 4), 0x55, dtype=torch.uint8, device=DEV)
    km = torch.full((3, 2, 2, D), 7.0, dtype=BF, device=DEV)
    bidx = torch.from_numpy(golden_npz[p + "boost_idx"]).to(DEV)
    KK.quantize_key_page(bf(key), bidx, K, sent, kl[2][1], kh[2][1], km[2, 1, 0], km[2, 1, 1])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kl[2, 1].cpu().numpy(), golden_npz[p + "low"])
    np.testing.assert_array_equal(kh[2, 1].cpu().numpy(), golden_npz[p + "high"])
    np.testing.assert_array_equal(meta_by_value(f32(km[2, 1, 0])), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(f32(km[2, 1, 1])), meta_by_value(golden_npz[p + "zero"]))
    assert (kl[:2] == 0xAA).all() and (km[:2] == 7.0).all()
    out = torch.empty(D, G, dtype=BF, device=DEV)
    KK.dequantize_key_page(kl[2, 1], kh[2, 1], km[2, 1, 0].contiguous(), km[2, 1, 1].contiguous(), bidx, K, out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(f32(out), O.bf16_round(golden_npz[p + "dequant"]))


@pytest.mark.parametrize("name", KEYS)
def test_key_functional_form_returns_fp16_metadata(golden_npz, name):
    p = f"bf16key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    key, bidx = golden_npz[p + "key"], golden_npz[p + "boost_idx"]
    low, high, sc, zp = KK.quantize_key_page_torch(bf(key), torch.from_numpy(bidx).to(DEV), K, sent)
    torch.cuda.synchronize()
    assert sc.dtype == torch.float16 and zp.dtype == torch.float16
    el, eh, es, ez = O.quantize_key_page(key, bidx, K, sent, dtype="bfloat16", meta_dtype="float16")
    np.testing.assert_array_equal(low.cpu().numpy(), el)
    np.testing.assert_array_equal(high.cpu().numpy(), eh)
    np.testing.assert_array_equal(meta_by_value(sc.cpu().numpy()), meta_by_value(es))
    np.testing.assert_array_equal(meta_by_value(zp.cpu().numpy()), meta_by_value(ez))


@pytest.mark.parametrize("name", VALUES)
def test_value_launcher_into_stride2_bf16_views(golden_npz, name):
    p = f"bf16value/{name}/"
    val = golden_npz[p + "value"]
    G, D = val.shape
    vc = torch.zeros(2, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.full((2, G, 2), 5.0, dtype=BF, device=DEV)
    KK.quantize_value_page(bf(val), vc[1], vm[1, :, 0], vm[1, :, 1])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(vc[1].cpu().numpy(), golden_npz[p + "codes"])
    np.testing.assert_array_equal(meta_by_value(f32(vm[1, :, 0])), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(f32(vm[1, :, 1])), meta_by_value(golden_npz[p + "zero"]))
    codes, sc, zp = KK.quantize_value_page_torch(bf(val))
    torch.cuda.synchronize()
    ec, es, ez = O.quantize_value_page(val, dtype="bfloat16", meta_dtype="float16")
    assert sc.dtype == torch.float16
    np.testing.assert_array_equal(codes.cpu().numpy(), ec)
    np.testing.assert_array_equal(meta_by_value(sc.cpu().numpy()), meta_by_value(es))
    np.testing.assert_array_equal(meta_by_value(zp.cpu().numpy()), meta_by_value(ez))


def build_bf16_pools(case, phys_of, n_phys):
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    kl = torch.zeros(n_phys, H, D, G // 4, dtype=torch.uint8, device=DEV)
    kh = torch.zeros(n_phys, H, K, G // 4, dtype=torch.uint8, device=DEV)
    km = torch.zeros(n_phys, H, 2, D, dtype=BF, device=DEV)
    vc = torch.zeros(n_phys, H, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.zeros(n_phys, H, G, 2, dtype=BF, device=DEV)
    bidx = torch.from_numpy(case.boost_idx).to(DEV)
    for b, s in enumerate(case.seqs):
        if s.n_pages == 0:
            continue
        k, v = bf(s.k), bf(s.v)
        offs = torch.tensor([(s.sink + i * G) * D for i in range(s.n_pages)], dtype=torch.int64, device=DEV)
        dst = torch.from_numpy(phys_of[b]).to(DEV)
        KK.quantize_key_pages(k, offs, (k.stride(0), k.stride(1), k.stride(2)), bidx, K, case.sentinel, dst,
                              kl, kh, km, H, D, G)
        KK.quantize_value_pages(v, offs, (v.stride(0), v.stride(1), v.stride(2)), dst, vc, vm, H, D, G)
    torch.cuda.synchronize()
    return kl, kh, km, vc, vm


@pytest.fixture(params=["auto", "simt", "int8"])
def variant(request):
    prev = KK._lib.force_decode_variant(request.param)
    yield request.param
    KK._lib.force_decode_variant(prev)


@pytest.mark.parametrize("name", ["bf16_tiny", "bf16_d128"])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_decode_vs_reference(golden_npz, golden_manifest, name, splits, variant):
    """Pools built by the bf16 quantisers hash-identical to the reference's; decode over
    them (bf16 q, sinks and tails) vs the reference's float16 outputs."""
    e = golden_manifest["bf16_attention"][name]
    case = GC.bf16_case_from_manifest(e, O.bf16_round)
    phys_of = GC.phys_layout(case, e["phys_seed"], e["n_phys"])
    pools = build_bf16_pools(case, phys_of, e["n_phys"])
    assert sha(pools[0].cpu().numpy()) == e["pools_sha"]["key_low"]
    assert sha(pools[1].cpu().numpy()) == e["pools_sha"]["key_high"]
    assert sha(pools[3].cpu().numpy()) == e["pools_sha"]["val_codes"]
    assert sha(f32(pools[2]) + np.float32(0.0)) == e["pools_sha"]["key_meta_value"]
    assert sha(f32(pools[4]) + np.float32(0.0)) == e["pools_sha"]["val_meta_value"]
    sk, sv, sl, tk, tv, tl = GC.padded_regions(case, np.float32)
    bt, npg = GC.block_table(case, phys_of)
    c = lambda a: torch.from_numpy(a).to(DEV)
    out = KK.paged_attention_batched(bf(case.q), c(bt), c(npg), *pools, c(case.boost_idx), case.d_boost,
                                     sink_k=bf(sk), sink_v=bf(sv), sink_len=c(sl), tail_k=bf(tk), tail_v=bf(tv),
                                     tail_len=c(tl), num_splits=splits)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    np.testing.assert_allclose(out.float().cpu().numpy(), golden_npz[f"bf16attn/{name}/out"].astype(np.float32),
                               atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("Hq", [8, 32, 48, 64])
def test_random_d128_batches_vs_oracle(Hq, variant):
    """Longer contexts with the benchmark distribution (bf16): kernels vs the oracle."""
    case = synthetic.make_decode_case(77, 3, Hq, 8, 128, [32 + 9 * 128 + 50, 32 + 3 * 128, 20], sink=32, group=128,
                                      boost_rate=0.125)
    for s in case.seqs:
        s.k = O.bf16_round(s.k.astype(np.float32)); s.v = O.bf16_round(s.v.astype(np.float32))
    case.q = O.bf16_round(case.q.astype(np.float32))
    n_phys = sum(s.n_pages for s in case.seqs) + 2
    phys_of = GC.phys_layout(case, 5, n_phys)
    pools = build_bf16_pools(case, phys_of, n_phys)
    sk, sv, sl, tk, tv, tl = GC.padded_regions(case, np.float32)
    bt, npg = GC.block_table(case, phys_of)
    c = lambda a: torch.from_numpy(a).to(DEV)
    out = KK.paged_attention_batched(bf(case.q), c(bt), c(npg), *pools, c(case.boost_idx), case.d_boost,
                                     sink_k=bf(sk), sink_v=bf(sv), sink_len=c(sl), tail_k=bf(tk), tail_v=bf(tv),
                                     tail_len=c(tl))
    torch.cuda.synchronize()
    np_pools = [f32(p) if p.dtype == BF else p.cpu().numpy() for p in pools]
    exp = O.paged_attention_batched(case.q, bt, npg, np_pools, case.boost_idx, case.d_boost, sk, sv, sl, tk, tv, tl,
                                    dtype="bfloat16")
    np.testing.assert_allclose(out.float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)


def test_batched_cache_bf16_matches_oracle():
    """Device-resident cache with bfloat16 buffers and metadata: append steps and a
    prefill vs the oracle state machine (bit-exact), then decode vs the oracle."""
    cfg = KittyConfig(num_layers=1, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32, boost_rate=0.125,
                      max_seq_len=1024, dtype="bfloat16", device=DEV, local_value_window=0)
    rng = np.random.default_rng(31)
    bidx = O.boost_idx_from_scores(rng.random((1, 2, 128), dtype=np.float32), cfg.d_boost, cfg.sentinel)
    cache = BatchedKVCache(cfg, torch.from_numpy(bidx), max_seqs=3)
    hist = {}
    lens = [300, 40, 180]
    for s, n in enumerate(lens):
        k, v = (O.bf16_round(x.transpose(1, 0, 2).astype(np.float32)) for x in synthetic.make_kv(rng, 2, n + 5, 128))
        hist[s] = (k, v)
    cache.prefill(0, [0, 1, 2], bf(np.concatenate([hist[s][0][:lens[s]] for s in range(3)])),
                  bf(np.concatenate([hist[s][1][:lens[s]] for s in range(3)])), lens)
    for t in range(5):
        cache.append(0, [2, 0, 1], bf(np.stack([hist[s][0][lens[s] + t] for s in (2, 0, 1)])),
                     bf(np.stack([hist[s][1][lens[s] + t] for s in (2, 0, 1)])))
    torch.cuda.synchronize()
    cache.check_errors()
    for s in range(3):
        k, v = hist[s]
        exp = O.sequence_state(k, v, cfg.sink_size, cfg.q_buffer_size, bidx[0], cfg.d_boost, cfg.sentinel,
                               dtype="bfloat16")
        sl, npg, tl = O.cache_regions(k.shape[0], cfg.sink_size, cfg.q_buffer_size)
        got = cache.lengths(0)
        assert (int(got["sink_len"][s]), int(got["num_pages"][s]), int(got["tail_len"][s])) == (sl, npg, tl)
        np.testing.assert_array_equal(f32(cache.sink_k[0, s, :, :sl]), exp["sink_k"])
        np.testing.assert_array_equal(f32(cache.tail_v[0, s, :, :tl]), exp["tail_v"])
        for j, page in enumerate(cache.block_table[0, s, :npg].cpu().numpy()):
            e = exp["pages"][j]
            np.testing.assert_array_equal(cache.key_baseline[page].cpu().numpy(), e["key_low"])
            np.testing.assert_array_equal(cache.key_boost[page].cpu().numpy(), e["key_high"])
            np.testing.assert_array_equal(meta_by_value(f32(cache.key_metadata[page, :, 0])), meta_by_value(e["key_scale"]))
            np.testing.assert_array_equal(cache.value_pool[page].cpu().numpy(), e["val_codes"])
            np.testing.assert_array_equal(meta_by_value(f32(cache.value_metadata[page, :, :, 0])),
                                          meta_by_value(e["val_scale"]))
    q = O.bf16_round(synthetic.make_q(rng, (3, 8, 128)).astype(np.float32))
    ids = [1, 2, 0]
    out = cache.decode(0, bf(q), ids)
    torch.cuda.synchronize()
    pools = [cache.key_baseline.cpu().numpy(), cache.key_boost.cpu().numpy(), f32(cache.key_metadata),
             cache.value_pool.cpu().numpy(), f32(cache.value_metadata)]
    lens_now = cache.lengths(0)
    for i, s in enumerate(ids):
        sl, npg, tl = (int(lens_now[k][s]) for k in ("sink_len", "num_pages", "tail_len"))
        exp = O.paged_attention(q[i], cache.block_table[0, s, :npg].cpu().numpy(), *pools, bidx[0], cfg.d_boost,
                                f32(cache.sink_k[0, s, :, :sl]), f32(cache.sink_v[0, s, :, :sl]),
                                f32(cache.tail_k[0, s, :, :tl]), f32(cache.tail_v[0, s, :, :tl]), 8, 2, 128,
                                dtype="bfloat16")
        np.testing.assert_allclose(out[i].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)
