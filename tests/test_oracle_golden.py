"""Pin the numpy oracle to the reference: every recorded reference output must be
reproduced (codes bit-exact, metadata by value, dequantised floats exactly,
attention within float32 rounding noise)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import kitty_oracle as O

from conftest import meta_by_value, sha, small_case_names
import golden_cases as GC


@pytest.mark.parametrize("name", ["rand0", "rand1", "rand2", "rand3", "constant_channels", "all_zero",
                                  "wide_ranges", "permuted_boost", "duplicate_rows", "boost_eq_k",
                                  "known_answer_0123", "halfway", "d128_page", "nonfinite", "nonfinite_d128"])
def test_key_quantize_matches_reference(golden_npz, name):
    p = f"key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    low, high, sc, zp = O.quantize_key_page(golden_npz[p + "key"], golden_npz[p + "boost_idx"], K, sent)
    np.testing.assert_array_equal(low, golden_npz[p + "low"])
    np.testing.assert_array_equal(high, golden_npz[p + "high"])
    np.testing.assert_array_equal(meta_by_value(sc), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp), meta_by_value(golden_npz[p + "zero"]))
    rec = O.dequantize_key_page(low, high, sc, zp, golden_npz[p + "boost_idx"], K)
    np.testing.assert_array_equal(rec, golden_npz[p + "dequant"])


def test_every_small_case_is_covered(golden_npz):
    assert len(small_case_names(golden_npz, "key")) == 15
    assert len(small_case_names(golden_npz, "value")) == 11


@pytest.mark.parametrize("name", ["rand0", "rand1", "rand2", "constant_3", "all_zero", "constant_rows",
                                  "wide_ranges", "halfway", "d128_page", "nonfinite", "nonfinite_d128"])
def test_value_quantize_matches_reference(golden_npz, name):
    p = f"value/{name}/"
    codes, sc, zp = O.quantize_value_page(golden_npz[p + "value"])
    np.testing.assert_array_equal(codes, golden_npz[p + "codes"])
    np.testing.assert_array_equal(meta_by_value(sc), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp), meta_by_value(golden_npz[p + "zero"]))
    np.testing.assert_array_equal(O.dequantize_value_page(codes, sc, zp), golden_npz[p + "dequant"])


def test_known_answer_0123(golden_npz):
    """The reference's only known-answer test (tests/test_quantize.py:141-166)."""
    key = np.tile(np.array([0.0, 1.0, 2.0, 3.0], np.float16), (4, 1))
    low, high, sc, zp = O.quantize_key_page(key, np.full(4, 255, np.uint8), 0, 255)
    rec = O.dequantize_key_page(low, high, sc, zp, np.full(4, 255, np.uint8), 0)
    np.testing.assert_allclose(rec, np.tile([0.0, 1.0, 2.0, 3.0], (4, 1)), atol=1e-3)
    assert high.shape == (0, 1)


def test_batched_oracle_equals_single():
    rng = np.random.default_rng(5)
    keys = (rng.standard_normal((3, 2, 16, 8)) * rng.uniform(0.1, 9, (3, 2, 16, 1))).astype(np.float16)
    bidx = np.full((2, 16), 5, np.uint8); bidx[0, :4] = np.arange(4); bidx[1, [3, 7, 9, 1]] = np.arange(4)
    bidx[1, 12] = 2  # duplicate row
    low, high, sc, zp = O.quantize_key_pages(keys, bidx, 4, 5)
    for i in range(3):
        for h in range(2):
            a, b, c, d = O.quantize_key_page(keys[i, h], bidx[h], 4, 5)
            np.testing.assert_array_equal(low[i, h], a)
            np.testing.assert_array_equal(high[i, h], b)
            np.testing.assert_array_equal(sc[i, h], c)
            np.testing.assert_array_equal(meta_by_value(zp[i, h]), meta_by_value(d))
            np.testing.assert_array_equal(O.dequantize_key_pages(low[i, h][None], high[i, h][None], sc[i, h][None],
                                                                 zp[i, h][None], bidx[h], 4)[0],
                                          O.dequantize_key_page(a, b, c, d, bidx[h], 4))
    vals = rng.standard_normal((3, 2, 8, 16)).astype(np.float16)
    codes, vs, vz = O.quantize_value_pages(vals)
    for i in range(3):
        for h in range(2):
            a, b, c = O.quantize_value_page(vals[i, h])
            np.testing.assert_array_equal(codes[i, h], a)
            np.testing.assert_array_equal(vs[i, h], b)
            np.testing.assert_array_equal(meta_by_value(vz[i, h]), meta_by_value(c))


def _oracle_pools(case, phys_of, n_phys):
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    kl = np.zeros((n_phys, H, D, G // 4), np.uint8); kh = np.zeros((n_phys, H, K, G // 4), np.uint8)
    km = np.zeros((n_phys, H, 2, D), np.float16); vc = np.zeros((n_phys, H, G, D // 4), np.uint8)
    vm = np.zeros((n_phys, H, G, 2), np.float16)
    for b, s in enumerate(case.seqs):
        if s.n_pages == 0:
            continue
        low, high, sc, zp = O.quantize_key_pages(s.page_keys(), case.boost_idx, K, case.sentinel)
        codes, vs, vz = O.quantize_value_pages(s.page_values())
        p = phys_of[b]
        kl[p] = low; kh[p] = high; km[p, :, 0] = sc; km[p, :, 1] = zp
        vc[p] = codes; vm[p, :, :, 0] = vs; vm[p, :, :, 1] = vz
    return kl, kh, km, vc, vm


@pytest.mark.parametrize("name", ["tiny_mixed", "tiny_sink_only", "tiny_no_sink", "tiny_tail_only", "tiny_gqa8",
                                  "d128_short", "config1", "batched_pro"])
def test_attention_pools_and_outputs_match_reference(golden_npz, golden_manifest, name):
    e = golden_manifest["attention"][name]
    case = GC.decode_case_from_manifest(e)
    phys_of = GC.phys_layout(case, e["phys_seed"], e["n_phys"])
    pools = _oracle_pools(case, phys_of, e["n_phys"])
    names = ["key_low", "key_high", "key_meta", "val_codes", "val_meta"]
    for n, p in zip(names, pools):
        if n in ("key_meta", "val_meta"):
            assert sha(meta_by_value(p)) == e["pools_sha"][n + "_value"], n
        else:
            assert sha(p) == e["pools_sha"][n], n
    sk, sv, sl, tk, tv, tl = GC.padded_regions(case)
    bt, npg = GC.block_table(case, phys_of)
    out = O.paged_attention_batched(case.q, bt, npg, pools, case.boost_idx, case.d_boost, sk, sv, sl, tk, tv, tl)
    ref = golden_npz[f"attn/{name}/out"]
    np.testing.assert_allclose(out.astype(np.float32), ref.astype(np.float32), atol=1e-3, rtol=1e-3)


def test_config3_sample_quantization_matches_reference(golden_manifest):
    """Config-3-shaped pages (K=32): oracle outputs hash-identical to the reference's."""
    e = golden_manifest["quant"]["config3_sample"]
    rng = np.random.default_rng(e["seed"])
    H, D, T, K, S, G = e["num_kv_heads"], e["head_dim"], e["tokens"], e["d_boost"], e["sink"], e["group"]
    seqs = [GC.synthetic.make_kv(rng, H, T, D) for _ in range(e["n_seq"])]
    assert [sha(s[0]) for s in seqs] == e["inputs_sha"]["k"]
    bidx = GC.synthetic.boost_idx_from_scores(GC.synthetic.channel_scores([s[0] for s in seqs]), K, e["sentinel"])
    assert sha(bidx) == e["inputs_sha"]["boost_idx"]
    n = e["n_pages"]
    for (k, v), ref in zip(seqs, e["outputs_sha"]):
        sq = GC.synthetic.SequenceKV(k=k, v=v, sink=S, n_pages=n, tail=(T - S) - n * G, group=G)
        low, high, sc, zp = O.quantize_key_pages(sq.page_keys(), bidx, K, e["sentinel"])
        codes, vs, vz = O.quantize_value_pages(sq.page_values())
        assert sha(low) == ref["key_low"]
        assert sha(high) == ref["key_high"]
        assert sha(sc) == ref["key_scale"]
        assert sha(meta_by_value(zp)) == ref["key_zero_value"]
        assert sha(codes) == ref["val_codes"]
        assert sha(vs) == ref["val_scale"]
        assert sha(meta_by_value(vz)) == ref["val_zero_value"]


def test_profiler_rule_matches_reference(golden_manifest):
    """boost index from channel scores == the reference profiler's compute()."""
    assert golden_manifest["profiler"]["equal"]
    rng = np.random.default_rng(golden_manifest["profiler"]["seed"])
    keys = [GC.synthetic.make_kv(rng, 4, 256, 128)[0] for _ in range(2)]
    mine = np.stack([O.boost_idx_from_scores(GC.synthetic.channel_scores([k]), 16, 17) for k in keys])
    assert sha(mine) == golden_manifest["profiler"]["boost_idx_sha"]


@pytest.mark.parametrize("name", ["tiny", "d128"])
def test_sequence_state_matches_reference_pipeline(golden_npz, golden_manifest, name):
    """The cache state machine of the oracle (sinks, key pages, key tail after T pushes)
    against the reference pipeline driven over the same tokens: counters, the page
    count, the key pool bytes and the fp16 sink / Key Q-buffer contents.  (Value pages
    are not compared: the reference quantises its value window's evictions, the
    batched cache the values of the page's own tokens.)"""
    import synthetic
    e = golden_manifest["pipeline"][name]
    cfg = e["config"]
    H, D, G, S = cfg["num_kv_heads"], cfg["head_dim"], cfg["q_buffer_size"], cfg["sink_size"]
    K = round(cfg["boost_rate"] * D)
    sent = min(K + 1, 255)
    rng = np.random.default_rng(e["seed"])
    k, v = synthetic.make_kv(rng, H, e["steps"], D)
    bidx = synthetic.boost_idx_from_scores(synthetic.channel_scores([k]), K, sent)
    st = O.sequence_state(k.transpose(1, 0, 2), v.transpose(1, 0, 2), S, G, bidx, K, sent)
    s, n, t = O.cache_regions(e["steps"], S, G)
    assert (s, t) == (e["state"]["sink_fill"], e["state"]["key_qbuf_len"])
    assert n == len(e["page_list"]) == len(st["pages"])
    P = ((cfg["max_seq_len"] - S) // G + 2)
    low = np.zeros((P, H, D, G // 4), np.uint8)
    high = np.zeros((P, H, K, G // 4), np.uint8)
    meta = np.zeros((P, H, 2, D), np.float16)
    for j, page in enumerate(e["page_list"]):
        pg = st["pages"][j]
        low[page], high[page] = pg["key_low"], pg["key_high"]
        meta[page, :, 0], meta[page, :, 1] = pg["key_scale"], pg["key_zero"]
    assert sha(low) == e["pools_sha"]["key_low"]
    assert sha(high) == e["pools_sha"]["key_high"]
    assert sha(meta_by_value(meta)) == e["pools_sha"]["key_meta_value"]
    sink = np.zeros((1, H, S, D), np.float16)
    sink[0, :, :s] = st["sink_k"]
    assert sha(sink) == e["buffers_sha"]["sink_k"]
    qbuf = np.zeros((1, H, G, D), np.float16)
    qbuf[0, :, :t] = st["tail_k"]
    assert sha(qbuf) == e["buffers_sha"]["key_qbuf"]


# ----------------------------------------------------------------- bfloat16 cache

BF16_KEY = ["rand0", "rand1", "rand2", "rand3", "constant_channels", "all_zero", "wide_ranges", "permuted_boost",
            "duplicate_rows", "boost_eq_k", "known_answer_0123", "halfway", "d128_page"]
BF16_VALUE = ["rand0", "rand1", "rand2", "constant_3", "all_zero", "constant_rows", "wide_ranges", "halfway",
              "d128_page"]


def test_bf16_sets_are_recorded(golden_manifest):
    assert sorted(n for k, n in golden_manifest["bf16_small"] if k == "bf16key") == sorted(BF16_KEY)
    assert sorted(n for k, n in golden_manifest["bf16_small"] if k == "bf16value") == sorted(BF16_VALUE)


def test_bf16_round_matches_torch():
    """bf16_round == torch's float32 -> bfloat16 conversion (ties, overflow, subnormals)."""
    import torch
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-40, 38, 20000),
                        np.array([1.0, 1.00390625, 1.005859375, 1.0078125, 65504.0, 3.4e38, 3.3e38, np.inf, -np.inf,
                                  -0.0, 1e-40, -1e-45], np.float32)]).astype(np.float32)
    exp = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.bf16_round(x), exp)
    assert np.isnan(O.bf16_round(np.array([np.nan], np.float32)))[0]


@pytest.mark.parametrize("name", BF16_KEY)
def test_bf16_key_quantize_matches_reference(golden_npz, name):
    p = f"bf16key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    low, high, sc, zp = O.quantize_key_page(golden_npz[p + "key"], golden_npz[p + "boost_idx"], K, sent,
                                            dtype="bfloat16")
    np.testing.assert_array_equal(low, golden_npz[p + "low"])
    np.testing.assert_array_equal(high, golden_npz[p + "high"])
    np.testing.assert_array_equal(meta_by_value(sc), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp), meta_by_value(golden_npz[p + "zero"]))
    rec = O.dequantize_key_page(low, high, sc, zp, golden_npz[p + "boost_idx"], K, dtype="bfloat16")
    np.testing.assert_array_equal(rec, golden_npz[p + "dequant"])


@pytest.mark.parametrize("name", BF16_VALUE)
def test_bf16_value_quantize_matches_reference(golden_npz, name):
    p = f"bf16value/{name}/"
    codes, sc, zp = O.quantize_value_page(golden_npz[p + "value"], dtype="bfloat16")
    np.testing.assert_array_equal(codes, golden_npz[p + "codes"])
    np.testing.assert_array_equal(meta_by_value(sc), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp), meta_by_value(golden_npz[p + "zero"]))
    np.testing.assert_array_equal(O.dequantize_value_page(codes, sc, zp, dtype="bfloat16"), golden_npz[p + "dequant"])


def bf16_oracle_pools(case, phys_of, n_phys):
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    kl = np.zeros((n_phys, H, D, G // 4), np.uint8); kh = np.zeros((n_phys, H, K, G // 4), np.uint8)
    km = np.zeros((n_phys, H, 2, D), np.float32); vc = np.zeros((n_phys, H, G, D // 4), np.uint8)
    vm = np.zeros((n_phys, H, G, 2), np.float32)
    for b, s in enumerate(case.seqs):
        if s.n_pages == 0:
            continue
        low, high, sc, zp = O.quantize_key_pages(s.page_keys(), case.boost_idx, K, case.sentinel, dtype="bfloat16")
        codes, vs, vz = O.quantize_value_pages(s.page_values(), dtype="bfloat16")
        p = phys_of[b]
        kl[p] = low; kh[p] = high; km[p, :, 0] = sc; km[p, :, 1] = zp
        vc[p] = codes; vm[p, :, :, 0] = vs; vm[p, :, :, 1] = vz
    return kl, kh, km, vc, vm


@pytest.mark.parametrize("name", ["bf16_tiny", "bf16_d128"])
def test_bf16_attention_pools_and_outputs_match_reference(golden_npz, golden_manifest, name):
    e = golden_manifest["bf16_attention"][name]
    case = GC.bf16_case_from_manifest(e, O.bf16_round)
    phys_of = GC.phys_layout(case, e["phys_seed"], e["n_phys"])
    pools = bf16_oracle_pools(case, phys_of, e["n_phys"])
    assert sha(pools[0]) == e["pools_sha"]["key_low"]
    assert sha(pools[1]) == e["pools_sha"]["key_high"]
    assert sha(pools[3]) == e["pools_sha"]["val_codes"]
    assert sha(pools[2] + np.float32(0.0)) == e["pools_sha"]["key_meta_value"]
    assert sha(pools[4] + np.float32(0.0)) == e["pools_sha"]["val_meta_value"]
    sk, sv, sl, tk, tv, tl = GC.padded_regions(case, np.float32)
    bt, npg = GC.block_table(case, phys_of)
    out = O.paged_attention_batched(case.q, bt, npg, pools, case.boost_idx, case.d_boost, sk, sv, sl, tk, tv, tl,
                                    dtype="bfloat16")
    np.testing.assert_allclose(out.astype(np.float32), golden_npz[f"bf16attn/{name}/out"].astype(np.float32),
                               atol=1e-3, rtol=1e-3)
