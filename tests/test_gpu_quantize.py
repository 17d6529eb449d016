"""GPU parity of the page quantise/pack kernels (through the C ABI) against the
reference's recorded outputs: codes and high planes bit-exact, fp16 metadata
equal by value (+0 == -0)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kitty import kernels as KK
import synthetic
from oracle import kitty_oracle as O

from conftest import meta_by_value, sha
import golden_cases as GC

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

KEY_CASES = ["rand0", "rand1", "rand2", "rand3", "constant_channels", "all_zero", "wide_ranges",
             "permuted_boost", "duplicate_rows", "boost_eq_k", "known_answer_0123", "halfway", "d128_page",
             "nonfinite", "nonfinite_d128"]
VALUE_CASES = ["rand0", "rand1", "rand2", "constant_3", "all_zero", "constant_rows", "wide_ranges",
               "halfway", "d128_page", "nonfinite", "nonfinite_d128"]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("name", KEY_CASES)
def test_key_page_functional(golden_npz, name):
    p = f"key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    low, high, sc, zp = KK.quantize_key_page_torch(cuda(golden_npz[p + "key"]), cuda(golden_npz[p + "boost_idx"]),
                                                   K, sent)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(low.cpu().numpy(), golden_npz[p + "low"])
    np.testing.assert_array_equal(high.cpu().numpy(), golden_npz[p + "high"])
    np.testing.assert_array_equal(meta_by_value(sc.cpu().numpy()), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp.cpu().numpy()), meta_by_value(golden_npz[p + "zero"]))


@pytest.mark.parametrize("name", KEY_CASES)
def test_key_page_into_pool_views_and_dequant(golden_npz, name):
    """Reference launcher signature writing into pool views (kitty/pipeline.py:214-230),
    with a transposed (non-contiguous) key source, then dequantise."""
    p = f"key/{name}/"
    K, sent = (int(x) for x in golden_npz[p + "params"])
    key = golden_npz[p + "key"]
    D, G = key.shape
    P, H = 3, 2
    kl = torch.full((P, H, D, G // 4), 0xAA, dtype=torch.uint8, device=DEV)
    kh = torch.full((P, H, K, G // 4), 0x55, dtype=torch.uint8, device=DEV)
    km = torch.full((P, H, 2, D), 7.0, dtype=torch.float16, device=DEV)
    src = cuda(np.ascontiguousarray(key.T)).T       # (D, G) view with token stride 1
    KK.quantize_key_page(src, cuda(golden_npz[p + "boost_idx"]), K, sent, kl[2][1], kh[2][1], km[2, 1, 0], km[2, 1, 1])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kl[2, 1].cpu().numpy(), golden_npz[p + "low"])
    np.testing.assert_array_equal(kh[2, 1].cpu().numpy(), golden_npz[p + "high"])
    np.testing.assert_array_equal(meta_by_value(km[2, 1, 0].cpu().numpy()), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(km[2, 1, 1].cpu().numpy()), meta_by_value(golden_npz[p + "zero"]))
    assert (kl[:2] == 0xAA).all() and (kl[2, 0] == 0xAA).all(), "wrote outside the target page-head"
    out = torch.empty(D, G, dtype=torch.float16, device=DEV)
    KK.dequantize_key_page(kl[2, 1], kh[2, 1], km[2, 1, 0], km[2, 1, 1], cuda(golden_npz[p + "boost_idx"]), K, out)
    torch.cuda.synchronize()
    ref = golden_npz[p + "dequant"].astype(np.float16)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("name", VALUE_CASES)
def test_value_page_functional_and_views(golden_npz, name):
    p = f"value/{name}/"
    v = golden_npz[p + "value"]
    codes, sc, zp = KK.quantize_value_page_torch(cuda(v))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), golden_npz[p + "codes"])
    np.testing.assert_array_equal(meta_by_value(sc.cpu().numpy()), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(zp.cpu().numpy()), meta_by_value(golden_npz[p + "zero"]))
    G, D = v.shape
    vc = torch.zeros(2, 2, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.zeros(2, 2, G, 2, dtype=torch.float16, device=DEV)
    # stride-2 metadata views, as the reference pipeline passes them (kitty/pipeline.py:245-250)
    KK.quantize_value_page(cuda(v), vc[1][0], vm[1, 0, :, 0], vm[1, 0, :, 1])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(vc[1, 0].cpu().numpy(), golden_npz[p + "codes"])
    np.testing.assert_array_equal(meta_by_value(vm[1, 0, :, 0].cpu().numpy()), meta_by_value(golden_npz[p + "scale"]))
    np.testing.assert_array_equal(meta_by_value(vm[1, 0, :, 1].cpu().numpy()), meta_by_value(golden_npz[p + "zero"]))
    assert (vc[0] == 0).all() and (vm[0] == 0).all()


def test_cpu_tensors_raise():
    with pytest.raises(RuntimeError, match="CUDA"):
        KK.quantize_key_page_torch(torch.zeros(16, 8, dtype=torch.float16), torch.zeros(16, dtype=torch.uint8), 4, 5)


def test_batched_pool_quantization_matches_reference_hashes(golden_manifest):
    """Config-1 and batched Kitty-Pro pools built by the batched CUDA entry points from a
    token-major (H, T, D) source are hash-identical to the reference's pools."""
    for name in ("config1", "batched_pro", "d128_short"):
        e = golden_manifest["attention"][name]
        case = GC.decode_case_from_manifest(e)
        phys_of = GC.phys_layout(case, e["phys_seed"], e["n_phys"])
        pools = build_pools_gpu(case, phys_of, e["n_phys"])
        names = ["key_low", "key_high", "key_meta", "val_codes", "val_meta"]
        for n, p in zip(names, pools):
            arr = p.cpu().numpy()
            if n in ("key_meta", "val_meta"):
                assert sha(meta_by_value(arr)) == e["pools_sha"][n + "_value"], (name, n)
            else:
                assert sha(arr) == e["pools_sha"][n], (name, n)


def build_pools_gpu(case, phys_of, n_phys):
    """Quantise all page-heads of ``case`` with the batched kernels (one launch per
    sequence per tensor), reading straight from the (H, T, D) fp16 cache."""
    H, D, G, K = case.num_kv_heads, case.head_dim, case.group, case.d_boost
    kl = torch.zeros(n_phys, H, D, G // 4, dtype=torch.uint8, device=DEV)
    kh = torch.zeros(n_phys, H, K, G // 4, dtype=torch.uint8, device=DEV)
    km = torch.zeros(n_phys, H, 2, D, dtype=torch.float16, device=DEV)
    vc = torch.zeros(n_phys, H, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.zeros(n_phys, H, G, 2, dtype=torch.float16, device=DEV)
    bidx = cuda(case.boost_idx)
    for b, s in enumerate(case.seqs):
        if s.n_pages == 0:
            continue
        k = cuda(s.k); v = cuda(s.v)
        offs = torch.tensor([(s.sink + i * G) * D for i in range(s.n_pages)], dtype=torch.int64, device=DEV)
        dst = torch.from_numpy(phys_of[b]).to(DEV)
        KK.quantize_key_pages(k, offs, (k.stride(0), k.stride(1), k.stride(2)), bidx, K, case.sentinel, dst,
                              kl, kh, km, H, D, G)
        KK.quantize_value_pages(v, offs, (v.stride(0), v.stride(1), v.stride(2)), dst, vc, vm, H, D, G)
    torch.cuda.synchronize()
    return kl, kh, km, vc, vm


def test_config3_sample_bit_exact(golden_manifest):
    """Benchmark config 3 (K=32) on the recorded 2-sequence sample: every page-head's
    outputs hash-identical to the reference's."""
    e = golden_manifest["quant"]["config3_sample"]
    rng = np.random.default_rng(e["seed"])
    H, D, T, K, S, G = e["num_kv_heads"], e["head_dim"], e["tokens"], e["d_boost"], e["sink"], e["group"]
    seqs = [synthetic.make_kv(rng, H, T, D) for _ in range(e["n_seq"])]
    bidx = synthetic.boost_idx_from_scores(synthetic.channel_scores([s[0] for s in seqs]), K, e["sentinel"])
    assert sha(bidx) == e["inputs_sha"]["boost_idx"]
    n = e["n_pages"]
    for (k, v), ref in zip(seqs, e["outputs_sha"]):
        kt, vt = cuda(k), cuda(v)
        kl = torch.zeros(n, H, D, G // 4, dtype=torch.uint8, device=DEV)
        kh = torch.zeros(n, H, K, G // 4, dtype=torch.uint8, device=DEV)
        km = torch.zeros(n, H, 2, D, dtype=torch.float16, device=DEV)
        vc = torch.zeros(n, H, G, D // 4, dtype=torch.uint8, device=DEV)
        vm = torch.zeros(n, H, G, 2, dtype=torch.float16, device=DEV)
        offs = torch.arange(n, dtype=torch.int64, device=DEV) * (G * D) + S * D
        dst = torch.arange(n, dtype=torch.int32, device=DEV)
        KK.quantize_key_pages(kt, offs, (T * D, D, 1), cuda(bidx), K, e["sentinel"], dst, kl, kh, km, H, D, G)
        KK.quantize_value_pages(vt, offs, (T * D, D, 1), dst, vc, vm, H, D, G)
        torch.cuda.synchronize()
        assert sha(kl.cpu().numpy()) == ref["key_low"]
        assert sha(kh.cpu().numpy()) == ref["key_high"]
        assert sha(km[:, :, 0].cpu().numpy()) == ref["key_scale"]
        assert sha(meta_by_value(km[:, :, 1].cpu().numpy())) == ref["key_zero_value"]
        assert sha(vc.cpu().numpy()) == ref["val_codes"]
        assert sha(vm[..., 0].cpu().numpy()) == ref["val_scale"]
        assert sha(meta_by_value(vm[..., 1].cpu().numpy())) == ref["val_zero_value"]


def test_nonfinite_pages_on_the_token_major_path(golden_npz):
    """The D = G = 128 page quantisers (token-major source, batched entry points: the path
    a cache flush and a prefill take) on pages holding +-inf and NaN: channels (keys) and
    tokens (values) with a non-finite range take the exact per-element path and must
    still equal the reference's recorded pages byte for byte (metadata by value)."""
    pk, pv = "key/nonfinite_d128/", "value/nonfinite_d128/"
    key, bidx = golden_npz[pk + "key"], golden_npz[pk + "boost_idx"]
    K, sent = (int(x) for x in golden_npz[pk + "params"])
    D, G = key.shape
    H, S = 1, 32
    # (H, T, D) caches: S leading tokens, then the page
    kt = torch.zeros(H, S + G, D, dtype=torch.float16, device=DEV)
    kt[0, S:] = cuda(np.ascontiguousarray(key.T))
    vt = torch.zeros(H, S + G, D, dtype=torch.float16, device=DEV)
    vt[0, S:] = cuda(golden_npz[pv + "value"])
    offs = torch.tensor([S * D], dtype=torch.int64, device=DEV)
    dst = torch.tensor([1], dtype=torch.int32, device=DEV)
    kl = torch.zeros(2, H, D, G // 4, dtype=torch.uint8, device=DEV)
    kh = torch.zeros(2, H, K, G // 4, dtype=torch.uint8, device=DEV)
    km = torch.zeros(2, H, 2, D, dtype=torch.float16, device=DEV)
    vc = torch.zeros(2, H, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.zeros(2, H, G, 2, dtype=torch.float16, device=DEV)
    KK.quantize_key_pages(kt, offs, tuple(kt.stride()), cuda(bidx[None, :]), K, sent, dst, kl, kh, km, H, D, G)
    KK.quantize_value_pages(vt, offs, tuple(vt.stride()), dst, vc, vm, H, D, G)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kl[1, 0].cpu().numpy(), golden_npz[pk + "low"])
    np.testing.assert_array_equal(kh[1, 0].cpu().numpy(), golden_npz[pk + "high"])
    np.testing.assert_array_equal(meta_by_value(km[1, 0, 0].cpu().numpy()), meta_by_value(golden_npz[pk + "scale"]))
    np.testing.assert_array_equal(meta_by_value(km[1, 0, 1].cpu().numpy()), meta_by_value(golden_npz[pk + "zero"]))
    np.testing.assert_array_equal(vc[1, 0].cpu().numpy(), golden_npz[pv + "codes"])
    np.testing.assert_array_equal(meta_by_value(vm[1, 0, :, 0].cpu().numpy()), meta_by_value(golden_npz[pv + "scale"]))
    np.testing.assert_array_equal(meta_by_value(vm[1, 0, :, 1].cpu().numpy()), meta_by_value(golden_npz[pv + "zero"]))
    assert (kl[0] == 0).all() and (vc[0] == 0).all()


def test_value_partial_buffer_zero_padding():
    """n_valid < G: tokens beyond are quantised as zeros (kitty/pipeline.py:238-243)."""
    rng = np.random.default_rng(3)
    H, G, D = 2, 128, 128
    buf = rng.standard_normal((H, G, D)).astype(np.float16)
    vc = torch.zeros(1, H, G, D // 4, dtype=torch.uint8, device=DEV)
    vm = torch.zeros(1, H, G, 2, dtype=torch.float16, device=DEV)
    src = cuda(buf)
    KK.quantize_value_pages(src, torch.zeros(1, dtype=torch.int64, device=DEV), (G * D, D, 1),
                            torch.zeros(1, dtype=torch.int32, device=DEV), vc, vm, H, D, G,
                            n_valid=torch.tensor([37], dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    padded = buf.copy(); padded[:, 37:] = 0
    for h in range(H):
        codes, sc, zp = O.quantize_value_page(padded[h])
        np.testing.assert_array_equal(vc[0, h].cpu().numpy(), codes)
        np.testing.assert_array_equal(vm[0, h, :, 0].cpu().numpy(), sc)
        np.testing.assert_array_equal(meta_by_value(vm[0, h, :, 1].cpu().numpy()), meta_by_value(zp))


@pytest.mark.parametrize("shape", [(16, 8, 4), (64, 32, 16), (128, 128, 16), (128, 128, 32), (96, 64, 12),
                                   (256, 128, 32)])
def test_random_shapes_match_oracle(shape):
    D, G, K = shape
    rng = np.random.default_rng(D * 1000 + G + K)
    n = 5
    keys = (rng.standard_normal((n, D, G)) * rng.uniform(0.05, 20, (n, D, 1))).astype(np.float16)
    bidx = np.full(D, K + 1, np.uint8); bidx[rng.permutation(D)[:K]] = np.arange(K)
    for i in range(n):
        got = KK.quantize_key_page_torch(cuda(keys[i]), cuda(bidx), K, K + 1)
        exp = O.quantize_key_page(keys[i], bidx, K, K + 1)
        for a, b in zip(got[:2], exp[:2]):
            np.testing.assert_array_equal(a.cpu().numpy(), b)
        for a, b in zip(got[2:], exp[2:]):
            np.testing.assert_array_equal(meta_by_value(a.cpu().numpy()), meta_by_value(b))
        vals = keys[i].T.copy()
        got = KK.quantize_value_page_torch(cuda(vals))
        exp = O.quantize_value_page(vals)
        np.testing.assert_array_equal(got[0].cpu().numpy(), exp[0])
        np.testing.assert_array_equal(meta_by_value(got[1].cpu().numpy()), meta_by_value(exp[1]))
        np.testing.assert_array_equal(meta_by_value(got[2].cpu().numpy()), meta_by_value(exp[2]))


@pytest.mark.parametrize("name", VALUE_CASES)
def test_value_dequant_functional_vs_reference(golden_npz, name):
    """dequantize_value_page_torch (reference quantize_value.py:97-133) on the CUDA value
    dequantiser: float32 (G, D) equal bit for bit to the reference's recorded output,
    from contiguous metadata and from the stride-2 views of a value_metadata pool."""
    p = f"value/{name}/"
    codes, sc, zp, exp = (golden_npz[p + n] for n in ("codes", "scale", "zero", "dequant"))
    got = KK.dequantize_value_page_torch(cuda(codes), cuda(sc), cuda(zp))
    torch.cuda.synchronize()
    assert got.dtype == torch.float32 and tuple(got.shape) == exp.shape
    np.testing.assert_array_equal(got.cpu().numpy(), exp)
    G = codes.shape[0]
    vm = torch.zeros(3, G, 2, dtype=torch.float16, device=DEV)
    vm[1, :, 0] = cuda(sc); vm[1, :, 1] = cuda(zp)
    got = KK.dequantize_value_page_torch(cuda(codes), vm[1, :, 0], vm[1, :, 1])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), exp)


@pytest.mark.parametrize("name", KEY_CASES)
def test_key_dequant_functional_vs_reference(golden_npz, name):
    """dequantize_key_page_torch (reference dequantize_key.py:35-97) on the CUDA key
    dequantiser with float32 output: equal bit for bit to the reference's recorded output."""
    p = f"key/{name}/"
    K = int(golden_npz[p + "params"][0])
    got = KK.dequantize_key_page_torch(cuda(golden_npz[p + "low"]), cuda(golden_npz[p + "high"]),
                                       cuda(golden_npz[p + "scale"]), cuda(golden_npz[p + "zero"]),
                                       cuda(golden_npz[p + "boost_idx"]), K)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    np.testing.assert_array_equal(got.cpu().numpy(), golden_npz[p + "dequant"])


@pytest.mark.parametrize("kind", ["bf16key", "bf16value"])
def test_dequant_functional_bf16_metadata_vs_reference(golden_npz, kind):
    """The same functional forms over bfloat16 metadata (a bfloat16 cache): float32 equal
    to the reference's recorded output for every recorded page."""
    names = sorted({k.split("/")[1] for k in golden_npz if k.startswith(kind + "/")})
    assert names
    for name in names:
        p = f"{kind}/{name}/"
        bf = lambda a: cuda(a.astype(np.float32)).to(torch.bfloat16)
        if kind == "bf16key":
            K = int(golden_npz[p + "params"][0])
            got = KK.dequantize_key_page_torch(cuda(golden_npz[p + "low"]), cuda(golden_npz[p + "high"]),
                                               bf(golden_npz[p + "scale"]), bf(golden_npz[p + "zero"]),
                                               cuda(golden_npz[p + "boost_idx"]), K)
        else:
            got = KK.dequantize_value_page_torch(cuda(golden_npz[p + "codes"]), bf(golden_npz[p + "scale"]),
                                                 bf(golden_npz[p + "zero"]))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), golden_npz[p + "dequant"], err_msg=p)
