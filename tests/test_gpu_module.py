"""GPU tests of the drop-in module stack (KittyAttentionFactory -> pipeline ->
kernels) and of the reference's own test behaviours (tests/test_attention.py,
tests/test_quantize.py in bitxwolf/kitty-kv) run on the CUDA path.

* the reference pipeline driven token by token with ``align_values=False`` writes
  pool bytes identical to the reference's recorded ones (``num_layers == 1``);
* decode steps through ``KittyPagedAttention.forward`` (T == 1) match the oracle
  over the same cache contents within atol 2e-3 / rtol 1e-2;
* a prefill (T > 1) returns causal attention over the raw keys and values and leaves
  the same cache as pushing the tokens one by one;
* quantisation properties the reference tests check (round-trip error bounds, boosted
  channels more accurate, constant values exact, shapes).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import kitty
from kitty import KittyAttentionFactory, KittyConfig
from kitty import kernels as KK
import synthetic
from oracle import kitty_oracle as O

from conftest import meta_by_value, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 2e-3, 1e-2


@pytest.mark.parametrize("name", ["tiny", "d128"])
def test_reference_mode_pipeline_pool_bytes(golden_manifest, name):
    """align_values=False reproduces the reference pipeline's pool bytes on the GPU."""
    e = golden_manifest["pipeline"][name]
    cfgd = dict(e["config"]); cfgd["device"] = DEV
    cfg = KittyConfig(**cfgd)
    H, D = cfg.num_kv_heads, cfg.head_dim
    rng = np.random.default_rng(e["seed"])
    k, v = synthetic.make_kv(rng, H, e["steps"], D)
    bidx = synthetic.boost_idx_from_scores(synthetic.channel_scores([k]), cfg.d_boost, cfg.sentinel)[None]
    layout, pipe, layers = KittyAttentionFactory.from_config(cfg, torch.from_numpy(bidx), e["num_q_heads"],
                                                             align_values=False)
    for t in range(e["steps"]):
        pipe.push_token(0, torch.from_numpy(k[:, t]).to(DEV), torch.from_numpy(v[:, t]).to(DEV))
    torch.cuda.synchronize()
    assert layout.get_page_list(0, 0) == e["page_list"]
    assert {"sink_fill": pipe.sink_fill, "key_qbuf_len": pipe.key_qbuf_len, "val_local_len": pipe.val_local_len,
            "val_qbuf_len": pipe.val_qbuf_len} == e["state"]
    pools = [layout.key_baseline, layout.key_boost, layout.key_metadata, layout.value_pool, layout.value_metadata]
    for n, p in zip(["key_low", "key_high", "val_codes"], [pools[0], pools[1], pools[3]]):
        assert sha(p.cpu().numpy()) == e["pools_sha"][n], n
    assert sha(meta_by_value(pools[2].cpu().numpy())) == e["pools_sha"]["key_meta_value"]
    assert sha(meta_by_value(pools[4].cpu().numpy())) == e["pools_sha"]["val_meta_value"]


def _module_stack(seed, **kw):
    cfg = KittyConfig(device=DEV, **kw)
    rng = np.random.default_rng(seed)
    bidx = O.boost_idx_from_scores(rng.random((cfg.num_layers, cfg.num_kv_heads, cfg.head_dim), dtype=np.float32),
                                   cfg.d_boost, cfg.sentinel)
    return cfg, rng, bidx


def _oracle_from_pipeline(pipe, layout, cfg, bidx, q, l):
    ctx = pipe.get_attention_context(l, 0)
    pools = [t.cpu().numpy() for t in (layout.key_baseline, layout.key_boost, layout.key_metadata,
                                       layout.value_pool, layout.value_metadata)]
    return O.paged_attention(q, ctx["page_list"], *pools, bidx[l], cfg.d_boost, ctx["sink_k"].cpu().numpy(),
                             ctx["sink_v"].cpu().numpy(), ctx["key_qbuf"].cpu().numpy(),
                             ctx["value_tail"].cpu().numpy(), q.shape[0], cfg.num_kv_heads, cfg.head_dim)


def test_decode_steps_through_the_module_match_oracle():
    cfg, rng, bidx = _module_stack(3, num_layers=2, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32,
                                   local_value_window=128, boost_rate=0.125, max_seq_len=1024)
    Hq, H, D = 8, cfg.num_kv_heads, cfg.head_dim
    layout, pipe, layers = KittyAttentionFactory.from_config(cfg, torch.from_numpy(bidx), Hq)
    T = 32 + 2 * 128 + 20
    k, v = synthetic.make_kv(rng, H, T, D)
    checks = {31, 32 + 127, 32 + 128, T - 1}
    for t in range(T):
        q = synthetic.make_q(rng, (Hq, D))
        for l, layer in enumerate(layers):
            out = layer(torch.from_numpy(q).to(DEV).view(1, Hq, 1, D), torch.from_numpy(k[:, t]).to(DEV).view(1, H, 1, D),
                        torch.from_numpy(v[:, t]).to(DEV).view(1, H, 1, D))
            assert out.shape == (1, Hq, 1, D) and out.dtype == torch.float16
            if t in checks:
                torch.cuda.synchronize()
                exp = _oracle_from_pipeline(pipe, layout, cfg, bidx, q, l)
                np.testing.assert_allclose(out[0, :, 0].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL,
                                           rtol=RTOL)
    assert pipe.layer_state(0) == pipe.layer_state(1)
    assert len(layout.get_page_list(0, 0)) == 2 and len(layout.get_page_list(0, 1)) == 2


def test_prefill_then_decode():
    cfg, rng, bidx = _module_stack(4, num_layers=1, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32,
                                   local_value_window=128, boost_rate=0.125, max_seq_len=2048)
    Hq, H, D = 4, cfg.num_kv_heads, cfg.head_dim
    T = 32 + 3 * 128 + 50
    k, v = synthetic.make_kv(rng, H, T + 1, D)
    q = synthetic.make_q(rng, (Hq, T + 1, D))
    kt, vt, qt = (torch.from_numpy(x).to(DEV) for x in (k, v, q))
    layout, pipe, (layer,) = KittyAttentionFactory.from_config(cfg, torch.from_numpy(bidx), Hq)
    out = layer(qt[None, :, :T], kt[None, :, :T], vt[None, :, :T])
    torch.cuda.synchronize()
    assert out.shape == (1, Hq, T, D)
    # causal attention over the raw fp16 keys and values (float32 check on a few rows)
    g = Hq // H
    for qh in range(Hq):
        for t in (0, 31, 200, T - 1):
            s = (q[qh, t].astype(np.float32) @ k[qh // g, :t + 1].astype(np.float32).T) / math.sqrt(D)
            w = np.exp(s - s.max()); w /= w.sum()
            exp = w @ v[qh // g, :t + 1].astype(np.float32)
            np.testing.assert_allclose(out[0, qh, t].float().cpu().numpy(), exp, atol=ATOL, rtol=RTOL)
    # the cache equals token-by-token pushes
    layout2, pipe2, _ = KittyAttentionFactory.from_config(cfg, torch.from_numpy(bidx), Hq)
    for t in range(T):
        pipe2.push_token(0, kt[:, t], vt[:, t])
    torch.cuda.synchronize()
    assert pipe.layer_state(0) == pipe2.layer_state(0)
    for name in ("sink_k", "sink_v", "key_qbuf", "val_tail", "val_local", "val_qbuf"):
        assert torch.equal(getattr(pipe, name), getattr(pipe2, name)), name
    p1, p2 = layout.get_page_list(0, 0), layout2.get_page_list(0, 0)
    assert len(p1) == len(p2) == 3
    for a, b in zip(p1, p2):
        for pool in ("key_baseline", "key_boost", "value_pool"):
            assert torch.equal(getattr(layout, pool)[a], getattr(layout2, pool)[b]), pool
        for pool in ("key_metadata", "value_metadata"):
            assert torch.equal(getattr(layout, pool)[a].float() + 0.0, getattr(layout2, pool)[b].float() + 0.0), pool
    # and a decode step after the prefill
    dq = layer(qt[None, :, T:T + 1], kt[None, :, T:T + 1], vt[None, :, T:T + 1])
    torch.cuda.synchronize()
    exp = _oracle_from_pipeline(pipe, layout, cfg, bidx, q[:, T], 0)
    np.testing.assert_allclose(dq[0, :, 0].float().cpu().numpy(), exp.astype(np.float32), atol=ATOL, rtol=RTOL)


def test_sink_only_context_is_finite():
    """test_attention.py: attention with only sinks (no pages) works and is finite."""
    cfg, rng, bidx = _module_stack(5, num_layers=1, num_kv_heads=2, head_dim=128, q_buffer_size=128, sink_size=32)
    layout, pipe, (layer,) = KittyAttentionFactory.from_config(cfg, torch.from_numpy(bidx), 2)
    for t in range(cfg.sink_size):
        out = layer(torch.randn(1, 2, 1, 128, device=DEV, dtype=torch.float16),
                    torch.randn(1, 2, 1, 128, device=DEV, dtype=torch.float16),
                    torch.randn(1, 2, 1, 128, device=DEV, dtype=torch.float16))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and layout.get_page_list(0, 0) == []


def test_key_round_trip_error_bounds_and_boost():
    """test_quantize.py: |x - dequant(quant(x))| stays within one quantisation step per
    channel (half a step except where the zero-point rounding clamps the top code; plus
    fp16 rounding), and INT4 (boosted) channels reconstruct more accurately than INT2."""
    rng = np.random.default_rng(9)
    D, G, K = 16, 8, 8
    sent = K + 1
    bidx = np.full(D, sent, np.uint8); bidx[:K] = np.arange(K)
    errs_b, errs_n = [], []
    for _ in range(20):
        key = rng.standard_normal((D, G)).astype(np.float16)
        kt = torch.from_numpy(key).to(DEV)
        low, high, sc, zp = KK.quantize_key_page_torch(kt, torch.from_numpy(bidx).to(DEV), K, sent)
        out = torch.empty(D, G, dtype=torch.float16, device=DEV)
        KK.dequantize_key_page(low, high, sc, zp, torch.from_numpy(bidx).to(DEV), K, out)
        torch.cuda.synchronize()
        err = np.abs(key.astype(np.float32) - out.float().cpu().numpy())
        s = sc.float().cpu().numpy()
        assert (err <= s[:, None] + np.abs(key.astype(np.float32)) * 2e-3 + 1e-3).all()
        errs_b.append((err[:K] ** 2).mean()); errs_n.append((err[K:] ** 2).mean())
    assert np.mean(errs_b) < np.mean(errs_n)


def test_value_constant_and_shapes():
    """test_quantize.py: a constant token reconstructs exactly; output shapes."""
    G, D = 128, 128
    val = torch.full((G, D), 3.0, dtype=torch.float16, device=DEV)
    packed, sc, zp = KK.quantize_value_page_torch(val)
    torch.cuda.synchronize()
    assert packed.shape == (G, D // 4) and packed.dtype == torch.uint8 and sc.shape == (G,) and zp.shape == (G,)
    rec = KK.dequantize_value_page_torch(packed, sc, zp)
    assert (rec - rec[:, :1]).abs().max().item() < 1e-3
    v = torch.from_numpy(np.random.default_rng(2).standard_normal((G, D)).astype(np.float16)).to(DEV)
    packed, sc, zp = KK.quantize_value_page_torch(v)
    rec = KK.dequantize_value_page_torch(packed, sc, zp)
    assert ((v.float() - rec).abs() <= sc.float()[:, None] + 2e-3).all()
