"""CPU tests of the host-side mirror of the reference API: config, layout manager
(allocation policy, pools, accessors, block tables), the pipeline state machine
(with the two quantise launches replaced by a recorder, since the kernels need
a GPU) and the sensitivity profiler.  Behaviour follows the reference's own
tests (tests/test_layout.py, tests/test_attention.py, tests/test_quantize.py)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn

import kitty
from kitty import pipeline as pipeline_mod
from kitty.config import KittyConfig
from kitty.layout import PageCentricKVLayoutManager
from kitty.pipeline import KittyInferencePipeline
from kitty.sensitivity import KittySensitivityProfiler, _ChannelAccumulator
from oracle import kitty_oracle as O


def cfg(**kw):
    d = dict(num_layers=1, num_kv_heads=2, head_dim=16, q_buffer_size=8, sink_size=4, local_value_window=8,
             boost_rate=0.25, device="cpu")
    d.update(kw)
    return KittyConfig(**d)


def bidx_for(c):
    b = torch.full((c.num_layers, c.num_kv_heads, c.head_dim), c.sentinel, dtype=torch.uint8)
    b[:, :, :c.d_boost] = torch.arange(c.d_boost, dtype=torch.uint8)
    return b


# ----------------------------------------------------------------- config

def test_config_derived_values_and_io(tmp_path):
    c = KittyConfig(device="cpu")
    assert c.d_boost == 16 and c.sentinel == 17
    assert c.max_pages == ((32768 - 32) // 128 + 2) * 1 == 257
    p = KittyConfig.kitty_pro(device="cpu")
    assert p.d_boost == 32 and p.variant == "kitty-pro"
    c.save(tmp_path / "c.json")
    assert KittyConfig.load(tmp_path / "c.json") == c
    with pytest.raises(AssertionError):
        KittyConfig(boost_rate=1.0)
    with pytest.raises(AssertionError):
        KittyConfig(head_dim=18)
    with pytest.raises(AssertionError):
        KittyConfig(q_buffer_size=6)
    assert "d_boost=16" in repr(c)


def test_public_api_names():
    for n in ["KittyConfig", "KittySensitivityProfiler", "PageCentricKVLayoutManager", "KittyInferencePipeline",
              "KittyPagedAttention", "KittyAttentionFactory"]:
        assert hasattr(kitty, n)
    from kitty import kernels
    for n in ["quantize_key_page", "quantize_key_page_torch", "dequantize_key_page", "dequantize_key_page_torch",
              "quantize_value_page", "quantize_value_page_torch", "dequantize_value_page_torch", "paged_attention",
              "paged_attention_reference", "paged_attention_batched", "quantize_key_pages", "quantize_value_pages"]:
        assert callable(getattr(kernels, n))


def test_kernels_reject_cpu_tensors():
    from kitty import kernels
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.quantize_value_page_torch(torch.zeros(8, 16, dtype=torch.float16))


# ----------------------------------------------------------------- layout

def test_pool_shapes_and_dtypes():
    c = cfg()
    lay = PageCentricKVLayoutManager(c, bidx_for(c))
    P, H, D, G, K = c.max_pages, c.num_kv_heads, c.head_dim, c.q_buffer_size, c.d_boost
    assert lay.key_baseline.shape == (P, H, D, G // 4) and lay.key_baseline.dtype == torch.uint8
    assert lay.key_boost.shape == (P, H, K, G // 4)
    assert lay.key_metadata.shape == (P, H, 2, D) and lay.key_metadata.dtype == torch.float16
    assert lay.value_pool.shape == (P, H, G, D // 4)
    assert lay.value_metadata.shape == (P, H, G, 2)
    assert lay.key_baseline_page(0).shape == (H, D, G // 4)
    assert lay.key_boost_page(0).shape == (H, K, G // 4)
    assert lay.key_meta_page(0).shape == (H, 2, D)
    assert lay.value_page(0).shape == (H, G, D // 4)
    assert lay.value_meta_page(0).shape == (H, G, 2)


def test_allocation_policy_matches_reference():
    c = cfg()
    lay = PageCentricKVLayoutManager(c, bidx_for(c))
    pages = [lay.allocate_page(0, 0, i) for i in range(5)]
    assert [p.physical_idx for p in pages] == [0, 1, 2, 3, 4]
    lay.free_page(0, 0, 1)
    lay.free_page(0, 0, 3)
    assert lay.allocate_page(1, 0, 0).physical_idx == 1          # lowest free first
    assert lay.allocate_page(1, 0, 1).physical_idx == 3
    assert lay.allocate_page(1, 0, 2).physical_idx == 5
    assert lay.get_page_list(1, 0) == [1, 3, 5]
    assert lay.get_page_list(0, 0) == [0]                        # stops at the gap (page 1 freed)
    assert lay.get_physical_idx(0, 0, 2) == 2
    with pytest.raises(KeyError):
        lay.get_physical_idx(9, 0, 0)
    lay.free_sequence(1)
    assert lay.memory_stats()["pages_used"] == 3
    lay.free_page(5, 5, 5)                                        # unknown page: no-op


def test_pool_exhaustion_raises():
    c = cfg()
    lay = PageCentricKVLayoutManager(c, bidx_for(c))
    for i in range(c.max_pages):
        lay.allocate_page(0, 0, i)
    with pytest.raises(RuntimeError, match="exhausted"):
        lay.allocate_page(0, 0, c.max_pages)


def test_block_table():
    c = cfg()
    lay = PageCentricKVLayoutManager(c, bidx_for(c))
    for i in range(3):
        lay.allocate_page(0, 0, i)
    for i in range(2):
        lay.allocate_page(4, 0, i)
    bt, n = lay.block_table([4, 0, 9], 0, width=4)
    assert bt.tolist() == [[3, 4, 0, 0], [0, 1, 2, 0], [0, 0, 0, 0]]
    assert n.tolist() == [2, 3, 0]
    with pytest.raises(RuntimeError):
        lay.block_table([0], 0, width=2)


# ----------------------------------------------------------------- pipeline

class Recorder:
    """Stands in for the two quantise launches: records what the flush passes."""

    def __init__(self):
        self.key_calls, self.value_calls = [], []

    def key(self, src, offs, strides, bidx, K, sent, dst, kl, kh, km, H, D, G):
        self.key_calls.append(dict(src=src.clone(), strides=strides, dst=dst.clone(), K=K, sent=sent,
                                   bidx=bidx.clone()))

    def value(self, src, offs, strides, dst, vc, vm, H, D, G, n_valid=None):
        self.value_calls.append(dict(src=src.clone(), dst=dst.clone(),
                                     n_valid=None if n_valid is None else int(n_valid[0])))


@pytest.fixture
def recorder(monkeypatch):
    r = Recorder()
    monkeypatch.setattr(pipeline_mod, "quantize_key_pages", r.key)
    monkeypatch.setattr(pipeline_mod, "quantize_value_pages", r.value)
    return r


def make_pipe(c, align=True):
    lay = PageCentricKVLayoutManager(c, bidx_for(c))
    return KittyInferencePipeline(c, lay, bidx_for(c), align_values=align), lay


def tok(i, H=2, D=16):
    return torch.full((H, D), float(i), dtype=torch.float16)


def test_sink_then_qbuf(recorder):
    c = cfg()
    p, lay = make_pipe(c)
    for t in range(c.sink_size):
        p.push_token(0, tok(t), tok(-t))
    assert p.sink_fill == 4 and p.key_qbuf_len == 0
    for t in range(3):
        p.push_token(0, tok(10 + t), tok(20 + t))
    assert p.key_qbuf_len == 3 and p.val_local_len == 3
    assert not recorder.key_calls


@pytest.mark.parametrize("align", [True, False])
def test_flush_at_G_and_sources(recorder, align):
    c = cfg()
    p, lay = make_pipe(c, align)
    n = c.sink_size + 3 * c.q_buffer_size + 2
    for t in range(n):
        p.push_token(0, tok(t), tok(1000 + t))
    assert len(recorder.key_calls) == 3 and len(recorder.value_calls) == 3
    assert lay.get_page_list(0, 0) == [0, 1, 2]
    assert p.key_qbuf_len == 2
    G, S, R = c.q_buffer_size, c.sink_size, c.local_value_window
    for i, call in enumerate(recorder.key_calls):
        assert int(call["dst"][0]) == i
        toks = call["src"][0, :, 0].float().tolist()                # (H, G, D) buffer, head 0, channel 0
        assert toks == [float(S + i * G + j) for j in range(G)]
    for i, call in enumerate(recorder.value_calls):
        vals = call["src"][0, :, 0].float().tolist()
        if align:
            assert call["n_valid"] is None
            assert vals == [float(1000 + S + i * G + j) for j in range(G)]   # same tokens as key page i
        else:
            # reference order: evicted values; page 0 is all padding when R == G
            nv = call["n_valid"]
            assert nv == (0 if i == 0 else G)
            if i > 0:
                assert vals == [float(1000 + S + (i - 1) * G + j) for j in range(G)]
    ctx = p.get_attention_context(0)
    assert ctx["key_qbuf"].shape == (2, 2, 16)
    assert ctx["page_list"] == [0, 1, 2]
    if align:
        assert ctx["value_tail"][0, :, 0].float().tolist() == [1000.0 + n - 2, 1000.0 + n - 1]
    assert ctx["val_local"].shape[1] == R


def test_reset_and_per_layer_counters(recorder):
    c = cfg(num_layers=2)
    p, lay = make_pipe(c)
    for t in range(c.sink_size + c.q_buffer_size):
        for l in range(2):
            p.push_token(l, tok(t + 100 * l), tok(t))
    assert len(recorder.key_calls) == 2                              # one flush per layer
    assert lay.get_page_list(0, 0) == [0] and lay.get_page_list(0, 1) == [1]
    # layer 1 wrote its own tokens at the same positions as layer 0
    assert p.sink_k[1, 0, :, 0].tolist() == [100.0 + t for t in range(c.sink_size)]
    assert recorder.key_calls[1]["src"][0, :, 0].tolist() == [100.0 + c.sink_size + j for j in range(8)]
    assert p.layer_state(1) == p.layer_state(0)
    p.reset_sequence(0)
    assert p.sink_fill == 0 and p.key_qbuf_len == 0 and lay.memory_stats()["pages_used"] == 0
    assert p.stats()["pages_used"] == 0


# ----------------------------------------------------------------- profiler

def test_profiler_compute_matches_oracle_rule():
    c = KittyConfig(num_layers=2, num_kv_heads=4, head_dim=32, boost_rate=0.25, device="cpu")
    prof = KittySensitivityProfiler(c)
    rng = np.random.default_rng(0)
    keys = []
    for l in range(2):
        k = (rng.standard_normal((1, 4, 50, 32)) * rng.uniform(0.1, 5, (1, 4, 1, 32))).astype(np.float32)
        acc = _ChannelAccumulator(4, 32, "cpu")
        acc.update(torch.from_numpy(k))
        prof._accumulators[l] = acc
        keys.append(k[0])
    prof.compute()
    exp = np.stack([O.boost_idx_from_scores(np.abs(k).mean(axis=1), c.d_boost, c.sentinel) for k in keys])
    np.testing.assert_array_equal(prof.boost_idx_uint8.numpy(), exp)
    assert prof.boost_masks.sum().item() == 2 * 4 * c.d_boost


class PageRecorder:
    """Stands in for the quantise launches and materialises each job's (H, G, D) block
    from (source, offsets, strides), so flushes from a buffer and pages quantised
    straight from a prefill source can be compared."""

    def __init__(self):
        self.keys, self.values = {}, {}

    @staticmethod
    def _blocks(src, offs, strides, dst, H, D, G):
        flat = src.reshape(-1) if src.is_contiguous() else src.contiguous().reshape(-1)
        if not src.is_contiguous():
            raise AssertionError("sources are passed contiguous")
        sh, st, sc = strides
        h = torch.arange(H).view(H, 1, 1) * sh
        t = torch.arange(G).view(1, G, 1) * st
        c = torch.arange(D).view(1, 1, D) * sc
        return {int(p): flat[int(o) + h + t + c].clone() for o, p in zip(offs.tolist(), dst.tolist())}

    def key(self, src, offs, strides, bidx, K, sent, dst, kl, kh, km, H, D, G):
        self.keys.update(self._blocks(src, offs, strides, dst, H, D, G))

    def value(self, src, offs, strides, dst, vc, vm, H, D, G, n_valid=None):
        assert n_valid is None
        self.values.update(self._blocks(src, offs, strides, dst, H, D, G))


@pytest.mark.parametrize("R", [8, 3, 0])
@pytest.mark.parametrize("chunks", [[1, 2, 30, 5], [4, 8, 8, 1], [17, 3, 0, 25], [2, 40]])
def test_bulk_push_equals_token_by_token(monkeypatch, R, chunks):
    """push_tokens (aligned values) leaves the same buffers, counters, value window,
    value Q-buffer, page list and page contents as pushing the same tokens one by one."""
    c = cfg(local_value_window=R)
    H, D = c.num_kv_heads, c.head_dim
    total = sum(chunks)
    g = torch.Generator().manual_seed(R * 100 + total)
    keys = torch.randn(H, total, D, generator=g).to(torch.float16)
    vals = torch.randn(H, total, D, generator=g).to(torch.float16)
    results = []
    for bulk in (False, True):
        rec = PageRecorder()
        monkeypatch.setattr(pipeline_mod, "quantize_key_pages", rec.key)
        monkeypatch.setattr(pipeline_mod, "quantize_value_pages", rec.value)
        p, lay = make_pipe(c, True)
        t = 0
        for n in chunks:
            if bulk:
                p.push_tokens(0, keys[:, t:t + n], vals[:, t:t + n])
            else:
                for j in range(t, t + n):
                    p.push_token(0, keys[:, j], vals[:, j])
            t += n
        results.append((p, lay, rec))
    (a, la, ra), (b, lb, rb) = results
    assert a.layer_state(0) == b.layer_state(0)
    for name in ("sink_k", "sink_v", "key_qbuf", "val_tail", "val_local", "val_qbuf"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    assert la.get_page_list(0, 0) == lb.get_page_list(0, 0)
    assert ra.keys.keys() == rb.keys.keys() == set(la.get_page_list(0, 0))
    for pg in ra.keys:
        assert torch.equal(ra.keys[pg], rb.keys[pg]) and torch.equal(ra.values[pg], rb.values[pg])


def test_bulk_push_reference_mode_goes_token_by_token(recorder):
    c = cfg()
    p, lay = make_pipe(c, align=False)
    H, D = c.num_kv_heads, c.head_dim
    n = c.sink_size + 2 * c.q_buffer_size + 3
    p.push_tokens(0, torch.arange(n, dtype=torch.float16).view(1, n, 1).expand(H, n, D),
                  (1000 + torch.arange(n, dtype=torch.float16)).view(1, n, 1).expand(H, n, D))
    assert len(recorder.key_calls) == 2 and [cl["n_valid"] for cl in recorder.value_calls] == [0, c.q_buffer_size]


class _Attn(nn.Module):
    def __init__(self, dm, H, D):
        super().__init__()
        self.q_proj = nn.Linear(dm, 2 * H * D, bias=False)
        self.k_proj = nn.Linear(dm, H * D, bias=False)


class _Block(nn.Module):
    def __init__(self, dm, H, D):
        super().__init__()
        self.self_attn = _Attn(dm, H, D)
        self.mlp = nn.Linear(dm, dm)

    def forward(self, x):
        self.self_attn.k_proj(x)
        return x + self.mlp(x)


class _ToyModel(nn.Module):
    def __init__(self, L, dm, H, D):
        super().__init__()
        self.embed = nn.ModuleList([nn.Linear(dm, dm)])       # a ModuleList without k_proj comes first
        self.layers = nn.ModuleList([_Block(dm, H, D) for _ in range(L)])

    def forward(self, x):
        for blk in self.layers:
            x = blk(x)
        return x


def test_profiler_hooks_find_the_key_projections_and_rank_them():
    """register_hooks locates layer i's k_proj by walking the model, the hooks see every
    calibration token, and compute() applies the rank rule to mean |K| of the projection
    outputs (checked against the oracle's rule on the same outputs); save / load round
    trip the four files."""
    import tempfile
    torch.manual_seed(0)
    L, dm, H, D = 3, 24, 2, 16
    c = KittyConfig(num_layers=L, num_kv_heads=H, head_dim=D, boost_rate=0.25, device="cpu")
    model = _ToyModel(L, dm, H, D)
    xs = [torch.randn(2, 7, dm), torch.randn(1, 5, dm)]
    outs = {0: [], 2: []}
    with torch.no_grad():
        for x in xs:                              # the inputs each layer's k_proj sees in forward
            for i, blk in enumerate(model.layers):
                if i in outs:
                    outs[i].append(blk.self_attn.k_proj(x).reshape(-1, H, D))
                x = x + blk.mlp(x)
    prof = KittySensitivityProfiler(c, model)
    prof.register_hooks([0, 2])
    with torch.no_grad():
        for x in xs:
            model(x)
    prof.remove_hooks()
    with torch.no_grad():
        model(xs[0])                              # hooks removed: no more tokens counted
    assert prof._accumulators[0].token_count == 2 * 7 + 5
    prof.compute()
    for i in (0, 2):
        k = torch.cat(outs[i]).abs().double().mean(dim=0).float().numpy()
        np.testing.assert_array_equal(prof.boost_idx_uint8[i].numpy(), O.boost_idx_from_scores(k, c.d_boost,
                                                                                              c.sentinel))
    assert (prof.boost_idx_uint8[1] == torch.tensor([0, 1, 2, 3] + [c.sentinel] * (D - 4),
                                                    dtype=torch.uint8)).all()   # no data: channel order
    assert prof.boost_masks.sum().item() == L * H * c.d_boost
    with tempfile.TemporaryDirectory() as d:
        prof.save(d)
        back = KittySensitivityProfiler.load(d, c)
        assert torch.equal(back.boost_idx_uint8, prof.boost_idx_uint8) and torch.equal(back.scores_, prof.scores_)
        assert json.loads((Path(d) / "meta.json").read_text())["token_count"] == {"0": 19, "2": 19}
    with pytest.raises(RuntimeError, match="key_proj_getter"):
        KittySensitivityProfiler(c, nn.Sequential(nn.Linear(4, 4))).register_hooks([0])
    custom = KittySensitivityProfiler(c, model)
    custom.register_hooks([1], key_proj_getter=lambda m, i: m.layers[i].self_attn.k_proj)
    model(xs[1])
    assert custom._accumulators[1].token_count == 5
