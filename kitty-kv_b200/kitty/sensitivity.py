"""KittySensitivityProfiler - offline choice of the INT4 ("boosted") key channels.

API-compatible with the reference (``kitty/sensitivity.py:74-332``): forward
hooks on the key projections accumulate sum |K| per (layer, head, channel);
``compute`` ranks channels by mean |K| and gives the top K ranks 0..K-1 in the
boost index (all others get the sentinel); ``save``/``load`` use the same file
names.  Offline calibration is not on the decode path, so this stays plain
PyTorch.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.nn as nn

from .config import KittyConfig


class _ChannelAccumulator:
    def __init__(self, num_kv_heads: int, head_dim: int, device) -> None:
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.sum_abs = torch.zeros(num_kv_heads, head_dim, dtype=torch.float32, device=device)
        self.token_count = 0

    @torch.no_grad()
    def update(self, key: torch.Tensor) -> None:
        """key (batch, num_kv_heads, seq_len, head_dim)."""
        n = key.shape[0] * key.shape[2]
        flat = key.transpose(1, 2).reshape(-1, self.num_kv_heads, self.head_dim)
        self.sum_abs += flat.abs().float().sum(dim=0)
        self.token_count += n

    def scores(self) -> torch.Tensor:
        if self.token_count == 0:
            raise RuntimeError("No tokens have been accumulated yet.")
        return self.sum_abs / self.token_count


class KittySensitivityProfiler:
    def __init__(self, config: KittyConfig, model: Optional[nn.Module] = None) -> None:
        self.config = config
        self.model = model
        self._accumulators: Dict[int, _ChannelAccumulator] = {}
        self._hooks: List = []
        self.scores_: Optional[torch.Tensor] = None
        self.boost_masks_: Optional[torch.Tensor] = None
        self.boost_idx_uint8_: Optional[torch.Tensor] = None

    def register_hooks(self, layer_indices: Sequence[int],
                       key_proj_getter: Optional[Callable[[nn.Module, int], nn.Module]] = None) -> None:
        if self.model is None:
            raise RuntimeError("A model must be provided to KittySensitivityProfiler to register hooks. "
                               "Pass model= at construction time.")
        for layer_idx in layer_indices:
            acc = _ChannelAccumulator(self.config.num_kv_heads, self.config.head_dim, self.config.device)
            self._accumulators[layer_idx] = acc
            proj = self._find_key_proj(layer_idx, key_proj_getter)

            def hook(module, inp, out, acc=acc):
                B, T, _ = out.shape
                acc.update(out.detach().reshape(B, T, acc.num_kv_heads, acc.head_dim).permute(0, 2, 1, 3))

            self._hooks.append(proj.register_forward_hook(hook))

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()

    def compute(self) -> None:
        cfg = self.config
        L, H, D, K = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.d_boost
        if not self._accumulators:
            raise RuntimeError("No accumulators found.  Did you call register_hooks() and "
                               "forward the model over the calibration data?")
        scores = torch.zeros(L, H, D, dtype=torch.float32)
        for layer_idx, acc in self._accumulators.items():
            scores[layer_idx] = acc.scores().cpu()
        masks = torch.zeros(L, H, D, dtype=torch.bool)
        masks.scatter_(-1, scores.topk(K, dim=-1).indices, True)
        order = scores.argsort(dim=-1, descending=True, stable=True)
        bidx = torch.full((L, H, D), cfg.sentinel, dtype=torch.uint8)
        ranks = torch.arange(K, dtype=torch.uint8).expand(L, H, K)
        bidx.scatter_(-1, order[..., :K], ranks)
        self.scores_, self.boost_masks_, self.boost_idx_uint8_ = scores, masks, bidx

    def save(self, directory) -> None:
        if self.scores_ is None:
            self.compute()
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        torch.save(self.scores_, d / "scores.pt")
        torch.save(self.boost_masks_, d / "boost_masks.pt")
        torch.save(self.boost_idx_uint8_, d / "boost_idx.pt")
        meta = {"num_layers": self.config.num_layers, "num_kv_heads": self.config.num_kv_heads,
                "head_dim": self.config.head_dim, "d_boost": self.config.d_boost,
                "boost_rate": self.config.boost_rate,
                "token_count": {k: v.token_count for k, v in self._accumulators.items()}}
        (d / "meta.json").write_text(json.dumps(meta, indent=2))
        print(f"[KittySensitivityProfiler] Saved to {d}")

    @classmethod
    def load(cls, directory, config: KittyConfig) -> "KittySensitivityProfiler":
        d = Path(directory)
        p = cls(config)
        p.scores_ = torch.load(d / "scores.pt", weights_only=True)
        p.boost_masks_ = torch.load(d / "boost_masks.pt", weights_only=True)
        p.boost_idx_uint8_ = torch.load(d / "boost_idx.pt", weights_only=True)
        print(f"[KittySensitivityProfiler] Loaded from {d}")
        return p

    @property
    def boost_masks(self) -> torch.Tensor:
        if self.boost_masks_ is None:
            self.compute()
        return self.boost_masks_

    @property
    def boost_idx_uint8(self) -> torch.Tensor:
        if self.boost_idx_uint8_ is None:
            self.compute()
        return self.boost_idx_uint8_

    def _find_key_proj(self, layer_idx: int, getter) -> nn.Module:
        if getter is not None:
            return getter(self.model, layer_idx)
        for fn in (lambda m, i: m.layers[i].self_attn.k_proj,
                   lambda m, i: m.model.layers[i].self_attn.k_proj,
                   lambda m, i: m.transformer.h[i].attn.k_proj,
                   lambda m, i: m.transformer.h[i].attn.c_attn):
            try:
                mod = fn(self.model, layer_idx)
                if isinstance(mod, nn.Module):
                    return mod
            except (AttributeError, IndexError, TypeError):
                continue
        raise RuntimeError(f"Could not automatically find the Key Projection layer for layer {layer_idx}. "
                           "Please pass a key_proj_getter callable.")

    def summary(self) -> str:
        if self.scores_ is None:
            return "KittySensitivityProfiler — not yet computed."
        cfg = self.config
        return "\n".join([
            "KittySensitivityProfiler Summary",
            f"  Layers: {cfg.num_layers}, KV Heads: {cfg.num_kv_heads}, Head Dim: {cfg.head_dim}",
            f"  Boost rate: {cfg.boost_rate:.1%} → {cfg.d_boost} INT4 channels/head",
            f"  Sentinel value: {cfg.sentinel}",
            f"  Max channel score: {self.scores_.max().item():.4f}",
            f"  Mean channel score: {self.scores_.mean().item():.4f}",
        ])
