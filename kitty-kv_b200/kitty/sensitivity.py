"""Offline choice of the INT4 ("boosted") key channels.

Interface of the reference's ``KittySensitivityProfiler``
(``kitty/sensitivity.py:74-332``): the class name, its constructor, the
``register_hooks`` / ``remove_hooks`` / ``compute`` / ``save`` / ``load`` methods,
the ``boost_masks`` / ``boost_idx_uint8`` properties and ``scores_`` /
``boost_masks_`` / ``boost_idx_uint8_`` attributes, the saved file set
(``scores.pt``, ``boost_masks.pt``, ``boost_idx.pt``, ``meta.json`` with the
config snapshot and per-layer token counts) and the ranking rule of ``compute``
(``:164-207``): the channel with the r-th largest mean |K| of a (layer, KV head)
gets boost index r for r < d_boost, every other channel the sentinel.

Design of this implementation:

* statistics are kept per layer as one float64 running sum of |K| per (KV head,
  channel) on the projection's own device, fed by a forward hook that sees the
  projection output (B, T, H*D) and reduces over batch and time in one call;
* the key projection of a layer is found by walking the model: the first
  ``nn.ModuleList`` whose entries each hold a submodule named ``k_proj`` is taken
  as the layer stack, and entry i's ``k_proj`` is layer i's projection (a fused
  QKV projection has no ``k_proj`` and needs ``key_proj_getter``);
* ranking is one stable descending sort per (layer, head) and a scatter.

Offline calibration is not on the decode path, so this module is plain PyTorch.
"""

from __future__ import annotations

import json
import logging
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.nn as nn

from .config import KittyConfig

log = logging.getLogger(__name__)

_FILES = ("scores.pt", "boost_masks.pt", "boost_idx.pt")


class _ChannelAccumulator:
    """Running mean of |K| per (KV head, channel) of one layer.

    ``update`` takes keys laid out (batch, num_kv_heads, seq_len, head_dim); the
    hook below feeds it the projection output viewed that way.  Sums are float64
    so that long calibration runs do not lose the small channels' mass.
    """

    def __init__(self, num_kv_heads: int, head_dim: int, device) -> None:
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.sum_abs = torch.zeros(num_kv_heads, head_dim, dtype=torch.float64, device=device)
        self.token_count = 0

    @torch.no_grad()
    def update(self, key: torch.Tensor) -> None:
        if key.dim() != 4 or key.shape[1] != self.num_kv_heads or key.shape[3] != self.head_dim:
            raise ValueError(f"expected keys (batch, {self.num_kv_heads}, seq, {self.head_dim}), "
                             f"got {tuple(key.shape)}")
        self.sum_abs += key.detach().abs().sum(dim=(0, 2), dtype=torch.float64).to(self.sum_abs.device)
        self.token_count += key.shape[0] * key.shape[2]

    def scores(self) -> torch.Tensor:
        """(num_kv_heads, head_dim) float32 mean |K|."""
        if self.token_count == 0:
            raise RuntimeError("this layer's hook has not seen any tokens")
        return (self.sum_abs / self.token_count).float()


def _layer_stack(model: nn.Module) -> Optional[nn.ModuleList]:
    """The first ModuleList (in definition order) whose every entry holds a
    submodule named ``k_proj``."""
    for mod in model.modules():
        if isinstance(mod, nn.ModuleList) and len(mod) > 0 and all(
                any(name.rsplit(".", 1)[-1] == "k_proj" for name, _ in entry.named_modules()) for entry in mod):
            return mod
    return None


def _k_proj_of(entry: nn.Module) -> nn.Module:
    for name, sub in entry.named_modules():
        if name.rsplit(".", 1)[-1] == "k_proj":
            return sub
    raise LookupError("no k_proj submodule")


class KittySensitivityProfiler:
    """Collects mean |K| per (layer, KV head, channel) over calibration data and turns
    it into boost indices.

    Typical use: ``register_hooks(range(L))``, run the model over calibration
    batches, ``remove_hooks()``, then ``save(dir)`` or read ``boost_idx_uint8``.
    """

    def __init__(self, config: KittyConfig, model: Optional[nn.Module] = None) -> None:
        self.config = config
        self.model = model
        self._accumulators: Dict[int, _ChannelAccumulator] = {}
        self._hooks: List[torch.utils.hooks.RemovableHandle] = []
        self.scores_: Optional[torch.Tensor] = None            # (L, H, D) float32
        self.boost_masks_: Optional[torch.Tensor] = None       # (L, H, D) bool
        self.boost_idx_uint8_: Optional[torch.Tensor] = None   # (L, H, D) uint8

    # ------------------------------------------------------------------ hooks

    def register_hooks(self, layer_indices: Sequence[int],
                       key_proj_getter: Optional[Callable[[nn.Module, int], nn.Module]] = None) -> None:
        """Hook the key projection of every listed layer.  ``key_proj_getter(model, i)``
        overrides the search for models whose layers are not a ModuleList of blocks
        with a ``k_proj`` (fused QKV projections, custom containers)."""
        if self.model is None:
            raise RuntimeError("register_hooks needs the model: construct the profiler with model=...")
        stack = None if key_proj_getter is not None else _layer_stack(self.model)
        H, D = self.config.num_kv_heads, self.config.head_dim
        for i in layer_indices:
            if key_proj_getter is not None:
                proj = key_proj_getter(self.model, i)
            elif stack is None or not 0 <= i < len(stack):
                raise RuntimeError(f"layer {i}: no layer stack of blocks with a k_proj was found in the model "
                                   f"(or the index is out of range); pass key_proj_getter=(model, i) -> module")
            else:
                proj = _k_proj_of(stack[i])
            acc = self._accumulators.setdefault(i, _ChannelAccumulator(H, D, self.config.device))

            def hook(_mod, _inp, out, acc=acc):
                # (B, T, H*D) -> (B, H, T, D)
                B, T = out.shape[0], out.shape[1]
                acc.update(out.reshape(B, T, acc.num_kv_heads, acc.head_dim).transpose(1, 2))

            self._hooks.append(proj.register_forward_hook(hook))

    def remove_hooks(self) -> None:
        while self._hooks:
            self._hooks.pop().remove()

    # ---------------------------------------------------------------- ranking

    def compute(self) -> None:
        """Scores, boost masks and boost indices from the accumulated statistics.
        Layers without statistics keep score 0 (their ranks follow channel order)."""
        cfg = self.config
        if not self._accumulators:
            raise RuntimeError("nothing to compute: register_hooks() and run calibration data first")
        L, H, D, K = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.d_boost
        scores = torch.zeros(L, H, D, dtype=torch.float32)
        for i, acc in self._accumulators.items():
            scores[i] = acc.scores().cpu()
        ranked = torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :K]
        idx = torch.full((L, H, D), cfg.sentinel, dtype=torch.uint8)
        idx.scatter_(-1, ranked, torch.arange(K, dtype=torch.uint8).expand(L, H, K).contiguous())
        masks = torch.zeros(L, H, D, dtype=torch.bool)
        masks.scatter_(-1, ranked, True)
        self.scores_, self.boost_masks_, self.boost_idx_uint8_ = scores, masks, idx

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

    # -------------------------------------------------------------------- I/O

    def save(self, directory) -> None:
        if self.scores_ is None:
            self.compute()
        out = Path(directory)
        out.mkdir(parents=True, exist_ok=True)
        for name, t in zip(_FILES, (self.scores_, self.boost_masks_, self.boost_idx_uint8_)):
            torch.save(t, out / name)
        cfg = self.config
        meta = {"num_layers": cfg.num_layers, "num_kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
                "d_boost": cfg.d_boost, "boost_rate": cfg.boost_rate,
                "token_count": {i: a.token_count for i, a in self._accumulators.items()}}
        (out / "meta.json").write_text(json.dumps(meta, indent=2))
        log.info("sensitivity profile written to %s", out)

    @classmethod
    def load(cls, directory, config: KittyConfig) -> "KittySensitivityProfiler":
        src = Path(directory)
        prof = cls(config)
        prof.scores_, prof.boost_masks_, prof.boost_idx_uint8_ = (
            torch.load(src / name, weights_only=True) for name in _FILES)
        log.info("sensitivity profile read from %s", src)
        return prof

    def summary(self) -> str:
        if self.scores_ is None:
            return "sensitivity profile: not computed"
        cfg, s = self.config, self.scores_
        return (f"sensitivity profile: {cfg.num_layers} layers x {cfg.num_kv_heads} KV heads x {cfg.head_dim} "
                f"channels; {cfg.d_boost} INT4 channels per head (rate {cfg.boost_rate:g}, sentinel "
                f"{cfg.sentinel}); mean |K| max {s.max().item():.4f}, mean {s.mean().item():.4f}")
