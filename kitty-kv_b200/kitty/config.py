"""KittyConfig - the configuration dataclass of the Kitty KV cache.

Same fields, defaults, derived properties, JSON save/load and validation as
the reference (``kitty/config.py:18-152`` in bitxwolf/kitty-kv), so configs
and saved JSON files move between the two unchanged.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Literal


@dataclass
class KittyConfig:
    """Kitty KV-cache configuration.

    num_layers / num_kv_heads / head_dim: model shape (KV heads after GQA).
    sink_size (S): leading tokens kept in fp16 forever.
    q_buffer_size (G): fp16 Key Q-buffer length; a full buffer becomes one page.
    local_value_window (R): most recent values kept in fp16.
    boost_rate: fraction of key channels stored at INT4 (0.125 Kitty, 0.25 Kitty-Pro).
    max_seq_len / max_batch_size: sizing of the page pool.
    dtype: buffer / metadata type, "float16" or "bfloat16" (the B200 kernels take
    both; decode outputs are float16 either way, as in the reference).
    device: CUDA device of the pools and buffers.
    """

    num_layers: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    sink_size: int = 32
    q_buffer_size: int = 128
    local_value_window: int = 128
    boost_rate: float = 0.125
    max_seq_len: int = 32768
    max_batch_size: int = 1
    dtype: Literal["float16", "bfloat16"] = "float16"
    device: str = "cuda:0"
    profile_save_dir: str = "kitty_profiles"
    variant: Literal["kitty", "kitty-pro"] = "kitty"

    @property
    def d_boost(self) -> int:
        """K = round(boost_rate * head_dim) INT4 channels per head."""
        return round(self.boost_rate * self.head_dim)

    @property
    def max_pages(self) -> int:
        """Pool size in pages: ((max_seq_len - S) // G + 2) * max_batch_size.

        Same formula as the reference (``config.py:91-103``); note that it has
        no layer factor while every flush takes one page per layer.
        """
        return ((self.max_seq_len - self.sink_size) // self.q_buffer_size + 2) * self.max_batch_size

    @property
    def sentinel(self) -> int:
        """Boost-index value marking a non-boosted channel: min(K + 1, 255)."""
        return min(self.d_boost + 1, 255)

    def save(self, path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(asdict(self), indent=2))

    @classmethod
    def load(cls, path) -> "KittyConfig":
        return cls(**json.loads(Path(path).read_text()))

    @classmethod
    def kitty_pro(cls, **kwargs) -> "KittyConfig":
        """Kitty-Pro: 25% boosted channels."""
        return cls(boost_rate=0.25, variant="kitty-pro", **kwargs)

    def __post_init__(self) -> None:
        assert 0 < self.boost_rate < 1, "boost_rate must be in (0, 1)"
        assert self.head_dim % 4 == 0, "head_dim must be divisible by 4 (packing)"
        assert self.q_buffer_size % 4 == 0, "q_buffer_size (G) must be divisible by 4 (uint8 packing)"
        assert self.sink_size >= 0
        assert self.local_value_window >= 0
        assert self.dtype in ("float16", "bfloat16")

    def __repr__(self) -> str:
        return (f"KittyConfig(variant={self.variant!r}, num_layers={self.num_layers}, "
                f"num_kv_heads={self.num_kv_heads}, head_dim={self.head_dim}, "
                f"boost_rate={self.boost_rate} -> d_boost={self.d_boost}, "
                f"G={self.q_buffer_size}, S={self.sink_size}, R={self.local_value_window})")
