"""KittyPagedAttention - drop-in attention module over the Kitty cache.

Same constructor, ``forward`` contract and factory as the reference
(``kitty/attention.py:28-257``).  Decode (T == 1) pushes the token into the
pipeline and runs the fused CUDA decode kernel over sinks + quantised pages +
fp16 tail; prefill (T > 1) appends the tokens to the pipeline in one bulk call
and returns causal SDPA over the raw fp16 K/V, as the reference does.
"""

from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import KittyConfig
from .kernels.attention import paged_attention
from .layout import PageCentricKVLayoutManager
from .pipeline import KittyInferencePipeline


class KittyPagedAttention(nn.Module):
    def __init__(self, config: KittyConfig, num_q_heads: int, layout: PageCentricKVLayoutManager,
                 pipeline: KittyInferencePipeline, layer_id: int) -> None:
        super().__init__()
        self.config = config
        self.num_q_heads = num_q_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self.q_per_kv = num_q_heads // config.num_kv_heads
        self.layer_id = layer_id
        self.layout = layout
        self.pipeline = pipeline
        self.scale = 1.0 / math.sqrt(config.head_dim)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_id: int = 0,
                attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q (B, Hq, T, D), k/v (B, H, T, D) -> (B, Hq, T, D); B must be 1 (the
        pipeline holds one sequence; use ``kitty.kernels.paged_attention_batched``
        for batched decode over many sequences)."""
        B, nqh, T, D = q.shape
        assert B == 1, "KittyPagedAttention currently supports batch_size=1"
        assert nqh == self.num_q_heads
        assert D == self.head_dim
        if T == 1:
            return self._decode_step(q, k, v, seq_id)
        return self._prefill(q, k, v, seq_id)

    def _decode_step(self, q, k, v, seq_id: int) -> torch.Tensor:
        self.pipeline.push_token(layer_id=self.layer_id, key=k[0, :, 0, :], value=v[0, :, 0, :], seq_id=seq_id)
        ctx = self.pipeline.get_attention_context(self.layer_id, seq_id)
        tail_v = ctx["value_tail"] if "value_tail" in ctx else ctx["val_local"]
        out = paged_attention(
            q=q[0, :, 0, :], page_list=ctx["page_list"],
            key_baseline=self.layout.key_baseline, key_boost=self.layout.key_boost,
            key_meta=self.layout.key_metadata, value_pool=self.layout.value_pool,
            value_meta=self.layout.value_metadata,
            boost_idx=self.pipeline._boost_idx_dev()[self.layer_id], D_boost=self.config.d_boost,
            sink_k=ctx["sink_k"], sink_v=ctx["sink_v"], qbuf_k=ctx["key_qbuf"], qbuf_v=tail_v,
            num_q_heads=self.num_q_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim)
        return out.unsqueeze(0).unsqueeze(2)

    def _prefill(self, q, k, v, seq_id: int) -> torch.Tensor:
        # all T tokens in one call (full pages quantised straight from k / v)
        self.pipeline.push_tokens(layer_id=self.layer_id, keys=k[0], values=v[0], seq_id=seq_id)
        k_exp = k.repeat_interleave(self.q_per_kv, dim=1)
        v_exp = v.repeat_interleave(self.q_per_kv, dim=1)
        return F.scaled_dot_product_attention(q, k_exp, v_exp, attn_mask=None, dropout_p=0.0,
                                              is_causal=True, scale=self.scale)


class KittyAttentionFactory:
    """Builds the layout manager, the pipeline and one module per layer."""

    @classmethod
    def from_config(cls, config: KittyConfig, boost_idx_uint8: torch.Tensor, num_q_heads: int,
                    align_values: bool = True
                    ) -> Tuple[PageCentricKVLayoutManager, KittyInferencePipeline, List[KittyPagedAttention]]:
        layout = PageCentricKVLayoutManager(config, boost_idx_uint8)
        pipeline = KittyInferencePipeline(config, layout, boost_idx_uint8, align_values=align_values)
        layers = [KittyPagedAttention(config=config, num_q_heads=num_q_heads, layout=layout,
                                      pipeline=pipeline, layer_id=i) for i in range(config.num_layers)]
        return layout, pipeline, layers
