"""CDC-03 decode attention inside Hugging Face models.

The reference has no model hook for CDC-03: its harness calls
``hybrid_pq_attention`` (compressed_attention.py:315-412) per head on NumPy
arrays, while the model attends the dense cache.  Here:

* ``CDC03Cache`` is a ``CompressedKVCache`` (same lifecycle, same
  ``layer_states``) that also mirrors every compressed layer into a
  ``cdc03.CDC03Store``: it calibrates the layer's PQ codebooks on its first
  ``calibration_tokens`` tokens and gives PQ codes to the tokens that leave the
  hot window, on the device, as they arrive;
* ``cdc03_attention_forward`` is registered with transformers as the attention
  implementation ``"cdc03"``: a decode step (one query token) of a compressed,
  calibrated layer runs the CDC-03 kernels on the store (top-k of the cold
  range with sinks, plus the exact hot window); prefill, exact layers and
  layers still calibrating use SDPA on the exact K/V.

Usage::

    cache = CDC03Cache(OnlineKVConfig(pq_subspaces=8), n_layers, batch=1,
                       kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                       capacity=4096, dtype=torch.float16)
    cache.attach(model)          # sets model.config._attn_implementation = "cdc03"
    model.generate(ids, past_key_values=cache, max_new_tokens=256)

Decode steps assume unpadded batches (every sequence has the same length).
"""

from __future__ import annotations

from typing import Optional

import torch
from transformers import AttentionInterface
from transformers.integrations.sdpa_attention import sdpa_attention_forward

from .cdc03 import CDC03Store
from .compressed_cache import CompressedKVCache
from .config import OnlineKVConfig


class CDC03Cache(CompressedKVCache):
    """CompressedKVCache with device-resident CDC-03 tiers for compressed layers."""

    def __init__(self, config: OnlineKVConfig, n_layers: int, batch: int, kv_heads: int, head_dim: int,
                 capacity: int, dtype=torch.float16, n_subspaces: Optional[int] = None,
                 top_k: Optional[int] = None, sink_tokens: Optional[int] = None):
        super().__init__(config, n_layers)
        M = n_subspaces or config.pq_subspaces
        if M <= 0:
            raise ValueError("CDC-03 needs pq_subspaces > 0")
        self.store = CDC03Store(batch, n_layers, kv_heads, head_dim, capacity, n_subspaces=M, dtype=dtype)
        self.top_k = config.top_k if top_k is None else top_k
        self.sink_tokens = config.sink_tokens if sink_tokens is None else sink_tokens
        self.hot_window = config.hot_window
        self._len = [0] * n_layers         # tokens of the layer in the store
        self._coded = [0] * n_layers       # leading tokens of the layer with PQ codes
        self._calibrated = [False] * n_layers

    def ready(self, layer_idx) -> bool:
        """True when decode steps of this layer run CDC-03."""
        return (layer_idx is not None and 0 <= layer_idx < len(self._len)
                and not self.layer_states[layer_idx].is_exact and self._calibrated[layer_idx])

    def update(self, key_states, value_states, layer_idx: int, cache_kwargs: Optional[dict] = None):
        k_out, v_out = super().update(key_states, value_states, layer_idx, cache_kwargs)
        if self.layer_states[layer_idx].is_exact:
            return k_out, v_out
        st = self.store
        T = key_states.shape[2]
        s0 = self._len[layer_idx]
        if key_states.shape[0] != st.B or key_states.shape[1] != st.H or key_states.shape[3] != st.D:
            raise ValueError(f"Expected shape [{st.B}, {st.H}, *, {st.D}], got {tuple(key_states.shape)}")
        if s0 + T > st.cap:
            raise ValueError(f"CDC-03 store capacity {st.cap} exceeded ({s0 + T} tokens)")
        st.k[layer_idx, :, :, s0:s0 + T] = key_states.detach()
        st.v[layer_idx, :, :, s0:s0 + T] = value_states.detach()
        n = self._len[layer_idx] = s0 + T
        n_cal = self.config.calibration_tokens
        if not self._calibrated[layer_idx] and n >= n_cal:
            st.calibrate(layer_idx, n_cal, max_iters=self.config.pq_max_iters, rtol=self.config.pq_rtol)
            self._calibrated[layer_idx] = True
        if self._calibrated[layer_idx]:
            cold = max(0, n - self.hot_window)   # AgingPolicy.tier_boundary (aging_policy.py:54-56)
            if cold > self._coded[layer_idx]:
                st.assign(layer_idx, self._coded[layer_idx], cold)
                self._coded[layer_idx] = cold
        return k_out, v_out

    def attach(self, model) -> "CDC03Cache":
        """Route the model's attention through ``"cdc03"`` with this cache."""
        n = 0
        for mod in model.modules():
            if hasattr(mod, "layer_idx") and hasattr(mod, "q_proj"):
                mod._cdc03_cache = self
                n += 1
        if n == 0:
            raise ValueError("no attention modules with a layer_idx found")
        model.config._attn_implementation = "cdc03"
        for mod in model.modules():
            cfg = getattr(mod, "config", None)
            if cfg is not None and hasattr(cfg, "_attn_implementation"):
                cfg._attn_implementation = "cdc03"
        return self


def cdc03_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                            scaling: Optional[float] = None, is_causal: Optional[bool] = None, **kwargs):
    """Attention interface ``"cdc03"``: query [B, H_q, q_len, D] -> ([B, q_len, H_q, D], None)."""
    cache = getattr(module, "_cdc03_cache", None)
    layer = getattr(module, "layer_idx", None)
    if cache is not None and query.shape[2] == 1 and cache.ready(layer):
        st = cache.store
        st.seq_len.fill_(cache._len[layer])
        scale = scaling if scaling is not None else query.shape[-1] ** -0.5
        out = st.decode(layer, query[:, :, 0, :].contiguous(), scale, cache.top_k, cache.sink_tokens,
                        cache.hot_window, out_dtype=query.dtype)
        return out.unsqueeze(1), None
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


AttentionInterface.register("cdc03", cdc03_attention_forward)
