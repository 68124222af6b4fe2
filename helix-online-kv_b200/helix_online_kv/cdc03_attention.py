"""CDC-03 decode attention inside Hugging Face models.

The reference has no model hook for CDC-03: its harness calls
``hybrid_pq_attention`` (compressed_attention.py:315-412) per head on NumPy
arrays, while the model attends the dense cache.  Here:

* ``CDC03Cache`` is a ``CompressedKVCache`` (same constructor arguments first,
  same ``layer_states`` and lifecycle properties) whose compressed layers live
  in a ``cdc03.CDC03Store`` only: their cache layer holds views into the
  store's exact tiers (the single copy of their K/V, no parent
  ``DynamicCache`` copy), the layer's PQ codebooks are calibrated on its first
  ``calibration_tokens`` tokens and the tokens that leave the hot window get
  their PQ codes, on the device, as they arrive.  Exact layers stay in the
  parent ``DynamicCache``;
* ``cdc03_attention_forward`` is registered with transformers as the attention
  implementation ``"cdc03"``: a decode step (one query token) of a compressed,
  calibrated layer runs the CDC-03 kernels on the store (top-k of the cold
  range with sinks, plus the exact hot window); prefill (several query tokens,
  no padding mask) of every layer runs ``prefill.prefill_attention`` on the
  exact K/V (for compressed layers, the store's views); single-token steps of
  exact layers and of layers still calibrating, and head dims or dtypes that
  kernel does not take, use SDPA.

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
from transformers.cache_utils import DynamicLayer
from transformers.integrations.sdpa_attention import sdpa_attention_forward

from .cdc03 import CDC03Store
from .compressed_cache import CompressedKVCache
from .config import OnlineKVConfig
from .layer_state import LayerPhase
from .prefill import prefill_attention, supported


class _StoreLayer(DynamicLayer):
    """A compressed layer's K/V: views [B, H_kv, n, D] into the CDC-03 store."""

    def __init__(self, cache: "CDC03Cache", layer_idx: int):
        super().__init__()
        self._cache, self._layer = cache, layer_idx

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.keys, self.values = self._cache._store_append(self._layer, key_states, value_states)
        return self.keys, self.values

    def crop(self, max_length: int) -> None:
        n = self._cache._len[self._layer]
        if max_length < 0:
            max_length = n - abs(max_length)
        if n <= max_length:
            return
        self._cache._truncate(self._layer, max_length)
        self.keys, self.values = self._cache._views(self._layer)

    def batch_repeat_interleave(self, repeats: int) -> None:
        raise ValueError("CDC03Cache keeps each sequence's tiers in place; it cannot repeat the batch (beam search)")

    def batch_select_indices(self, indices) -> None:
        raise ValueError("CDC03Cache keeps each sequence's tiers in place; it cannot select batch rows (beam search)")


class CDC03Cache(CompressedKVCache):
    """CompressedKVCache whose compressed layers live in device-resident CDC-03 tiers."""

    def __init__(self, config: OnlineKVConfig, n_layers: int, batch: int, kv_heads: int, head_dim: int,
                 capacity: int, dtype=torch.float16, n_subspaces: Optional[int] = None,
                 top_k: Optional[int] = None, sink_tokens: Optional[int] = None):
        super().__init__(config, n_layers)
        M = n_subspaces or config.pq_subspaces
        if M <= 0:
            raise ValueError("CDC-03 needs pq_subspaces > 0")
        # store slots for the compressed layers only
        self._slot = {}
        for i in range(n_layers):
            if not self.layer_states[i].is_exact:
                self._slot[i] = len(self._slot)
        self.store = CDC03Store(batch, max(1, len(self._slot)), kv_heads, head_dim, capacity, n_subspaces=M,
                                dtype=dtype)
        self.top_k = config.top_k if top_k is None else top_k
        self.sink_tokens = config.sink_tokens if sink_tokens is None else sink_tokens
        self.hot_window = config.hot_window
        self._len = [0] * n_layers         # tokens of the layer in the store
        self._coded = [0] * n_layers       # leading tokens of the layer with PQ codes
        self._calibrated = [False] * n_layers
        self.layers = [_StoreLayer(self, i) if i in self._slot else DynamicLayer() for i in range(n_layers)]
        self.layer_class_to_replicate = None

    def slot(self, layer_idx: int) -> int:
        """The store layer that holds a compressed model layer."""
        return self._slot[layer_idx]

    def ready(self, layer_idx) -> bool:
        """True when decode steps of this layer run CDC-03."""
        return layer_idx is not None and layer_idx in self._slot and self._calibrated[layer_idx]

    @property
    def calibration_complete(self) -> bool:
        return all(self._calibrated[i] for i in self._slot)

    def update(self, key_states, value_states, layer_idx: int, cache_kwargs: Optional[dict] = None):
        if layer_idx not in self._slot:
            return super().update(key_states, value_states, layer_idx, cache_kwargs)
        if layer_idx == 0:
            self._total_tokens += key_states.shape[2]
        return self.layers[layer_idx].update(key_states, value_states)

    def _views(self, layer_idx: int):
        st, sl, n = self.store, self._slot[layer_idx], self._len[layer_idx]
        return st.k[sl, :, :, :n], st.v[sl, :, :, :n]

    def _truncate(self, layer_idx: int, n: int):
        self._len[layer_idx] = n
        self._coded[layer_idx] = min(self._coded[layer_idx], max(0, n - self.hot_window))

    def _store_append(self, layer_idx: int, key_states, value_states):
        st, sl = self.store, self._slot[layer_idx]
        T = key_states.shape[2]
        s0 = self._len[layer_idx]
        if key_states.shape[0] != st.B or key_states.shape[1] != st.H or key_states.shape[3] != st.D:
            raise ValueError(f"Expected shape [{st.B}, {st.H}, *, {st.D}], got {tuple(key_states.shape)}")
        if s0 + T > st.cap:
            raise ValueError(f"CDC-03 store capacity {st.cap} exceeded ({s0 + T} tokens)")
        st.k[sl, :, :, s0:s0 + T] = key_states.detach()
        st.v[sl, :, :, s0:s0 + T] = value_states.detach()
        n = self._len[layer_idx] = s0 + T
        ls = self.layer_states[layer_idx]
        ls._tokens_seen = n
        n_cal = self.config.calibration_tokens
        if not self._calibrated[layer_idx] and n >= n_cal:
            st.calibrate(sl, n_cal, max_iters=self.config.pq_max_iters, rtol=self.config.pq_rtol)
            self._calibrated[layer_idx] = True
            ls.phase = LayerPhase.STREAMING
        if self._calibrated[layer_idx]:
            cold = max(0, n - self.hot_window)   # AgingPolicy.tier_boundary (aging_policy.py:54-56)
            if cold > self._coded[layer_idx]:
                st.assign(sl, self._coded[layer_idx], cold)
                self._coded[layer_idx] = cold
        return self._views(layer_idx)

    def state_dict(self) -> dict:
        """The CompressedKVCache state of the exact layers, the CDC-03 store and
        the per-layer counters, as CPU tensors."""
        import dataclasses
        store = {k: (v.detach().cpu() if isinstance(v, torch.Tensor) else v) for k, v in self.store.state_dict().items()}
        return {"config": dataclasses.asdict(self.config), "n_layers": self.n_layers_expected,
                "total_tokens": self._total_tokens, "calibration_stats": list(self._calibration_stats),
                "layer_states": [ls.state_dict() for ls in self.layer_states],
                "exact_kv": self._exact_layers_state(skip=self._slot), "store": store,
                "len": list(self._len), "coded": list(self._coded), "calibrated": list(self._calibrated),
                "budget": (self.top_k, self.sink_tokens, self.hot_window)}

    def load_state_dict(self, state: dict) -> None:
        import dataclasses
        mine = dataclasses.asdict(self.config)
        if state["config"] != mine or state["n_layers"] != self.n_layers_expected:
            raise ValueError(f"Expected shape {(mine, self.n_layers_expected)}, got "
                             f"{(state['config'], state['n_layers'])}")
        self.store.load_state_dict(state["store"])
        self._total_tokens = int(state["total_tokens"])
        self._calibration_stats = list(state["calibration_stats"])
        for ls, st in zip(self.layer_states, state["layer_states"]):
            ls.load_state_dict(st)
        self._load_exact_kv(state["exact_kv"], skip=self._slot)
        self._len, self._coded, self._calibrated = list(state["len"]), list(state["coded"]), list(state["calibrated"])
        self.top_k, self.sink_tokens, self.hot_window = state["budget"]
        for i in self._slot:
            layer = _StoreLayer(self, i)
            if self._len[i] > 0:
                layer.dtype, layer.device, layer.is_initialized = self.store.k.dtype, self.store.k.device, True
                layer.keys, layer.values = self._views(i)
            self.layers[i] = layer

    def memory_report(self) -> dict:
        """Device bytes: exact layers in the parent, the store's exact tiers for
        compressed layers, and their PQ codes and codebooks; the keys of the
        reference's report (compressed_cache.py:107-130)."""
        st = self.store
        exact = 0
        for i, layer in enumerate(self.layers):
            if i in self._slot:
                continue
            for t in (getattr(layer, "keys", None), getattr(layer, "values", None)):
                if isinstance(t, torch.Tensor):
                    exact += t.element_size() * t.nelement()
        tiers = st.k.element_size() * st.k.nelement() + st.v.element_size() * st.v.nelement()
        codes = (st.codes.nelement() + st.codebook.element_size() * st.codebook.nelement()
                 + st.cb_k.element_size() * st.cb_k.nelement())
        return {
            "exact_bytes": exact + tiers,
            "compressed_bytes": codes,
            "total_bytes": exact + tiers + codes,
            "n_layers": self.n_layers_expected,
            "total_tokens": self._total_tokens,
            "calibration_complete": self.calibration_complete,
        }

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
        out = st.decode(cache.slot(layer), query[:, :, 0, :].contiguous(), scale, cache.top_k, cache.sink_tokens,
                        cache.hot_window, out_dtype=query.dtype)
        return out.unsqueeze(1), None
    if query.shape[2] > 1 and attention_mask is None and dropout == 0.0 and supported(query, key, value):
        # prefill, and multi-token steps of any layer: exact attention on the tensor cores
        causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
        if not causal or key.shape[2] >= query.shape[2]:
            return prefill_attention(query, key, value, scaling, is_causal=bool(causal)), None
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


AttentionInterface.register("cdc03", cdc03_attention_forward)
