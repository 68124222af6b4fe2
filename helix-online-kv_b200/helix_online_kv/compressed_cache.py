"""CompressedKVCache: a DynamicCache that compresses on the device.

Drop-in for the reference (helix_online_kv/compressed_cache.py:34-130).  The
parent DynamicCache still stores exact K/V and returns them, so HF attention
is unchanged.  Where the reference copied every new token to the host one at
a time (compressed_cache.py:97-103), ``update`` here hands the whole
[B, H, S_new, D] block to the layer state as a [S_new, B*H*D] CUDA view:
calibration, codebook fitting and assignment run as CUDA kernels and the
indices stay on the device.  ``memory_report`` works with transformers 5.x
(the reference's ``self[layer_idx]`` raises TypeError there).
"""

from __future__ import annotations

from typing import Optional

try:
    import torch
    from transformers.cache_utils import DynamicCache
    _HAS_TORCH = True
except ImportError:  # pragma: no cover
    _HAS_TORCH = False
    DynamicCache = object

from .aging_policy import AgingPolicy
from .config import OnlineKVConfig
from .layer_state import KVLayerState


def _require_torch():
    if not _HAS_TORCH:
        raise ImportError(
            "CompressedKVCache requires torch and transformers. "
            "Install with: pip install helix-online-kv[torch]"
        )


class CompressedKVCache(DynamicCache):
    """Online compressed KV cache -- a DynamicCache subclass (compressed_cache.py:34-130).

    Lifecycle: the first ``calibration_tokens`` tokens of each compressed layer
    calibrate its codebooks, later tokens are assigned uint8 indices; layers in
    ``exact_layers`` stay exact.
    """

    def __init__(self, config: OnlineKVConfig, n_layers: int):
        _require_torch()
        super().__init__()
        self.config = config
        self.n_layers_expected = n_layers
        self.aging = AgingPolicy(hot_window=config.hot_window)
        self.layer_states: list[KVLayerState] = [KVLayerState(i, config) for i in range(n_layers)]
        self._total_tokens = 0
        self._calibration_stats: list[dict] = []

    @property
    def total_tokens(self) -> int:
        return self._total_tokens

    @property
    def calibration_complete(self) -> bool:
        """True when every non-exact layer has finalized codebooks."""
        return all(ls.is_streaming or ls.is_exact for ls in self.layer_states)

    def update(self, key_states, value_states, layer_idx: int, cache_kwargs: Optional[dict] = None):
        """Store exact K/V (parent), then feed the new tokens to the layer state on the device."""
        k_out, v_out = super().update(key_states, value_states, layer_idx, cache_kwargs)
        if layer_idx == 0:
            self._total_tokens += key_states.shape[2]
        ls = self.layer_states[layer_idx]
        if ls.is_exact:
            return k_out, v_out
        T = key_states.shape[2]
        k_rows = key_states.detach().permute(2, 0, 1, 3).reshape(T, -1)
        v_rows = value_states.detach().permute(2, 0, 1, 3).reshape(T, -1)
        self._calibration_stats.extend(ls.feed_tokens(k_rows, v_rows))
        return k_out, v_out

    # ---- checkpoint / resume (the reference has no serialization) ------------
    def _exact_layers_state(self, skip=()):
        out = []
        for i, layer in enumerate(getattr(self, "layers", [])):
            k, v = getattr(layer, "keys", None), getattr(layer, "values", None)
            if i in skip or not isinstance(k, torch.Tensor) or k.numel() == 0:
                out.append(None)
            else:
                out.append((k.detach().cpu(), v.detach().cpu()))
        return out

    def state_dict(self) -> dict:
        """Configuration, token count, every layer state (codebooks and indices)
        and the exact K/V the parent DynamicCache holds, as CPU tensors."""
        import dataclasses
        return {"config": dataclasses.asdict(self.config), "n_layers": self.n_layers_expected,
                "total_tokens": self._total_tokens, "calibration_stats": list(self._calibration_stats),
                "layer_states": [ls.state_dict() for ls in self.layer_states],
                "exact_kv": self._exact_layers_state()}

    def _load_exact_kv(self, exact_kv, skip=()):
        from transformers.cache_utils import DynamicLayer
        from . import _lib as L
        for i, kv in enumerate(exact_kv):
            if i in skip:
                continue
            while len(self.layers) <= i:
                self.layers.append(DynamicLayer())
            layer = DynamicLayer()
            if kv is not None:
                layer.update(L.to_dev(kv[0], kv[0].dtype), L.to_dev(kv[1], kv[1].dtype))
            self.layers[i] = layer

    def load_state_dict(self, state: dict) -> None:
        import dataclasses
        mine = dataclasses.asdict(self.config)
        if state["config"] != mine or state["n_layers"] != self.n_layers_expected:
            raise ValueError(f"Expected shape {(mine, self.n_layers_expected)}, got "
                             f"{(state['config'], state['n_layers'])}")
        self._total_tokens = int(state["total_tokens"])
        self._calibration_stats = list(state["calibration_stats"])
        for ls, st in zip(self.layer_states, state["layer_states"]):
            ls.load_state_dict(st)
        self._load_exact_kv(state["exact_kv"])

    def memory_report(self) -> dict:
        """Exact (parent) and compressed bytes (compressed_cache.py:107-130)."""
        compressed = sum(ls.memory_bytes()["total_bytes"] for ls in self.layer_states)
        exact = 0
        for layer in getattr(self, "layers", []):
            for t in (getattr(layer, "keys", None), getattr(layer, "values", None)):
                if isinstance(t, torch.Tensor):
                    exact += t.element_size() * t.nelement()
        return {
            "exact_bytes": exact,
            "compressed_bytes": compressed,
            "total_bytes": exact + compressed,
            "n_layers": self.n_layers_expected,
            "total_tokens": self._total_tokens,
            "calibration_complete": self.calibration_complete,
        }
