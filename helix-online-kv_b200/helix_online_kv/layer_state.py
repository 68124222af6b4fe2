"""Per-layer compression state: scalar K/V codebooks and index buffers.

Drop-in for the reference (helix_online_kv/layer_state.py).  ``feed_token``
keeps the reference's one-token NumPy interface; ``feed_tokens`` takes a
whole [T, entry] CUDA tensor per call, which is what ``CompressedKVCache``
uses so that no key/value ever leaves the device.  Both follow the same phase
machine: calibrate on the first ``calibration_tokens`` tokens, fit both
codebooks on the token that completes calibration, then assign.
Calibration tokens keep no indices (layer_state.py:106-109).
"""

from __future__ import annotations

from enum import Enum

import numpy as np

from .codebook import OnlineCodebook
from .config import OnlineKVConfig

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


class LayerPhase(Enum):
    CALIBRATING = "calibrating"
    STREAMING = "streaming"
    EXACT = "exact"  # Layer excluded from compression


class KVLayerState:
    """Per-layer state: codebooks for K and V, phase, compressed index buffers."""

    def __init__(self, layer_idx: int, config: OnlineKVConfig):
        self.layer_idx = layer_idx
        self.config = config
        if layer_idx in config.exact_layers:
            self.phase = LayerPhase.EXACT
            self.k_codebook = None
            self.v_codebook = None
        else:
            self.phase = LayerPhase.CALIBRATING
            kw = dict(n_clusters=config.n_clusters, max_iters=config.max_kmeans_iters, rtol=config.rtol,
                      drift_threshold=config.drift_threshold, drift_ema_alpha=config.drift_ema_alpha)
            self.k_codebook = OnlineCodebook(**kw)
            self.v_codebook = OnlineCodebook(**kw)
        self._k_indices: list = []   # NumPy rows (feed_token) or CUDA [T, entry] blocks (feed_tokens)
        self._v_indices: list = []
        self._n_compressed = 0
        self._tokens_seen = 0

    @property
    def tokens_seen(self) -> int:
        return self._tokens_seen

    @property
    def is_exact(self) -> bool:
        return self.phase == LayerPhase.EXACT

    @property
    def is_calibrating(self) -> bool:
        return self.phase == LayerPhase.CALIBRATING

    @property
    def is_streaming(self) -> bool:
        return self.phase == LayerPhase.STREAMING

    @property
    def compressed_token_count(self) -> int:
        """Number of tokens stored as compressed indices."""
        return self._n_compressed

    def _finalize(self):
        k_stats = self.k_codebook.finalize_calibration()
        v_stats = self.v_codebook.finalize_calibration()
        self.phase = LayerPhase.STREAMING
        return {"layer": self.layer_idx, "k_calibration": k_stats, "v_calibration": v_stats}

    def feed_token(self, k_values, v_values):
        """Process one token's flat K/V values (layer_state.py:78-123).

        Returns the calibration stats dict when this token completes calibration.
        """
        self._tokens_seen += 1
        if self.phase == LayerPhase.EXACT:
            return None
        if self.phase == LayerPhase.CALIBRATING:
            self.k_codebook.feed_calibration(k_values)
            self.v_codebook.feed_calibration(v_values)
            if self._tokens_seen >= self.config.calibration_tokens:
                return self._finalize()
            return None
        self._k_indices.append(self.k_codebook.assign(k_values))
        self._v_indices.append(self.v_codebook.assign(v_values))
        self._n_compressed += 1
        return None

    def feed_tokens(self, k_rows, v_rows) -> list:
        """Process T tokens at once: ``k_rows``/``v_rows`` are [T, entry] CUDA tensors.

        Same phase semantics as T calls of ``feed_token``; returns the list of
        calibration stats dicts produced (0 or 1).
        """
        T = int(k_rows.shape[0])
        if T == 0:
            return []
        if self.phase == LayerPhase.EXACT:
            self._tokens_seen += T
            return []
        out = []
        i = 0
        if self.phase == LayerPhase.CALIBRATING:
            need = max(self.config.calibration_tokens - self._tokens_seen, 1)
            take = min(need, T)
            self.k_codebook.feed_calibration(k_rows[:take])
            self.v_codebook.feed_calibration(v_rows[:take])
            self._tokens_seen += take
            i = take
            if self._tokens_seen >= self.config.calibration_tokens:
                out.append(self._finalize())
        if i < T and self.phase == LayerPhase.STREAMING:
            kr, vr = k_rows[i:], v_rows[i:]
            self._k_indices.append(self.k_codebook.assign(kr.reshape(-1)).reshape(kr.shape))
            self._v_indices.append(self.v_codebook.assign(vr.reshape(-1)).reshape(vr.shape))
            self._n_compressed += T - i
            self._tokens_seen += T - i
        return out

    def _stack(self, parts):
        if torch is not None and parts and isinstance(parts[0], torch.Tensor):
            return torch.cat([p.reshape(-1, p.shape[-1]) for p in parts], 0)
        return np.stack(parts)

    def get_compressed_kv(self, token_offset: int):
        """Decoded K/V of one compressed token (layer_state.py:125-140)."""
        if self.phase == LayerPhase.EXACT:
            raise RuntimeError(f"Layer {self.layer_idx} is exact — no compressed data")
        if not self.k_codebook.finalized:
            raise RuntimeError("Codebook not finalized yet")
        k_all = self._stack(self._k_indices)
        v_all = self._stack(self._v_indices)
        return self.k_codebook.decode(k_all[token_offset]), self.v_codebook.decode(v_all[token_offset])

    def get_all_compressed_k(self):
        """All compressed K decoded, [n_compressed, entry] (layer_state.py:142-151)."""
        if not self._k_indices:
            return None
        return self.k_codebook.decode(self._stack(self._k_indices))

    def get_all_compressed_v(self):
        """All compressed V decoded (layer_state.py:153-162)."""
        if not self._v_indices:
            return None
        return self.v_codebook.decode(self._stack(self._v_indices))

    # ---- checkpoint / resume (the reference has no serialization) ------------
    def state_dict(self) -> dict:
        """Phase, counters, both codebooks and the index blocks (CPU uint8)."""
        def blocks(parts):
            if not parts:
                return None
            if isinstance(parts[0], np.ndarray):
                return ("numpy", torch.from_numpy(np.stack(parts)))
            return ("device", torch.cat([p.reshape(-1, p.shape[-1]) for p in parts], 0).cpu())
        return {"layer_idx": self.layer_idx, "phase": self.phase.value, "tokens_seen": self._tokens_seen,
                "n_compressed": self._n_compressed,
                "k_codebook": None if self.k_codebook is None else self.k_codebook.state_dict(),
                "v_codebook": None if self.v_codebook is None else self.v_codebook.state_dict(),
                "k_indices": blocks(self._k_indices), "v_indices": blocks(self._v_indices)}

    def load_state_dict(self, state: dict) -> None:
        if state["layer_idx"] != self.layer_idx or (state["phase"] == LayerPhase.EXACT.value) != self.is_exact:
            raise ValueError(f"Expected shape of layer {self.layer_idx} ({self.phase.value}), got layer "
                             f"{state['layer_idx']} ({state['phase']})")
        self.phase = LayerPhase(state["phase"])
        self._tokens_seen = int(state["tokens_seen"])
        self._n_compressed = int(state["n_compressed"])
        for name in ("k_codebook", "v_codebook"):
            if state[name] is not None:
                getattr(self, name).load_state_dict(state[name])

        def unblock(b):
            if b is None:
                return []
            kind, t = b
            if kind == "numpy":
                return [row for row in t.numpy()]
            from . import _lib as L
            return [L.to_dev(t, torch.uint8)]
        self._k_indices = unblock(state["k_indices"])
        self._v_indices = unblock(state["v_indices"])

    def memory_bytes(self) -> dict:
        """Codebook and index bytes of this layer (layer_state.py:164-182)."""
        if self.phase == LayerPhase.EXACT:
            return {"codebook_bytes": 0, "index_bytes": 0, "total_bytes": 0}
        cb = 0
        for c in (self.k_codebook, self.v_codebook):
            if c is not None and c.centroids is not None:
                cb += c.centroids.nbytes
        idx = 0
        for p in self._k_indices + self._v_indices:
            idx += p.nbytes if isinstance(p, np.ndarray) else p.numel() * p.element_size()
        return {"codebook_bytes": cb, "index_bytes": idx, "total_bytes": cb + idx}
