"""Configuration of the compressed KV cache.

Same fields and defaults as the reference ``OnlineKVConfig``
(helix_online_kv/config.py:8-30); the CDC-03 fields after ``exact_layers`` are
additions with defaults, so existing callers are unaffected.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class OnlineKVConfig:
    """Configuration for CompressedKVCache.

    Attributes:
        calibration_tokens: Tokens accumulated before the codebooks are fitted.
        hot_window: Most recent tokens kept exact and always attended (Tier 0).
        n_clusters: Codebook size (at most 256: indices are uint8).
        max_kmeans_iters: Lloyd iterations of the scalar calibration.
        rtol: Relative convergence tolerance of the scalar calibration.
        drift_threshold: MSE above which the EMA centroid update runs.
        drift_ema_alpha: EMA factor of the centroid update.
        exact_layers: Layer indices that are never compressed.
        pq_subspaces: PQ subspaces of the CDC-03 key codebooks (0 disables CDC-03).
        pq_max_iters: Lloyd iterations of the PQ calibration.
        pq_rtol: Relative tolerance of the PQ calibration.
        top_k: CDC-03 token budget per query head, sinks included.
        sink_tokens: Leading tokens always attended.
    """
    calibration_tokens: int = 128
    hot_window: int = 256
    n_clusters: int = 256
    max_kmeans_iters: int = 10
    rtol: float = 0.001
    drift_threshold: float = 0.01
    drift_ema_alpha: float = 0.05
    exact_layers: list[int] = field(default_factory=lambda: [0])
    pq_subspaces: int = 8
    pq_max_iters: int = 30
    pq_rtol: float = 1e-4
    top_k: int = 128
    sink_tokens: int = 4
