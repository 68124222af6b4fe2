"""Aging policy: Tier 0 (exact) -> Tier 1 (compressed).

Host arithmetic, as in the reference (helix_online_kv/aging_policy.py:8-56).
The boundary it computes is applied on the device by
``CompressedKVCache`` (the reference computes it but never moves tokens).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class AgingPolicy:
    """When tokens age from Tier 0 (exact) to Tier 1 (compressed).

    Attributes:
        hot_window: Number of most recent tokens kept exact.
        min_age_tokens: Minimum age before a token may be compressed
            (defaults to hot_window).
    """
    hot_window: int = 256
    min_age_tokens: int | None = None

    @property
    def effective_min_age(self) -> int:
        return self.min_age_tokens if self.min_age_tokens is not None else self.hot_window

    def should_compress(self, token_age: int) -> bool:
        """True if a token that many steps old belongs in Tier 1 (aging_policy.py:30-40)."""
        return token_age >= self.effective_min_age

    def tier_boundary(self, total_tokens: int) -> int:
        """First Tier 0 index: [0, b) compressed, [b, total) exact (aging_policy.py:42-56)."""
        if total_tokens <= self.effective_min_age:
            return 0
        return total_tokens - self.effective_min_age
