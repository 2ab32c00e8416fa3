"""``from tiledattention.sdpa import sdpa`` (reference: src/tiledattention/sdpa.py:14)."""

from tiledattention_b200.sdpa import sdpa, sdpa_with_lse  # noqa: F401
