"""k_eff from the coverage floor.

Mirrors ``adaptive_k_window`` (Seqev/dcr-attention_v3,
dcr_attention/models/llama/adaptive.py:39): the same integer function, so the kernels see
the same k_eff as the reference's hook (attention.py:776-780). At N=32768, c=0.15 it gives
4916 (floor 4915 rounded up to even).
"""
from __future__ import annotations


def adaptive_k_window(k_window_min: int, n_kv: int, coverage_floor: float) -> int:
    """k_eff = min(n_kv, max(k_window_min, floor(n_kv * c))), odd values rounded up to even
    and capped at n_kv."""
    if n_kv <= 0:
        raise ValueError(f"n_kv must be > 0, got {n_kv}")
    if not (0.0 <= coverage_floor <= 1.0):
        raise ValueError(f"coverage_floor must be in [0, 1], got {coverage_floor}")
    k_eff = max(k_window_min, int(n_kv * coverage_floor))
    k_eff = min(k_eff, n_kv)
    if k_eff % 2 == 1:
        k_eff = min(k_eff + 1, n_kv)
    return k_eff
