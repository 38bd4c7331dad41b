"""Kernel API of dcr_b200 (mirrors dcr_attention.kernel of the reference)."""
