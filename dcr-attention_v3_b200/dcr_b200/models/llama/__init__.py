"""Llama decode-side helpers (mirrors dcr_attention.models.llama of the reference)."""
