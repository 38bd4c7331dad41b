"""Model-side helpers of dcr_b200 (mirrors dcr_attention.models of the reference)."""
