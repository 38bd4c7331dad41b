"""CUDA (sm_100a) implementations of the reference's Triton kernel API
(dcr_attention/kernel/triton/__init__.py of Seqev/dcr-attention_v3)."""
from dcr_b200.kernel.cuda.fused_attn import fused_topk_attention
from dcr_b200.kernel.cuda.projected import (project_keys, topk_qaxis_attention_projected,
                                            topk_qaxis_select_projected)
from dcr_b200.kernel.cuda.topk_axis import compute_u_Q, topk_qaxis_attention, topk_qaxis_select
from dcr_b200.kernel.cuda.topk_axis_pass1 import topk_pass1_projection
from dcr_b200.kernel.cuda.topk_axis_pass2 import topk_pass2_select

__all__ = [
    "compute_u_Q",
    "fused_topk_attention",
    "project_keys",
    "topk_pass1_projection",
    "topk_pass2_select",
    "topk_qaxis_attention",
    "topk_qaxis_attention_projected",
    "topk_qaxis_select",
    "topk_qaxis_select_projected",
]
