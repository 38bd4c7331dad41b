"""Pass 3 — fused gather + online-softmax attention on the B200 (CUDA, sm_100a).

Drop-in for ``fused_topk_attention``
(Seqev/dcr-attention_v3, dcr_attention/kernel/triton/fused_attn.py:158):
``O[b, h] = softmax(K[b, h//G, idx] . f32(Q[b, h]) / sqrt(D)) @ V[b, h//G, idx]`` with an
fp32 running state and one rounding at the output. The kernel (csrc/dcr_attend.cu) splits
each (b, h) index list across CTAs and merges the partial (m, l, o) states on the device.
The output has Q's dtype (the reference only accepts bf16, so for bf16 inputs it is the
same).
"""
from __future__ import annotations

from typing import Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import (HEAD_DIM, cache_strides, check_dtype, check_groups,
                                          check_k_range, require, workspace, workspace_bytes)


def fused_topk_attention(
    Q: torch.Tensor,            # [B, H, D]
    K_cache: torch.Tensor,      # [B, H_kv, N, D]
    V_cache: torch.Tensor,      # [B, H_kv, N, D]
    indices: torch.Tensor,      # [B, H, k_eff] int32 (from Pass 2)
    *,
    workspace_buf: Optional[torch.Tensor] = None,
) -> torch.Tensor:              # [B, H, D], Q's dtype
    """Attention of each query head over its selected cache rows."""
    _lib.require_cuda(Q, K_cache, V_cache, indices)
    require(Q.dim() == 3, f"Q must be [B, H, D], got {tuple(Q.shape)}")
    B, H, D = Q.shape
    require(K_cache.dim() == 4 and V_cache.dim() == 4, "K_cache/V_cache must be 4-D")
    B_k, H_kv, N, D_k = K_cache.shape
    require(indices.dim() == 3, f"indices must be [B, H, k_eff], got {tuple(indices.shape)}")
    B_i, H_i, k_eff = indices.shape
    dt = check_dtype(Q, "Q")
    require(K_cache.dtype == Q.dtype and V_cache.dtype == Q.dtype,
            f"Q, K_cache and V_cache must share a dtype, got {Q.dtype}, {K_cache.dtype}, "
            f"{V_cache.dtype}")
    require(indices.dtype == torch.int32, f"indices must be int32, got {indices.dtype}")
    require(Q.is_contiguous(), "Q must be contiguous")
    require(indices.is_contiguous(), "indices must be contiguous")
    require(B == B_k == B_i and H == H_i and D == D_k, "Q / K_cache / indices shape mismatch")
    require(tuple(V_cache.shape) == tuple(K_cache.shape), "V_cache must match K_cache's shape")
    require(D == HEAD_DIM, f"spec locked at D={HEAD_DIM}; got D={D}")
    check_groups(H, H_kv)
    check_k_range(k_eff, N)
    ksb, ksh = cache_strides(K_cache, "K_cache")
    vsb, vsh = cache_strides(V_cache, "V_cache")
    O = torch.empty(B, H, D, dtype=Q.dtype, device=Q.device)
    nbytes = workspace_bytes(B, H, H_kv, N, k_eff)
    ws = workspace(Q.device, nbytes, workspace_buf)
    with torch.cuda.device(Q.device):
        st = _lib.load().dcr_attend(Q.data_ptr(), K_cache.data_ptr(), V_cache.data_ptr(), dt,
                                    ksb, ksh, vsb, vsh, indices.data_ptr(), B, H, H_kv, N,
                                    HEAD_DIM, k_eff, O.data_ptr(), ws.data_ptr(), ws.numel(),
                                    _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_attend")
    return O
