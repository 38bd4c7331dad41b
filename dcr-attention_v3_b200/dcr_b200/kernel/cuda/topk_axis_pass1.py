"""Pass 1 — projection scores on the B200 (CUDA, sm_100a).

Drop-in for ``topk_pass1_projection``
(Seqev/dcr-attention_v3, dcr_attention/kernel/triton/topk_axis_pass1.py:104):
``scores[b, h, n] = bf16(sum_d f32(K[b, h // G, n, d]) * u_Q[b, h, d])``.
The kernel (csrc/dcr_score.cu) streams the K cache with TMA tile loads and scores the
G = H / H_kv query heads of each KV head from the same rows.
"""
from __future__ import annotations

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import (HEAD_DIM, cache_strides, check_dtype, check_groups,
                                          require)


def topk_pass1_projection(
    K_cache: torch.Tensor,   # [B, H_kv, N, D] bf16 / fp16 / fp32, rows contiguous
    u_Q: torch.Tensor,       # [B, H, D] fp32
) -> torch.Tensor:           # [B, H, N] bf16
    """Project every cached key on the unit query of each query head; bf16 scores."""
    _lib.require_cuda(K_cache, u_Q)
    B, H_kv, N, D = K_cache.shape
    require(u_Q.dim() == 3 and u_Q.shape[0] == B and u_Q.shape[2] == D,
            f"u_Q must be [B, H, D] = [{B}, H, {D}], got {tuple(u_Q.shape)}")
    H = u_Q.shape[1]
    dt = check_dtype(K_cache, "K_cache")
    require(u_Q.dtype == torch.float32, f"u_Q must be fp32, got {u_Q.dtype}")
    require(u_Q.is_contiguous(), "u_Q must be contiguous")
    require(K_cache.device == u_Q.device, "K_cache and u_Q must be on the same device")
    ksb, ksh = cache_strides(K_cache, "K_cache")
    check_groups(H, H_kv)
    scores = torch.empty(B, H, N, dtype=torch.bfloat16, device=K_cache.device)
    with torch.cuda.device(K_cache.device):
        st = _lib.load().dcr_score(K_cache.data_ptr(), dt, ksb, ksh, u_Q.data_ptr(), None, 0.0,
                                   B, H, H_kv, N, HEAD_DIM, scores.data_ptr(), N,
                                   _lib.stream_ptr(K_cache.device))
    _lib.check(st, "dcr_score")
    return scores
