"""Top-K Q-axis sparse decode attention on the B200 — the drop-in entry points.

Same names and signatures as the reference's Triton pipeline
(Seqev/dcr-attention_v3, dcr_attention/kernel/triton/topk_axis.py):

* :func:`topk_qaxis_select` (topk_axis.py:20) - Pass 1 + 2, int32 indices ascending.
* :func:`topk_qaxis_attention` (topk_axis.py:58) - Pass 1 + 2 + 3, the attention output.

Differences from the reference, all supersets: fp16 and fp32 caches are accepted (the
reference asserts bf16); H / H_kv may be 1, 2, 4 or 8 (the reference hard-codes 4); cache
views whose rows are contiguous are accepted without a copy; the output keeps Q's dtype.
The unit query is computed on the device inside Pass 1 (the reference computes it with
torch ops on the host side, topk_axis.py:47).
"""
from __future__ import annotations

from typing import Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import (HEAD_DIM, cache_strides, check_dtype, check_groups,
                                          check_k_range, require, workspace, workspace_bytes)


def _check_qk(Q: torch.Tensor, K_cache: torch.Tensor):
    _lib.require_cuda(Q, K_cache)
    require(Q.dim() == 3, f"Q must be [B, H, D], got {tuple(Q.shape)}")
    require(K_cache.dim() == 4, f"K_cache must be [B, H_kv, N, D], got {tuple(K_cache.shape)}")
    B, H, D = Q.shape
    B_k, H_kv, N, D_k = K_cache.shape
    dt = check_dtype(Q, "Q")
    require(K_cache.dtype == Q.dtype, f"K_cache must have Q's dtype {Q.dtype}, got "
            f"{K_cache.dtype}")
    require(B == B_k and D == D_k, "Q and K_cache batch/head-dim mismatch")
    require(D == HEAD_DIM, f"spec locked at D={HEAD_DIM}; got D={D}")
    require(Q.is_contiguous(), "Q must be contiguous")
    require(Q.device == K_cache.device, "Q and K_cache must be on the same device")
    check_groups(H, H_kv)
    return B, H, H_kv, N, dt


def check_attention_args(Q: torch.Tensor, K_cache: torch.Tensor, V_cache: torch.Tensor,
                         k_eff: int):
    """The argument checks of :func:`topk_qaxis_attention` (the reference's
    topk_axis.py:37-44 and fused_attn.py:170-193, widened as the module docstring says).
    Returns (B, H, H_kv, N, dtype code, K's batch and head strides, V's)."""
    B, H, H_kv, N, dt = _check_qk(Q, K_cache)
    _lib.require_cuda(V_cache)
    require(tuple(V_cache.shape) == tuple(K_cache.shape), "V_cache must match K_cache's shape")
    require(V_cache.dtype == Q.dtype, f"V_cache must have Q's dtype {Q.dtype}")
    check_k_range(int(k_eff), N)
    ksb, ksh = cache_strides(K_cache, "K_cache")
    vsb, vsh = cache_strides(V_cache, "V_cache")
    return B, H, H_kv, N, dt, ksb, ksh, vsb, vsh


def compute_u_Q(Q: torch.Tensor, eps: float = 1e-12) -> torch.Tensor:
    """u = f32(Q) / max(||f32(Q)||, eps) on the device (``_compute_u_Q``,
    qaxis_topk_reference.py:42)."""
    _lib.require_cuda(Q)
    require(Q.dim() >= 1 and Q.shape[-1] == HEAD_DIM, f"Q must be [..., {HEAD_DIM}]")
    dt = check_dtype(Q, "Q")
    Qc = Q.contiguous()
    u = torch.empty(Q.shape, dtype=torch.float32, device=Q.device)
    rows = Qc.numel() // HEAD_DIM
    with torch.cuda.device(Q.device):
        st = _lib.load().dcr_unit_query(Qc.data_ptr(), dt, rows, 1, HEAD_DIM, float(eps),
                                        u.data_ptr(), _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_unit_query")
    return u


def topk_qaxis_select(
    Q: torch.Tensor,         # [B, H, D]
    K_cache: torch.Tensor,   # [B, H_kv, N, D]
    k_eff: int,
    *,
    eps: float = 1e-12,
    workspace_buf: Optional[torch.Tensor] = None,
) -> torch.Tensor:           # [B, H, k_eff] int32, sorted ascending
    """Top-K key indices per query head via the Q-axis projection (Pass 1 + 2)."""
    B, H, H_kv, N, dt = _check_qk(Q, K_cache)
    check_k_range(int(k_eff), N)
    ksb, ksh = cache_strides(K_cache, "K_cache")
    idx = torch.empty(B, H, k_eff, dtype=torch.int32, device=Q.device)
    ws = workspace(Q.device, workspace_bytes(B, H, H_kv, N, k_eff), workspace_buf)
    with torch.cuda.device(Q.device):
        st = _lib.load().dcr_select_indices(Q.data_ptr(), K_cache.data_ptr(), dt, ksb, ksh, B, H,
                                            H_kv, N, HEAD_DIM, int(k_eff), float(eps),
                                            idx.data_ptr(), ws.data_ptr(), ws.numel(),
                                            _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_select_indices")
    return idx


def topk_qaxis_attention(
    Q: torch.Tensor,            # [B, H, D]
    K_cache: torch.Tensor,      # [B, H_kv, N, D]
    V_cache: torch.Tensor,      # [B, H_kv, N, D]
    k_eff: int,
    *,
    eps: float = 1e-12,
    out: Optional[torch.Tensor] = None,
    workspace_buf: Optional[torch.Tensor] = None,
) -> torch.Tensor:              # [B, H, D], Q's dtype
    """Full decode step: unit query, Pass 1 scores, Pass 2 top-K, Pass 3 attention."""
    B, H, H_kv, N, dt, ksb, ksh, vsb, vsh = check_attention_args(Q, K_cache, V_cache, k_eff)
    if out is None:
        out = torch.empty(B, H, HEAD_DIM, dtype=Q.dtype, device=Q.device)
    else:
        require(out.shape == (B, H, HEAD_DIM) and out.dtype == Q.dtype and out.is_contiguous()
                and out.device == Q.device, "out must be a contiguous [B, H, D] tensor like Q")
    ws = workspace(Q.device, workspace_bytes(B, H, H_kv, N, k_eff), workspace_buf)
    with torch.cuda.device(Q.device):
        st = _lib.load().dcr_decode(Q.data_ptr(), K_cache.data_ptr(), V_cache.data_ptr(), dt,
                                    ksb, ksh, vsb, vsh, B, H, H_kv, N, HEAD_DIM, int(k_eff),
                                    float(eps), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                    _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_decode")
    return out
