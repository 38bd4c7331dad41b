"""Projected-score mode of the sparse decode attention (rank-16 key projection).

The reference's Pass 1 reads every 64-dim key to score it against the unit query
(dcr_attention/kernel/triton/topk_axis_pass1.py:29). Here the cache also keeps
``KP = K . P`` (P: a fixed [64, 16] fp32 matrix), written when tokens are appended, and
Pass 1 scores ``bf16(KP . (u . P))`` from 32-byte rows. Pass 2 and Pass 3 are those of
:func:`topk_qaxis_attention`. The reference has no such mode; the kernels follow the CPU
restatement in ``oracle/dcr_oracle.c`` bit for bit.

Functions mirror the exact-mode ones and add the projected cache and P:

* :func:`project_keys` (prefill): KP of an existing cache.
* :func:`topk_qaxis_select_projected`: Pass 1 (projected) + Pass 2.
* :func:`topk_qaxis_attention_projected`: the full step.
"""
from __future__ import annotations

from typing import Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import (HEAD_DIM, cache_strides, check_dtype, check_groups,
                                          check_k_range, require, workspace, workspace_bytes)

PROJ_RANK = 16


def check_projection(P: torch.Tensor, device: torch.device) -> torch.Tensor:
    require(P.dim() == 2 and tuple(P.shape) == (HEAD_DIM, PROJ_RANK),
            f"P must be [{HEAD_DIM}, {PROJ_RANK}], got {tuple(P.shape)}")
    require(P.dtype == torch.float32 and P.is_contiguous() and P.device == device,
            "P must be a contiguous fp32 tensor on the cache's device")
    return P


def kp_strides(KP: torch.Tensor, name: str = "KP_cache"):
    require(KP.dim() == 4 and KP.shape[-1] == PROJ_RANK,
            f"{name} must be [B, H_kv, N, {PROJ_RANK}], got {tuple(KP.shape)}")
    require(KP.stride(-1) == 1 and (KP.shape[2] <= 1 or KP.stride(-2) == PROJ_RANK),
            f"{name} rows must be contiguous")
    return KP.stride(0), KP.stride(1)


def project_keys(K_cache: torch.Tensor, P: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """KP [B, H_kv, N, 16] in K's dtype: the projection of every cached key."""
    _lib.require_cuda(K_cache)
    dt = check_dtype(K_cache, "K_cache")
    B, H_kv, N, _ = K_cache.shape
    ksb, ksh = cache_strides(K_cache, "K_cache")
    check_projection(P, K_cache.device)
    if out is None:
        out = torch.empty(B, H_kv, N, PROJ_RANK, dtype=K_cache.dtype, device=K_cache.device)
    psb, psh = kp_strides(out, "out")
    with torch.cuda.device(K_cache.device):
        st = _lib.load().dcr_project_keys(K_cache.data_ptr(), dt, ksb, ksh, B, H_kv, N, HEAD_DIM,
                                          P.data_ptr(), PROJ_RANK, out.data_ptr(), psb, psh,
                                          _lib.stream_ptr(K_cache.device))
    _lib.check(st, "dcr_project_keys")
    return out


def _check_q_kp(Q, KP_cache, P):
    _lib.require_cuda(Q, KP_cache)
    require(Q.dim() == 3 and Q.shape[-1] == HEAD_DIM and Q.is_contiguous(),
            f"Q must be a contiguous [B, H, {HEAD_DIM}] tensor")
    dt = check_dtype(Q, "Q")
    require(KP_cache.dtype == Q.dtype, "KP_cache must have Q's dtype")
    B, H, _ = Q.shape
    B_k, H_kv, N, _ = KP_cache.shape
    require(B == B_k, "Q and KP_cache batch mismatch")
    check_groups(H, H_kv)
    check_projection(P, Q.device)
    psb, psh = kp_strides(KP_cache)
    return B, H, H_kv, N, dt, psb, psh


def topk_qaxis_select_projected(Q: torch.Tensor, KP_cache: torch.Tensor, P: torch.Tensor,
                                k_eff: int, *, eps: float = 1e-12,
                                workspace_buf: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[B, H, k_eff] int32 ascending: the top-K of the projected scores."""
    B, H, H_kv, N, dt, psb, psh = _check_q_kp(Q, KP_cache, P)
    check_k_range(int(k_eff), N)
    idx = torch.empty(B, H, k_eff, dtype=torch.int32, device=Q.device)
    ws = workspace(Q.device, workspace_bytes(B, H, H_kv, N, k_eff), workspace_buf)
    with torch.cuda.device(Q.device):
        st = _lib.load().dcr_select_indices_projected(
            Q.data_ptr(), KP_cache.data_ptr(), dt, psb, psh, P.data_ptr(), PROJ_RANK, None, B, H,
            H_kv, N, HEAD_DIM, int(k_eff), float(eps), idx.data_ptr(), ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_select_indices_projected")
    return idx


def topk_qaxis_attention_projected(Q: torch.Tensor, K_cache: torch.Tensor,
                                   V_cache: torch.Tensor, KP_cache: torch.Tensor,
                                   P: torch.Tensor, k_eff: int, *, eps: float = 1e-12,
                                   out: Optional[torch.Tensor] = None,
                                   workspace_buf: Optional[torch.Tensor] = None,
                                   qp: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode step with the projected Pass 1: O [B, H, D] in Q's dtype. ``qp`` (optional):
    the projected unit queries [B, H, 16] fp32 from :func:`decode_prologue`."""
    B, H, H_kv, N, dt, psb, psh = _check_q_kp(Q, KP_cache, P)
    _lib.require_cuda(K_cache, V_cache)
    require(tuple(K_cache.shape) == (B, H_kv, N, HEAD_DIM) and
            tuple(V_cache.shape) == (B, H_kv, N, HEAD_DIM),
            "K_cache and V_cache must be [B, H_kv, N, D] matching KP_cache")
    require(K_cache.dtype == Q.dtype and V_cache.dtype == Q.dtype, "caches must have Q's dtype")
    check_k_range(int(k_eff), N)
    ksb, ksh = cache_strides(K_cache, "K_cache")
    vsb, vsh = cache_strides(V_cache, "V_cache")
    if out is None:
        out = torch.empty(B, H, HEAD_DIM, dtype=Q.dtype, device=Q.device)
    else:
        require(out.shape == (B, H, HEAD_DIM) and out.dtype == Q.dtype and out.is_contiguous(),
                "out must be a contiguous [B, H, D] tensor like Q")
    ws = workspace(Q.device, workspace_bytes(B, H, H_kv, N, k_eff), workspace_buf)
    with torch.cuda.device(Q.device):
        qp_ptr = None
        if qp is not None:
            require(qp.dtype == torch.float32 and qp.is_contiguous() and
                    tuple(qp.shape) == (B, H, PROJ_RANK), "qp must be a contiguous fp32 [B, H, 16]")
            qp_ptr = qp.data_ptr()
        st = _lib.load().dcr_decode_projected(
            Q.data_ptr(), K_cache.data_ptr(), V_cache.data_ptr(), KP_cache.data_ptr(), dt, ksb,
            ksh, vsb, vsh, psb, psh, P.data_ptr(), PROJ_RANK, qp_ptr, B, H, H_kv, N, HEAD_DIM,
            int(k_eff), float(eps), out.data_ptr(), ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(Q.device))
    _lib.check(st, "dcr_decode_projected")
    return out
