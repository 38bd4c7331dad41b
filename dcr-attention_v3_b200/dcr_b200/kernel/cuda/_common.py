"""Argument checks and workspace handling shared by the CUDA kernel wrappers.

The checks mirror the reference's Python wrappers
(dcr_attention/kernel/triton/topk_axis.py:37-44, topk_axis_pass1.py:114-130,
topk_axis_pass2.py:30-36, fused_attn.py:170-193): shape, dtype and layout problems raise
AssertionError, non-CUDA tensors raise RuntimeError, and ``N <= k_eff`` raises
:class:`KEffRangeError`, which is both the oracle's ValueError
(qaxis_topk_reference.py:236-241) and the Triton wrappers' AssertionError.
The checks are explicit ``raise`` statements, so they also hold under ``python -O``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from dcr_b200 import _lib

HEAD_DIM = 64
SUPPORTED_GROUPS = (1, 2, 4, 8)


class KEffRangeError(ValueError, AssertionError):
    """k_eff is not in (0, N): the caller must dispatch to SDPA."""


def require(cond: bool, msg: str) -> None:
    if not cond:
        raise AssertionError(msg)


def check_dtype(t: torch.Tensor, name: str) -> int:
    require(t.dtype in _lib.DTYPE_CODES,
            f"{name} must be bfloat16, float16 or float32, got {t.dtype}")
    return _lib.DTYPE_CODES[t.dtype]


def check_k_range(k_eff: int, N: int) -> None:
    if not (0 < k_eff < N):
        raise KEffRangeError(
            f"kernel invoked with N={N} <= k_eff={k_eff}; caller must dispatch to SDPA"
            if k_eff >= N else f"k_eff must be > 0, got {k_eff}")


def cache_strides(t: torch.Tensor, name: str) -> Tuple[int, int]:
    """(batch stride, head stride) in elements of a [B, H_kv, N, D] cache whose rows are
    contiguous; any batch/head strides are accepted (e.g. a cache allocated for N_max)."""
    require(t.dim() == 4, f"{name} must be [B, H_kv, N, D], got shape {tuple(t.shape)}")
    require(t.shape[-1] == HEAD_DIM, f"spec locked at D={HEAD_DIM}; got D={t.shape[-1]}")
    require(t.stride(-1) == 1 and (t.shape[2] <= 1 or t.stride(-2) == HEAD_DIM),
            f"{name} rows must be contiguous (stride D along N, 1 along D)")
    return t.stride(0), t.stride(1)


def check_groups(H: int, H_kv: int) -> None:
    require(H % H_kv == 0, f"H={H} must be divisible by H_kv={H_kv}")
    require(H // H_kv in SUPPORTED_GROUPS,
            f"n_per_kv={H // H_kv} not supported (supported: {SUPPORTED_GROUPS})")


def workspace(device: torch.device, nbytes: int,
              ws: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Caller-provided workspace (checked) or a fresh uint8 buffer from torch's allocator."""
    if ws is not None:
        require(ws.is_cuda and ws.device == device and ws.dtype == torch.uint8 and
                ws.is_contiguous() and ws.numel() >= nbytes,
                f"workspace must be a contiguous uint8 CUDA tensor of >= {nbytes} bytes "
                f"on {device}")
        return ws
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


def workspace_bytes(B: int, H: int, H_kv: int, N: int, k_eff: int) -> int:
    return int(_lib.load().dcr_workspace_bytes(B, H, H_kv, N, HEAD_DIM, k_eff))
