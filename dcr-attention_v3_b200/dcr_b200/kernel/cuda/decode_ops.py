"""The layers around the attention in a decode step, on this package's kernels.

A decode step of a Llama model runs, per layer, a residual add and HF ``LlamaRMSNorm``
twice, four ``nn.Linear`` projections of the attention, the SwiGLU MLP and, at the end, a
norm and the LM head (transformers' ``modeling_llama``; the reference keeps them in torch).
With B = 1-8 tokens these are matrix-vector products and kilobyte-sized elementwise ops:
:func:`linear_skinny` streams each weight once, :func:`add_rmsnorm` and :func:`silu_mul`
replace the chains of small torch kernels with one launch each, with torch's rounding of the
same op sequence (see ``csrc/dcr_decode_ops.cu``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import check_dtype, require

SKINNY_MAX_M = 8


def _dt(x: torch.Tensor) -> int:
    return check_dtype(x, "tensor")


def add_rmsnorm(h: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor,
                eps: float, *, h_out: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
    """(h + delta, RMSNorm(h + delta)) over the last dim (delta None: (h, RMSNorm(h))).
    ``h_out`` (optional, may be ``h``) receives the sum."""
    _lib.require_cuda(h, weight)
    require(h.is_contiguous() and weight.is_contiguous() and weight.dim() == 1 and
            weight.shape[0] == h.shape[-1], "h [..., dim] and weight [dim], contiguous")
    require(weight.dtype == h.dtype, "weight must have h's dtype")
    dim = h.shape[-1]
    rows = h.numel() // dim
    y = torch.empty_like(h)
    if delta is not None:
        require(delta.shape == h.shape and delta.dtype == h.dtype and delta.is_contiguous(),
                "delta must match h")
        if h_out is None:
            h_out = torch.empty_like(h)
        require(h_out.shape == h.shape and h_out.dtype == h.dtype and h_out.is_contiguous(),
                "h_out must match h")
    with torch.cuda.device(h.device):
        st = _lib.load().dcr_add_rmsnorm(
            h.data_ptr(), None if delta is None else delta.data_ptr(), weight.data_ptr(), _dt(h),
            rows, dim, float(eps), None if delta is None else h_out.data_ptr(), y.data_ptr(),
            _lib.stream_ptr(h.device))
    _lib.check(st, "dcr_add_rmsnorm")
    return (h if delta is None else h_out), y


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up with torch's rounding (LlamaMLP's ``act_fn(gate_proj(x)) * up_proj(x)``)."""
    _lib.require_cuda(gate, up)
    require(gate.shape == up.shape and gate.dtype == up.dtype and gate.is_contiguous() and
            up.is_contiguous(), "gate and up must be contiguous tensors of one shape and dtype")
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        st = _lib.load().dcr_silu_mul(gate.data_ptr(), up.data_ptr(), _dt(gate), gate.numel(),
                                      out.data_ptr(), _lib.stream_ptr(gate.device))
    _lib.check(st, "dcr_silu_mul")
    return out


def linear_skinny(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """x [..., K] @ weight[N, K]^T for at most 8 rows of x (nn.Linear without bias),
    16-bit dtypes, K a multiple of 256."""
    _lib.require_cuda(x, weight)
    K = x.shape[-1]
    M = x.numel() // K
    require(weight.dim() == 2 and weight.shape[1] == K, "weight must be [N, K]")
    require(x.is_contiguous() and weight.is_contiguous(), "x and weight must be contiguous")
    require(x.dtype == weight.dtype and x.dtype in (torch.bfloat16, torch.float16),
            "x and weight must share a 16-bit dtype")
    require(1 <= M <= SKINNY_MAX_M and K % 256 == 0,
            f"need 1 <= rows <= {SKINNY_MAX_M} and K % 256 == 0, got rows={M}, K={K}")
    N = weight.shape[0]
    y = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    with torch.cuda.device(x.device):
        st = _lib.load().dcr_linear_skinny(x.data_ptr(), weight.data_ptr(), _dt(x), M, N, K,
                                           y.data_ptr(), _lib.stream_ptr(x.device))
    _lib.check(st, "dcr_linear_skinny")
    return y


def skinny_ok(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether :func:`linear_skinny` takes this product (else use a library GEMM)."""
    K = x.shape[-1]
    M = x.numel() // K
    return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and
            weight.dtype == x.dtype and 1 <= M <= SKINNY_MAX_M and K % 256 == 0 and
            x.is_contiguous() and weight.is_contiguous() and M * K * 2 <= 200 * 1024)
