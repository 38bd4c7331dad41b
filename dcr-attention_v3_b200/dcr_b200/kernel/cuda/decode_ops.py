"""The layers around the attention in a decode step, on this package's kernels.

A decode step of a Llama model runs, per layer, a residual add and HF ``LlamaRMSNorm``
twice, the attention's projections, the SwiGLU MLP and, at the end, a norm and the LM head
(transformers' ``modeling_llama``; the reference keeps them in torch). With B = 1-8 tokens
the norms and activations are kilobyte-sized: :func:`add_rmsnorm` and :func:`silu_mul`
replace chains of small torch kernels with one launch each, with torch's rounding of the
same op sequence (see ``csrc/dcr_decode_ops.cu``). :func:`pack_linears` lets one library
GEMM compute several projections of the same input (q/k/v, gate/up).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import check_dtype, require

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


def silu_mul_packed(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up from one [..., 2 * inter] tensor holding gate then up (the output of
    one GEMM over the concatenated gate and up weights) -> [..., inter]."""
    _lib.require_cuda(gate_up)
    require(gate_up.is_contiguous() and gate_up.shape[-1] % 2 == 0,
            "gate_up must be contiguous with an even last dim")
    inter = gate_up.shape[-1] // 2
    rows = gate_up.numel() // gate_up.shape[-1]
    out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        st = _lib.load().dcr_silu_mul_packed(gate_up.data_ptr(), _dt(gate_up), rows, inter,
                                             out.data_ptr(), _lib.stream_ptr(gate_up.device))
    _lib.check(st, "dcr_silu_mul_packed")
    return out


def pack_linears(*layers: torch.nn.Linear) -> torch.Tensor:
    """Puts the weights of bias-free linear layers over one input into one [sum N, K]
    tensor and makes each layer's weight a view of its rows, so one GEMM computes all of
    them (weights loaded later, e.g. by load_state_dict, land in the packed tensor)."""
    K = layers[0].weight.shape[1]
    require(all(l.weight.shape[1] == K and l.bias is None for l in layers),
            "packed layers must share the input size and have no bias")
    w0 = layers[0].weight
    packed = torch.empty(sum(l.weight.shape[0] for l in layers), K, dtype=w0.dtype,
                         device=w0.device)
    r = 0
    with torch.no_grad():
        for l in layers:
            n = l.weight.shape[0]
            packed[r:r + n].copy_(l.weight)
            l.weight = torch.nn.Parameter(packed[r:r + n], requires_grad=l.weight.requires_grad)
            r += n
    return packed
