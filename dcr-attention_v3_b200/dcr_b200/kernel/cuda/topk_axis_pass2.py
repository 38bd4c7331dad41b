"""Pass 2 — exact top-K selection on the B200 (CUDA, sm_100a).

Drop-in for ``topk_pass2_select``
(Seqev/dcr-attention_v3, dcr_attention/kernel/triton/topk_axis_pass2.py:16): the k_eff
positions a stable descending argsort of ``f32(scores)`` puts first (ties -> lower
index), returned in ascending order as int32. The kernel (csrc/dcr_select.cu) finds the
k-th largest 16-bit key by radix select and emits the set in index order, with no sort.
Past one wave of rows (B x H x N above 148 x 32768) the same selection runs as chunked
grid-wide kernels (csrc/dcr_select_stream.cu) over a workspace allocated here.
"""
from __future__ import annotations

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import check_k_range, require


def topk_pass2_select(
    scores: torch.Tensor,    # [B, H, N] bf16 (from Pass 1)
    k_eff: int,
) -> torch.Tensor:           # [B, H, k_eff] int32, sorted ascending
    """Top-k_eff indices per (b, h) row, ties broken by lower index, ascending."""
    _lib.require_cuda(scores)
    require(scores.dim() == 3, f"scores must be [B, H, N], got {tuple(scores.shape)}")
    B, H, N = scores.shape
    require(scores.dtype == torch.bfloat16, f"scores must be bf16, got {scores.dtype}")
    check_k_range(int(k_eff), N)
    s = scores if (scores.stride(-1) == 1 and scores.stride(0) == H * scores.stride(1)) \
        else scores.contiguous()
    stride = s.stride(1)
    idx = torch.empty(B, H, k_eff, dtype=torch.int32, device=scores.device)
    lib = _lib.load()
    ws_bytes = int(lib.dcr_select_workspace_bytes(B * H, N))
    with torch.cuda.device(scores.device):
        if ws_bytes == 0:
            st = lib.dcr_select(s.data_ptr(), stride, B * H, N, int(k_eff), idx.data_ptr(),
                                _lib.stream_ptr(scores.device))
        else:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=scores.device)
            st = lib.dcr_select_ws(s.data_ptr(), stride, B * H, N, int(k_eff), idx.data_ptr(),
                                   ws.data_ptr(), ws_bytes, _lib.stream_ptr(scores.device))
    _lib.check(st, "dcr_select_ws" if ws_bytes else "dcr_select")
    return idx
