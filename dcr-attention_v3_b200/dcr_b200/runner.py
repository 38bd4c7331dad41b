"""One decode step replayed as a CUDA graph, host buffers in and out.

The reference's hook calls its kernels from Python every step
(dcr_attention/models/llama/attention.py:805-813, kernel/triton/topk_axis.py:58): four
launches, argument checks and allocations per call. :class:`DecodeRunner` is the same
step for a serving loop that keeps its caches in place: the copy of the step's query from
a pinned host buffer, the three passes and the copy of O back to a pinned host buffer are
captured once into a CUDA graph and replayed per step, so a step costs one graph launch
and one synchronisation on the host. The graph bakes in the cache tensors and the context
length N: capture a runner per length bucket (or re-capture when N changes).
"""
from __future__ import annotations

from typing import Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import HEAD_DIM, check_k_range, require, workspace_bytes


class DecodeRunner:
    """``O = runner(q_host)``: the decode step of :func:`topk_qaxis_attention` (or of the
    projected mode when ``KP`` and ``P`` are given) over fixed caches."""

    def __init__(self, K_cache: torch.Tensor, V_cache: torch.Tensor, k_eff: int, H: int, *,
                 KP: Optional[torch.Tensor] = None, P: Optional[torch.Tensor] = None,
                 eps: float = 1e-12):
        from dcr_b200.kernel.cuda.projected import topk_qaxis_attention_projected
        from dcr_b200.kernel.cuda.topk_axis import topk_qaxis_attention

        _lib.require_cuda(K_cache, V_cache)
        B, H_kv, N, D = K_cache.shape
        require(D == HEAD_DIM, f"head dim must be {HEAD_DIM}")
        check_k_range(int(k_eff), N)
        self.device = K_cache.device
        self.dtype = K_cache.dtype
        self.shape = (B, H, HEAD_DIM)
        self.q_host = torch.empty(self.shape, dtype=self.dtype).pin_memory()
        self.o_host = torch.empty(self.shape, dtype=self.dtype).pin_memory()
        self.q_dev = torch.zeros(self.shape, dtype=self.dtype, device=self.device)
        self.o_dev = torch.empty(self.shape, dtype=self.dtype, device=self.device)
        self.ws = torch.empty(workspace_bytes(B, H, H_kv, N, k_eff), dtype=torch.uint8,
                              device=self.device)

        def step():
            self.q_dev.copy_(self.q_host, non_blocking=True)
            if KP is not None:
                topk_qaxis_attention_projected(self.q_dev, K_cache, V_cache, KP, P, k_eff,
                                               eps=eps, out=self.o_dev, workspace_buf=self.ws)
            else:
                topk_qaxis_attention(self.q_dev, K_cache, V_cache, k_eff, eps=eps,
                                     out=self.o_dev, workspace_buf=self.ws)
            self.o_host.copy_(self.o_dev, non_blocking=True)

        self.stream = torch.cuda.Stream(self.device)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            step()  # warm-up outside the capture (one-time setup inside the library)
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                step()

    def __call__(self, q: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Runs one step for the host query q [B, H, D]; returns O [B, H, D] on the host
        (``out`` if given, else a view of the runner's pinned buffer, valid until the next
        call)."""
        require(tuple(q.shape) == self.shape and q.dtype == self.dtype,
                f"q must be {self.dtype} {self.shape}")
        self.q_host.copy_(q)
        with torch.cuda.stream(self.stream):  # replay() launches on the current stream
            self.graph.replay()
        self.stream.synchronize()
        if out is not None:
            out.copy_(self.o_host)
            return out
        return self.o_host

    def close(self) -> None:
        self.graph = None
