"""One decode step replayed as a CUDA graph, host buffers in and out.

The reference's hook calls its kernels from Python every step
(dcr_attention/models/llama/attention.py:805-813, kernel/triton/topk_axis.py:58): four
launches, argument checks and allocations per call. :class:`DecodeRunner` is the same
step for a serving loop that keeps its caches in place, on the library's native runner
(dcr_runner_create / dcr_runner_step): the copy of the step's query from pinned staging,
the three passes and the copy of O back are captured once into a CUDA graph, and a step is
one C call — a host copy into the staging, one graph launch, one synchronisation, a host
copy out. Inside the graph two small kernels move Q from the pinned staging to the device
and O back, reading and writing the mapped host buffers over the bus: copy-engine nodes
cost several microseconds each to start, a 16 KB kernel copy about one. The graph bakes in the cache tensors and the context length N: keep a runner per
length bucket (or make a new one when N changes).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import HEAD_DIM, cache_strides, check_dtype, check_k_range, require


class DecodeRunner:
    """``O = runner(q)``: the decode step of :func:`topk_qaxis_attention` (or of the
    projected mode when ``KP`` and ``P`` are given) over fixed caches, q and O on the host."""

    def __init__(self, K_cache: torch.Tensor, V_cache: torch.Tensor, k_eff: int, H: int, *,
                 KP: Optional[torch.Tensor] = None, P: Optional[torch.Tensor] = None,
                 eps: float = 1e-12):
        _lib.require_cuda(K_cache, V_cache)
        B, H_kv, N, D = K_cache.shape
        require(D == HEAD_DIM, f"head dim must be {HEAD_DIM}")
        require(tuple(V_cache.shape) == (B, H_kv, N, D) and V_cache.dtype == K_cache.dtype,
                "V_cache must match K_cache")
        require((KP is None) == (P is None), "give both KP and P, or neither")
        check_k_range(int(k_eff), N)
        dt = check_dtype(K_cache, "K_cache")
        ksb, ksh = cache_strides(K_cache, "K_cache")
        vsb, vsh = cache_strides(V_cache, "V_cache")
        psb = psh = 0
        if KP is not None:
            from dcr_b200.kernel.cuda.projected import check_projection, kp_strides
            check_projection(P, K_cache.device)
            psb, psh = kp_strides(KP)
        self.device = K_cache.device
        self.dtype = K_cache.dtype
        self.shape = torch.Size((B, H, HEAD_DIM))
        self._keep = (K_cache, V_cache, KP, P)  # the graph reads these buffers
        self._lib = _lib.load()
        self._step = self._lib.dcr_runner_step
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            st = self._lib.dcr_runner_create(
                K_cache.data_ptr(), V_cache.data_ptr(), None if KP is None else KP.data_ptr(),
                None if P is None else P.data_ptr(), dt, ksb, ksh, vsb, vsh, psb, psh, B, H,
                H_kv, N, HEAD_DIM, int(k_eff), float(eps), ctypes.byref(handle))
        _lib.check(st, "dcr_runner_create")
        self._h = handle.value
        n = B * H * HEAD_DIM
        esz = torch.empty(0, dtype=self.dtype).element_size()

        def pinned(ptr):  # a tensor view of the runner's own pinned buffer
            buf = (ctypes.c_uint8 * (n * esz)).from_address(ptr)
            return torch.frombuffer(buf, dtype=self.dtype).view(self.shape)

        self.q_host = pinned(self._lib.dcr_runner_query_buffer(self._h))
        self.o_host = pinned(self._lib.dcr_runner_output_buffer(self._h))

    def __call__(self, q: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Runs one step for the host query q [B, H, D]; returns O [B, H, D] on the host
        (``out`` if given, else a view of the runner's pinned buffer, valid until the next
        call)."""
        # the checks run on every step, so their messages are only formatted on failure
        if self._h is None:
            raise AssertionError("runner is closed")
        if not self._host_ok(q):
            raise AssertionError(f"q must be a contiguous host {self.dtype} {self.shape}")
        dst = self.o_host
        if out is not None:
            if not self._host_ok(out):
                raise AssertionError(f"out must be a contiguous host {self.dtype} {self.shape}")
            dst = out
        st = self._step(self._h, q.data_ptr(), dst.data_ptr())
        if st != 0:
            _lib.check(st, "dcr_runner_step")
        return dst

    def _host_ok(self, t: torch.Tensor) -> bool:
        return (t.shape == self.shape and t.dtype == self.dtype and not t.is_cuda and
                t.is_contiguous())

    def close(self) -> None:
        """Frees the runner (graph, stream, buffers); its pinned-buffer views die with it."""
        if self._h is not None:
            self.q_host = self.o_host = None
            self._lib.dcr_runner_destroy(self._h)
            self._h = None
        self._keep = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
