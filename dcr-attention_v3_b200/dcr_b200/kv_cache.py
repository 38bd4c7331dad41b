"""Preallocated decode KV cache written in place (optionally with projected keys).

The reference's Llama hook keeps K and V in HF ``DynamicCache`` (dcr_attention/models/
llama/compat.py:208-254; attention.py:422), whose ``update`` concatenates the whole cache
with the new token every step (an O(N) copy), and then repeats or strides the KV heads
for the kernel (attention.py:425-426, :810-811). :class:`StaticKVCache` allocates
``[B, H_kv, N_max, D]`` K and V once and appends new tokens in place with one kernel
(dcr_cache_append), which also writes the rank-16 projected keys ``KP = K . P`` used by
the projected-score mode. The views it hands out (``K``, ``V``, ``KP``: the first
``length`` positions) are strided views that every kernel of this package accepts
without a copy.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import HEAD_DIM, cache_strides, check_dtype, require
from dcr_b200.kernel.cuda.projected import PROJ_RANK, check_projection, kp_strides


class StaticKVCache:
    """One layer's K/V (and projected-key) cache for ``B`` sequences of up to ``N_max``
    positions, filled from position 0 by :meth:`append`."""

    def __init__(self, B: int, H_kv: int, N_max: int, *, dtype: torch.dtype, device,
                 P: Optional[torch.Tensor] = None):
        self.device = torch.device(device)
        check_dtype(torch.empty(0, dtype=dtype), "cache")
        self.B, self.H_kv, self.N_max, self.dtype = B, H_kv, N_max, dtype
        shape = (B, H_kv, N_max, HEAD_DIM)
        self.k = torch.empty(shape, dtype=dtype, device=self.device)
        self.v = torch.empty(shape, dtype=dtype, device=self.device)
        self.P = check_projection(P, self.device) if P is not None else None
        self.kp = (torch.empty(B, H_kv, N_max, PROJ_RANK, dtype=dtype, device=self.device)
                   if P is not None else None)
        self.length = 0

    @property
    def K(self) -> torch.Tensor:
        return self.k[:, :, :self.length]

    @property
    def V(self) -> torch.Tensor:
        return self.v[:, :, :self.length]

    @property
    def KP(self) -> Optional[torch.Tensor]:
        return None if self.kp is None else self.kp[:, :, :self.length]

    def append(self, K_new: torch.Tensor, V_new: torch.Tensor) -> None:
        """Writes ``[B, H_kv, n_new, D]`` new keys and values (and their projections) at
        positions ``[length, length + n_new)``; stream-ordered, no synchronisation."""
        _lib.require_cuda(K_new, V_new)
        require(tuple(K_new.shape) == tuple(V_new.shape) and K_new.dim() == 4 and
                K_new.shape[0] == self.B and K_new.shape[1] == self.H_kv,
                f"K_new and V_new must be [{self.B}, {self.H_kv}, n_new, {HEAD_DIM}]")
        require(K_new.dtype == self.dtype and V_new.dtype == self.dtype,
                f"new rows must be {self.dtype}")
        n_new = K_new.shape[2]
        require(self.length + n_new <= self.N_max,
                f"cache full: {self.length} + {n_new} > N_max={self.N_max}")
        nsb, nsh = cache_strides(K_new, "K_new")
        require(cache_strides(V_new, "V_new") == (nsb, nsh) or n_new == 1 or
                V_new.stride() == K_new.stride(), "K_new and V_new must share strides")
        csb, csh = cache_strides(self.k, "K_cache")
        if self.kp is not None:
            psb, psh = kp_strides(self.kp)
            P_ptr, kp_ptr = self.P.data_ptr(), self.kp.data_ptr()
        else:
            psb = psh = 0
            P_ptr = kp_ptr = None
        with torch.cuda.device(self.device):
            st = _lib.load().dcr_cache_append(
                K_new.data_ptr(), V_new.data_ptr(), _lib.DTYPE_CODES[self.dtype], nsb, nsh,
                self.B, self.H_kv, n_new, HEAD_DIM, self.k.data_ptr(), self.v.data_ptr(), csb,
                csh, self.length, self.N_max, P_ptr, PROJ_RANK, kp_ptr, psb, psh,
                _lib.stream_ptr(self.device))
        _lib.check(st, "dcr_cache_append")
        self.length += n_new

    def append_rotated(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       cos: torch.Tensor, sin: torch.Tensor, *, want_qp: bool = False,
                       eps: float = 1e-12) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """The decode prologue of one step in one launch (dcr_decode_prologue_strided; q, k, v
        may be slices of one packed q/k/v row per batch entry): RoPE of the
        step's q [B, H, D] and k [B, H_kv, D] rows with the position embeddings cos, sin
        [B, D] (HF apply_rotary_pos_emb, dcr_attention/models/llama/compat.py:63), the
        rotated k and v appended at position ``length`` (with their projection when the
        cache keeps KP). Returns (rotated q [B, H, D], projected unit queries [B, H, 16]
        fp32 when ``want_qp`` and the cache has P, else None)."""
        _lib.require_cuda(q, k, v, cos, sin)
        B, H, D = q.shape
        require(D == HEAD_DIM and B == self.B and tuple(k.shape) == (B, self.H_kv, D) and
                tuple(v.shape) == (B, self.H_kv, D), "q [B, H, D], k and v [B, H_kv, D]")
        require(all(t.dtype == self.dtype for t in (q, k, v, cos, sin)),
                f"q, k, v, cos, sin must be {self.dtype}")
        require(tuple(cos.shape) == (B, D) and tuple(sin.shape) == (B, D), "cos, sin [B, D]")
        require(self.length < self.N_max, f"cache full: N_max={self.N_max}")

        def rows_ok(t):  # [B, h, D] with contiguous heads, any batch stride
            return t.stride(-1) == 1 and (t.shape[1] == 1 or t.stride(1) == D)
        if not rows_ok(q):
            q = q.contiguous()
        if not (rows_ok(k) and rows_ok(v) and k.stride(0) == v.stride(0)):
            k, v = k.contiguous(), v.contiguous()
        cos, sin = cos.contiguous(), sin.contiguous()
        q_out = torch.empty(B, H, D, dtype=q.dtype, device=q.device)
        qp = None
        if want_qp:
            require(self.P is not None, "want_qp needs a cache with a projection P")
            qp = torch.empty(B, H, PROJ_RANK, dtype=torch.float32, device=self.device)
        csb, csh = cache_strides(self.k, "K_cache")
        if self.kp is not None:
            psb, psh = kp_strides(self.kp)
            kp_ptr = self.kp.data_ptr()
        else:
            psb = psh = 0
            kp_ptr = None
        P_ptr = self.P.data_ptr() if self.P is not None else None
        with torch.cuda.device(self.device):
            st = _lib.load().dcr_decode_prologue_strided(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0) if B > 1 else 0,
                k.stride(0) if B > 1 else 0, cos.data_ptr(), sin.data_ptr(),
                _lib.DTYPE_CODES[self.dtype], B, H, self.H_kv, HEAD_DIM, q_out.data_ptr(),
                self.k.data_ptr(), self.v.data_ptr(), csb, csh, self.length, self.N_max, P_ptr,
                PROJ_RANK, kp_ptr, psb, psh, None if qp is None else qp.data_ptr(), float(eps),
                _lib.stream_ptr(self.device))
        _lib.check(st, "dcr_decode_prologue")
        self.length += 1
        return q_out, qp
