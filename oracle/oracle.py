"""CPU oracle for DCR-Attention's sparse decode attention (ctypes wrapper of dcr_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker used by ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s ``cpu_baseline`` leg. The product path (``dcr_b200``) never imports it.

Every function takes and returns numpy arrays. 16-bit tensors are passed as their raw bits
(``uint16``) with a dtype name (``"bf16"``, ``"f16"``), fp32 tensors as ``float32``.
Each function restates one step of the reference's oracle
(Seqev/dcr-attention_v3, ``dcr_attention/kernel/qaxis_topk_reference.py``):

===================  =================================  ==========================
function             reference step                     file:line
===================  =================================  ==========================
``unit_query``       ``_compute_u_Q``                   qaxis_topk_reference.py:42
``scores``           ``_compute_projection_scores``     qaxis_topk_reference.py:58
``select``           ``_select_topk_indices``           qaxis_topk_reference.py:91
``attend``           ``_gather_kv`` +                   qaxis_topk_reference.py:111,
                     ``_fused_softmax_attention``       :148
``decode``           ``topk_qaxis_attention_reference`` qaxis_topk_reference.py:200
===================  =================================  ==========================

The sums of ``unit_query`` and ``scores`` follow the CUDA kernels' order (documented in
``dcr_oracle.c``), so their outputs are bit-identical to the kernels'. They differ from the
reference's torch einsum only where torch's own summation order rounds differently (at
most one bf16 ulp, measured in ``tests/test_oracle_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_DTYPES = {"bf16": 0, "f16": 1, "f32": 2}
_lib = None


def build(force: bool = False) -> str:
    """Compile dcr_oracle.c into oracle/build/liboracle.so (gcc, OpenMP)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "dcr_oracle.c"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "all"], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        lib.oracle_unit_query.argtypes = [vp, i32, i32, f32, vp]
        lib.oracle_unit_query.restype = None
        lib.oracle_scores.argtypes = [vp, i32, i64, i64, vp, i32, i32, i32, i32, vp, i64]
        lib.oracle_scores.restype = None
        lib.oracle_select.argtypes = [vp, i64, i32, i32, i32, vp]
        lib.oracle_select.restype = i32
        lib.oracle_attend.argtypes = [vp, vp, vp, i32, i64, i64, i64, i64, vp, i32, i32, i32,
                                      i32, i32, i32, vp]
        lib.oracle_attend.restype = None
        lib.oracle_project_keys.argtypes = [vp, i32, i64, i64, i32, i32, i32, vp, i32, vp, i64,
                                            i64]
        lib.oracle_project_keys.restype = None
        lib.oracle_query_projection.argtypes = [vp, i32, vp, i32, vp]
        lib.oracle_query_projection.restype = None
        lib.oracle_scores_projected.argtypes = [vp, i32, i64, i64, vp, i32, i32, i32, i32, i32,
                                                vp, i64]
        lib.oracle_scores_projected.restype = None
        lib.oracle_adaptive_k_window.argtypes = [i32, i32, ctypes.c_double]
        lib.oracle_adaptive_k_window.restype = i32
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _check(a: np.ndarray, dtype: str) -> np.ndarray:
    want = np.float32 if dtype == "f32" else np.uint16
    a = np.ascontiguousarray(a)
    assert a.dtype == want, f"{dtype} tensors are passed as {want.__name__}, got {a.dtype}"
    return a


def unit_query(Q: np.ndarray, dtype: str, eps: float = 1e-12) -> np.ndarray:
    """u = f32(Q) / max(||f32(Q)||, eps); Q [..., 64] -> float32 of the same shape."""
    Q = _check(Q, dtype)
    rows = Q.size // 64
    u = np.empty(Q.shape, dtype=np.float32)
    _load().oracle_unit_query(_ptr(Q), _DTYPES[dtype], rows, eps, _ptr(u))
    return u


def scores(K: np.ndarray, dtype: str, u: np.ndarray) -> np.ndarray:
    """bf16 projection scores (raw bits) [B*H, N] from K [B, H_kv, N, 64] and u [B, H, 64]."""
    K = _check(K, dtype)
    u = np.ascontiguousarray(u, dtype=np.float32)
    B, H_kv, N, D = K.shape
    H = u.shape[1]
    assert D == 64 and H % H_kv == 0
    out = np.empty((B * H, N), dtype=np.uint16)
    _load().oracle_scores(_ptr(K), _DTYPES[dtype], H_kv * N * 64, N * 64, _ptr(u), B, H, H_kv,
                          N, _ptr(out), N)
    return out


def select(scores_bits: np.ndarray, k: int) -> np.ndarray:
    """Top-k indices [rows, k] int32 ascending; ties go to the lower index."""
    s = np.ascontiguousarray(scores_bits, dtype=np.uint16)
    rows, N = s.reshape(-1, s.shape[-1]).shape
    out = np.empty((rows, k), dtype=np.int32)
    bad = _load().oracle_select(_ptr(s), N, rows, N, k, _ptr(out))
    if bad:
        raise ValueError(f"oracle_select failed for N={N}, k={k}")
    return out


def attend(Q: np.ndarray, K: np.ndarray, V: np.ndarray, dtype: str, idx: np.ndarray,
           tile: int = 64) -> np.ndarray:
    """fp32 attention output [B, H, 64] over the rows idx [B*H, k] (64-key online softmax)."""
    Q, K, V = _check(Q, dtype), _check(K, dtype), _check(V, dtype)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    B, H, _ = Q.shape
    _, H_kv, N, _ = K.shape
    k = idx.shape[-1]
    O = np.empty((B, H, 64), dtype=np.float32)
    _load().oracle_attend(_ptr(Q), _ptr(K), _ptr(V), _DTYPES[dtype], H_kv * N * 64, N * 64,
                          H_kv * N * 64, N * 64, _ptr(idx), B, H, H_kv, N, k, tile, _ptr(O))
    return O


def decode(Q: np.ndarray, K: np.ndarray, V: np.ndarray, dtype: str, k: int,
           eps: float = 1e-12):
    """Full step: returns (u, score bits, indices, fp32 output)."""
    N = K.shape[2]
    if N <= k:
        raise ValueError(f"kernel invoked with N={N} <= k_eff={k}; caller must dispatch to SDPA")
    u = unit_query(Q, dtype, eps)
    s = scores(K, dtype, u)
    idx = select(s, k)
    O = attend(Q, K, V, dtype, idx)
    return u, s, idx, O


# ---- projected-score mode (no counterpart in the reference) -------------------------
def project_keys(K: np.ndarray, dtype: str, P: np.ndarray) -> np.ndarray:
    """KP [B, H_kv, N, R] in K's storage (bits for 16-bit types): round(K . P)."""
    K = _check(K, dtype)
    P = np.ascontiguousarray(P, dtype=np.float32)
    B, H_kv, N, D = K.shape
    R = P.shape[1]
    assert D == 64 and P.shape[0] == 64
    KP = np.empty((B, H_kv, N, R), dtype=K.dtype)
    _load().oracle_project_keys(_ptr(K), _DTYPES[dtype], H_kv * N * 64, N * 64, B, H_kv, N,
                                _ptr(P), R, _ptr(KP), H_kv * N * R, N * R)
    return KP


def query_projection(u: np.ndarray, P: np.ndarray) -> np.ndarray:
    """qp [..., R] = u . P (fp32)."""
    u = np.ascontiguousarray(u, dtype=np.float32)
    P = np.ascontiguousarray(P, dtype=np.float32)
    R = P.shape[1]
    rows = u.size // 64
    qp = np.empty(u.shape[:-1] + (R,), dtype=np.float32)
    _load().oracle_query_projection(_ptr(u), rows, _ptr(P), R, _ptr(qp))
    return qp


def scores_projected(KP: np.ndarray, dtype: str, qp: np.ndarray) -> np.ndarray:
    """bf16 score bits [B*H, N] from KP [B, H_kv, N, R] and qp [B, H, R]."""
    KP = _check(KP, dtype)
    qp = np.ascontiguousarray(qp, dtype=np.float32)
    B, H_kv, N, R = KP.shape
    H = qp.shape[1]
    out = np.empty((B * H, N), dtype=np.uint16)
    _load().oracle_scores_projected(_ptr(KP), _DTYPES[dtype], H_kv * N * R, N * R, _ptr(qp), R,
                                    B, H, H_kv, N, _ptr(out), N)
    return out


def decode_projected(Q, K, V, KP, P, dtype: str, k: int, eps: float = 1e-12):
    """Projected-mode step: (qp, score bits, indices, fp32 output)."""
    N = K.shape[2]
    if N <= k:
        raise ValueError(f"kernel invoked with N={N} <= k_eff={k}; caller must dispatch to SDPA")
    qp = query_projection(unit_query(Q, dtype, eps), P)
    s = scores_projected(KP, dtype, qp)
    idx = select(s, k)
    O = attend(Q, K, V, dtype, idx)
    return qp, s, idx, O


def adaptive_k_window(k_window_min: int, n_kv: int, coverage_floor: float) -> int:
    return int(_load().oracle_adaptive_k_window(k_window_min, n_kv, coverage_floor))


# ---- bit helpers (numpy) ------------------------------------------------------------
def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (torch's .to(torch.bfloat16))."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r
