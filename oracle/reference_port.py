"""numpy restatement of the reference's CPU implementation of the hot path.

TEST INFRASTRUCTURE ONLY: ``bench.py --impl reference`` times it (the reference itself is
Python and cannot travel to the GPU box), and ``tests/`` pin it against the reference's
golden vectors. The product path never imports it.

It mirrors ``topk_qaxis_attention_reference``
(Seqev/dcr-attention_v3, ``dcr_attention/kernel/qaxis_topk_reference.py:200``) op for op:

* ``compute_u_Q``          - ``_compute_u_Q`` (:42): fp32 norm, clamp at eps, divide.
* ``compute_projection_scores`` - ``_compute_projection_scores`` (:58): per KV head an fp32
  ``einsum('bnd,bhd->bnh')`` (here a BLAS matmul), rounded to bf16.
* ``select_topk_indices``  - ``_select_topk_indices`` (:91): stable descending argsort,
  first k, re-sorted ascending.
* ``gather_kv`` / ``fused_softmax_attention`` - ``_gather_kv`` (:111) and
  ``_fused_softmax_attention`` (:148): 64-key tiles, fp32 (m, l, o), unnormalised Q.

The BLAS summation order differs from torch's, so single scores may differ by one bf16 ulp
from the reference's; tests/test_oracle_golden.py bounds that.
"""
from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from oracle.oracle import f32_to_bf16_bits, bf16_bits_to_f32  # noqa: F401


def compute_u_Q(Q: np.ndarray, eps: float = 1e-12) -> np.ndarray:
    q = np.asarray(Q, dtype=np.float32)
    n = np.linalg.norm(q, axis=-1, keepdims=True).astype(np.float32)
    return q / np.maximum(n, np.float32(eps))


def _scores_group(K_g: np.ndarray, u_g: np.ndarray) -> np.ndarray:
    # K_g [N, D] fp32, u_g [G, D] fp32 -> bf16 bits [G, N]
    s = u_g @ K_g.T
    return f32_to_bf16_bits(s)


def compute_projection_scores(K: np.ndarray, u: np.ndarray, pool=None) -> np.ndarray:
    """K [B, H_kv, N, D] fp32, u [B, H, D] fp32 -> bf16 bits [B, H, N]."""
    B, H_kv, N, D = K.shape
    H = u.shape[1]
    G = H // H_kv
    out = np.empty((B, H, N), dtype=np.uint16)
    jobs = [(b, hk) for b in range(B) for hk in range(H_kv)]

    def run(job):
        b, hk = job
        out[b, hk * G:(hk + 1) * G] = _scores_group(K[b, hk], u[b, hk * G:(hk + 1) * G])

    if pool is None:
        for j in jobs:
            run(j)
    else:
        list(pool.map(run, jobs))
    return out


def select_topk_indices(scores_bits: np.ndarray, k: int, pool=None) -> np.ndarray:
    """bf16 bits [B, H, N] -> int64 [B, H, k] ascending (stable descending argsort)."""
    s = bf16_bits_to_f32(scores_bits)
    B, H, N = s.shape
    out = np.empty((B, H, k), dtype=np.int64)

    def run(bh):
        b, h = divmod(bh, H)
        order = np.argsort(-s[b, h], kind="stable")[:k]
        out[b, h] = np.sort(order)

    if pool is None:
        for bh in range(B * H):
            run(bh)
    else:
        list(pool.map(run, range(B * H)))
    return out


def fused_softmax_attention(K_sel: np.ndarray, V_sel: np.ndarray, Q: np.ndarray,
                            B_block: int = 64) -> np.ndarray:
    """K_sel, V_sel [B, H, k, D] fp32, Q [B, H, D] fp32 -> fp32 [B, H, D]."""
    B, H, k, D = K_sel.shape
    scale = np.float32(1.0 / math.sqrt(D))
    m = np.full((B, H), -np.inf, dtype=np.float32)
    l = np.zeros((B, H), dtype=np.float32)
    o = np.zeros((B, H, D), dtype=np.float32)
    q = Q.astype(np.float32)
    for t0 in range(0, k, B_block):
        t1 = min(t0 + B_block, k)
        Kb = K_sel[:, :, t0:t1]
        Vb = V_sel[:, :, t0:t1]
        z = np.einsum("bhd,bhjd->bhj", q, Kb).astype(np.float32) * scale
        m_new = np.maximum(m, z.max(axis=-1))
        alpha = np.exp(m - m_new)
        beta = np.exp(z - m_new[..., None])
        l = alpha * l + beta.sum(axis=-1)
        o = alpha[..., None] * o + np.einsum("bhj,bhjd->bhd", beta, Vb)
        m = m_new
    return (o / l[..., None]).astype(np.float32)


def topk_qaxis_attention_reference(Q: np.ndarray, K: np.ndarray, V: np.ndarray, k: int,
                                   eps: float = 1e-12, threads: int = 1):
    """Full step on fp32 arrays (exact widenings of the stored dtype).

    Returns (scores bits [B,H,N], indices int64 [B,H,k], O fp32 [B,H,D]).
    """
    B, H, D = Q.shape
    _, H_kv, N, _ = K.shape
    if N <= k:
        raise ValueError(f"kernel invoked with N={N} <= k_eff={k}; caller must dispatch to SDPA")
    G = H // H_kv
    pool = ThreadPoolExecutor(threads) if threads > 1 else None
    try:
        u = compute_u_Q(Q, eps)
        s = compute_projection_scores(K, u, pool)
        idx = select_topk_indices(s, k, pool)
        # gather per query head from its KV head
        hk = np.arange(H) // G
        K_sel = K[np.arange(B)[:, None, None], hk[None, :, None], idx]
        V_sel = V[np.arange(B)[:, None, None], hk[None, :, None], idx]
        O = fused_softmax_attention(K_sel, V_sel, Q)
    finally:
        if pool is not None:
            pool.shutdown()
    return s, idx, O
