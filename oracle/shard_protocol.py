"""CPU restatement of the sequence-sharded decode step (TEST INFRASTRUCTURE ONLY).

Used by ``tests/`` as the per-rank compute of the sequence split when the collectives
run on CPU (``gloo``), and as the checker of the CUDA phases. The product path
(``dcr_b200``) never imports it.

The reference has no multi-GPU decode; the sharded step must reproduce its single-GPU
result: the selected set of ``_select_topk_indices``
(``dcr_attention/kernel/qaxis_topk_reference.py:91``, stable descending argsort, first
k) over the concatenated context, and ``_fused_softmax_attention`` (:148) over that set.
:class:`OracleSequenceShardStep` mirrors the four phases of the CUDA path
(``dcr_shard_score``, ``_refine``, ``_attend``, ``_combine``) with numpy:

* keys: the order-preserving 16-bit map of the bf16 scores (-0 -> +0, NaN -> 0xffff);
* phase 1: per-row 256-bin histogram of ``key >> 8``;
* phase 2: the bin BH holding the k-th largest key of the summed histogram; per-row
  histogram of ``key & 0xff`` over the local keys in BH;
* phase 3: T from the summed low-byte histograms, ``need = k - #{key > T}``, this rank's
  tie quota ``clamp(need - #{key == T on lower ranks}, 0, #{key == T here})``; the local
  selection and its attention state ``(m, l, o)`` with m in base-2 units of the scaled
  scores (``z * 0.125 * log2(e)``), as the CUDA kernels store it;
* phase 4: ``O = sum_r 2^{m_r - M} o_r / sum_r 2^{m_r - M} l_r``.

Tensors crossing the collectives are torch CPU tensors (int32 histograms, fp32 states).
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle

LOG2E = 1.4426950408889634


def order_keys(bits: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 keys of raw bf16 score bits (the CUDA kernels' map)."""
    b = np.asarray(bits, dtype=np.uint32) & 0xFFFF
    mag = b & 0x7FFF
    b = np.where(mag == 0, 0, b)
    key = np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)
    return np.where(mag > 0x7F80, 0xFFFF, key).astype(np.uint32)


def _find_bin(hist: np.ndarray, k: int):
    """Bin B (0..255, counted from the top) with #{above B} < k <= #{above B-1}, and
    #{above B}; (-1, 0) if the histogram holds fewer than k keys."""
    above = 0
    for b in range(255, -1, -1):
        c = int(hist[b])
        if above < k <= above + c:
            return b, above
        above += c
    return -1, 0


def _to_bits(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


class OracleSequenceShardStep:
    """One rank's share of a sequence-sharded step, on the CPU."""

    def __init__(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, k_eff: int,
                 eps: float = 1e-12):
        self.dtype_name = {torch.bfloat16: "bf16", torch.float16: "f16",
                           torch.float32: "f32"}[Q.dtype]
        self.Q, self.K, self.V = Q, K, V
        self.B, self.H, _ = Q.shape
        self.N = K.shape[2]
        self.G = self.H // K.shape[1]
        self.k = int(k_eff)
        q = _to_bits(Q)
        u = oracle.unit_query(q, self.dtype_name, eps)
        self.scores = oracle.scores(_to_bits(K), self.dtype_name, u)   # [rows, N] bf16 bits
        self.keys = order_keys(self.scores)
        self.rows = self.keys.shape[0]
        self.sel = None

    def score(self, out=None) -> torch.Tensor:
        h = np.zeros((self.rows, 256), dtype=np.int32)
        for r in range(self.rows):
            h[r] = np.bincount(self.keys[r] >> 8, minlength=256)
        return torch.from_numpy(h)

    def refine(self, hist_hi_sum: torch.Tensor, out=None) -> torch.Tensor:
        hs = hist_hi_sum.numpy()
        h = np.zeros((self.rows, 256), dtype=np.int32)
        self.bh = np.zeros(self.rows, dtype=np.int64)
        self.above = np.zeros(self.rows, dtype=np.int64)
        for r in range(self.rows):
            bh, above = _find_bin(hs[r], self.k)
            if bh < 0:
                raise ValueError("fewer than k_eff keys over all ranks")
            self.bh[r], self.above[r] = bh, above
            kr = self.keys[r]
            h[r] = np.bincount(kr[(kr >> 8) == bh] & 0xFF, minlength=256)
        return torch.from_numpy(h)

    def attend(self, hist_lo_all: torch.Tensor, world: int, rank: int,
               out=None) -> torch.Tensor:
        lo = hist_lo_all.numpy()                         # [world, rows, 256]
        state = np.zeros((self.rows, 66), dtype=np.float32)
        self.sel = []
        Qf = self.Q.float().numpy().reshape(self.rows, 64).astype(np.float64)
        Kf = self.K.float().numpy().astype(np.float64)
        Vf = self.V.float().numpy().astype(np.float64)
        H_kv = self.K.shape[1]
        for r in range(self.rows):
            bl, above_lo = _find_bin(lo[:, r].sum(axis=0), self.k - int(self.above[r]))
            T = (int(self.bh[r]) << 8) | bl
            need = self.k - int(self.above[r]) - above_lo
            eq_lower = int(lo[:rank, r, bl].sum())
            quota = max(0, min(need - eq_lower, int(lo[rank, r, bl])))
            kr = self.keys[r]
            gt = np.nonzero(kr > T)[0]
            eq = np.nonzero(kr == T)[0][:quota]
            sel = np.sort(np.concatenate([gt, eq])).astype(np.int64)
            self.sel.append(sel)
            if sel.size == 0:
                state[r, 0] = -np.inf
                continue
            b, h = divmod(r, self.H)
            kv = h // self.G
            z = (Kf[b, kv, sel] @ Qf[r]) * 0.125 * LOG2E
            m = z.max()
            p = np.exp2(z - m)
            state[r, 0] = m
            state[r, 1] = p.sum()
            state[r, 2:] = p @ Vf[b, kv, sel]
        assert H_kv * self.G == self.H
        return torch.from_numpy(state)

    def combine(self, states: torch.Tensor, out=None) -> torch.Tensor:
        s = states.numpy().astype(np.float64)            # [world, rows, 66]
        M = s[:, :, 0].max(axis=0)
        w = np.where(np.isneginf(s[:, :, 0]), 0.0, np.exp2(s[:, :, 0] - M[None]))
        L = (w * s[:, :, 1]).sum(axis=0)
        o = (w[:, :, None] * s[:, :, 2:]).sum(axis=0) / L[:, None]
        return torch.from_numpy(o.astype(np.float32).reshape(self.B, self.H, 64))

    def selection(self):
        return self.sel


def global_selection(scores_chunks, k: int) -> np.ndarray:
    """The reference's selection over the concatenated context: [rows, k] ascending."""
    return oracle.select(np.concatenate(scores_chunks, axis=1), k)
