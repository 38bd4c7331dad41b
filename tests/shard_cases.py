"""Seeded cases for the sharded decode tests (CPU gloo protocol tests and GPU parity).

A case is a full single-layer decode input (Q [B,H,D], K and V [B,H_kv,N,D]), the chunk
lengths of the ranks (sequence split, in rank order) and the global k_eff. The cases cover
the edges of the exact global top-K: ragged chunks, a chunk shorter than one 16-byte
vector, ties at the threshold that straddle a chunk boundary (the lowest-index rule across
ranks), a rank that contributes nothing, GQA groups 1/4/8, and every dtype.
"""
from __future__ import annotations

import torch

from dcr_b200.synthetic import make_decode_inputs

_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _k(N, c):
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    return adaptive_k_window(64, N, c)


# name -> (B, H, H_kv, splits, k_eff or coverage, dtype, kind)
CASES = {
    "bf16_2r": (1, 4, 1, [600, 400], 150, "bf16", "plain"),
    "f16_3r_ragged": (2, 8, 2, [700, 13, 787], 0.15, "f16", "plain"),
    "ties_2r": (1, 4, 1, [256, 256], 200, "bf16", "ties"),
    "gqa8_f32_4r": (1, 8, 1, [512, 512, 512, 512], 308, "f32", "plain"),
    "empty_rank_2r": (1, 1, 1, [400, 200], 100, "bf16", "empty_rank"),
    "gqa2_bf16_2r": (2, 4, 2, [1031, 997], 0.3, "bf16", "plain"),
    # a chunk longer than one CTA's 32768 keys: the peer step's accumulating phase kernels
    "long_2r": (1, 4, 1, [40000, 30008], 0.05, "bf16", "plain"),
}

CASES_BY_WORLD = {}
for _name, _c in CASES.items():
    CASES_BY_WORLD.setdefault(len(_c[3]), []).append(_name)


def make_case(name: str, seed: int = 5):
    """(Q, K, V, splits, k_eff) on the CPU."""
    B, H, H_kv, splits, kc, dtn, kind = CASES[name]
    N = sum(splits)
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.float32, seed=seed)
    if kind == "ties":
        # 312 identical key rows (100..411) that head 0 scores above everything else: with
        # k = 200 the threshold falls inside the tie group, across the chunk boundary at 256.
        v = Q[0, 0] / Q[0, 0].norm() * 12.0
        K[:, :, 100:412] = v
    elif kind == "empty_rank":
        # rank 1's keys point away from the query: it holds none of the top k
        K[0, 0, splits[0]:] = -Q[0, 0] / Q[0, 0].norm() * 8.0 + 0.01 * K[0, 0, splits[0]:]
    k = kc if isinstance(kc, int) else _k(N, kc)
    dt = _DT[dtn]
    return Q.to(dt), K.to(dt), V.to(dt), list(splits), k


def chunk(t: torch.Tensor, splits, rank: int) -> torch.Tensor:
    off = sum(splits[:rank])
    return t[:, :, off:off + splits[rank]].contiguous()
