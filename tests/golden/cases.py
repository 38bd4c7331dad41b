"""Golden-vector cases: shapes, seeds and the deterministic input construction.

Shared by ``make_golden.py`` (which runs the reference on these inputs, in the build
container) and the tests (which rebuild the same inputs from the same seeds with torch's
CPU generator and check them against the stored SHA-256 before use).
"""
from __future__ import annotations

import hashlib
import os
import sys

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "dcr-attention_v3_b200")
if _SRC not in sys.path:
    sys.path.insert(0, _SRC)

from dcr_b200.synthetic import make_decode_inputs  # noqa: E402

DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}

# name -> (B, H, H_kv, N, k_eff, dtype, seed, kind)
CASES = {
    # B=1, N=4096, 32/8 heads, fp32, c=0.15 -> k=614
    "config0_f32": (1, 32, 8, 4096, 614, "f32", 0, "synthetic"),
    "bf16_b2_n1000": (2, 32, 8, 1000, 500, "bf16", 42, "synthetic"),
    "bf16_n63": (1, 32, 8, 63, 31, "bf16", 7, "synthetic"),
    "bf16_n65": (1, 32, 8, 65, 32, "bf16", 7, "synthetic"),
    "bf16_n4096_c15": (1, 32, 8, 4096, 614, "bf16", 0, "synthetic"),
    "bf16_n8192_half": (1, 32, 8, 8192, 4096, "bf16", 100, "synthetic"),
    "f16_n2000": (1, 32, 8, 2000, 600, "f16", 100, "synthetic"),
    "f16_b2_n4096": (2, 32, 8, 4096, 614, "f16", 5, "synthetic"),
    "gqa1_bf16": (1, 4, 4, 300, 100, "bf16", 3, "synthetic"),
    "gqa2_bf16": (1, 8, 4, 500, 150, "bf16", 4, "synthetic"),
    "gqa8_bf16": (1, 16, 2, 700, 210, "bf16", 5, "synthetic"),
    "minimal_h4_hkv1": (1, 4, 1, 1000, 100, "bf16", 7, "synthetic"),
    "near_full_kNm1": (1, 32, 8, 100, 99, "bf16", 0, "synthetic"),
    "ties_bf16": (1, 8, 2, 1000, 300, "bf16", 11, "ties"),
    "zero_query_bf16": (1, 8, 2, 128, 40, "bf16", 12, "zero_query"),
}


def build_inputs(name: str):
    """(Q, K, V) for a case, in the case's dtype, on the CPU."""
    B, H, H_kv, N, k, dt, seed, kind = CASES[name]
    dtype = DTYPES[dt]
    Q, K, V = make_decode_inputs(B, H, H_kv, N, 64, dtype=dtype, seed=seed)
    if kind == "ties":
        # u = e_0 for every head, so score[n] = K[n, 0] exactly; K[n, 0] takes 4 values,
        # which puts hundreds of equal scores across every selection threshold.
        g = torch.Generator().manual_seed(seed + 1000)
        Q = torch.zeros(B, H, 64)
        Q[..., 0] = 1.0
        K = K.float()
        K[..., 0] = torch.randint(0, 4, (B, H_kv, N), generator=g).float() * 0.5
        Q, K = Q.to(dtype), K.to(dtype)
    elif kind == "zero_query":
        Q = Q.clone()
        Q[:, ::2] = 0  # every other head has an all-zero query (eps clamp path)
    return Q, K, V


def input_sha256(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in (Q, K, V):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes()
                 if t.dtype != torch.float32 else t.contiguous().numpy().tobytes())
    return h.hexdigest()


def fixture_path(name: str) -> str:
    return os.path.join(_HERE, f"{name}.npz")
