"""Loading golden fixtures and converting torch tensors for the oracle (test helper)."""
from __future__ import annotations

import json

import numpy as np
import torch

from cases import CASES, build_inputs, fixture_path, input_sha256


def load_case(name: str):
    """(meta, (Q, K, V) torch CPU tensors, fixture arrays dict)."""
    z = np.load(fixture_path(name))
    meta = json.loads(str(z["meta"]))
    Q, K, V = build_inputs(name)
    sha = input_sha256(Q, K, V)
    assert sha == meta["input_sha256"], (
        f"{name}: rebuilt inputs differ from the ones the golden vectors were made from "
        f"(torch {torch.__version__} vs {meta['torch']})")
    arrays = {k: z[k] for k in z.files if k != "meta"}
    return meta, (Q, K, V), arrays


def to_np(t: torch.Tensor) -> np.ndarray:
    """Raw bits (uint16) for 16-bit tensors, float32 for fp32 — the oracle's convention."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.float().numpy()


def dtype_name(t: torch.Tensor) -> str:
    return {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[t.dtype]


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def half_ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """Half an ulp of |x| in the given output dtype: the most one rounding can move it."""
    mant = {"bf16": 7, "f16": 10, "f32": 23}[dtype]
    a = np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -126)
    e = np.floor(np.log2(a))
    return 2.0 ** (e - mant - 1)


def attention_close(got: np.ndarray, want: np.ndarray, max_abs: float = 2e-3,
                    min_cos: float = 0.9999, got_rounded_to: str | None = None):
    """The north-star gate for attention outputs, against the reference's unrounded fp32
    output: max|d| <= 2e-3 and cosine >= 0.9999 per (b, h) row, plus the reference's own
    RMSE^2 <= 1e-6 (kernel_spec.md section 5.1.2). If ``got`` was rounded to a 16-bit
    output dtype, half an ulp of that dtype is added to the 2e-3 per element (the rounding
    the reference's own bf16 output also carries)."""
    g = got.reshape(-1, 64).astype(np.float64)
    w = want.reshape(-1, 64).astype(np.float64)
    d = np.abs(g - w)
    if got_rounded_to is not None and got_rounded_to != "f32":
        d = np.maximum(d - half_ulp(w, got_rounded_to), 0.0)
    cos = (g * w).sum(-1) / (np.linalg.norm(g, axis=-1) * np.linalg.norm(w, axis=-1) + 1e-30)
    stats = dict(max_abs=float(d.max()), min_cos=float(cos.min()), rmse2=float((d ** 2).mean()))
    ok = stats["max_abs"] <= max_abs and stats["min_cos"] >= min_cos and stats["rmse2"] <= 1e-6
    return ok, stats


ALL_CASES = list(CASES)
