"""Seeded synthetic decode inputs with the reference's measurement distribution.

There is no dataset or checkpoint here, so benchmarks and parity tests use Gaussian inputs
shaped like Llama-3.2-1B decode (H=32, H_kv=8, D=64) with the two features real caches have:
the keys of tokens 0-3 scaled x4 (attention sinks) and two random key channels scaled x6
(outlier channels). Drawing order (one generator): Q, K, V, then the outlier channels
(``randperm(D)[:2]``); then, for multi-step runs, one fresh Q per step.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

SINK_ROWS = 4
SINK_SCALE = 4.0
OUTLIER_CHANNELS = 2
OUTLIER_SCALE = 6.0


def outlier_channels(D: int = 64, seed: int = 0,
                     device: str | torch.device = "cpu") -> torch.Tensor:
    """The outlier key channels of a sequence (``randperm(D)[:2]`` of a seeded generator)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randperm(D, generator=g, device=device)[:OUTLIER_CHANNELS]


def make_decode_inputs(B: int, H: int, H_kv: int, N: int, D: int = 64,
                       dtype: torch.dtype = torch.bfloat16, seed: int = 0,
                       device: str | torch.device = "cpu",
                       generator: Optional[torch.Generator] = None,
                       sink_rows: int = SINK_ROWS,
                       channels: Optional[torch.Tensor] = None
                       ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(Q [B,H,D], K [B,H_kv,N,D], V [B,H_kv,N,D]) in ``dtype`` on ``device``.

    For one chunk of a longer sequence (a rank's share in a sequence split) pass the
    sequence's ``channels`` (``outlier_channels``) and ``sink_rows=0`` for every chunk but
    the first: a sequence has one set of outlier channels and its sinks at positions 0-3."""
    g = generator if generator is not None else torch.Generator(device=device).manual_seed(seed)
    Q = torch.randn(B, H, D, generator=g, device=device)
    K = torch.randn(B, H_kv, N, D, generator=g, device=device)
    V = torch.randn(B, H_kv, N, D, generator=g, device=device)
    K[:, :, :sink_rows, :] *= SINK_SCALE
    ch = channels if channels is not None else \
        torch.randperm(D, generator=g, device=device)[:OUTLIER_CHANNELS]
    K[..., ch] *= OUTLIER_SCALE
    return Q.to(dtype), K.to(dtype), V.to(dtype)


def fresh_queries(steps: int, B: int, H: int, D: int = 64, dtype: torch.dtype = torch.bfloat16,
                  seed: int = 1, device: str | torch.device = "cpu") -> torch.Tensor:
    """[steps, B, H, D] fresh N(0,1) queries (one per decode step)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(steps, B, H, D, generator=g, device=device).to(dtype)


def projection_matrix(D: int = 64, rank: int = 16, seed: int = 0,
                      device: str | torch.device = "cpu") -> torch.Tensor:
    """Seeded Gaussian projection P [D, rank] (fp32) for the projected-score mode."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(D, rank, generator=g, device=device)
