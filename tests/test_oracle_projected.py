"""The projected-score oracle (CPU): its roundings and sums are checked against torch.

The reference has no projected mode, so these pin the restatement itself: the stored
projection rounds like torch's fp32 -> fp16 / bf16 conversions (round to nearest even,
subnormals, overflow to inf), and scores and the selection agree with a float64
computation up to the bf16 rounding of the scores.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import to_np


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dt,name", [(torch.float16, "f16"), (torch.bfloat16, "bf16")])
def test_projection_rounds_like_torch(oracle_mod, dt, name):
    g = torch.Generator().manual_seed(3)
    mags = torch.tensor([1e-7, 3e-6, 1e-4, 1e-2, 1.0, 50.0, 3e3, 6e4])
    x = torch.randn(64 * 4096, generator=g) * mags[torch.randint(0, 8, (64 * 4096,), generator=g)]
    K = x.clamp(-6e4, 6e4).to(dt).view(1, 1, 4096, 64)  # finite: inf * 0 would give NaN
    K = torch.where(K == 0, torch.ones_like(K), K)          # keep the sign of zero out of it
    c = torch.tensor([1 / 3, 3.7, 1e-3, 1.0e3, 0.999, 7.0, 1e-5, 20.0])
    P = torch.zeros(64, 16)
    P[0, :8] = c                                             # KP[..., j] = round(K[..., 0] * c_j)
    P[1, 8:] = c
    KP = oracle_mod.project_keys(to_np(K), name, P.numpy())
    want = torch.cat([(K[..., 0:1].float() * c).to(dt), (K[..., 1:2].float() * c).to(dt)], -1)
    assert np.array_equal(KP, _bits16(want))


def test_projection_f32_and_sums(oracle_mod):
    g = torch.Generator().manual_seed(4)
    K = torch.randn(2, 3, 100, 64, generator=g)
    P = torch.randn(64, 16, generator=g)
    KP = oracle_mod.project_keys(K.numpy(), "f32", P.numpy())
    ref = K.double() @ P.double()
    assert np.allclose(KP, ref.numpy(), rtol=1e-5, atol=1e-4)


def test_projected_scores_and_selection(oracle_mod):
    from dcr_b200.synthetic import make_decode_inputs, projection_matrix
    Q, K, V = make_decode_inputs(1, 8, 2, 700, dtype=torch.bfloat16, seed=8)
    P = projection_matrix(seed=0)
    KP = oracle_mod.project_keys(to_np(K), "bf16", P.numpy())
    qp, s, idx, O = oracle_mod.decode_projected(to_np(Q), to_np(K), to_np(V), KP, P.numpy(),
                                                "bf16", 106)
    # qp = u . P, with u the unit query
    u = Q.float() / Q.float().norm(dim=-1, keepdim=True)
    assert np.allclose(qp, (u.double() @ P.double()).numpy(), rtol=1e-5, atol=1e-5)
    # scores: bf16 of KP . qp, within one bf16 rounding of the float64 product
    kpf = torch.from_numpy(KP.view(np.int16)).view(torch.bfloat16).double()
    ref = torch.einsum("bknr,bkgr->bkgn", kpf, torch.from_numpy(qp).double().view(1, 2, 4, 16))
    got = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).double().view(1, 2, 4, 700)
    assert ((got - ref).abs() <= ref.abs() * 2 ** -8 + 1e-30).all()
    # selection: stable descending argsort of the scores, first k, ascending
    sf = got.view(8, 700).float()
    want = torch.sort(torch.argsort(-sf, dim=-1, stable=True)[:, :106], dim=-1).values
    assert np.array_equal(idx, want.numpy().astype(np.int32))
