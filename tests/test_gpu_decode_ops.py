"""The decode-step kernels around the attention (csrc/dcr_decode_ops.cu) against torch:
residual add + HF LlamaRMSNorm, SiLU-gated product, and the skinny linear layer."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _hf_rmsnorm(x, w, eps):
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(x.dtype)


def _ulps_apart(a, b):
    """Distance in units of the last place of 16-bit floats of one sign."""
    ai = a.contiguous().view(torch.int16).int()
    bi = b.contiguous().view(torch.int16).int()
    return (ai - bi).abs()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm_matches_hf(dt, with_delta):
    from dcr_b200.kernel.cuda.decode_ops import add_rmsnorm
    g = torch.Generator(device=DEV).manual_seed(1)
    h = (torch.randn(4, 1, 2048, generator=g, device=DEV) * 3).to(dt)
    d = (torch.randn(4, 1, 2048, generator=g, device=DEV)).to(dt) if with_delta else None
    w = torch.randn(2048, generator=g, device=DEV).to(dt)
    h2, y = add_rmsnorm(h, d, w, 1e-5)
    h_ref = h + d if with_delta else h
    assert torch.equal(h2, h_ref)
    y_ref = _hf_rmsnorm(h_ref, w, 1e-5)
    # fp32 statistics summed in another order: rarely one ulp apart
    assert (y == y_ref).float().mean().item() >= 0.99
    assert _ulps_apart(y, y_ref).max().item() <= 1


def test_add_rmsnorm_in_place():
    from dcr_b200.kernel.cuda.decode_ops import add_rmsnorm
    h = torch.randn(3, 256, device=DEV).to(torch.bfloat16)
    d = torch.randn(3, 256, device=DEV).to(torch.bfloat16)
    want = h + d
    h2, _ = add_rmsnorm(h, d, torch.ones(256, device=DEV, dtype=torch.bfloat16), 1e-5, h_out=h)
    assert h2.data_ptr() == h.data_ptr() and torch.equal(h, want)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_silu_mul_matches_torch(dt):
    from dcr_b200.kernel.cuda.decode_ops import silu_mul
    g = torch.Generator(device=DEV).manual_seed(2)
    a = (torch.randn(4, 8192, generator=g, device=DEV) * 4).to(dt)
    b = torch.randn(4, 8192, generator=g, device=DEV).to(dt)
    got = silu_mul(a, b)
    want = F.silu(a) * b
    assert (got == want).float().mean().item() >= 0.999
    assert _ulps_apart(got, want).max().item() <= 1


@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("N,K", [(2048, 2048), (8192, 2048), (2048, 8192), (77, 512)])
def test_linear_skinny_matches_fp32_product(M, N, K):
    from dcr_b200.kernel.cuda.decode_ops import linear_skinny
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    got = linear_skinny(x, w).float()
    want = x.float() @ w.float().T
    tol = 1e-2 * want.abs().max().item() + 1e-3
    assert (got - want).abs().max().item() <= tol
    assert torch.allclose(got, F.linear(x, w).float(), rtol=2e-2, atol=tol)


def test_linear_skinny_rejects_unsupported_shapes():
    from dcr_b200 import _lib
    from dcr_b200.kernel.cuda.decode_ops import linear_skinny
    x = torch.randn(9, 512, device=DEV).to(torch.bfloat16)
    w = torch.randn(64, 512, device=DEV).to(torch.bfloat16)
    with pytest.raises(Exception):
        linear_skinny(x, w)                      # 9 rows
    lib = _lib.load()
    assert lib.dcr_linear_skinny(x.data_ptr(), w.data_ptr(), 0, 4, 64, 300, x.data_ptr(),
                                 None) == _lib.DCR_ERR_SHAPE  # K % 256 != 0
