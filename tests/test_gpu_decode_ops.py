"""The decode-step kernels around the attention (csrc/dcr_decode_ops.cu) against torch:
residual add + HF LlamaRMSNorm, the SiLU-gated product (plain and from packed gate/up
weights), and the prologue reading q/k/v as strided slices of one packed GEMM output."""
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


def test_silu_mul_packed_and_packed_linears():
    from dcr_b200.kernel.cuda.decode_ops import pack_linears, silu_mul_packed
    g = torch.Generator(device=DEV).manual_seed(4)
    gate = torch.nn.Linear(512, 1024, bias=False, device=DEV, dtype=torch.bfloat16)
    up = torch.nn.Linear(512, 1024, bias=False, device=DEV, dtype=torch.bfloat16)
    wg, wu = gate.weight.detach().clone(), up.weight.detach().clone()
    packed = pack_linears(gate, up)
    assert torch.equal(gate.weight, wg) and torch.equal(up.weight, wu)
    assert gate.weight.data_ptr() == packed.data_ptr()
    x = torch.randn(3, 512, generator=g, device=DEV).to(torch.bfloat16)
    gu = F.linear(x, packed)
    got = silu_mul_packed(gu)
    want = F.silu(gu[:, :1024].contiguous()) * gu[:, 1024:].contiguous()
    assert torch.equal(got, want) or _ulps_apart(got, want).max().item() <= 1
    with torch.no_grad():
        up.weight.mul_(2)   # writes land in the packed tensor
    assert torch.equal(packed[1024:], 2 * wu)


def test_prologue_reads_packed_qkv_slices():
    """append_rotated on q/k/v views into one [B, (H + 2 H_kv) D] GEMM output gives the
    same cache rows and rotated query as on contiguous copies."""
    from dcr_b200.kv_cache import StaticKVCache
    from dcr_b200.models.llama.attention import llama3_inv_freq, rope_cos_sin
    B, H, H_kv, D = 3, 8, 2, 64
    g = torch.Generator(device=DEV).manual_seed(6)
    qkv = torch.randn(B, (H + 2 * H_kv) * D, generator=g, device=DEV).to(torch.bfloat16)
    q = qkv[:, :H * D].view(B, H, D)
    k = qkv[:, H * D:(H + H_kv) * D].view(B, H_kv, D)
    v = qkv[:, (H + H_kv) * D:].view(B, H_kv, D)
    cos, sin = rope_cos_sin(torch.tensor([5, 6, 7], device=DEV), llama3_inv_freq().to(DEV),
                            torch.bfloat16)
    a = StaticKVCache(B, H_kv, 16, dtype=torch.bfloat16, device=DEV)
    b = StaticKVCache(B, H_kv, 16, dtype=torch.bfloat16, device=DEV)
    a.length = b.length = 4
    qa, _ = a.append_rotated(q, k, v, cos, sin)
    qb, _ = b.append_rotated(q.contiguous(), k.contiguous(), v.contiguous(), cos, sin)
    assert torch.equal(qa, qb)
    assert torch.equal(a.k[:, :, 4], b.k[:, :, 4]) and torch.equal(a.v[:, :, 4], b.v[:, :, 4])
