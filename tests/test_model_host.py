"""Host-side pieces of the Llama decode model (no GPU): the architecture constants and the
HF RMSNorm formula."""
from __future__ import annotations

import torch


def test_config_is_llama_3_2_1b():
    from dcr_b200.models.llama.model import LlamaDecodeConfig
    c = LlamaDecodeConfig()
    assert (c.vocab, c.hidden, c.intermediate, c.layers, c.heads, c.kv_heads) == \
        (128256, 2048, 8192, 16, 32, 8)
    assert c.rope_theta == 500000.0 and c.rms_eps == 1e-5
    assert c.hidden == c.heads * 64


def test_rmsnorm_is_hf_llama_rmsnorm():
    from dcr_b200.models.llama.model import RMSNorm
    torch.manual_seed(0)
    n = RMSNorm(64, 1e-5, torch.bfloat16, "cpu")
    with torch.no_grad():
        n.weight.copy_(torch.randn(64).to(torch.bfloat16))
    x = (torch.randn(3, 64) * 5).to(torch.bfloat16)
    # transformers' LlamaRMSNorm.forward, written out
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + 1e-5)
    want = n.weight * h.to(torch.bfloat16)
    assert torch.equal(n(x), want)


def test_rmsnorm_matches_transformers():
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    from dcr_b200.models.llama.model import RMSNorm
    torch.manual_seed(1)
    ours = RMSNorm(128, 1e-5, torch.bfloat16, "cpu")
    hf = LlamaRMSNorm(128, eps=1e-5).to(torch.bfloat16)
    w = torch.randn(128).to(torch.bfloat16)
    with torch.no_grad():
        ours.weight.copy_(w)
        hf.weight.copy_(w)
    x = (torch.randn(2, 3, 128) * 3).to(torch.bfloat16)
    assert torch.equal(ours(x), hf(x))
