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


def test_tensor_parallel_shards_cover_the_full_model():
    """Each rank's TP shard holds its slice of the unsplit weights (CPU, no kernels run): the
    concatenated q/k/v/gate/up rows and o/down columns of the ranks give back the full
    layer, KV heads [r*H_kv/W, (r+1)*H_kv/W) are rank r's, replicated tensors are equal."""
    from dcr_b200.models.llama.model import (DCRLlamaDecoder, LlamaDecodeConfig,
                                              TPDCRLlamaDecoder)
    cfg = LlamaDecodeConfig(vocab=300, hidden=256, intermediate=512, layers=2, heads=4,
                            kv_heads=2)
    full = DCRLlamaDecoder(cfg, device="cpu", seed=3)
    world = 2
    shards = [TPDCRLlamaDecoder(cfg, world=world, rank=r, device="cpu", seed=9).load_from(full)
              for r in range(world)]
    assert [list(s.kv_heads_held()) for s in shards] == [[0], [1]]
    for i, layer in enumerate(full.layers):
        ls = [s.layers[i] for s in shards]
        cat0 = lambda f: torch.cat([f(l) for l in ls], dim=0)  # noqa: E731
        cat1 = lambda f: torch.cat([f(l) for l in ls], dim=1)  # noqa: E731
        a = layer.self_attn
        assert torch.equal(cat0(lambda l: l.self_attn.q_proj.weight), a.q_proj.weight)
        assert torch.equal(cat0(lambda l: l.self_attn.k_proj.weight), a.k_proj.weight)
        assert torch.equal(cat0(lambda l: l.self_attn.v_proj.weight), a.v_proj.weight)
        assert torch.equal(cat1(lambda l: l.self_attn.o_proj.weight), a.o_proj.weight)
        assert torch.equal(cat0(lambda l: l.gate_proj.weight), layer.gate_proj.weight)
        assert torch.equal(cat0(lambda l: l.up_proj.weight), layer.up_proj.weight)
        assert torch.equal(cat1(lambda l: l.down_proj.weight), layer.down_proj.weight)
        for l in ls:
            # packed storage: the q/k/v and gate/up weights are views of one tensor each
            assert l.self_attn.q_proj.weight.data_ptr() == l.self_attn._qkv.data_ptr()
            assert l.gate_proj.weight.data_ptr() == l._gate_up.data_ptr()
    for s in shards:
        assert torch.equal(s.embed_tokens.weight, full.embed_tokens.weight)
