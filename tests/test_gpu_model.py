"""The Llama decode model on the GPU: per-step CUDA graphs reproduce eager decode bit for
bit, the dense mode matches a plain-torch restatement of the decoder (HF RMSNorm, RoPE,
GQA attention, SwiGLU), and the sparse mode runs the three-pass step in every layer."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _small(attention="dcr", mode="exact", seed=0):
    from dcr_b200.models.llama.model import DCRLlamaDecoder, LlamaDecodeConfig
    cfg = LlamaDecodeConfig(vocab=1000, hidden=256, intermediate=512, layers=2, heads=4,
                            kv_heads=2)
    return DCRLlamaDecoder(cfg, attention=attention, mode=mode, T_dispatch=1024,
                           dtype=torch.bfloat16, device=DEV, seed=seed)


def _caches(model, B, N0, steps, P=None):
    caches = model.new_caches(B, N0 + steps + 1, P=P)
    model.prefill_synthetic(caches, N0, seed=11)
    return caches


@pytest.mark.parametrize("mode", ["exact", "projected"])
def test_graph_replay_matches_eager_decode(mode):
    from dcr_b200.models.llama.model import GreedyDecodeGraphs
    from dcr_b200.synthetic import projection_matrix
    B, N0, steps = 2, 3000, 4
    model = _small(mode=mode)
    P = projection_matrix(seed=0, device=DEV) if mode == "projected" else None
    ca, cb = _caches(model, B, N0, steps, P), _caches(model, B, N0, steps, P)
    first = torch.tensor([3, 7])
    # eager
    cos, sin = model.rope_table(N0 + steps)
    tok = first.to(DEV)
    eager = []
    for t in range(steps):
        logits = model.step(tok, ca, cos[N0 + t].expand(B, 64).contiguous(),
                            sin[N0 + t].expand(B, 64).contiguous())
        tok = logits.argmax(-1)
        eager.append(tok.cpu())
    # graphs
    runner = GreedyDecodeGraphs(model, cb, steps)
    got = runner.run(first)
    assert torch.equal(got, torch.stack(eager))
    assert all(c.length == N0 + steps for c in cb)
    for x, y in zip(ca, cb):
        assert torch.equal(x.K, y.K) and torch.equal(x.V, y.V)
    assert model.layers[0].self_attn.last_branch == "dcr"
    runner.close()


def _rotate_half(x):
    return torch.cat((-x[..., 32:], x[..., :32]), dim=-1)


def test_dense_step_matches_torch_restatement():
    """Dense mode against the decoder written out with torch ops (HF LlamaRMSNorm, HF RoPE,
    SDPA over the repeated KV heads, SwiGLU, tied head), from the same caches."""
    B, N0 = 2, 700
    model = _small(attention="dense")
    caches = _caches(model, B, N0, 1)
    K0 = [c.K.clone() for c in caches]
    V0 = [c.V.clone() for c in caches]
    tok = torch.tensor([5, 9], device=DEV)
    cos, sin = model.rope_table(N0 + 1)
    c1, s1 = cos[N0].expand(B, 64).contiguous(), sin[N0].expand(B, 64).contiguous()
    got = model.step(tok, caches, c1, s1).float()

    def rms(x, w, eps=1e-5):
        x32 = x.float()
        return w * (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)

    with torch.no_grad():
        h = model.embed_tokens(tok)
        for i, layer in enumerate(model.layers):
            a = layer.self_attn
            x = rms(h, layer.input_layernorm.weight)
            q = a.q_proj(x).view(B, 4, 64)
            k = a.k_proj(x).view(B, 2, 64)
            v = a.v_proj(x).view(B, 2, 64)
            q = q * c1[:, None] + _rotate_half(q) * s1[:, None]
            k = k * c1[:, None] + _rotate_half(k) * s1[:, None]
            K = torch.cat([K0[i], k[:, :, None]], dim=2).repeat_interleave(2, dim=1)
            V = torch.cat([V0[i], v[:, :, None]], dim=2).repeat_interleave(2, dim=1)
            o = F.scaled_dot_product_attention(q[:, :, None], K, V).reshape(B, 256)
            h = h + a.o_proj(o)
            x = rms(h, layer.post_attention_layernorm.weight)
            h = h + layer.down_proj(F.silu(layer.gate_proj(x)) * layer.up_proj(x))
        want = F.linear(rms(h, model.norm.weight), model.embed_tokens.weight).float()
    err = (got - want).abs().max().item()
    assert err <= 2e-2 * max(want.abs().max().item(), 1.0), err
    assert torch.equal(caches[0].K[:, :, :N0], K0[0])


def test_fused_kernels_match_the_torch_composition():
    """The model with the fused decode-step kernels (add_rmsnorm, silu_mul, skinny GEMMs)
    against the same weights run through torch's ops: the logits agree within bf16 noise."""
    from dcr_b200.models.llama.model import DCRLlamaDecoder, LlamaDecodeConfig
    B, N0 = 2, 3000
    cfg = LlamaDecodeConfig(vocab=1000, hidden=256, intermediate=512, layers=2, heads=4,
                            kv_heads=2)
    fast = DCRLlamaDecoder(cfg, T_dispatch=1024, device=DEV, seed=4, fast=True)
    slow = DCRLlamaDecoder(cfg, T_dispatch=1024, device=DEV, seed=4, fast=False)
    ca, cb = _caches(fast, B, N0, 1), _caches(slow, B, N0, 1)
    cos, sin = fast.rope_table(N0 + 1)
    c1, s1 = cos[N0].expand(B, 64).contiguous(), sin[N0].expand(B, 64).contiguous()
    tok = torch.tensor([11, 12], device=DEV)
    a = fast.step(tok, ca, c1, s1).float()
    b = slow.step(tok, cb, c1, s1).float()
    assert (a - b).abs().max().item() <= 3e-2 * max(b.abs().max().item(), 1.0)
