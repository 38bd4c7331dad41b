"""The decode layer on the GPU: the fused prologue (RoPE, cache append, projections) bit for
bit against torch's RoPE ops and the oracle, and the layer's decode step against the
reference's decode path (projections, HF RoPE, cache, routing, top-K attention, o_proj)
computed with torch and the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import attention_close, dtype_name, to_np

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _rotate_half(x):
    return torch.cat((-x[..., 32:], x[..., :32]), dim=-1)


def _hf_rope(x, cos, sin):
    """HF apply_rotary_pos_emb for one row per (batch, head): x [B, h, D], cos/sin [B, D]."""
    return x * cos[:, None] + _rotate_half(x) * sin[:, None]


def _cos_sin(B, pos, dt):
    from dcr_b200.models.llama.attention import llama3_inv_freq, rope_cos_sin
    return rope_cos_sin(torch.tensor([pos + 17 * b for b in range(B)]), llama3_inv_freq(), dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_prologue_bit_exact(oracle_mod, cuda_lib, dt):
    from dcr_b200 import _lib
    from dcr_b200.kv_cache import StaticKVCache
    from dcr_b200.synthetic import projection_matrix
    B, H, H_kv, N_max, pos = 3, 16, 4, 300, 123
    g = torch.Generator().manual_seed(5)
    q = (torch.randn(B, H, 64, generator=g) * 3).to(dt)
    k = (torch.randn(B, H_kv, 64, generator=g) * 3).to(dt)
    v = torch.randn(B, H_kv, 64, generator=g).to(dt)
    cos, sin = _cos_sin(B, pos, dt)
    P = projection_matrix(seed=0)
    cache = StaticKVCache(B, H_kv, N_max, dtype=dt, device=DEV, P=P.to(DEV))
    cache.length = pos
    q_rot, qp = cache.append_rotated(q.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV),
                                     want_qp=True)
    assert _lib.read_device_status(clear=True) == 0
    q_ref, k_ref = _hf_rope(q, cos, sin), _hf_rope(k, cos, sin)
    assert torch.equal(q_rot.cpu(), q_ref)
    assert torch.equal(cache.k[:, :, pos].cpu(), k_ref)
    assert torch.equal(cache.v[:, :, pos].cpu(), v)
    assert cache.length == pos + 1
    n = dtype_name(q)
    kp_ref = oracle_mod.project_keys(to_np(k_ref[:, :, None]), n, P.numpy())[:, :, 0]
    assert np.array_equal(to_np(cache.kp[:, :, pos].cpu()), kp_ref)
    qp_ref = oracle_mod.query_projection(oracle_mod.unit_query(to_np(q_ref), n), P.numpy())
    assert np.array_equal(qp.cpu().numpy(), qp_ref)


def _prefilled_layer(mode, dt, N0, T_dispatch, seed=3):
    from dcr_b200.kv_cache import StaticKVCache
    from dcr_b200.models.llama.attention import DCRDecodeAttention
    from dcr_b200.synthetic import make_decode_inputs, projection_matrix
    torch.manual_seed(seed)
    B, H, H_kv, hidden = 2, 32, 8, 512
    layer = DCRDecodeAttention(hidden, H, H_kv, T_dispatch=T_dispatch, mode=mode, dtype=dt,
                               device=DEV)
    for lin in (layer.q_proj, layer.k_proj, layer.v_proj, layer.o_proj):
        torch.nn.init.normal_(lin.weight, std=hidden ** -0.5)
    P = projection_matrix(seed=0, device=DEV)
    cache = StaticKVCache(B, H_kv, N0 + 8, dtype=dt, device=DEV, P=P)
    _, K, V = make_decode_inputs(B, H_kv, H_kv, N0, dtype=dt, seed=seed, device=DEV)
    cache.append(K, V)
    return layer, cache


@pytest.mark.parametrize("mode", ["exact", "projected"])
def test_layer_decode_step_vs_reference_path(oracle_mod, cuda_lib, mode):
    from dcr_b200 import _lib
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    dt = torch.bfloat16
    layer, cache = _prefilled_layer(mode, dt, 6000, 1024)
    B = cache.B
    x = torch.randn(B, 1, layer.hidden, device=DEV).to(dt)
    cos, sin = _cos_sin(B, cache.length, dt)
    K_before = cache.K.clone()
    with torch.no_grad():
        out = layer(x, cos[:, None].to(DEV), sin[:, None].to(DEV), cache)
        # the reference's path with torch and the oracle
        q = layer.q_proj(x[:, 0]).view(B, 32, 64)
        k = layer.k_proj(x[:, 0]).view(B, 8, 64)
        v = layer.v_proj(x[:, 0]).view(B, 8, 64)
    assert layer.last_branch == "dcr"
    assert _lib.read_device_status(clear=True) == 0
    cs, sn = cos.to(DEV), sin.to(DEV)
    q_ref, k_ref = _hf_rope(q, cs, sn), _hf_rope(k, cs, sn)
    K_ref = torch.cat([K_before, k_ref[:, :, None]], dim=2)
    V_ref = torch.cat([cache.V[:, :, :-1], v[:, :, None]], dim=2)
    assert torch.equal(cache.K, K_ref) and torch.equal(cache.V, V_ref)
    N = cache.length
    kk = adaptive_k_window(64, N, 0.15)
    if mode == "exact":
        O_ref = oracle_mod.decode(to_np(q_ref.cpu()), to_np(K_ref.cpu()), to_np(V_ref.cpu()),
                                  "bf16", kk)[3]
    else:
        kp = to_np(cache.KP.cpu())
        O_ref = oracle_mod.decode_projected(to_np(q_ref.cpu()), to_np(K_ref.cpu()),
                                            to_np(V_ref.cpu()), kp, cache.P.cpu().numpy(),
                                            "bf16", kk)[3]
    O_ref_t = torch.from_numpy(O_ref).to(DEV)
    with torch.no_grad():
        out_ref = layer.o_proj(O_ref_t.to(dt).reshape(B, 1, 32 * 64))
    err = (out.float() - out_ref.float()).abs().max().item()
    scale = out_ref.float().abs().max().item()
    assert err <= 2e-2 * max(scale, 1.0), (err, scale)
    # the attention output itself, before o_proj
    O = layer.attend(q_ref.contiguous(), None, cache) if mode == "exact" else None
    if O is not None:
        ok, st = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to="bf16")
        assert ok, st


def test_layer_routes_short_context_to_sdpa(cuda_lib):
    dt = torch.bfloat16
    layer, cache = _prefilled_layer("exact", dt, 500, 4096)
    B = cache.B
    x = torch.randn(B, 1, layer.hidden, device=DEV).to(dt)
    cos, sin = _cos_sin(B, cache.length, dt)
    with torch.no_grad():
        out = layer(x, cos[:, None].to(DEV), sin[:, None].to(DEV), cache)
    assert layer.last_branch == "sdpa"
    assert torch.isfinite(out.float()).all()


def test_kv_head_parallel_partials_sum_to_the_layer(cuda_lib):
    """Two emulated ranks on one GPU (each its own KV heads and cache): the partial o_proj
    outputs summed equal the unsplit layer's output up to bf16 summation order."""
    from dcr_b200.kv_cache import StaticKVCache
    from dcr_b200.models.llama.attention import KVHeadParallelDecodeAttention
    dt = torch.bfloat16
    full, cache = _prefilled_layer("exact", dt, 6000, 1024)
    B = cache.B
    x = torch.randn(B, 1, full.hidden, device=DEV).to(dt)
    cos, sin = _cos_sin(B, cache.length, dt)
    partials = []
    for r in range(2):
        shard = KVHeadParallelDecodeAttention(full.hidden, 32, 8, world=2, rank=r,
                                              all_reduce=lambda t: t, T_dispatch=1024,
                                              dtype=dt, device=DEV).load_shard(full)
        c = StaticKVCache(B, 4, cache.N_max, dtype=dt, device=DEV)
        c.append(cache.K[:, 4 * r:4 * r + 4], cache.V[:, 4 * r:4 * r + 4])
        with torch.no_grad():
            partials.append(shard(x, cos[:, None].to(DEV), sin[:, None].to(DEV), c).float())
    with torch.no_grad():
        out = full(x, cos[:, None].to(DEV), sin[:, None].to(DEV), cache).float()
    err = (partials[0] + partials[1] - out).abs().max().item()
    assert err <= 2e-2 * max(out.abs().max().item(), 1.0), err
