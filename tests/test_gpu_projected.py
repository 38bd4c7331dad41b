"""Projected-score mode and the static KV cache on the GPU, against the CPU restatement.

The projected keys (append and prefill kernels), the projected scores and the selected
indices must equal the oracle's bit for bit; O must pass the attention tolerance against
the oracle's fp32 attention over the same indices. Appending into StaticKVCache must
leave exactly the appended rows in the caches, and the whole append + decode step must
replay from a CUDA graph.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import attention_close, dtype_name, to_np

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
DTS = [torch.bfloat16, torch.float16, torch.float32]


def _P(seed=0):
    from dcr_b200.synthetic import projection_matrix
    return projection_matrix(seed=seed)


@pytest.mark.parametrize("dt", DTS)
def test_project_keys_bit_exact(oracle_mod, cuda_lib, dt):
    from dcr_b200.kernel.cuda import project_keys
    from dcr_b200.synthetic import make_decode_inputs
    _, K, _ = make_decode_inputs(2, 8, 4, 1003, dtype=dt, seed=12)
    P = _P()
    got = project_keys(K.to(DEV), P.to(DEV)).cpu()
    want = oracle_mod.project_keys(to_np(K), dtype_name(K), P.numpy())
    assert np.array_equal(to_np(got), want)


def test_project_keys_strided_cache_view(oracle_mod, cuda_lib):
    """A cache allocated for N_max positions, passed as its first N positions."""
    from dcr_b200.kernel.cuda import project_keys
    from dcr_b200.synthetic import make_decode_inputs
    _, K, _ = make_decode_inputs(2, 4, 4, 777, dtype=torch.float16, seed=13)
    big = torch.zeros(2, 4, 1000, 64, dtype=torch.float16, device=DEV)
    big[:, :, :777] = K.to(DEV)
    kp_big = torch.zeros(2, 4, 1000, 16, dtype=torch.float16, device=DEV)
    project_keys(big[:, :, :777], _P().to(DEV), out=kp_big[:, :, :777])
    want = oracle_mod.project_keys(to_np(K), "f16", _P().numpy())
    assert np.array_equal(to_np(kp_big[:, :, :777].cpu()), want)
    assert not kp_big[:, :, 777:].any()


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("B,H,H_kv,N,k", [(1, 32, 8, 4096, 614), (2, 16, 2, 2001, 300),
                                          (3, 8, 8, 517, 78), (1, 64, 8, 3000, 450),
                                          (2, 8, 4, 9000, 1200)])
def test_projected_select_and_decode_vs_oracle(oracle_mod, cuda_lib, dt, B, H, H_kv, N, k):
    from dcr_b200 import _lib
    from dcr_b200.kernel.cuda import (project_keys, topk_qaxis_attention_projected,
                                      topk_qaxis_select_projected)
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=dt, seed=14)
    P = _P()
    Qd, Kd, Vd, Pd = Q.to(DEV), K.to(DEV), V.to(DEV), P.to(DEV)
    KP = project_keys(Kd, Pd)
    n = dtype_name(Q)
    kp_o = oracle_mod.project_keys(to_np(K), n, P.numpy())
    qp, s, idx, O_ref = oracle_mod.decode_projected(to_np(Q), to_np(K), to_np(V), kp_o,
                                                    P.numpy(), n, k)
    # scores bit-exact
    scores = torch.empty(B * H, N, dtype=torch.int16, device=DEV)
    psb, psh = KP.stride(0), KP.stride(1)
    st = cuda_lib.dcr_score_projected(KP.data_ptr(), _lib.DTYPE_CODES[dt], psb, psh,
                                      Qd.data_ptr(), 1e-12, Pd.data_ptr(), 16, None, B, H, H_kv,
                                      N, 64, scores.data_ptr(), N, None)
    assert st == 0
    assert np.array_equal(scores.cpu().numpy().view(np.uint16), s)
    sel = topk_qaxis_select_projected(Qd, KP, Pd, k)
    assert np.array_equal(sel.view(B * H, k).cpu().numpy(), idx)
    O = topk_qaxis_attention_projected(Qd, Kd, Vd, KP, Pd, k)
    assert _lib.read_device_status(clear=True) == 0
    ok, stats = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to=n)
    assert ok, stats


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_projected_scores_reject_unaligned_kp(cuda_lib, dt):
    """Projected Pass 1 reads KP rows with 16-byte vector loads: a KP view that does not
    start on a 16-byte boundary is refused with DCR_ERR_ALIGN, and the same rows copied to
    an aligned buffer score normally."""
    from dcr_b200 import _lib
    from dcr_b200.kernel.cuda import project_keys
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, N = 2, 16, 4, 3001
    Q, K, _ = make_decode_inputs(B, H, H_kv, N, dtype=dt, seed=17, device=DEV)
    Pd = _P().to(DEV)
    KP = project_keys(K, Pd)
    esz = KP.element_size()
    flat = torch.empty(KP.numel() + 16 // esz, dtype=dt, device=DEV)
    off = 8 // esz
    KPu = flat[off:off + KP.numel()].view(KP.shape)
    KPu.copy_(KP)
    assert KPu.data_ptr() % 16 == 8

    def score(kp):
        out = torch.empty(B * H, N, dtype=torch.int16, device=DEV)
        return cuda_lib.dcr_score_projected(kp.data_ptr(), _lib.DTYPE_CODES[dt], kp.stride(0),
                                            kp.stride(1), Q.data_ptr(), 1e-12, Pd.data_ptr(),
                                            16, None, B, H, H_kv, N, 64, out.data_ptr(), N, None)

    assert score(KPu) == _lib.DCR_ERR_ALIGN
    assert score(KP) == 0
    assert _lib.read_device_status(clear=True) == 0


@pytest.mark.slow
def test_projected_hero_indices_bit_exact(oracle_mod, cuda_lib):
    """Hero shape (B=4, N=32768, 32/8 heads, fp16, k=4916): every index set bit-exact."""
    from dcr_b200.kernel.cuda import project_keys, topk_qaxis_select_projected
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, N, k = 4, 32, 8, 32768, 4916
    Q, K, _ = make_decode_inputs(B, H, H_kv, N, dtype=torch.float16, seed=15)
    P = _P()
    KP = project_keys(K.to(DEV), P.to(DEV))
    kp_o = oracle_mod.project_keys(to_np(K), "f16", P.numpy())
    assert np.array_equal(to_np(KP.cpu()), kp_o)
    qp = oracle_mod.query_projection(oracle_mod.unit_query(to_np(Q), "f16"), P.numpy())
    idx = oracle_mod.select(oracle_mod.scores_projected(kp_o, "f16", qp), k)
    sel = topk_qaxis_select_projected(Q.to(DEV), KP, P.to(DEV), k)
    assert np.array_equal(sel.view(B * H, k).cpu().numpy(), idx)


def test_static_cache_append_and_graph_replay(oracle_mod, cuda_lib):
    """Prefill 1000 positions, append 3 single tokens, then capture append + decode in a
    CUDA graph and replay it for 2 more tokens."""
    from dcr_b200 import _lib
    from dcr_b200.kernel.cuda import topk_qaxis_attention_projected
    from dcr_b200.kv_cache import StaticKVCache
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs
    B, H, H_kv, N_max = 2, 16, 4, 1100
    _, K, V = make_decode_inputs(B, H_kv, H_kv, 1005, dtype=torch.bfloat16, seed=16)
    Qs = fresh_queries(6, B, H, dtype=torch.bfloat16, seed=17)
    P = _P()
    cache = StaticKVCache(B, H_kv, N_max, dtype=torch.bfloat16, device=DEV, P=P.to(DEV))
    Kd, Vd = K.to(DEV), V.to(DEV)
    cache.append(Kd[:, :, :1000], Vd[:, :, :1000])
    for t in range(1000, 1003):
        cache.append(Kd[:, :, t:t + 1], Vd[:, :, t:t + 1])
    assert cache.length == 1003
    assert torch.equal(cache.K, Kd[:, :, :1003]) and torch.equal(cache.V, Vd[:, :, :1003])
    kp_o = oracle_mod.project_keys(to_np(K[:, :, :1003]), "bf16", P.numpy())
    assert np.array_equal(to_np(cache.KP.cpu()), kp_o)

    # graph: append token t (fixed buffers), then decode over the first t + 1 positions
    k_new = torch.empty(B, H_kv, 1, 64, dtype=torch.bfloat16, device=DEV)
    v_new = torch.empty_like(k_new)
    Qd = torch.empty(B, H, 64, dtype=torch.bfloat16, device=DEV)
    Od = torch.empty_like(Qd)
    outs = []
    for t in (1003, 1004):
        k_new.copy_(Kd[:, :, t:t + 1])
        v_new.copy_(Vd[:, :, t:t + 1])
        Qd.copy_(Qs[t - 1003].to(DEV))
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(DEV)
        side.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                cache.append(k_new, v_new)
                topk_qaxis_attention_projected(Qd, cache.K, cache.V, cache.KP, cache.P, 150,
                                               out=Od)
            g.replay()
            side.synchronize()
        outs.append(Od.clone())
        del g
    assert cache.length == 1005     # two appends captured, each replayed once
    assert _lib.read_device_status(clear=True) == 0
    kp_o = oracle_mod.project_keys(to_np(K), "bf16", P.numpy())
    assert np.array_equal(to_np(cache.KP.cpu()), kp_o)
    for t, O in zip((1003, 1004), outs):
        _, _, _, O_ref = oracle_mod.decode_projected(
            to_np(Qs[t - 1003]), to_np(K[:, :, :t + 1]), to_np(V[:, :, :t + 1]),
            kp_o[:, :, :t + 1], P.numpy(), "bf16", 150)
        ok, st = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to="bf16")
        assert ok, (t, st)


def test_append_errors(cuda_lib):
    from dcr_b200 import _lib
    lib = cuda_lib
    k = torch.zeros(1, 2, 4, 64, dtype=torch.float16, device=DEV)
    c = torch.zeros(1, 2, 10, 64, dtype=torch.float16, device=DEV)
    args = (k.data_ptr(), k.data_ptr(), 1, 2 * 4 * 64, 4 * 64, 1, 2, 4, 64, c.data_ptr(),
            c.data_ptr(), 2 * 10 * 64, 10 * 64)
    assert lib.dcr_cache_append(*args, 7, 10, None, 16, None, 0, 0, None) == _lib.DCR_ERR_SHAPE
    assert lib.dcr_cache_append(*args, 6, 10, None, 16, None, 0, 0, None) == 0
    P = torch.zeros(64, 16, device=DEV)
    kp = torch.zeros(1, 2, 10, 16, dtype=torch.float16, device=DEV)
    assert lib.dcr_cache_append(*args, 0, 10, P.data_ptr(), 8, kp.data_ptr(), 320, 160,
                                None) == _lib.DCR_ERR_SHAPE      # rank must be 16
    torch.cuda.synchronize()
