"""DecodeRunner: the graph-replayed decode step with host buffers returns exactly what the
per-call API returns, step after step, in the exact and the projected mode."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.mark.parametrize("projected,B", [(False, 2), (True, 2), (False, 20)])
def test_runner_matches_per_call_api(cuda_lib, projected, B):
    """B = 20: an 80 KB query and output per step (several copy CTAs each way)."""
    from dcr_b200.kernel.cuda import (project_keys, topk_qaxis_attention,
                                      topk_qaxis_attention_projected)
    from dcr_b200.runner import DecodeRunner
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs, projection_matrix
    H, H_kv, N, k = 32, 8, 6000, 900
    _, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.float16, seed=41, device=DEV)
    Qs = fresh_queries(4, B, H, dtype=torch.float16, seed=42)
    kw = {}
    if projected:
        P = projection_matrix(seed=0, device=DEV)
        kw = dict(KP=project_keys(K, P), P=P)
    runner = DecodeRunner(K, V, k, H, **kw)
    for i in range(4):
        got = runner(Qs[i]).clone()
        q = Qs[i].to(DEV)
        want = (topk_qaxis_attention_projected(q, K, V, kw["KP"], kw["P"], k) if projected
                else topk_qaxis_attention(q, K, V, k)).cpu()
        assert torch.equal(got, want), i
    runner.close()
