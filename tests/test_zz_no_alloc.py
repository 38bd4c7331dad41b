"""dcr_decode_noalloc: the decode step for callers that cannot allocate device memory.

Some callers of this library cannot allocate GPU memory where they run a decode step (an
engine plugin whose enqueue must not allocate, a host callback, a serving loop that cannot
pay for cudaMalloc's implicit synchronisation). dcr_decode_noalloc serves them from a
16 MiB scratch array inside the library instead of a caller workspace. This test calls it
through the C ABI twice in a row (the second call finds the first call's leftovers in the
shared scratch) and checks both outputs against dcr_decode with a normal workspace, with
the attention tolerance the other tests use. It also checks that a shape needing more than
the array is refused before anything runs.

The file name makes pytest collect it last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import attention_close

pytestmark = pytest.mark.gpu


def _decode_args(Q, K, V, k):
    B, H, _ = Q.shape
    _, H_kv, N, D = K.shape
    code = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[Q.dtype]
    return (Q.data_ptr(), K.data_ptr(), V.data_ptr(), code, K.stride(0), K.stride(1),
            V.stride(0), V.stride(1), B, H, H_kv, N, D, k, 1e-12)


def test_noalloc_matches_decode_on_two_calls(cuda_lib):
    from dcr_b200 import _lib
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs

    dev = torch.device("cuda:0")
    lib = cuda_lib
    B, H, H_kv, N, k = 4, 32, 8, 8192, 1229
    _, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.float16, seed=21, device=dev)
    Qs = fresh_queries(2, B, H, dtype=torch.float16, seed=22, device=dev)
    assert lib.dcr_workspace_bytes(B, H, H_kv, N, 64, k) <= (16 << 20)
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = torch.empty(lib.dcr_workspace_bytes(B, H, H_kv, N, 64, k), dtype=torch.uint8,
                     device=dev)

    for step in range(2):
        Q = Qs[step].contiguous()
        want = torch.empty(B, H, 64, dtype=Q.dtype, device=dev)
        got = torch.empty_like(want)
        got.fill_(float("nan"))
        st = lib.dcr_decode(*_decode_args(Q, K, V, k), want.data_ptr(), ws.data_ptr(),
                            ws.numel(), stream)
        assert st == 0, _lib.status_string(st)
        st = lib.dcr_decode_noalloc(*_decode_args(Q, K, V, k), got.data_ptr(), stream)
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        assert _lib.read_device_status(clear=True) == 0
        ok, stats = attention_close(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                    got_rounded_to="f16")
        assert ok, (step, stats)
        assert torch.isfinite(got.float()).all()


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_lib):
    from dcr_b200 import _lib

    lib = cuda_lib
    # B=4, N=131072: the scores alone need 32 MiB > 16 MiB. Refused before any launch, so
    # the (never dereferenced) pointers below are never used.
    B, H, H_kv, N, k = 4, 32, 8, 131072, 19660
    assert lib.dcr_workspace_bytes(B, H, H_kv, N, 64, k) > (16 << 20)
    p = 256
    st = lib.dcr_decode_noalloc(p, p, p, 1, H_kv * N * 64, N * 64, H_kv * N * 64, N * 64, B, H,
                                H_kv, N, 64, k, 1e-12, p, None)
    assert st == _lib.DCR_ERR_NOALLOC_LIMIT
    assert "16 MiB" in _lib.status_string(st)
    assert np.isscalar(st)
