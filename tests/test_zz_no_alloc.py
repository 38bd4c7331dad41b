"""dcr_decode_noalloc: the decode step for callers that cannot allocate device memory.

Some callers of this library cannot allocate GPU memory where they run a decode step: an
inference-engine plugin whose enqueue must not allocate because the engine owns all device
memory, or a serving loop that cannot pay for cudaMalloc's implicit synchronisation.
dcr_decode_noalloc serves them from a 16 MiB scratch array inside the library instead of a
caller workspace. It runs the same kernels on the same workspace layout as dcr_decode, so
its output must be bit-identical to dcr_decode's.

These tests call it through the C ABI several times in a row, so later calls find earlier
calls' leftovers in the shared scratch: two steps of one shape, then a large shape followed
by a small one. fp16 and bf16 take the union Pass 3 (selection bitmaps); fp32 takes the
per-head Pass 3 with split-K tickets that every call must reset. A shape needing more than
the array is refused before anything runs.

The file name makes pytest collect it last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def _decode_args(Q, K, V, k):
    B, H, _ = Q.shape
    _, H_kv, N, D = K.shape
    code = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[Q.dtype]
    return (Q.data_ptr(), K.data_ptr(), V.data_ptr(), code, K.stride(0), K.stride(1),
            V.stride(0), V.stride(1), B, H, H_kv, N, D, k, 1e-12)


def _run_pair(lib, Q, K, V, k, stream):
    """One dcr_decode (fresh workspace) and one dcr_decode_noalloc on the same inputs."""
    from dcr_b200 import _lib

    B, H, _ = Q.shape
    _, H_kv, N, D = K.shape
    nbytes = lib.dcr_workspace_bytes(B, H, H_kv, N, D, k)
    assert 0 < nbytes <= (16 << 20)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=Q.device)
    want = torch.empty(B, H, D, dtype=Q.dtype, device=Q.device)
    got = torch.full_like(want, float("nan"))
    st = lib.dcr_decode(*_decode_args(Q, K, V, k), want.data_ptr(), ws.data_ptr(), ws.numel(),
                        stream)
    assert st == 0, _lib.status_string(st)
    st = lib.dcr_decode_noalloc(*_decode_args(Q, K, V, k), got.data_ptr(), stream)
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()
    assert _lib.read_device_status(clear=True) == 0
    return want, got


@pytest.mark.parametrize("dt", sorted(DTYPES))
def test_noalloc_matches_decode_on_two_calls(cuda_lib, dt):
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs

    dev = torch.device("cuda:0")
    dtype = DTYPES[dt]
    B, H, H_kv, N, k = 4, 32, 8, 8192, 1229
    _, K, V = make_decode_inputs(B, H, H_kv, N, dtype=dtype, seed=21, device=dev)
    Qs = fresh_queries(2, B, H, dtype=dtype, seed=22, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for step in range(2):
        want, got = _run_pair(cuda_lib, Qs[step].contiguous(), K, V, k, stream)
        assert torch.isfinite(got.float()).all()
        assert torch.equal(got, want), (dt, step)


@pytest.mark.parametrize("dt", ["f16", "f32"])
def test_noalloc_large_then_small_shape(cuda_lib, dt):
    """A small call after a large one finds the large call's data in the scratch."""
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs

    dev = torch.device("cuda:0")
    dtype = DTYPES[dt]
    stream = torch.cuda.current_stream(dev).cuda_stream
    # Large: B=2, N=32768 (scores 4 MiB, bitmaps and partials on top); small: B=1, N=2000.
    for (B, N, k, seed) in [(2, 32768, 4916, 31), (1, 2000, 300, 32), (1, 2000, 300, 33)]:
        _, K, V = make_decode_inputs(B, 32, 8, N, dtype=dtype, seed=seed, device=dev)
        Q = fresh_queries(1, B, 32, dtype=dtype, seed=seed + 100, device=dev)[0].contiguous()
        want, got = _run_pair(cuda_lib, Q, K, V, k, stream)
        assert torch.equal(got, want), (dt, B, N)


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
