"""The C ABI (CPU only): the library loads, exports every symbol include/dcr_b200.h
declares, and the host-side entry points that launch nothing behave like the reference.
No call here touches a GPU: argument errors return before any CUDA call."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dcr_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dcr_[a-z_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from dcr_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_matches_binding_table():
    from dcr_b200 import _lib
    assert _declared() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    from dcr_b200.build import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (dcr_\w+)", out))
    missing = [s for s in _declared() if s not in exported]
    assert not missing, missing
    for s in _declared():
        assert hasattr(lib, s)


def test_library_is_built_for_sm100a_only():
    """The build compiles one architecture, sm_100a, with no PTX for other targets; the
    GPU test test_gpu_parity.py::test_binary_version asks the runtime the same question."""
    from dcr_b200 import build
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version_and_status_strings(lib):
    assert lib.dcr_version() == 1
    assert b"SDPA" in lib.dcr_status_string(3)
    assert lib.dcr_status_string(999) == b"unknown status"


@pytest.mark.parametrize("n,c", [(64, 0.8), (100, 0.8), (256, 0.8), (1000, 0.8), (4096, 0.8),
                                 (4096, 0.15), (32768, 0.15), (262144, 0.05), (131072, 0.30),
                                 (8192, 0.05), (65, 0.5), (63, 0.0), (1, 1.0), (7, 0.9)])
def test_adaptive_k_window_agrees(lib, oracle_mod, n, c):
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    py = adaptive_k_window(64, n, c)
    assert lib.dcr_adaptive_k_window(64, n, c) == py == oracle_mod.adaptive_k_window(64, n, c)


def test_adaptive_k_window_reference_values():
    """Values the reference's adaptive_k_window returns (docstring table at
    adaptive.py:55-63 and the hero/long-context operating points)."""
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    assert [adaptive_k_window(64, n, 0.8) for n in (64, 100, 256, 1000, 4096)] == \
        [64, 80, 204, 800, 3276]
    assert adaptive_k_window(64, 4096, 0.15) == 614
    assert adaptive_k_window(64, 32768, 0.15) == 4916
    assert adaptive_k_window(64, 262144, 0.05) == 13108
    with pytest.raises(ValueError):
        adaptive_k_window(64, 0, 0.1)
    with pytest.raises(ValueError):
        adaptive_k_window(64, 10, 1.5)


def test_workspace_bytes(lib):
    assert lib.dcr_workspace_bytes(4, 32, 8, 32768, 64, 4916) > 4 * 32 * 32768 * 2
    assert lib.dcr_workspace_bytes(4, 32, 8, 32768, 32, 4916) == 0   # D != 64
    assert lib.dcr_workspace_bytes(4, 32, 5, 32768, 64, 4916) == 0   # H % H_kv
    assert lib.dcr_workspace_bytes(4, 48, 4, 32768, 64, 4916) == 0   # G = 12


def _decode(lib, B=1, H=32, H_kv=8, N=128, D=64, k=10, dtype=0, q=16, kk=16, v=16, o=16,
            ws=16, ws_bytes=1 << 20, kstride=None):
    ksb, ksh = kstride if kstride else (H_kv * N * 64, N * 64)
    return lib.dcr_decode(q, kk, v, dtype, ksb, ksh, ksb, ksh, B, H, H_kv, N, D, k, 1e-12, o,
                          ws, ws_bytes, None)


def test_argument_errors_return_before_any_launch(lib):
    # Fake, never-dereferenced but aligned pointers: every call must fail validation.
    assert _decode(lib, D=32) == 2
    assert _decode(lib, H=48, H_kv=4) == 2           # n_per_kv = 12 unsupported
    assert _decode(lib, H=32, H_kv=5) == 2
    assert _decode(lib, k=128) == 3                   # k_eff == N
    assert _decode(lib, k=0) == 3
    assert _decode(lib, dtype=7) == 4
    assert _decode(lib, q=0) == 1
    assert _decode(lib, kk=0) == 1
    assert _decode(lib, kk=24) == 5                   # misaligned cache
    assert _decode(lib, kstride=(8 * 128 * 64, 100 * 64 + 4)) == 5   # misaligned stride
    assert _decode(lib, kstride=(8 * 128 * 64, 64 * 64)) == 2        # heads overlap
    assert _decode(lib, ws=0) == 6
    assert _decode(lib, ws_bytes=16) == 6
    assert lib.dcr_select(16, 100, 4, 100, 100, 16, None) == 3
    assert lib.dcr_select(16, 50, 4, 100, 10, 16, None) == 2         # stride < N
    assert lib.dcr_unit_query(16, 0, 1, 1, 32, ctypes.c_float(1e-12), 16, None) == 2
    # the step-prefix diagnostic takes 1, 2 or 3 passes and validates like dcr_decode
    for passes in (0, 4):
        assert lib.dcr_decode_prefix(16, 16, 16, 0, 8 * 128 * 64, 128 * 64, 8 * 128 * 64,
                                     128 * 64, 1, 32, 8, 128, 64, 10, 1e-12, 16, 16, 1 << 20,
                                     None, passes) == 2
    assert lib.dcr_decode_prefix(16, 16, 16, 0, 8 * 128 * 64, 128 * 64, 8 * 128 * 64, 128 * 64,
                                 1, 32, 8, 128, 32, 10, 1e-12, 16, 16, 1 << 20, None, 1) == 2
