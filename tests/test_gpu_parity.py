"""Parity of the CUDA path (through the C ABI) with the reference and the oracle (B200).

Gates (north star + the reference's own kernel_spec.md section 5):
* unit query, Pass 1 scores, Pass 2 / end-to-end indices: bit-exact against the oracle;
  indices also bit-exact against the reference's golden vectors;
* Pass 1 scores vs the reference's einsum: at most one bf16 ulp, RMSE^2 <= 1e-6;
* attention outputs: max|d| <= 2e-3 beyond the output rounding, cosine >= 0.9999,
  RMSE^2 <= 1e-6 against the reference's unrounded fp32 output (or the oracle's).
At full size (3 and one GPU's shard of config 4) the oracle is run too,
and the size-independent properties of an exact top-K are checked on the device.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from golden_io import ALL_CASES, attention_close, bf16_bits_to_f32, dtype_name, load_case, to_np

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(cuda_lib):
    from dcr_b200 import _lib
    _lib.read_device_status(clear=True)
    yield
    assert _lib.read_device_status(clear=True) == 0, "a kernel raised a device status"


def _api():
    from dcr_b200.kernel import cuda as api
    return api


def _bf16_tensor(bits: np.ndarray, shape) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).reshape(shape)


def test_binary_version(cuda_lib):
    """The runtime reports the library's device code as built for compute capability 10.0
    (sm_100a), the only architecture the build compiles."""
    import ctypes
    v = ctypes.c_int(0)
    assert cuda_lib.dcr_binary_version(ctypes.byref(v)) == 0
    assert v.value == 100


# ---------------------------------------------------------------------------------------
# Golden vectors (made by the reference itself)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", ALL_CASES)
def test_unit_query_bit_exact(oracle_mod, name):
    meta, (Q, K, V), g = load_case(name)
    u = _api().compute_u_Q(Q.to(DEV)).cpu().numpy()
    assert np.array_equal(u.view(np.uint32), oracle_mod.unit_query(to_np(Q), dtype_name(Q)).view(np.uint32))
    ulp = np.spacing(np.abs(g["u"]).astype(np.float32))
    assert np.all(np.abs(u - g["u"]) <= 2 * ulp + 1e-30)


@pytest.mark.parametrize("name", ALL_CASES)
def test_pass1_scores(oracle_mod, name):
    meta, (Q, K, V), g = load_case(name)
    B, H, N = meta["B"], meta["H"], meta["N"]
    s = _api().topk_pass1_projection(K.to(DEV), torch.from_numpy(g["u"]).to(DEV))
    assert s.shape == (B, H, N) and s.dtype == torch.bfloat16
    bits = to_np(s).reshape(B * H, N)
    want_oracle = oracle_mod.scores(to_np(K), dtype_name(K), g["u"])
    assert np.array_equal(bits, want_oracle), "Pass 1 scores differ from the oracle's bits"
    got, ref = bf16_bits_to_f32(bits), bf16_bits_to_f32(g["scores"])
    d = np.abs(got - ref)
    assert d.max() <= 1e-2 and (d ** 2).mean() <= 1e-6          # reference gate
    assert np.all(d <= np.spacing(np.abs(ref)) * 2 ** 16 + 1e-30)  # <= one bf16 ulp


@pytest.mark.parametrize("name", ALL_CASES)
def test_pass2_bit_exact_on_reference_scores(name):
    meta, _, g = load_case(name)
    B, H, N, k = meta["B"], meta["H"], meta["N"], meta["k"]
    idx = _api().topk_pass2_select(_bf16_tensor(g["scores"], (B, H, N)).to(DEV), k)
    assert idx.dtype == torch.int32 and idx.shape == (B, H, k)
    assert np.array_equal(idx.cpu().numpy().reshape(B * H, k), g["idx"])


@pytest.mark.parametrize("name", ALL_CASES)
def test_pass3_on_reference_indices(name):
    meta, (Q, K, V), g = load_case(name)
    B, H, k = meta["B"], meta["H"], meta["k"]
    idx = torch.from_numpy(g["idx"].reshape(B, H, k)).to(DEV)
    O = _api().fused_topk_attention(Q.to(DEV), K.to(DEV), V.to(DEV), idx)
    assert O.dtype == Q.dtype and O.shape == (B, H, 64)
    ok, st = attention_close(O.float().cpu().numpy(), g["O_f32"], got_rounded_to=dtype_name(Q))
    assert ok, st


@pytest.mark.parametrize("name", ALL_CASES)
def test_full_pipeline_vs_reference(oracle_mod, name):
    meta, (Q, K, V), g = load_case(name)
    B, H, k = meta["B"], meta["H"], meta["k"]
    Qd, Kd, Vd = Q.to(DEV), K.to(DEV), V.to(DEV)
    idx = _api().topk_qaxis_select(Qd, Kd, k).cpu().numpy().reshape(B * H, k)
    _, _, idx_oracle, O_oracle = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dtype_name(Q), k)
    assert np.array_equal(idx, idx_oracle), "indices differ from the oracle"
    assert np.array_equal(idx, g["idx"]), "indices differ from the reference's"
    O = _api().topk_qaxis_attention(Qd, Kd, Vd, k).float().cpu().numpy()
    ok, st = attention_close(O, g["O_f32"], got_rounded_to=dtype_name(Q))
    assert ok, st
    if dtype_name(Q) == "bf16":
        # Against the reference's own bf16 output: both sides are one rounding away from
        # nearly equal fp32 values, so they agree on almost every bit and never differ by
        # more than the 2e-3 gate plus one bf16 ulp (near zero the fp32 summation-order
        # noise can exceed the ulp, hence the absolute part).
        ref = bf16_bits_to_f32(g["O_ref"])
        assert np.mean(O == ref) >= 0.98
        assert np.all(np.abs(O - ref) <= 2e-3 + np.spacing(np.abs(ref)) * 2 ** 16)


# ---------------------------------------------------------------------------------------
# Shapes, dtypes and edge cases against the oracle
# ---------------------------------------------------------------------------------------
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
SWEEP = [
    # B, H, H_kv, N, k, dtype
    (1, 4, 4, 2, 1, "bf16"),
    (1, 8, 2, 9, 3, "bf16"),
    (1, 8, 8, 64, 63, "f16"),
    (3, 32, 8, 257, 100, "bf16"),
    (2, 16, 2, 513, 256, "f16"),
    (1, 32, 8, 1023, 511, "f32"),
    (2, 8, 1, 5000, 2500, "bf16"),
    (8, 32, 8, 5000, 2500, "bf16"),      # reference test_edge_case_b8_production
    (1, 32, 8, 20000, 10000, "bf16"),    # reference test_fp32_softmax_state_long_context
    (1, 32, 8, 20000, 1, "f16"),
    (2, 64, 8, 3000, 450, "bf16"),       # G = 8
    (1, 32, 8, 4096, 614, "f32"),        # config 0
    (4, 32, 8, 32771, 4916, "bf16"),     # just past 32768: one 1024-thread CTA per row
    (4, 32, 8, 40960, 6144, "f16"),      # the longest row that shape covers
    (4, 32, 8, 40961, 6144, "bf16"),     # two-CTA clusters
    (1, 4, 1, 262209, 13112, "bf16"),    # past 262144: 8-CTA clusters of 1024 threads
    (8, 32, 8, 20000, 3000, "bf16"),     # past one wave of rows: one CTA per row, in waves
    (8, 32, 8, 20000, 3000, "f32"),      # the same writing index lists
    (4, 64, 8, 20001, 3001, "f16"),      # G = 8, two waves of rows
    (4, 32, 8, 50000, 7500, "bf16"),     # long rows past one wave: the chunked Pass 2, bitmaps
    (2, 32, 8, 81921, 12289, "f32"),     # the chunked Pass 2 writing index lists
    (1, 64, 8, 90000, 13500, "f16"),     # G = 8 over the chunked selection
]


def _check_vs_oracle(oracle_mod, Q, K, V, k, dt):
    Qd, Kd, Vd = Q.to(DEV), K.to(DEV), V.to(DEV)
    B, H = Q.shape[:2]
    idx = _api().topk_qaxis_select(Qd, Kd, k).cpu().numpy().reshape(B * H, k)
    O = _api().topk_qaxis_attention(Qd, Kd, Vd, k).float().cpu().numpy()
    _, _, idx_o, O_o = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dt, k)
    assert np.array_equal(idx, idx_o)
    ok, st = attention_close(O, O_o, got_rounded_to=dt)
    assert ok, st


@pytest.mark.parametrize("B,H,H_kv,N,k,dt", SWEEP)
def test_sweep_vs_oracle(oracle_mod, B, H, H_kv, N, k, dt):
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=DT[dt], seed=N + k)
    _check_vs_oracle(oracle_mod, Q, K, V, k, dt)


@pytest.mark.parametrize("B,H,H_kv,N,k,dt", [
    (1, 32, 8, 65536, 9830, "bf16"),   # Pass 2 in clusters of 4 CTAs: bitmaps per segment
    (8, 32, 8, 16384, 2457, "f16"),    # more rows than SMs
    (2, 16, 2, 2001, 300, "bf16"),     # G = 8, index lists searched (no bitmaps)
])
def test_union_pass3_shapes_vs_oracle(oracle_mod, B, H, H_kv, N, k, dt):
    """The decode step's Pass 3 over each KV head's union of selections (bitmaps from Pass 2,
    or the heads' index lists where Pass 2 cannot write whole words) against the oracle."""
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=DT[dt], seed=N + k + 1)
    _check_vs_oracle(oracle_mod, Q, K, V, k, dt)


@pytest.mark.parametrize("B,H,H_kv,N,k,dt", [
    (4, 32, 8, 8192, 1229, "f16"),     # 16 positions per Pass 2 thread: words from lane pairs
    (4, 32, 8, 4000, 600, "bf16"),     # 8 positions per thread (4 lanes a word), ragged end
    (2, 8, 4, 4096, 614, "f16"),       # G = 2, 8-CTA clusters per row, 4 groups
    (16, 16, 8, 512, 8, "bf16"),       # 128 small groups, more rows than SMs
    (2, 64, 8, 8192, 1229, "bf16"),    # G = 8
    (4, 32, 8, 1024, 1023, "f16"),     # k = N - 1: nearly every position in every union
    (4, 32, 8, 4096, 1, "f16"),        # k = 1: at most G rows per union
    (4, 32, 8, 32800, 4920, "bf16"),   # 40 positions per thread (a model step past 32768)
    (1, 4, 1, 262209, 13112, "f16"),   # 40 per thread in 8-CTA clusters, segments on words
    (2, 8, 2, 64777, 9717, "bf16"),    # clustered rows, segments rounded up to whole words
    (1, 4, 4, 100, 15, "f16"),         # G = 1, 8-CTA clusters of which the last 4 are empty
])
def test_union_pass3_from_bitmaps_vs_oracle(oracle_mod, B, H, H_kv, N, k, dt):
    """The decode step's union Pass 3 reading the selection bitmaps that Pass 2 writes when
    its threads hold 8 or 16 positions each (lanes sharing a word OR their bits), 40 (ORed
    into the CTA's words in shared memory) or whole words, against the oracle: small and
    ragged rows, clusters, G = 1, 2 and 8, many small groups, k = N - 1 and k = 1."""
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=DT[dt], seed=N + k + 2)
    _check_vs_oracle(oracle_mod, Q, K, V, k, dt)


@pytest.mark.parametrize("N", [5000, 4096])  # 4096: bitmaps; 5000: index lists searched
def test_union_pass3_keeps_nonfinite_v_rows_to_their_heads(oracle_mod, N):
    """A V row holding inf or NaN that only one head of a KV group selected reaches that
    head's output and no other (the union kernel scores every union row for all heads, so
    the rows a head did not select must not be multiplied in, not even by a weight of 0)."""
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, k = 2, 32, 8, 750
    G = H // H_kv
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.float16, seed=21)
    idx = _api().topk_qaxis_select(Q.to(DEV), K.to(DEV), k).cpu()
    planted = 0
    for b in range(B):
        for hk in range(H_kv):
            sel = [set(idx[b, hk * G + j].tolist()) for j in range(G)]
            only0 = sorted(sel[0] - set().union(*sel[1:]))
            if only0:
                V[b, hk, only0[0], 3] = float("inf")
                V[b, hk, only0[-1], 60] = float("nan")
                planted += 1
    assert planted > 0
    O = _api().topk_qaxis_attention(Q.to(DEV), K.to(DEV), V.to(DEV), k).float().cpu()
    _, _, _, O_o = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), "f16", k)
    O_o = torch.from_numpy(np.asarray(O_o, dtype=np.float32)).reshape(O.shape)
    assert torch.equal(torch.isfinite(O), torch.isfinite(O_o))
    rows = torch.isfinite(O_o.reshape(-1, 64)).all(-1)
    assert 0 < int((~rows).sum()) < rows.numel()
    ok, st = attention_close(O.reshape(-1, 64)[rows].numpy(), O_o.reshape(-1, 64)[rows].numpy(),
                             got_rounded_to="f16")
    assert ok, st


def test_strided_cache_view_matches_contiguous(oracle_mod):
    """A cache allocated for N_max positions is used through a view, without a copy."""
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, N, k = 2, 32, 8, 3000, 450
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=9)
    Kb = torch.zeros(B, H_kv, N + 40, 64, dtype=K.dtype, device=DEV)
    Vb = torch.zeros_like(Kb)
    Kb[:, :, :N] = K.to(DEV)
    Vb[:, :, :N] = V.to(DEV)
    Kv, Vv = Kb[:, :, :N], Vb[:, :, :N]
    assert not Kv.is_contiguous()
    O1 = _api().topk_qaxis_attention(Q.to(DEV), Kv, Vv, k)
    O2 = _api().topk_qaxis_attention(Q.to(DEV), K.to(DEV), V.to(DEV), k)
    assert torch.equal(O1, O2)


def test_side_stream_and_determinism():
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(4, 32, 8, 8192, dtype=torch.float16, seed=3, device=DEV)
    O1 = _api().topk_qaxis_attention(Q, K, V, 1229)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        O2 = _api().topk_qaxis_attention(Q, K, V, 1229)
    s.synchronize()
    assert torch.equal(O1, O2)


def test_cuda_graph_capture_replay():
    from dcr_b200.kernel.cuda._common import workspace_bytes
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, N, k = 4, 32, 8, 8192, 1229
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=4, device=DEV)
    ws = torch.empty(workspace_bytes(B, H, H_kv, N, k), dtype=torch.uint8, device=DEV)
    out = torch.empty(B, H, 64, dtype=Q.dtype, device=DEV)
    want = _api().topk_qaxis_attention(Q, K, V, k)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _api().topk_qaxis_attention(Q, K, V, k, out=out, workspace_buf=ws)  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _api().topk_qaxis_attention(Q, K, V, k, out=out, workspace_buf=ws)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    Q.copy_(torch.randn_like(Q))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, _api().topk_qaxis_attention(Q, K, V, k))
    del g


def test_out_of_range_indices_are_skipped_and_reported():
    """Pass 3 checks every index against [0, N): a bad one is skipped (zero row) and
    raises DCR_ERR_DEVICE_INDEX instead of reading outside the cache."""
    from dcr_b200 import _lib
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(1, 8, 2, 256, dtype=torch.bfloat16, seed=1, device=DEV)
    idx = torch.arange(0, 64, dtype=torch.int32, device=DEV).repeat(1, 8, 1).contiguous()
    idx[0, 3, 5] = 256 + 7
    idx[0, 4, 9] = -3
    O = _api().fused_topk_attention(Q, K, V, idx)
    st = _lib.read_device_status(clear=True)
    assert st & _lib.DCR_ERR_DEVICE_INDEX
    assert torch.isfinite(O.float()).all()


def test_errors_mirror_reference():
    from dcr_b200.kernel.cuda._common import KEffRangeError
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(1, 4, 2, 16, dtype=torch.bfloat16, seed=1, device=DEV)
    with pytest.raises(ValueError, match="caller must dispatch to SDPA"):
        _api().topk_qaxis_attention(Q, K, V, 16)
    with pytest.raises(AssertionError):
        _api().topk_qaxis_attention(Q, K, V, 0)
    with pytest.raises(KEffRangeError):
        _api().topk_pass2_select(torch.zeros(1, 4, 16, dtype=torch.bfloat16, device=DEV), 20)
    with pytest.raises(AssertionError):
        _api().topk_qaxis_attention(Q, K.float(), V, 4)
    with pytest.raises(RuntimeError):
        _api().topk_qaxis_attention(Q.cpu(), K.cpu(), V.cpu(), 4)


def _stable_topk_reference(scores: torch.Tensor, k: int) -> torch.Tensor:
    """The reference's selection restated with torch: order keys of the bf16 bits (-0 as +0,
    every NaN on top), a stable descending sort, the first k positions, ascending."""
    x = scores.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    mag = x & 0x7FFF
    x = torch.where(mag == 0, torch.zeros_like(x), x)
    key = x ^ (((x >> 15) * 0x7FFF) | 0x8000)
    key = torch.where(mag > 0x7F80, torch.full_like(key, 0xFFFF), key)
    order = torch.sort(-key.to(torch.int64), dim=-1, stable=True).indices
    return torch.sort(order[..., :k], dim=-1).values.to(torch.int32)


def _adversarial_rows(kind: str, R: int, N: int, g: torch.Generator) -> torch.Tensor:
    if kind == "all_equal":
        s = torch.full((R, N), 0.75)
    elif kind == "three_values":
        s = torch.tensor([-1.0, 0.5, 2.0])[torch.randint(0, 3, (R, N), generator=g)]
    elif kind == "narrow":  # one exponent: every key shares the top 8 bits
        s = 1.0 + torch.rand(R, N, generator=g)
    elif kind == "raw_bits":  # every bf16 pattern: NaNs, +-inf, -0/+0, subnormals
        bits = torch.randint(0, 1 << 16, (R, N), generator=g, dtype=torch.int32)
        return (bits - ((bits >= 1 << 15).to(torch.int32) << 16)).to(torch.int16).view(
            torch.bfloat16)
    elif kind == "specials":
        vals = torch.tensor([float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1.0, -1.0])
        s = vals[torch.randint(0, len(vals), (R, N), generator=g)]
    else:  # decode-like: N(0, 1.45^2), the bench's score spread
        s = torch.randn(R, N, generator=g) * 1.45
    return s.to(torch.bfloat16)


@pytest.mark.parametrize("kind,R,N,k", [
    ("all_equal", 4, 1000, 300), ("three_values", 8, 40000, 17000), ("narrow", 8, 32768, 4916),
    ("raw_bits", 8, 5000, 2500), ("specials", 4, 3001, 1500), ("decode", 128, 32768, 4916),
    ("decode", 4, 32768, 1), ("decode", 4, 32768, 32767), ("three_values", 2, 70000, 30001),
    ("decode", 1, 300000, 45000), ("narrow", 2, 262209, 39331), ("raw_bits", 3, 65536, 9830),
    # more keys than 148 rows of 32768: the chunked selection of dcr_select_ws
    ("all_equal", 160, 32768, 4916), ("three_values", 64, 100000, 40000),
    ("narrow", 32, 262209, 39331), ("specials", 160, 33001, 16500), ("decode", 256, 32768, 1),
    ("decode", 160, 32768, 32767), ("raw_bits", 160, 32768, 9830), ("decode", 512, 32768, 4916),
])
def test_pass2_adversarial_distributions(kind, R, N, k):
    """Pass 2 on score rows built to stress the radix select (ties across and inside the
    threshold bin, every bf16 pattern, k = 1 and k = N, one- and multi-CTA rows, and the
    chunked grid-wide selection past one wave of rows, with ragged last chunks) against a
    stable torch sort of the same order keys: bit-exact."""
    g = torch.Generator().manual_seed(sum(map(ord, kind)) * 7919 + R * 131 + N + k)
    scores = _adversarial_rows(kind, R, N, g).reshape(1, R, N).to(DEV)
    idx = _api().topk_pass2_select(scores, k)
    assert torch.equal(idx, _stable_topk_reference(scores, k))


# ---------------------------------------------------------------------------------------
# Full size: BASELINE config 1 (hero), config 3 corners, one GPU's shard of config 4
# ---------------------------------------------------------------------------------------
def _topk_properties(scores: torch.Tensor, idx: torch.Tensor, k: int) -> None:
    """Exact top-K with lower-index tie-break, checked without a sort."""
    R, N = scores.shape
    s = scores.float()
    ix = idx.long()
    assert ix.shape == (R, k)
    assert bool((ix[:, 1:] > ix[:, :-1]).all()), "not strictly ascending"
    assert int(ix.min()) >= 0 and int(ix.max()) < N
    mask = torch.zeros(R, N, dtype=torch.bool, device=s.device)
    mask.scatter_(1, ix, True)
    assert bool((mask.sum(1) == k).all())
    sel_min = torch.where(mask, s, torch.full_like(s, float("inf"))).min(1).values
    uns_max = torch.where(~mask, s, torch.full_like(s, float("-inf"))).max(1).values
    assert bool((sel_min >= uns_max).all()), "an unselected score beats a selected one"
    pos = torch.arange(N, device=s.device).expand(R, N)
    tie = s == sel_min[:, None]
    last_sel_tie = torch.where(tie & mask, pos, torch.full_like(pos, -1)).max(1).values
    first_uns_tie = torch.where(tie & ~mask, pos, torch.full_like(pos, N)).min(1).values
    assert bool((last_sel_tie < first_uns_tie).all()), "ties not broken by lower index"


@pytest.mark.slow
@pytest.mark.parametrize("B,H,H_kv,N,c,dt", [
    (4, 32, 8, 32768, 0.15, "f16"),      # config 1 (hero)
    (4, 32, 8, 32768, 0.15, "bf16"),
    (16, 32, 8, 8192, 0.30, "f16"),      # config 3 corners
    (1, 32, 8, 131072, 0.05, "f16"),
    (8, 4, 1, 262144, 0.05, "bf16"),     # config 4: one GPU of the 8-way KV-head split
])
def test_full_size_vs_oracle(oracle_mod, B, H, H_kv, N, c, dt):
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    from dcr_b200.synthetic import make_decode_inputs
    k = adaptive_k_window(64, N, c)
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=DT[dt], seed=0, device=DEV)
    api = _api()
    u = api.compute_u_Q(Q)
    scores = api.topk_pass1_projection(K, u)
    idx = api.topk_qaxis_select(Q, K, k)
    _topk_properties(scores.reshape(B * H, N), idx.reshape(B * H, k), k)
    O = api.topk_qaxis_attention(Q, K, V, k).float().cpu().numpy()
    _, s_o, idx_o, O_o = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dt, k)
    assert np.array_equal(to_np(scores).reshape(B * H, N), s_o)
    assert np.array_equal(idx.cpu().numpy().reshape(B * H, k), idx_o)
    ok, st = attention_close(O, O_o, got_rounded_to=dt)
    assert ok, st


_GATHER_SCRIPT = r"""
import os, sys
sys.path[:0] = [sys.argv[2], os.path.join(sys.argv[2], "dcr-attention_v3_b200")]
import torch
from dcr_b200.kernel.cuda import topk_qaxis_attention
from dcr_b200.synthetic import make_decode_inputs
dev = torch.device("cuda:0")
outs = []
for dt, (B, H, H_kv, N, k) in [(torch.float16, (2, 32, 8, 5000, 750)),
                              (torch.bfloat16, (1, 16, 2, 3001, 450))]:
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=dt, seed=31, device=dev)
    outs.append(topk_qaxis_attention(Q, K, V, k).cpu())
    big = torch.zeros(B, H_kv, N + 77, 64, dtype=dt, device=dev)     # cache for N_max positions
    big[:, :, :N] = K
    bigv = torch.zeros_like(big)
    bigv[:, :, :N] = V
    outs.append(topk_qaxis_attention(Q, big[:, :, :N], bigv[:, :, :N], k).cpu())
torch.save(outs, sys.argv[1])
"""


def test_tma_gather_matches_cp_async(tmp_path):
    """Pass 3's two row-fetch paths (16-byte cp.async, the default, and the opt-in TMA
    gather4 for 16-bit caches with a uniform row pitch) give bit-identical outputs."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "gather.py"
    script.write_text(_GATHER_SCRIPT)
    res = {}
    for mode in ("tma", "cpasync"):
        env = dict(os.environ)
        env["DCR_ATTEND_GATHER"] = mode
        out = tmp_path / f"{mode}.pt"
        subprocess.run([sys.executable, str(script), str(out), root], env=env, check=True,
                       timeout=300)
        res[mode] = torch.load(out)
    for a, b in zip(res["tma"], res["cpasync"]):
        assert torch.equal(a, b)
