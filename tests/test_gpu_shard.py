"""Sequence- and KV-head-sharded decode on the GPU, through the C ABI (dcr_shard_*).

Single GPU: the ranks of a sequence split are emulated in lockstep on cuda:0 (each rank's
chunk in its own buffers, the collectives replaced by a sum and a stack on the device);
the CUDA phases must reproduce the oracle of the unsharded context: the union of the
ranks' selections bit-exact, O within the attention tolerance. At full size the union
is compared with the single-GPU CUDA selection (itself bit-exact against the oracle in
test_gpu_parity.py) and the selected counts must add up to k.

Two GPUs (skipped on a 1-GPU box): the real NCCL path, one process per GPU.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from golden_io import attention_close, dtype_name, to_np
from shard_cases import CASES, chunk, make_case

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def run_lockstep(Q, K, V, splits, k, eps=1e-12):
    """All ranks of a sequence split on one GPU. Returns (O, [(idx, cnt) per rank])."""
    from dcr_b200.sharded import CudaSequenceShardStep
    W = len(splits)
    B, H, _ = Q.shape
    H_kv = K.shape[1]
    Qd = Q.to(DEV)
    steps = []
    for r in range(W):
        Kc, Vc = chunk(K, splits, r).to(DEV), chunk(V, splits, r).to(DEV)
        steps.append(CudaSequenceShardStep(B, H, H_kv, splits[r], k, dtype=Q.dtype, device=DEV,
                                           eps=eps).bind(Qd, Kc, Vc))
    hist = torch.stack([s.score() for s in steps]).sum(0, dtype=torch.int32)
    lo_all = torch.stack([s.refine(hist) for s in steps])
    states = torch.stack([s.attend(lo_all, W, r) for r, s in enumerate(steps)])
    O = steps[0].combine(states)
    sels = [s.selection() for s in steps]
    torch.cuda.synchronize()
    return O, sels


def union_rows(sels, splits):
    """[rows, k] ascending global positions from the ranks' (idx, cnt)."""
    rows = sels[0][1].numel()
    out = []
    for r in range(rows):
        parts = []
        for w, (idx, cnt) in enumerate(sels):
            c = int(cnt.view(-1)[r])
            parts.append(idx.view(rows, -1)[r, :c].cpu().numpy().astype(np.int64) + sum(splits[:w]))
        out.append(np.concatenate(parts))
    return out


@pytest.mark.parametrize("name", list(CASES))
def test_lockstep_vs_oracle(oracle_mod, cuda_lib, name):
    from dcr_b200 import _lib
    Q, K, V, splits, k = make_case(name)
    O, sels = run_lockstep(Q, K, V, splits, k)
    assert _lib.read_device_status(clear=True) == 0
    _, _, idx, O_ref = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dtype_name(Q), k)
    for r, got in enumerate(union_rows(sels, splits)):
        assert got.shape == (k,) and np.all(np.diff(got) > 0), (name, r)
        assert np.array_equal(got, idx[r].astype(np.int64)), (name, r)
    ok, st = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to=dtype_name(Q))
    assert ok, (name, st)


@pytest.mark.parametrize("B,H,H_kv,splits,c,dt", [
    (2, 32, 8, [16385, 16383, 20000, 12768], 0.15, torch.float16),   # 4 ranks, ragged, 64K
    (1, 32, 8, [32768, 32768], 0.05, torch.bfloat16),                 # 2 ranks
    (3, 16, 2, [9000, 1, 7, 8200], 0.3, torch.bfloat16),              # 1- and 7-long chunks
])
def test_lockstep_medium_vs_oracle(oracle_mod, cuda_lib, B, H, H_kv, splits, c, dt):
    from dcr_b200 import _lib
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    from dcr_b200.synthetic import make_decode_inputs
    k = adaptive_k_window(64, sum(splits), c)
    Q, K, V = make_decode_inputs(B, H, H_kv, sum(splits), dtype=dt, seed=11)
    O, sels = run_lockstep(Q, K, V, splits, k)
    assert _lib.read_device_status(clear=True) == 0
    _, _, idx, O_ref = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dtype_name(Q), k)
    for r, got in enumerate(union_rows(sels, splits)):
        assert np.array_equal(got, idx[r].astype(np.int64)), r
    ok, st = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to=dtype_name(Q))
    assert ok, st


@pytest.mark.slow
@pytest.mark.parametrize("W", [2, 4, 8])
def test_lockstep_full_size_matches_single_gpu(cuda_lib, W):
    """Hero shape per rank (B=4, 32/8 heads, 32768 positions per rank, c=0.15 of the whole
    context): the union equals the single-GPU selection over the whole context."""
    from dcr_b200 import _lib
    from dcr_b200.kernel.cuda import topk_qaxis_attention, topk_qaxis_select
    from dcr_b200.models.llama.adaptive import adaptive_k_window
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, n = 4, 32, 8, 32768
    N = n * W
    k = adaptive_k_window(64, N, 0.15)
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.float16, seed=3, device=DEV)
    splits = [n] * W
    O, sels = run_lockstep(Q, K, V, splits, k)
    assert _lib.read_device_status(clear=True) == 0
    idx = topk_qaxis_select(Q, K, k).view(B * H, k).cpu().numpy().astype(np.int64)
    counts = torch.stack([c.view(-1) for _, c in sels]).sum(0)
    assert bool((counts == k).all())
    for r, got in enumerate(union_rows(sels, splits)):
        assert np.array_equal(got, idx[r]), r
    O1 = topk_qaxis_attention(Q, K, V, k)
    ok, st = attention_close(O.float().cpu().numpy(), O1.float().cpu().numpy(),
                             got_rounded_to="f16")
    assert ok, st


def test_shard_errors(cuda_lib):
    from dcr_b200 import _lib
    lib = cuda_lib
    B, H, H_kv, N, k = 1, 4, 1, 100, 10
    nb = lib.dcr_shard_workspace_bytes(B, H, H_kv, N, 64, k)
    assert nb > 0
    assert lib.dcr_shard_workspace_bytes(B, H, 3, N, 64, k) == 0      # H % H_kv != 0
    ws = torch.empty(nb, dtype=torch.uint8, device=DEV)
    hist = torch.empty(B * H, 256, dtype=torch.int32, device=DEV)
    st = lib.dcr_shard_refine(B, H, H_kv, N, 64, k, hist.data_ptr(), hist.data_ptr(),
                              ws.data_ptr(), nb - 1, None)
    assert st == _lib.DCR_ERR_WORKSPACE
    st = lib.dcr_shard_refine(B, H, H_kv, N, 64, 0, hist.data_ptr(), hist.data_ptr(),
                              ws.data_ptr(), nb, None)
    assert st == _lib.DCR_ERR_K_RANGE
    st = lib.dcr_shard_combine(None, 2, B, H, 64, 0, ws.data_ptr(), None)
    assert st == _lib.DCR_ERR_NULL
    st = lib.dcr_shard_combine(hist.data_ptr(), 2, B, H, 64, 9, ws.data_ptr(), None)
    assert st == _lib.DCR_ERR_DTYPE


def test_decoder_rejects_k_not_below_total(cuda_lib):
    """k_eff >= the whole context raises like the single-GPU path (the caller's SDPA case)."""
    from dcr_b200.kernel.cuda._common import KEffRangeError
    from dcr_b200.sharded import SequenceShardedDecoder

    class OneRank:
        world, rank = 1, 0

        def all_gather(self, t, out=None):
            return t.unsqueeze(0)

    with pytest.raises(KEffRangeError):
        SequenceShardedDecoder(1, 4, 1, 100, 100, dtype=torch.bfloat16, device=DEV,
                               comm=OneRank())


class _OneRank:
    world, rank = 1, 0

    def all_gather(self, t, out=None):
        return t.unsqueeze(0)

    def barrier(self):
        pass


@pytest.mark.parametrize("B,N,k", [(2, 5000, 750), (2, 20000, 3000), (24, 5000, 750)])
def test_peer_exchange_single_rank_steps(oracle_mod, cuda_lib, B, N, k):
    """The peer-exchange step with one rank: every kernel of the path (no peer to wait
    for), over consecutive steps (the epoch advances), eager and as a graph replay.
    N=5000 gives the fused selection 2 vectors of keys per thread (index lists, the
    per-head Pass 3); N=20000 gives it whole 32-bit words per thread, so it also writes
    bitmaps and the step runs the union Pass 3 with its state published into the buffer.
    B=24 gives 768 rows, more than one wave of the fused selection's CTAs, so the step
    runs the phase kernels (histograms, selection) with the same exchanges."""
    from dcr_b200 import _lib
    from dcr_b200.sharded import SequenceShardedDecoder
    from dcr_b200.synthetic import fresh_queries, make_decode_inputs
    H, H_kv = 32, 8
    _, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=4)
    Qs = fresh_queries(4, B, H, dtype=torch.bfloat16, seed=6)
    Kd, Vd = K.to(DEV), V.to(DEV)
    dec = SequenceShardedDecoder(B, H, H_kv, N, k, dtype=torch.bfloat16, device=DEV,
                                 comm=_OneRank(), exchange="peer")
    outs = []
    for i in range(3):
        Q = Qs[i].contiguous()
        O = dec(Q.to(DEV), Kd, Vd)
        idx, cnt = dec.selection_global()
        assert _lib.read_device_status(clear=True) == 0
        _, _, ref_idx, O_ref = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), "bf16", k)
        assert bool((cnt == k).all())
        assert np.array_equal(idx.view(B * H, k).cpu().numpy(), ref_idx.astype(np.int64))
        ok, st = attention_close(O.float().cpu().numpy(), O_ref, got_rounded_to="bf16")
        assert ok, (i, st)
        outs.append(O.clone())
    # the same three steps captured once and replayed
    Qd = torch.empty(B, H, 64, dtype=torch.bfloat16, device=DEV)
    Od = torch.empty_like(Qd)
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            dec(Qd, Kd, Vd, out=Od)
        for i in range(3):
            Qd.copy_(Qs[i].to(DEV))
            g.replay()
            side.synchronize()
            assert torch.equal(Od, outs[i]), i
    assert _lib.read_device_status(clear=True) == 0
    del g
    dec.close()


def test_peer_wait_expires_and_reports(cuda_lib):
    """Failure detection without a fault: a world-2 exchange in one process on one GPU
    whose 'peer' buffer nothing writes. The step's first wait must give up after its bound,
    raise DCR_ERR_DEVICE_TIMEOUT and set the abort word (every later wait returns at once),
    and after dcr_xchg_reset the context and the buffers work again."""
    import ctypes
    import time
    from dcr_b200 import _lib
    from dcr_b200.sharded import CudaSequenceShardStep
    from dcr_b200.synthetic import make_decode_inputs
    lib = cuda_lib
    B, H, H_kv, N, k = 1, 8, 2, 2048, 200
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=3, device=DEV)
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
    for b in bufs:
        assert lib.dcr_xchg_create(B, H, 2, ctypes.byref(b), handle) == 0
    peers = (ctypes.c_void_p * 2)(bufs[0].value, bufs[1].value)  # 'rank 1' never runs
    step = CudaSequenceShardStep(B, H, H_kv, N, k, dtype=torch.bfloat16, device=DEV).bind(Q, K, V)
    O = torch.empty(B, H, 64, dtype=torch.bfloat16, device=DEV)
    assert _lib.read_device_status(clear=True) == 0
    t0 = time.perf_counter()
    st = lib.dcr_shard_decode_peer(Q.data_ptr(), K.data_ptr(), V.data_ptr(), 0, step.ksb,
                                   step.ksh, step.vsb, step.vsh, B, H, H_kv, N, 64, k, 1e-12,
                                   peers, 2, 0, N, O.data_ptr(), step.ws.data_ptr(),
                                   step.ws_bytes, None)
    assert st == 0
    status = _lib.read_device_status(clear=True)       # synchronises
    elapsed = time.perf_counter() - t0
    assert status & _lib.DCR_ERR_DEVICE_TIMEOUT
    assert 1.5 < elapsed < 30.0                         # one bounded wait, then the abort word
    # after a reset of both buffers the single-rank step works again on the same context
    for b in bufs:
        assert lib.dcr_xchg_reset(b, B, H, 2, None) == 0
        assert lib.dcr_xchg_destroy(b) == 0
    one = ctypes.c_void_p()
    assert lib.dcr_xchg_create(B, H, 1, ctypes.byref(one), handle) == 0
    peers1 = (ctypes.c_void_p * 1)(one.value)
    st = lib.dcr_shard_decode_peer(Q.data_ptr(), K.data_ptr(), V.data_ptr(), 0, step.ksb,
                                   step.ksh, step.vsb, step.vsh, B, H, H_kv, N, 64, k, 1e-12,
                                   peers1, 1, 0, N, O.data_ptr(), step.ws.data_ptr(),
                                   step.ws_bytes, None)
    assert st == 0
    assert _lib.read_device_status(clear=True) == 0
    assert torch.isfinite(O.float()).all()
    assert lib.dcr_xchg_destroy(one) == 0


# ---- two GPUs: the real NCCL path ------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_gpus_nccl(oracle_mod, tmp_path):
    import shard_workers
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=shard_workers.nccl_rank, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(2)]
    for name, (Q, K, V, splits, k) in shard_workers.nccl_cases():
        _, _, idx, O_ref = oracle_mod.decode(to_np(Q), to_np(K), to_np(V), dtype_name(Q), k)
        rows = idx.shape[0]
        for r in range(rows):
            got = np.sort(np.concatenate([res[w][name]["sel"][r].numpy() for w in range(2)]))
            assert np.array_equal(got, idx[r].astype(np.int64)), (name, r)
        assert torch.equal(res[0][name]["O"], res[1][name]["O"])
        ok, st = attention_close(res[0][name]["O"].float().numpy(), O_ref,
                                 got_rounded_to=dtype_name(Q))
        assert ok, (name, st)
    # KV-head split: same O on both ranks; against the single-GPU step only the split-K
    # summation order differs (its split factor follows the rank's row count)
    for name, _ in shard_workers.nccl_cases():
        for w in range(2):     # peer-memory exchange: same selection and O as over NCCL
            assert torch.equal(res[w][name]["O_peer"], res[w][name]["O"]), (name, w)
            for a, b in zip(res[w][name]["sel_peer"], res[w][name]["sel"]):
                assert torch.equal(a, b), (name, w)
            assert res[w][name]["status"] == 0
    kv = res[0]["kv_head"]
    assert torch.equal(res[1]["kv_head"]["O"], kv["O"])
    ok, st = attention_close(kv["O"].float().numpy(), kv["O_single"].float().numpy(),
                             got_rounded_to="bf16")
    assert ok, st


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_tensor_parallel_model_on_two_gpus(tmp_path):
    """The Llama decode model split by KV head over 2 GPUs (two NCCL all-reduces per
    layer) gives the unsplit model's logits within bf16 noise, the same logits and greedy
    tokens on both ranks, and replays its steps as CUDA graphs holding the all-reduces."""
    import shard_workers
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=shard_workers.tp_model_rank, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(os.path.join(tmp_path, f"tp{r}.pt")) for r in range(2)]
    assert res[0]["held"] == [0] and res[1]["held"] == [1]
    assert torch.equal(res[0]["tokens"], res[1]["tokens"])
    for mode in ("dense", "dcr"):
        assert torch.equal(res[0]["tp_" + mode], res[1]["tp_" + mode])
    # dense attention: only the rounding of the split GEMMs and the bf16 all-reduce differ
    full, tp = res[0]["full_dense"], res[0]["tp_dense"]
    assert (tp - full).abs().max().item() <= 3e-2 * max(full.abs().max().item(), 1.0)
    # sparse: the same, plus top-K sets that may swap a near-tied boundary row when q and k
    # differ in their last bits
    full, tp = res[0]["full_dcr"], res[0]["tp_dcr"]
    assert ((tp - full).norm() / full.norm()).item() <= 5e-2
