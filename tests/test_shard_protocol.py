"""Host side of the multi-GPU splits, on CPU: world_size 2, 3 and 4 ``gloo`` ranks.

Each rank runs dcr_b200.sharded's collective protocol with the CPU restatement of the
per-rank phases (oracle/shard_protocol.py) and the single-GPU oracle for the KV-head
split. Checked against the oracle of the whole, unsharded context:
  - the union of the ranks' selected positions equals the reference selection over the
    concatenated context, bit-exact (ties at the threshold included);
  - O of the sequence split matches the oracle's fp32 attention; every rank gets the same O;
  - the KV-head split's O equals the single-process oracle's.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import shard_workers
from shard_cases import CASES_BY_WORLD, make_case


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    t = t.contiguous()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


def _dtn(t):
    return {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[t.dtype]


@pytest.fixture(scope="module", params=[2, 3, 4])
def gloo_results(request, tmp_path_factory, oracle_mod):
    world = request.param
    out = str(tmp_path_factory.mktemp(f"gloo{world}"))
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=shard_workers.gloo_rank, args=(r, world, port, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return world, [torch.load(os.path.join(out, f"rank{r}.pt")) for r in range(world)]


def test_sequence_split_selects_the_global_top_k(gloo_results, oracle_mod):
    world, res = gloo_results
    for name in CASES_BY_WORLD.get(world, []):
        Q, K, V, splits, k = make_case(name)
        _, _, idx, O_ref = oracle_mod.decode(_bits(Q), _bits(K), _bits(V), _dtn(Q), k)
        rows = idx.shape[0]
        for r in range(rows):
            got = np.sort(np.concatenate([res[w][name]["sel"][r].numpy() for w in range(world)]))
            assert got.shape == (k,), (name, r, got.shape)
            assert np.array_equal(got, idx[r].astype(np.int64)), (name, r)
        O0 = res[0][name]["O"].numpy()
        for w in range(1, world):
            assert np.array_equal(res[w][name]["O"].numpy(), O0), (name, w)
        np.testing.assert_allclose(O0.reshape(O_ref.shape), O_ref, rtol=2e-4, atol=2e-5,
                                   err_msg=name)


def test_ties_straddle_the_chunk_boundary(gloo_results):
    world, res = gloo_results
    if "ties_2r" not in CASES_BY_WORLD.get(world, []):
        pytest.skip("2-rank case")
    sel0 = res[0]["ties_2r"]["sel"][0].numpy()
    sel1 = res[1]["ties_2r"]["sel"][0].numpy()
    # head 0: the 200 lowest positions of the tie group 100..411, 156 on rank 0, 44 on rank 1
    assert np.array_equal(sel0, np.arange(100, 256))
    assert np.array_equal(sel1, np.arange(256, 300))


def test_rank_without_selected_keys(gloo_results):
    world, res = gloo_results
    if "empty_rank_2r" not in CASES_BY_WORLD.get(world, []):
        pytest.skip("2-rank case")
    assert res[1]["empty_rank_2r"]["sel"][0].numel() == 0
    assert torch.isfinite(res[1]["empty_rank_2r"]["O"]).all()


def test_kv_head_split_matches_unsharded(gloo_results, oracle_mod):
    world, res = gloo_results
    if 8 % world:
        pytest.skip("8 KV heads do not split over this many ranks")
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(2, 32, 8, 700, dtype=torch.bfloat16, seed=9)
    O_ref = oracle_mod.decode(_bits(Q), _bits(K), _bits(V), "bf16", 106)[3]
    for w in range(world):
        assert np.array_equal(res[w]["kv_head"]["O"].numpy(), O_ref)
