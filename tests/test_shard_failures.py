"""Failure detection of the sequence split, on the host: gloo ranks on CPU, world 2 and 3.

A rank of a sharded decode step can fail without any GPU fault: its host code raises in
the middle of a step, it leaves between steps, it stalls, or it was given another step
(k_eff, head counts) than its peers. Each case must end on every rank with a reported
error within the process group's timeout, never with a hang or a silently wrong result:

* a rank that raises or leaves: the others' next collective fails (connection closed or
  timed out) and raises;
* a rank that stalls: the others' collective times out after the process group's timeout;
* ranks that disagree on the step: the agreement all-gather at set-up
  (``dcr_b200.sharded.agree_on_step``) raises ShardMismatchError on every rank.

The faults are made on the host (a communicator that raises, a rank that exits or sleeps);
nothing here touches a GPU.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket

import pytest

import shard_workers

TIMEOUT_S = 5.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, scenario, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=shard_workers.gloo_fault_rank,
                         args=(r, world, port, str(tmp_path), scenario, TIMEOUT_S))
             for r in range(world)]
    for p in procs:
        p.start()
    hung = []
    for r, p in enumerate(procs):
        p.join(timeout=120)
        if p.is_alive():
            hung.append(r)
            p.kill()
            p.join()
    assert not hung, f"ranks {hung} still running after 120 s: a hang"
    recs = []
    for r in range(world):
        path = os.path.join(str(tmp_path), f"rank{r}.json")
        assert os.path.exists(path), f"rank {r} wrote no outcome (exit code {procs[r].exitcode})"
        recs.append(json.load(open(path)))
    return recs


@pytest.mark.parametrize("world", [2, 3])
def test_rank_raising_mid_step_fails_its_peers(world, tmp_path):
    recs = _run(world, "raise_mid_step", tmp_path)
    assert recs[-1]["outcome"] == "injected"
    for r in recs[:-1]:
        assert r["outcome"] == "error", r
        assert r["elapsed_s"] < TIMEOUT_S + 30, r


@pytest.mark.parametrize("world", [2, 3])
def test_rank_leaving_between_steps_fails_the_next_step(world, tmp_path):
    recs = _run(world, "leave_between_steps", tmp_path)
    assert recs[-1]["outcome"] == "left" and recs[-1]["steps_ok"] == 1
    for r in recs[:-1]:
        assert r["steps_ok"] == 1 and r["outcome"] == "error", r
        assert r["elapsed_s"] < TIMEOUT_S + 30, r


def test_stalled_rank_times_out_its_peers(tmp_path):
    recs = _run(2, "stall", tmp_path)
    r0 = recs[0]
    assert r0["steps_ok"] == 1 and r0["outcome"] == "error", r0
    # the peer waited for the process group's timeout, not for the stalled rank
    assert r0["elapsed_s"] < 3 * TIMEOUT_S, r0
    assert recs[1]["outcome"] in ("error", "ok"), recs[1]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("scenario,field", [("disagree_k", "k_eff"),
                                            ("disagree_heads", "H")])
def test_ranks_disagreeing_on_the_step_all_raise(world, scenario, field, tmp_path):
    recs = _run(world, scenario, tmp_path)
    for r in recs:
        assert r["outcome"] == "mismatch", r
        assert r["type"] == "ShardMismatchError" and field in r["msg"], r
        assert r["steps_ok"] == 0
