"""Rank bodies of the multi-process sharding tests (spawned processes, one per rank).

``gloo_rank`` runs the host side of both splits on CPU over ``gloo``: the collective
protocol of dcr_b200.sharded with the CPU restatement (oracle/shard_protocol.py) as each
rank's compute. ``nccl_rank`` runs the CUDA path over NCCL, one GPU per rank. Each rank
writes its results to ``out_dir/rank{r}.pt``; the test process checks them.
"""
from __future__ import annotations

import datetime
import os
import sys


def _paths():
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "dcr-attention_v3_b200"), here):
        if p not in sys.path:
            sys.path.insert(0, p)


def _bits(t):
    import numpy as np
    import torch
    t = t.contiguous()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


def gloo_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    _paths()
    import torch
    import torch.distributed as dist

    from dcr_b200.sharded import TorchComm, kv_head_sharded_attention, sequence_shard_step
    from oracle import oracle
    from oracle.shard_protocol import OracleSequenceShardStep
    from shard_cases import CASES_BY_WORLD, chunk, make_case

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = TorchComm()
    res = {}
    for name in CASES_BY_WORLD.get(world, []):
        Q, K, V, splits, k = make_case(name)
        step = OracleSequenceShardStep(Q, chunk(K, splits, rank), chunk(V, splits, rank), k)
        O = sequence_shard_step(step, comm)
        off = sum(splits[:rank])
        res[name] = {"O": O, "sel": [torch.from_numpy(s + off) for s in step.selection()]}

    # KV-head split: 8 KV heads over the ranks, the rank's heads through the oracle
    from dcr_b200.synthetic import make_decode_inputs
    B, H, H_kv, N, k = 2, 32, 8, 700, 106
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=9)
    hk = H_kv // world

    def local(Qr, Kr, Vr, k_eff, eps=1e-12):
        O = oracle.decode(_bits(Qr), _bits(Kr), _bits(Vr), "bf16", k_eff, eps)[3]
        return torch.from_numpy(O)

    if H_kv % world == 0:
        O_kv = kv_head_sharded_attention(Q, K[:, rank * hk:(rank + 1) * hk].contiguous(),
                                         V[:, rank * hk:(rank + 1) * hk].contiguous(), k,
                                         comm=comm, local_attention=local)
        res["kv_head"] = {"O": O_kv}
    torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def nccl_cases():
    """(name, (Q, K, V, splits, k)) of the 2-GPU test, on the CPU."""
    from shard_cases import make_case
    return [(n, make_case(n)) for n in ("bf16_2r", "ties_2r", "empty_rank_2r", "gqa2_bf16_2r",
                                        "long_2r")]


def nccl_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    _paths()
    import torch
    import torch.distributed as dist

    from dcr_b200.kernel.cuda import topk_qaxis_attention
    from dcr_b200.sharded import SequenceShardedDecoder, kv_head_sharded_attention
    from dcr_b200.synthetic import make_decode_inputs
    from shard_cases import chunk

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    from dcr_b200 import _lib
    res = {}
    for name, (Q, K, V, splits, k) in nccl_cases():
        B, H, _ = Q.shape
        Kc, Vc = chunk(K, splits, rank).to(dev), chunk(V, splits, rank).to(dev)
        r = {}
        for ex in ("nccl", "peer"):
            dec = SequenceShardedDecoder(B, H, K.shape[1], splits[rank], k, dtype=Q.dtype,
                                         device=dev, exchange=ex)
            for _ in range(3):   # repeated steps: the peer exchange's epochs advance
                O = dec(Q.to(dev), Kc, Vc)
            idx, cnt = dec.selection_global()
            idx, cnt = idx.view(B * H, -1).cpu(), cnt.view(-1).cpu()
            sfx = "" if ex == "nccl" else "_peer"
            r["O" + sfx] = O.cpu()
            r["sel" + sfx] = [idx[i, :int(cnt[i])].clone() for i in range(B * H)]
            dec.close()
        r["status"] = _lib.read_device_status(clear=True)
        res[name] = r
    B, H, H_kv, N, k = 2, 32, 8, 4096, 614
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=9, device=dev)
    hk = H_kv // world
    O = kv_head_sharded_attention(Q, K[:, rank * hk:(rank + 1) * hk], V[:, rank * hk:(rank + 1) * hk],
                                  k)
    res["kv_head"] = {"O": O.cpu(), "O_single": topk_qaxis_attention(Q, K, V, k).cpu()}
    torch.cuda.synchronize()
    torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def tp_model_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    """A small Llama decode model split across `world` GPUs by KV head (TPDCRLlamaDecoder
    over NCCL): one eager step's logits, the same model unsplit on every rank (its logits
    for comparison), and 3 greedy steps replayed as per-step CUDA graphs holding the
    all-reduces."""
    _paths()
    import torch
    import torch.distributed as dist

    from dcr_b200.models.llama.model import (DCRLlamaDecoder, GreedyDecodeGraphs,
                                              LlamaDecodeConfig, TPDCRLlamaDecoder)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = LlamaDecodeConfig(vocab=1000, hidden=512, intermediate=1024, layers=2, heads=8,
                            kv_heads=2)
    B, N0, steps = 2, 3000, 3
    full = DCRLlamaDecoder(cfg, T_dispatch=1024, device=dev, seed=5)
    tp = TPDCRLlamaDecoder(cfg, world=world, rank=rank, T_dispatch=1024, device=dev,
                           seed=6).load_from(full)
    cf = full.new_caches(B, N0 + steps + 1)
    full.prefill_synthetic(cf, N0, seed=21)
    ct = tp.new_caches(B, N0 + steps + 1)
    tp.prefill_synthetic(ct, N0, seed=21)
    cos, sin = full.rope_table(N0 + 1)
    c1, s1 = cos[N0].expand(B, 64).contiguous(), sin[N0].expand(B, 64).contiguous()
    tok = torch.tensor([4, 8], device=dev)
    res = {"held": list(tp.kv_heads_held())}
    for mode in ("dense", "dcr"):
        full.set_attention(mode)
        tp.set_attention(mode)
        for c in cf + ct:
            c.length = N0
        res["full_" + mode] = full.step(tok, cf, c1, s1).float().cpu()
        res["tp_" + mode] = tp.step(tok, ct, c1, s1).float().cpu()
    for c in ct:
        c.length = N0
    runner = GreedyDecodeGraphs(tp, ct, steps)
    res["tokens"] = runner.run(torch.tensor([4, 8]))
    runner.close()
    dist.barrier()
    torch.save(res, os.path.join(out_dir, f"tp{rank}.pt"))
    dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
# Host-side failure injection (gloo ranks on CPU; no GPU is involved)
# ---------------------------------------------------------------------------------------
class FaultyComm:
    """A TorchComm whose rank `victim` raises at its `fail_at`-th collective (0-based), the
    way a rank whose host code fails mid-step would leave its peers."""

    def __init__(self, comm, victim: int, fail_at: int):
        self.comm, self.victim, self.fail_at, self.calls = comm, victim, fail_at, 0
        self.world, self.rank = comm.world, comm.rank

    def _tick(self):
        n = self.calls
        self.calls += 1
        if self.rank == self.victim and n == self.fail_at:
            raise RuntimeError("injected fault on rank %d at collective %d" % (self.rank, n))

    def all_reduce_sum_(self, t):
        self._tick()
        return self.comm.all_reduce_sum_(t)

    def all_gather(self, t, out=None):
        self._tick()
        return self.comm.all_gather(t, out)

    def barrier(self):
        self._tick()
        self.comm.barrier()


def gloo_fault_rank(rank: int, world: int, port: int, out_dir: str, scenario: str,
                    timeout_s: float) -> None:
    """One rank of a sequence-split decode with a host-side fault in `scenario`:

    * ``raise_mid_step``: the last rank raises at its second collective of step 0;
    * ``leave_between_steps``: the last rank exits after step 0 without tearing down;
    * ``stall``: the last rank sleeps for 3 process-group timeouts before step 1;
    * ``disagree_k``: the last rank passes k_eff + 2;
    * ``disagree_heads``: the last rank passes other head counts.

    Writes ``rank{r}.json`` with what this rank saw, then leaves with os._exit."""
    _paths()
    import json
    import time

    import torch
    import torch.distributed as dist

    from dcr_b200.sharded import ShardMismatchError, TorchComm, agree_on_step, sequence_shard_step
    from dcr_b200.synthetic import make_decode_inputs
    from oracle.shard_protocol import OracleSequenceShardStep

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    victim = world - 1
    rec = {"rank": rank, "steps_ok": 0}

    def done(outcome, err=None, t0=None):
        rec["outcome"] = outcome
        if err is not None:
            rec["type"] = type(err).__name__
            rec["msg"] = str(err)[:300]
        if t0 is not None:
            rec["elapsed_s"] = time.perf_counter() - t0
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(rec, f)
        os._exit(0)

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    B, H, H_kv, n_local = 1, 8, 2, 300
    N = n_local * world
    k = 90
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=torch.bfloat16, seed=5)
    Kc = K[:, :, rank * n_local:(rank + 1) * n_local].contiguous()
    Vc = V[:, :, rank * n_local:(rank + 1) * n_local].contiguous()
    base = TorchComm()
    comm = FaultyComm(base, victim, 1) if scenario == "raise_mid_step" else base
    my_k = k + 2 if (scenario == "disagree_k" and rank == victim) else k
    my_H, my_Hkv = (16, 4) if (scenario == "disagree_heads" and rank == victim) else (H, H_kv)
    t0 = time.perf_counter()
    try:
        agree_on_step(base, B=B, H=my_H, H_kv=my_Hkv, N_local=n_local, k_eff=my_k,
                      dtype=torch.bfloat16)
    except ShardMismatchError as e:
        done("mismatch", e, t0)
    for step_i in range(2):
        if scenario == "leave_between_steps" and rank == victim and step_i == 1:
            done("left")
        if scenario == "stall" and rank == victim and step_i == 1:
            time.sleep(3 * timeout_s)
        t0 = time.perf_counter()
        try:
            step = OracleSequenceShardStep(Q, Kc, Vc, k)
            O = sequence_shard_step(step, comm)
            if not torch.isfinite(O).all():
                done("bad_output")
            rec["steps_ok"] += 1
        except RuntimeError as e:
            done("injected" if "injected fault" in str(e) else "error", e, t0)
    done("ok")
