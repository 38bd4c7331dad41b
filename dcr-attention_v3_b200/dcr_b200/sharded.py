"""Sparse decode attention over a KV cache split across the GPUs of one node.

The reference runs a layer's decode step on one GPU (topk_qaxis_attention,
dcr_attention/kernel/triton/topk_axis.py:58). Two splits across ranks keep its result:

* **KV-head split** (:func:`kv_head_sharded_attention`). Rank r of W owns KV heads
  [r*H_kv/W, (r+1)*H_kv/W) and the query heads that read them. The (b, h_kv) units are
  independent, so every rank runs the single-GPU step on its heads and one all-gather of
  the outputs ([B, H/W, D] per rank) assembles O. The selection is the single-GPU one;
  O differs from it only by fp32 summation order (Pass 3's split-K factor follows the
  number of rows a GPU holds).

* **Sequence split** (:class:`SequenceShardedDecoder`). Rank r holds positions
  [off_r, off_r + N_r) of every cache row, off_r increasing with r. The top-K is exact
  over the whole context: ranks exchange 256-bin histograms of the 16-bit score keys
  (all-reduce of the high byte, all-gather of the low byte within the threshold's bin),
  which fixes the k-th largest key T, how many keys above it there are, and, because
  lower ranks hold lower positions, how many of the keys equal to T each rank takes (the
  reference's lowest-index tie rule). Each rank attends to its share and publishes its
  unnormalised (m, l, o); an all-gather and a combine give O. The selected set is the
  reference's (_select_topk_indices, qaxis_topk_reference.py:91) over the concatenated
  context; O differs from a single-GPU step only by fp32 summation order.

The sequence split's exchanges run in one of two ways. ``exchange="peer"`` (default on
GPUs): the kernels push their histogram and state rows straight into the other ranks'
exchange buffers over NVLink (CUDA IPC peer memory, :class:`PeerExchange`) and wait on
per-row flags, so a step is one C call with no host collective (dcr_shard_decode_peer).
``exchange="nccl"``: the phases of :class:`CudaSequenceShardStep` with three
``torch.distributed`` collectives (:class:`TorchComm`) between them. There is no CPU path.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch

from dcr_b200 import _lib
from dcr_b200.kernel.cuda._common import (HEAD_DIM, cache_strides, check_dtype, check_groups,
                                          check_k_range, require)

STATE_FLOATS = HEAD_DIM + 2  # (m, l, o[64]) per (b, h) row


class TorchComm:
    """The three collectives of the sharded step over a ``torch.distributed`` group."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self._dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._gloo = dist.get_backend(group) == "gloo"

    def all_reduce_sum_(self, t: torch.Tensor) -> torch.Tensor:
        self._dist.all_reduce(t, op=self._dist.ReduceOp.SUM, group=self.group)
        return t

    def barrier(self) -> None:
        self._dist.barrier(group=self.group)

    def all_gather(self, t: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[world, *t.shape], rank-major."""
        if out is None:
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if self._gloo:
            self._dist.all_gather(list(out.unbind(0)), t.contiguous(), group=self.group)
        else:
            self._dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out


class ShardMismatchError(ValueError):
    """The ranks of a sharded step disagree on what the step is (raised on every rank)."""


_DTYPE_IDS = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def agree_on_step(comm, *, B: int, H: int, H_kv: int, N_local: int, k_eff: int,
                  dtype: torch.dtype, device=None):
    """Checks, with one all-gather, that every rank describes the same step, and returns
    (the ranks' chunk lengths, this rank's offset, the whole context's length).

    Every rank must pass the same B, H, H_kv, k_eff and dtype (N_local may differ: it is
    each rank's chunk). The exact global top-K depends on all of them: a rank with another
    k_eff would select from other histogram bins than its peers and the combined set would
    not be the reference's. Every rank sees the same gathered values, so every rank raises
    the same :class:`ShardMismatchError` (or none); no rank is left waiting in a later
    collective. Then ``0 < k_eff < sum(N_r)`` is checked as in the single-GPU step."""
    meta = torch.tensor([B, H, H_kv, int(N_local), int(k_eff), _DTYPE_IDS.get(dtype, -1)],
                        dtype=torch.int64, device=device if device is not None else "cpu")
    allm = comm.all_gather(meta).view(comm.world, -1).cpu()
    names = ("B", "H", "H_kv", "N_local", "k_eff", "dtype")
    for j, name in enumerate(names):
        if name == "N_local":
            continue
        vals = allm[:, j].tolist()
        if any(v != vals[0] for v in vals):
            raise ShardMismatchError(
                f"ranks disagree on {name}: {vals} (rank-ordered); every rank of a sharded "
                f"step must pass the same B, H, H_kv, k_eff and dtype")
    n_locals = [int(x) for x in allm[:, 3].tolist()]
    if any(n <= 0 for n in n_locals):
        raise ShardMismatchError(f"every rank needs a non-empty chunk, got N_local={n_locals}")
    n_total = sum(n_locals)
    check_k_range(int(k_eff), n_total)
    return n_locals, sum(n_locals[: comm.rank]), n_total


def sequence_shard_step(step, comm, bufs: Optional[dict] = None):
    """One decode step of the sequence split: the per-rank phases of ``step`` with the
    three collectives between them. Returns O [B, H, D] (identical on every rank).

    ``step`` provides ``score(hist_hi)``, ``refine(hist_hi_sum, hist_lo)``,
    ``attend(hist_lo_all, world, rank, state)`` and ``combine(states, out)``; ``bufs`` may
    hold preallocated ``hist_hi``, ``hist_lo``, ``hist_lo_all``, ``state``, ``states`` and
    ``out``."""
    bufs = bufs if bufs is not None else {}
    hist_hi = step.score(bufs.get("hist_hi"))
    comm.all_reduce_sum_(hist_hi)
    hist_lo = step.refine(hist_hi, bufs.get("hist_lo"))
    hist_lo_all = comm.all_gather(hist_lo, bufs.get("hist_lo_all"))
    state = step.attend(hist_lo_all, comm.world, comm.rank, bufs.get("state"))
    states = comm.all_gather(state, bufs.get("states"))
    return step.combine(states, bufs.get("out"))


class CudaSequenceShardStep:
    """This rank's share of a sequence-sharded step on its GPU (libdcr_b200 dcr_shard_*).

    Bind the step's tensors with :meth:`bind`, then the phases run in order; the
    workspace carries state from one phase to the next."""

    def __init__(self, B: int, H: int, H_kv: int, N_local: int, k_eff: int, *,
                 dtype: torch.dtype, device: torch.device, eps: float = 1e-12,
                 workspace_buf: Optional[torch.Tensor] = None):
        check_groups(H, H_kv)
        require(N_local > 0, f"N_local must be > 0, got {N_local}")
        require(k_eff > 0, f"k_eff must be > 0, got {k_eff}")
        self.B, self.H, self.H_kv, self.N, self.k = B, H, H_kv, N_local, int(k_eff)
        self.rows = B * H
        self.cap = min(self.k, N_local)
        self.dtype = dtype
        self.dt = _lib.DTYPE_CODES[dtype]
        self.device = torch.device(device)
        self.eps = float(eps)
        self.lib = _lib.load()
        self.ws_bytes = int(self.lib.dcr_shard_workspace_bytes(B, H, H_kv, N_local, HEAD_DIM,
                                                               self.k))
        require(self.ws_bytes > 0, "unsupported shard shape")
        if workspace_buf is not None:
            require(workspace_buf.is_cuda and workspace_buf.dtype == torch.uint8 and
                    workspace_buf.numel() >= self.ws_bytes, "workspace_buf too small")
            self.ws = workspace_buf
        else:
            self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=self.device)
        self.Q = self.K = self.V = None

    def bind(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> "CudaSequenceShardStep":
        _lib.require_cuda(Q, K, V)
        require(Q.shape == (self.B, self.H, HEAD_DIM) and Q.is_contiguous(),
                f"Q must be a contiguous [{self.B}, {self.H}, {HEAD_DIM}] tensor")
        want = (self.B, self.H_kv, self.N, HEAD_DIM)
        require(tuple(K.shape) == want and tuple(V.shape) == want,
                f"K and V chunks must be {want}, got {tuple(K.shape)}, {tuple(V.shape)}")
        require(Q.dtype == K.dtype == V.dtype == self.dtype, "Q, K, V must share the dtype")
        self.ksb, self.ksh = cache_strides(K, "K_chunk")
        self.vsb, self.vsh = cache_strides(V, "V_chunk")
        self.Q, self.K, self.V = Q, K, V
        return self

    def _stream(self) -> int:
        return _lib.stream_ptr(self.device)

    def _hist(self, out):
        if out is None:
            out = torch.empty(self.rows, 256, dtype=torch.int32, device=self.device)
        return out

    def score(self, hist_hi=None):
        hist_hi = self._hist(hist_hi)
        st = self.lib.dcr_shard_score(self.Q.data_ptr(), self.K.data_ptr(), self.dt, self.ksb,
                                      self.ksh, self.B, self.H, self.H_kv, self.N, HEAD_DIM,
                                      self.k, self.eps, hist_hi.data_ptr(), self.ws.data_ptr(),
                                      self.ws_bytes, self._stream())
        _lib.check(st, "dcr_shard_score")
        return hist_hi

    def refine(self, hist_hi_sum, hist_lo=None):
        hist_lo = self._hist(hist_lo)
        st = self.lib.dcr_shard_refine(self.B, self.H, self.H_kv, self.N, HEAD_DIM, self.k,
                                       hist_hi_sum.data_ptr(), hist_lo.data_ptr(),
                                       self.ws.data_ptr(), self.ws_bytes, self._stream())
        _lib.check(st, "dcr_shard_refine")
        return hist_lo

    def attend(self, hist_lo_all, world: int, rank: int, state=None):
        if state is None:
            state = torch.empty(self.rows, STATE_FLOATS, dtype=torch.float32, device=self.device)
        st = self.lib.dcr_shard_attend(self.Q.data_ptr(), self.K.data_ptr(), self.V.data_ptr(),
                                       self.dt, self.ksb, self.ksh, self.vsb, self.vsh, self.B,
                                       self.H, self.H_kv, self.N, HEAD_DIM, self.k,
                                       hist_lo_all.data_ptr(), world, rank, state.data_ptr(),
                                       self.ws.data_ptr(), self.ws_bytes, self._stream())
        _lib.check(st, "dcr_shard_attend")
        return state

    def combine(self, states, out=None):
        world = states.shape[0]
        if out is None:
            out = torch.empty(self.B, self.H, HEAD_DIM, dtype=self.dtype, device=self.device)
        st = self.lib.dcr_shard_combine(states.data_ptr(), world, self.B, self.H, HEAD_DIM,
                                        self.dt, out.data_ptr(), self._stream())
        _lib.check(st, "dcr_shard_combine")
        return out

    def selection(self):
        """(idx [B, H, min(k, N_local)] int32 local positions ascending, counts [B, H])
        chosen on this rank by the last :meth:`attend`."""
        idx = torch.empty(self.B, self.H, self.cap, dtype=torch.int32, device=self.device)
        cnt = torch.empty(self.B, self.H, dtype=torch.int32, device=self.device)
        st = self.lib.dcr_shard_selection(self.ws.data_ptr(), self.ws_bytes, self.B, self.H,
                                          self.H_kv, self.N, HEAD_DIM, self.k, idx.data_ptr(),
                                          cnt.data_ptr(), self._stream())
        _lib.check(st, "dcr_shard_selection")
        return idx, cnt


class PeerExchange:
    """This rank's exchange buffer and the mapped buffers of the other ranks (one node).

    Created collectively (every rank of ``comm``, same B and H): each rank allocates and
    zeroes its buffer (dcr_xchg_create), the IPC handles are all-gathered, and every rank
    maps the others' (dcr_xchg_open). :meth:`close` unmaps and frees, after a barrier."""

    def __init__(self, B: int, H: int, comm, device):
        self.lib = _lib.load()
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.B, self.H = B, H
        self.device = torch.device(device)
        require(1 <= self.world <= 8, f"peer exchange connects at most 8 ranks, got {self.world}")
        self.buf = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.dcr_xchg_create(B, H, self.world, ctypes.byref(self.buf), handle),
                       "dcr_xchg_create")
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
            allh = comm.all_gather(mine).cpu().numpy().tobytes()
            self.peers = (ctypes.c_void_p * self.world)()
            st = self.lib.dcr_xchg_open(allh, self.world, self.rank, self.buf, self.peers)
        if st:
            self.lib.dcr_xchg_destroy(self.buf)
            self.buf = None
            raise _lib.DCRError(st, "dcr_xchg_open")
        self._closed = False

    def close(self) -> None:
        if self._closed or self.buf is None:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        if hasattr(self.comm, "barrier"):
            self.comm.barrier()
        with torch.cuda.device(self.device):
            self.lib.dcr_xchg_close(self.peers, self.world, self.rank)
            self.lib.dcr_xchg_destroy(self.buf)

    def reset(self) -> None:
        """Clear the buffer (epoch, flags, abort word); every rank, between steps."""
        with torch.cuda.device(self.device):
            _lib.check(self.lib.dcr_xchg_reset(self.buf, self.B, self.H, self.world,
                                               _lib.stream_ptr(self.device)), "dcr_xchg_reset")


class SequenceShardedDecoder:
    """Decode steps of one layer whose KV cache is split by sequence across the ranks.

    Construct once per (shape, group): it learns every rank's chunk length with one
    all-gather that also checks that the ranks agree on the step (:func:`agree_on_step`),
    checks ``0 < k_eff < sum(N_r)`` (the reference's caller-side contract,
    dcr_attention/models/llama/attention.py:806) and allocates the step's buffers. Each
    call runs :func:`sequence_shard_step` and returns O [B, H, D] on every rank."""

    def __init__(self, B: int, H: int, H_kv: int, N_local: int, k_eff: int, *,
                 dtype: torch.dtype, device, group=None, comm=None, eps: float = 1e-12,
                 exchange: str = "peer"):
        require(exchange in ("peer", "nccl"), f"exchange must be 'peer' or 'nccl', got {exchange}")
        self.device = torch.device(device)
        self.comm = comm if comm is not None else TorchComm(group)
        self.exchange = exchange
        self.n_locals, self.offset, self.n_total = agree_on_step(
            self.comm, B=B, H=H, H_kv=H_kv, N_local=N_local, k_eff=k_eff, dtype=dtype,
            device=self.device)
        self.step = CudaSequenceShardStep(B, H, H_kv, N_local, k_eff, dtype=dtype,
                                          device=self.device, eps=eps)
        rows, W = B * H, self.comm.world
        dev = self.device
        self.bufs = {
            "hist_hi": torch.empty(rows, 256, dtype=torch.int32, device=dev),
            "hist_lo": torch.empty(rows, 256, dtype=torch.int32, device=dev),
            "hist_lo_all": torch.empty(W, rows, 256, dtype=torch.int32, device=dev),
            "state": torch.empty(rows, STATE_FLOATS, dtype=torch.float32, device=dev),
            "states": torch.empty(W, rows, STATE_FLOATS, dtype=torch.float32, device=dev),
        }
        self.peer = PeerExchange(B, H, self.comm, dev) if exchange == "peer" else None

    def close(self) -> None:
        """Release the peer exchange (collective: every rank)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def __call__(self, Q: torch.Tensor, K_chunk: torch.Tensor, V_chunk: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        self.step.bind(Q, K_chunk, V_chunk)
        if out is not None:
            require(out.shape == (self.step.B, self.step.H, HEAD_DIM) and out.dtype == Q.dtype
                    and out.is_contiguous() and out.device == self.device,
                    "out must be a contiguous [B, H, D] tensor like Q")
        with torch.cuda.device(self.device):
            if self.peer is None:
                return sequence_shard_step(self.step, self.comm, dict(self.bufs, out=out))
            st = self.step
            if out is None:
                out = torch.empty(st.B, st.H, HEAD_DIM, dtype=st.dtype, device=self.device)
            code = st.lib.dcr_shard_decode_peer(
                st.Q.data_ptr(), st.K.data_ptr(), st.V.data_ptr(), st.dt, st.ksb, st.ksh,
                st.vsb, st.vsh, st.B, st.H, st.H_kv, st.N, HEAD_DIM, st.k, st.eps,
                self.peer.peers, self.peer.world, self.peer.rank, max(self.n_locals),
                out.data_ptr(), st.ws.data_ptr(), st.ws_bytes, st._stream())
            _lib.check(code, "dcr_shard_decode_peer")
            return out

    def selection_global(self):
        """This rank's selected positions of the last step in global coordinates:
        (idx [B, H, cap] int64 with offset added, counts [B, H])."""
        idx, cnt = self.step.selection()
        return idx.to(torch.int64) + self.offset, cnt


def sequence_sharded_attention(Q: torch.Tensor, K_chunk: torch.Tensor, V_chunk: torch.Tensor,
                               k_eff: int, *, group=None, eps: float = 1e-12,
                               exchange: str = "nccl") -> torch.Tensor:
    """One-shot sequence-sharded decode step (see :class:`SequenceShardedDecoder`; a
    decoder kept across steps amortises its setup, which the peer exchange needs)."""
    B, H, _ = Q.shape
    _, H_kv, N_local, _ = K_chunk.shape
    dec = SequenceShardedDecoder(B, H, H_kv, N_local, k_eff, dtype=Q.dtype, device=Q.device,
                                 group=group, eps=eps, exchange=exchange)
    try:
        return dec(Q, K_chunk, V_chunk)
    finally:
        dec.close()


def kv_head_sharded_attention(Q: torch.Tensor, K_heads: torch.Tensor, V_heads: torch.Tensor,
                              k_eff: int, *, group=None, comm=None, eps: float = 1e-12,
                              local_attention: Optional[Callable] = None) -> torch.Tensor:
    """Decode step with the KV heads split across the ranks.

    Q is [B, H, D] (all query heads, the same on every rank); K_heads and V_heads are this
    rank's KV heads [B, H_kv / W, N, D], rank r owning heads [r*H_kv/W, (r+1)*H_kv/W).
    Returns O [B, H, D] on every rank. ``local_attention(Q_r, K_r, V_r, k_eff, eps=)``
    computes the rank's heads (default: the CUDA :func:`topk_qaxis_attention`)."""
    comm = comm if comm is not None else TorchComm(group)
    W, r = comm.world, comm.rank
    require(Q.dim() == 3 and Q.shape[-1] == HEAD_DIM, f"Q must be [B, H, {HEAD_DIM}]")
    check_dtype(Q, "Q")
    B, H, D = Q.shape
    H_kv_local = K_heads.shape[1]
    H_kv = H_kv_local * W
    require(H % H_kv == 0, f"H={H} must be divisible by H_kv={H_kv} (= {H_kv_local} x {W})")
    H_local = H // W
    if local_attention is None:
        from dcr_b200.kernel.cuda.topk_axis import topk_qaxis_attention as local_attention
    Q_r = Q[:, r * H_local:(r + 1) * H_local].contiguous()
    O_r = local_attention(Q_r, K_heads, V_heads, k_eff, eps=eps)
    O_all = comm.all_gather(O_r)                 # [W, B, H/W, D]
    return O_all.permute(1, 0, 2, 3).reshape(B, H, D)
