"""The decode step of DCR-Attention's Llama attention layer on the B200 kernels.

Mirrors the decode path of the reference's ``DCRLlamaAttention.forward``
(dcr_attention/models/llama/attention.py:386-454) for one new token per sequence:

1. q/k/v projections (attention.py:387-393): plain GEMMs (``torch.nn.Linear``, no bias),
   as in the reference;
2. RoPE and the cache update (:395-421): one launch (``StaticKVCache.append_rotated``,
   dcr_decode_prologue) instead of HF ``apply_rotary_pos_emb`` and a ``torch.cat`` of the
   whole cache, also writing the rank-16 projected key and, in projected mode, the
   projected unit query that the projected Pass 1 then reads instead of recomputing;
3. routing (:436, routing.py:28-70): dense attention (SDPA) when the cache is shorter than
   ``T_dispatch`` or ``k_eff >= N_kv``, else the sparse top-K step (``_dcr_forward``,
   attention.py:805-813) with ``k_eff = adaptive_k_window(k_window, N_kv, coverage_floor)``;
   no ``repeat_kv`` copy (the kernels read the un-repeated cache);
4. ``o_proj`` (:451-454): a plain GEMM.

:class:`KVHeadParallelDecodeAttention` is the same layer with its heads split across the
ranks of a group (tensor parallelism by KV head): each rank holds the projections of its
KV heads and their query heads and the matching input columns of ``o_proj``; the partial
outputs are summed with one all-reduce (the o_proj epilogue of a KV-head-parallel layout).
"""
from __future__ import annotations

import math
from typing import Callable, Optional, Tuple

import torch
import torch.nn.functional as F

from dcr_b200.kernel.cuda._common import HEAD_DIM, require
from dcr_b200.kv_cache import StaticKVCache
from dcr_b200.models.llama.adaptive import adaptive_k_window


def llama3_inv_freq(dim: int = HEAD_DIM, theta: float = 500000.0, factor: float = 32.0,
                    low_freq_factor: float = 1.0, high_freq_factor: float = 4.0,
                    original_max_position: int = 8192) -> torch.Tensor:
    """Llama-3 rotary inverse frequencies (fp32, [dim/2]) with the "llama3" frequency
    scaling of Llama-3.2 (wavelengths above original_max_position / low_freq_factor are
    divided by `factor`, those below original_max_position / high_freq_factor are kept,
    and the band between is interpolated)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    low_wavelen = original_max_position / low_freq_factor
    high_wavelen = original_max_position / high_freq_factor
    wavelen = 2 * math.pi / inv
    scaled = torch.where(wavelen > low_wavelen, inv / factor, inv)
    smooth = (original_max_position / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    smoothed = (1 - smooth) * scaled / factor + smooth * scaled
    medium = (wavelen >= high_wavelen) & (wavelen <= low_wavelen)
    return torch.where(medium, smoothed, scaled)


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor,
                 dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) [B, D] in ``dtype`` for the given positions [B] (HF's rotary embedding:
    angles in fp32, cat(freqs, freqs), cos/sin, cast to the model dtype)."""
    freqs = positions.float()[:, None] * inv_freq.to(positions.device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class DCRDecodeAttention(torch.nn.Module):
    """One Llama attention layer's decode step (one new token per sequence).

    ``mode``: ``"exact"`` (the reference's q-axis scores, ``axis_source="q_topk_triton"``)
    or ``"projected"`` (rank-16 projected scores; needs a cache built with P)."""

    def __init__(self, hidden: int, H: int, H_kv: int, *, k_window: int = 64,
                 coverage_floor: float = 0.15, T_dispatch: int = 4096, mode: str = "exact",
                 dtype: torch.dtype = torch.bfloat16, device="cuda", eps: float = 1e-12,
                 pack_qkv: bool = False):
        super().__init__()
        require(mode in ("exact", "projected"), f"mode must be 'exact' or 'projected', got {mode}")
        require(H % H_kv == 0, "H must be a multiple of H_kv")
        self.hidden, self.H, self.H_kv = hidden, H, H_kv
        self.k_window, self.coverage_floor, self.T_dispatch = k_window, coverage_floor, T_dispatch
        self.mode, self.eps = mode, eps
        kw = dict(bias=False, dtype=dtype, device=device)
        self.q_proj = torch.nn.Linear(hidden, H * HEAD_DIM, **kw)
        self.k_proj = torch.nn.Linear(hidden, H_kv * HEAD_DIM, **kw)
        self.v_proj = torch.nn.Linear(hidden, H_kv * HEAD_DIM, **kw)
        self.o_proj = torch.nn.Linear(H * HEAD_DIM, hidden, **kw)
        self.last_branch = None
        self._qkv = None
        if pack_qkv:  # q/k/v weights as row views of one tensor: one GEMM for all three
            from dcr_b200.kernel.cuda.decode_ops import pack_linears
            self._qkv = pack_linears(self.q_proj, self.k_proj, self.v_proj)

    def attend(self, q_rot: torch.Tensor, qp: Optional[torch.Tensor],
               cache: StaticKVCache) -> torch.Tensor:
        """O [B, H, D] over the cache (which already holds this step's key and value)."""
        N_kv = cache.length
        k_eff = adaptive_k_window(self.k_window, N_kv, self.coverage_floor)
        if N_kv < self.T_dispatch or k_eff >= N_kv:
            self.last_branch = "sdpa"
            # query head h reads KV head h // G, as the reference's repeat_kv (no copy)
            return F.scaled_dot_product_attention(q_rot[:, :, None], cache.K, cache.V,
                                                  enable_gqa=True).squeeze(2)
        self.last_branch = "dcr"
        if self.mode == "projected":
            from dcr_b200.kernel.cuda.projected import topk_qaxis_attention_projected
            return topk_qaxis_attention_projected(q_rot, cache.K, cache.V, cache.KP, cache.P,
                                                  k_eff, eps=self.eps, qp=qp)
        from dcr_b200.kernel.cuda.topk_axis import topk_qaxis_attention
        return topk_qaxis_attention(q_rot, cache.K, cache.V, k_eff, eps=self.eps)

    def forward(self, hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                cache: StaticKVCache) -> torch.Tensor:
        """hidden_states [B, 1, hidden], cos/sin [B, 1, D] (the model's position embeddings
        at the new position) -> [B, 1, hidden]; appends the step's key and value."""
        B, n_q, _ = hidden_states.shape
        require(n_q == 1, "decode step: one new token per sequence")
        x = hidden_states[:, 0]
        nq, nk = self.H * HEAD_DIM, self.H_kv * HEAD_DIM
        if self._qkv is not None:
            # one GEMM; the prologue reads q, k, v as strided slices of its rows
            qkv = F.linear(x, self._qkv)
            q = qkv[:, :nq].view(B, self.H, HEAD_DIM)
            k = qkv[:, nq:nq + nk].view(B, self.H_kv, HEAD_DIM)
            v = qkv[:, nq + nk:].view(B, self.H_kv, HEAD_DIM)
        else:
            q = self.q_proj(x).view(B, self.H, HEAD_DIM)
            k = self.k_proj(x).view(B, self.H_kv, HEAD_DIM)
            v = self.v_proj(x).view(B, self.H_kv, HEAD_DIM)
        q_rot, qp = cache.append_rotated(q, k, v, cos.reshape(B, HEAD_DIM),
                                         sin.reshape(B, HEAD_DIM),
                                         want_qp=self.mode == "projected", eps=self.eps)
        O = self.attend(q_rot, qp, cache)
        return self.o_proj(O.reshape(B, 1, self.H * HEAD_DIM))


class KVHeadParallelDecodeAttention(DCRDecodeAttention):
    """The layer with its KV heads split across the ranks of a group: rank r holds KV
    heads [r*H_kv/W, (r+1)*H_kv/W), their query heads, and the matching input columns of
    o_proj. ``forward`` returns the full output on every rank (one all-reduce)."""

    def __init__(self, hidden: int, H: int, H_kv: int, *, world: int, rank: int,
                 all_reduce: Optional[Callable[[torch.Tensor], torch.Tensor]] = None, **kw):
        require(H_kv % world == 0, f"H_kv={H_kv} must be a multiple of the world size {world}")
        super().__init__(hidden, H // world, H_kv // world, **kw)
        self.world, self.rank = world, rank
        self.full_H, self.full_H_kv = H, H_kv
        self._all_reduce = all_reduce

    @torch.no_grad()
    def load_shard(self, full: DCRDecodeAttention) -> "KVHeadParallelDecodeAttention":
        """Copies this rank's slices of an unsplit layer's weights."""
        hq = self.H * HEAD_DIM
        hk = self.H_kv * HEAD_DIM
        r = self.rank
        self.q_proj.weight.copy_(full.q_proj.weight[r * hq:(r + 1) * hq])
        self.k_proj.weight.copy_(full.k_proj.weight[r * hk:(r + 1) * hk])
        self.v_proj.weight.copy_(full.v_proj.weight[r * hk:(r + 1) * hk])
        self.o_proj.weight.copy_(full.o_proj.weight[:, r * hq:(r + 1) * hq])
        return self

    def forward(self, hidden_states, cos, sin, cache):
        partial = super().forward(hidden_states, cos, sin, cache)
        if self._all_reduce is not None:
            return self._all_reduce(partial)
        import torch.distributed as dist
        dist.all_reduce(partial, op=dist.ReduceOp.SUM)
        return partial
