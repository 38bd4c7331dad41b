"""Greedy decode of a Llama-3.2-1B-architecture model with DCR sparse attention.

The reference measures its end-to-end decode step as ``model(next_tok, past_key_values=past,
use_cache=True)`` on HF ``LlamaForCausalLM`` with ``DCRLlamaAttention`` installed in every
layer (dcr_attention/models/llama/attention.py:319; tests/kernel/test_m1_acceptance.py:198).
:class:`DCRLlamaDecoder` is that decode step on this package's pieces, with random-init
weights of the architecture (the checkpoint is not available here):

* token embedding; per layer HF ``LlamaRMSNorm`` (fp32 statistics, weight applied in the
  model dtype), the decode attention of :class:`~dcr_b200.models.llama.attention.DCRDecodeAttention`
  (q/k/v GEMMs, the fused RoPE + cache-append prologue, routing, the three-pass sparse step
  or SDPA, o_proj), a residual add, RMSNorm, the SwiGLU MLP ``down(silu(gate(x)) * up(x))``
  and a residual add; final RMSNorm; the LM head tied to the embedding (Llama-3.2-1B);
* one :class:`~dcr_b200.kv_cache.StaticKVCache` per layer instead of HF ``DynamicCache``.

``attention="dense"`` routes every layer to SDPA over the whole cache (the reference's SDPA
baseline); ``"dcr"`` uses the sparse step above ``T_dispatch`` positions, as the hook does.

:class:`GreedyDecodeGraphs` captures each of a run of decode steps as its own CUDA graph
(the cache length, hence the kernels' launch shapes and ``k_eff``, changes every step), so a
timed run replays one graph per step: the H2D copy of the step's tokens, 16 layers, the LM
head and argmax, and the D2H copy of the next tokens.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn.functional as F

from dcr_b200.kernel.cuda._common import HEAD_DIM, require
from dcr_b200.kv_cache import StaticKVCache
from dcr_b200.models.llama.attention import (DCRDecodeAttention, KVHeadParallelDecodeAttention,
                                             llama3_inv_freq)


@dataclass
class LlamaDecodeConfig:
    """Llama-3.2-1B's shape (hidden 2048, 16 layers, 32 q / 8 KV heads of 64, FFN 8192,
    vocab 128256, RoPE theta 500000 with llama3 frequency scaling, RMSNorm eps 1e-5)."""
    vocab: int = 128256
    hidden: int = 2048
    intermediate: int = 8192
    layers: int = 16
    heads: int = 32
    kv_heads: int = 8
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5


class RMSNorm(torch.nn.Module):
    """HF LlamaRMSNorm: x * rsqrt(mean(x^2) + eps) in fp32, cast back, times the weight."""

    def __init__(self, dim: int, eps: float, dtype, device):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim, dtype=dtype, device=device))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x32 = x.float()
        x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * x32.to(x.dtype)


class DecoderLayer(torch.nn.Module):
    def __init__(self, cfg: LlamaDecodeConfig, *, attention: str, mode: str, k_window: int,
                 coverage_floor: float, T_dispatch: int, dtype, device, fast: bool):
        super().__init__()
        kw = dict(bias=False, dtype=dtype, device=device)
        self.fast = fast
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, dtype, device)
        self.self_attn = DCRDecodeAttention(
            cfg.hidden, cfg.heads, cfg.kv_heads, k_window=k_window, coverage_floor=coverage_floor,
            T_dispatch=(1 << 62) if attention == "dense" else T_dispatch, mode=mode, dtype=dtype,
            device=device, pack_qkv=fast)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, dtype, device)
        self.gate_proj = torch.nn.Linear(cfg.hidden, cfg.intermediate, **kw)
        self.up_proj = torch.nn.Linear(cfg.hidden, cfg.intermediate, **kw)
        self.down_proj = torch.nn.Linear(cfg.intermediate, cfg.hidden, **kw)
        self._gate_up = None
        if fast:  # gate and up weights as row views of one tensor: one GEMM for both
            from dcr_b200.kernel.cuda.decode_ops import pack_linears
            self._gate_up = pack_linears(self.gate_proj, self.up_proj)

    def forward(self, h, delta, cos, sin, cache):
        """The layer on the residual stream h [B, 1, hidden] plus the previous layer's
        pending output ``delta`` (None for the first layer): returns (h, delta) with
        h = h_in + delta_in + attention, delta = this layer's MLP output (added by the next
        norm, as HF adds it at the end of the layer)."""
        if not self.fast:
            if delta is not None:
                h = h + delta
            h = h + self.self_attn(self.input_layernorm(h), cos, sin, cache)
            x = self.post_attention_layernorm(h)
            return h, self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
        from dcr_b200.kernel.cuda.decode_ops import add_rmsnorm, silu_mul_packed
        eps = self.input_layernorm.eps
        h, x = add_rmsnorm(h, delta, self.input_layernorm.weight, eps)
        a = self.self_attn(x, cos, sin, cache)
        h, x = add_rmsnorm(h, a, self.post_attention_layernorm.weight, eps)
        return h, self.down_proj(silu_mul_packed(F.linear(x, self._gate_up)))


class DCRLlamaDecoder(torch.nn.Module):
    """Decode-only Llama model (random init, std 0.02 as HF's initializer_range) whose
    attention layers run :class:`DCRDecodeAttention` over per-layer static caches."""

    def __init__(self, cfg: Optional[LlamaDecodeConfig] = None, *, attention: str = "dcr",
                 mode: str = "exact", k_window: int = 64, coverage_floor: float = 0.15,
                 T_dispatch: int = 4096, dtype: torch.dtype = torch.bfloat16, device="cuda",
                 seed: int = 0, fast: bool = True):
        super().__init__()
        self.fast = fast
        require(attention in ("dcr", "dense"), f"attention must be 'dcr' or 'dense', got {attention}")
        self.cfg = cfg = cfg or LlamaDecodeConfig()
        require(cfg.hidden == cfg.heads * HEAD_DIM, f"hidden must be heads x {HEAD_DIM}")
        self.dtype, self.device, self.mode = dtype, torch.device(device), mode
        self.T_dispatch = T_dispatch
        self.embed_tokens = torch.nn.Embedding(cfg.vocab, cfg.hidden, dtype=dtype, device=device)
        self.layers = torch.nn.ModuleList(
            self._make_layer(cfg, attention=attention, mode=mode, k_window=k_window,
                             coverage_floor=coverage_floor, T_dispatch=T_dispatch, dtype=dtype,
                             device=device, fast=fast)
            for _ in range(cfg.layers))
        self.norm = RMSNorm(cfg.hidden, cfg.rms_eps, dtype, device)
        self.inv_freq = llama3_inv_freq(HEAD_DIM, theta=cfg.rope_theta).to(self.device)
        g = torch.Generator(device=self.device).manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if p.dim() == 2:
                    p.normal_(0.0, 0.02, generator=g)
        self.set_attention(attention)

    def _make_layer(self, cfg, **kw) -> torch.nn.Module:
        return DecoderLayer(cfg, **kw)

    def set_attention(self, attention: str) -> None:
        """'dcr': sparse step at or above T_dispatch positions; 'dense': SDPA everywhere."""
        require(attention in ("dcr", "dense"), f"attention must be 'dcr' or 'dense', got {attention}")
        self.attention = attention
        for layer in self.layers:
            layer.self_attn.T_dispatch = (1 << 62) if attention == "dense" else self.T_dispatch

    def lm_head(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.embed_tokens.weight)  # tied to the embedding (Llama-3.2-1B)

    def new_caches(self, B: int, N_max: int, *, P: Optional[torch.Tensor] = None
                   ) -> List[StaticKVCache]:
        require(self.mode != "projected" or P is not None, "projected mode needs caches with P")
        return [StaticKVCache(B, len(self.kv_heads_held()), N_max, dtype=self.dtype,
                              device=self.device, P=P) for _ in self.layers]

    def kv_heads_held(self) -> range:
        """The global KV heads whose caches this model holds (all of them here)."""
        return range(self.cfg.kv_heads)

    @torch.no_grad()
    def prefill_synthetic(self, caches: List[StaticKVCache], n: int, *, seed: int = 0) -> None:
        """Fills the first n positions of every layer's cache with seeded synthetic keys and
        values (K, V ~ N(0,1), keys of tokens 0-3 x4, two key channels x6; one seed per
        (layer, global KV head), so a head's rows do not depend on how the heads are split
        across GPUs) and their projections; stands in for a prefill of real text."""
        from dcr_b200.synthetic import make_decode_inputs
        heads = self.kv_heads_held()
        for i, cache in enumerate(caches):
            require(cache.length == 0, "prefill_synthetic expects empty caches")
            require(cache.H_kv == len(heads), "cache heads do not match the model's")
            K = torch.empty(cache.B, cache.H_kv, n, HEAD_DIM, dtype=self.dtype, device=self.device)
            V = torch.empty_like(K)
            for j, h in enumerate(heads):
                _, K[:, j:j + 1], V[:, j:j + 1] = make_decode_inputs(
                    cache.B, 1, 1, n, dtype=self.dtype, seed=seed + 1000 * i + h,
                    device=self.device)
            cache.append(K, V)
            del K, V

    def rope_table(self, n_positions: int):
        """(cos, sin) [n_positions, D] in the model dtype for positions 0..n_positions-1."""
        from dcr_b200.models.llama.attention import rope_cos_sin
        return rope_cos_sin(torch.arange(n_positions, device=self.device), self.inv_freq,
                            self.dtype)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, caches: List[StaticKVCache], cos: torch.Tensor,
             sin: torch.Tensor) -> torch.Tensor:
        """One decode step for tokens [B] (int64, on the device) at the caches' common
        length, with that position's cos/sin [B, D]: appends every layer's key and value
        and returns the logits [B, vocab]."""
        B = tokens.shape[0]
        h = self.embed_tokens(tokens)[:, None]
        c, s = cos.reshape(B, 1, HEAD_DIM), sin.reshape(B, 1, HEAD_DIM)
        delta = None
        for layer, cache in zip(self.layers, caches):
            h, delta = layer(h, delta, c, s, cache)
        if self.fast:
            from dcr_b200.kernel.cuda.decode_ops import add_rmsnorm
            _, x = add_rmsnorm(h, delta, self.norm.weight, self.norm.eps)
        else:
            x = self.norm(h + delta)
        return self.lm_head(x[:, 0])


class TPDecoderLayer(DecoderLayer):
    """The decoder layer split across the `world` ranks of a group (tensor parallelism by
    KV head): the attention is :class:`KVHeadParallelDecodeAttention` (this rank's KV heads
    and their query heads, a row-split o_proj and one all-reduce); the MLP holds columns
    [r*I/W, (r+1)*I/W) of gate and up and the matching rows of down, whose partial output
    is all-reduced. Norms and the residual stream are replicated."""

    def __init__(self, cfg: LlamaDecodeConfig, *, world: int, rank: int, all_reduce,
                 attention: str, mode: str, k_window: int, coverage_floor: float,
                 T_dispatch: int, dtype, device, fast: bool):
        require(fast, "the tensor-parallel layer runs the fused decode path")
        require(cfg.intermediate % world == 0, "intermediate size must divide by the world")
        torch.nn.Module.__init__(self)
        kw = dict(bias=False, dtype=dtype, device=device)
        self.fast = True
        self.world, self.rank, self.all_reduce = world, rank, all_reduce
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, dtype, device)
        self.self_attn = KVHeadParallelDecodeAttention(
            cfg.hidden, cfg.heads, cfg.kv_heads, world=world, rank=rank, all_reduce=all_reduce,
            k_window=k_window, coverage_floor=coverage_floor,
            T_dispatch=(1 << 62) if attention == "dense" else T_dispatch, mode=mode, dtype=dtype,
            device=device, pack_qkv=True)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, dtype, device)
        inter = cfg.intermediate // world
        self.gate_proj = torch.nn.Linear(cfg.hidden, inter, **kw)
        self.up_proj = torch.nn.Linear(cfg.hidden, inter, **kw)
        self.down_proj = torch.nn.Linear(inter, cfg.hidden, **kw)
        from dcr_b200.kernel.cuda.decode_ops import pack_linears
        self._gate_up = pack_linears(self.gate_proj, self.up_proj)

    def forward(self, h, delta, cos, sin, cache):
        h, d = super().forward(h, delta, cos, sin, cache)
        if self.all_reduce is not None:
            return h, self.all_reduce(d)
        import torch.distributed as dist
        dist.all_reduce(d, op=dist.ReduceOp.SUM)
        return h, d

    @torch.no_grad()
    def load_shard(self, full: DecoderLayer) -> "TPDecoderLayer":
        """Copies this rank's slices of an unsplit layer's weights."""
        inter = self.gate_proj.weight.shape[0]
        r = self.rank
        self.input_layernorm.weight.copy_(full.input_layernorm.weight)
        self.post_attention_layernorm.weight.copy_(full.post_attention_layernorm.weight)
        self.self_attn.load_shard(full.self_attn)
        self.gate_proj.weight.copy_(full.gate_proj.weight[r * inter:(r + 1) * inter])
        self.up_proj.weight.copy_(full.up_proj.weight[r * inter:(r + 1) * inter])
        self.down_proj.weight.copy_(full.down_proj.weight[:, r * inter:(r + 1) * inter])
        return self


class TPDCRLlamaDecoder(DCRLlamaDecoder):
    """:class:`DCRLlamaDecoder` split across the ranks of a process group, one GPU each:
    every layer is a :class:`TPDecoderLayer` (KV heads [r*H_kv/W, (r+1)*H_kv/W) and their
    caches on rank r, two all-reduces per layer); the embedding, the norms and the tied LM
    head are replicated, so every rank computes the same logits and greedy tokens.
    ``all_reduce`` (optional) replaces torch.distributed's all-reduce (tests)."""

    def __init__(self, cfg: Optional[LlamaDecodeConfig] = None, *, world: int, rank: int,
                 all_reduce=None, **kw):
        self.world, self.rank, self._ar = world, rank, all_reduce
        super().__init__(cfg, **kw)

    def _make_layer(self, cfg, **kw) -> torch.nn.Module:
        return TPDecoderLayer(cfg, world=self.world, rank=self.rank, all_reduce=self._ar, **kw)

    def kv_heads_held(self) -> range:
        n = self.cfg.kv_heads // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    @torch.no_grad()
    def load_from(self, full: DCRLlamaDecoder) -> "TPDCRLlamaDecoder":
        """Copies this rank's shard of an unsplit model's weights."""
        self.embed_tokens.weight.copy_(full.embed_tokens.weight)
        self.norm.weight.copy_(full.norm.weight)
        for mine, theirs in zip(self.layers, full.layers):
            mine.load_shard(theirs)
        return self


class GreedyDecodeGraphs:
    """``steps`` consecutive greedy decode steps, each captured as one CUDA graph: the H2D
    copy of the step's tokens from a pinned buffer, the model step at that position, argmax
    and the D2H copy of the next tokens. Replaying them in order (``run``) advances the
    caches by ``steps`` positions; the graphs bake in the positions they were captured at."""

    def __init__(self, model: DCRLlamaDecoder, caches: List[StaticKVCache], steps: int):
        B = caches[0].B
        dev = model.device
        self.model, self.caches, self.steps = model, caches, steps
        self.pos0 = caches[0].length
        require(all(c.length == self.pos0 for c in caches), "caches must share one length")
        require(self.pos0 + steps <= caches[0].N_max, "caches too short for the steps")
        cos, sin = model.rope_table(self.pos0 + steps)
        self.cos = [cos[self.pos0 + t].expand(B, HEAD_DIM).contiguous() for t in range(steps)]
        self.sin = [sin[self.pos0 + t].expand(B, HEAD_DIM).contiguous() for t in range(steps)]
        self.tokens_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.next_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.next = torch.zeros(B, dtype=torch.int64, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))

        def body(t):
            self.tokens.copy_(self.tokens_host, non_blocking=True)
            logits = model.step(self.tokens, caches, self.cos[t], self.sin[t])
            self.next.copy_(logits.argmax(-1))
            self.next_host.copy_(self.next, non_blocking=True)

        with torch.cuda.stream(self.stream):
            body(0)  # warm-up outside the capture (it writes position pos0, rewritten later)
            self.stream.synchronize()
            self._reset(self.pos0)
            self.graphs = []
            pool = None
            for t in range(steps):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.stream, pool=pool):
                    body(t)
                pool = g.pool()
                self.graphs.append(g)
        self._reset(self.pos0)

    def _reset(self, length: int) -> None:
        for c in self.caches:
            c.length = length

    def run(self, first_tokens: torch.Tensor) -> torch.Tensor:
        """Replays the steps from the caches' start length; returns the greedy tokens
        [steps, B] (host). Each step syncs the host (its tokens come back before the next
        step's copy)."""
        out = torch.empty(self.steps, first_tokens.shape[0], dtype=torch.int64)
        cur = first_tokens.to(torch.int64).cpu()
        self._reset(self.pos0)
        with torch.cuda.stream(self.stream):
            for t, g in enumerate(self.graphs):
                self.tokens_host.copy_(cur)
                g.replay()
                self.stream.synchronize()
                cur = self.next_host.clone()
                out[t] = cur
        self._reset(self.pos0 + self.steps)
        return out

    def close(self) -> None:
        self.graphs = []
