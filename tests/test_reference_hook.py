"""The reference-side hook, run inside the reference's own attention module (CPU).

INTEGRATION.md gives the branch a maintainer adds to the reference's
``DCRLlamaAttention._dcr_forward`` (dcr_attention/models/llama/attention.py:805-813) and the
``"q_topk_cuda"`` value added to ``AxisSource`` and its validator
(dcr_attention/models/llama/config.py:14, :113-117). This test imports the reference, applies
exactly that change in memory (the branch is executed from INTEGRATION.md's own code block)
and runs the module's decode path on CPU with one stand-in: ``topk_qaxis_attention`` is
replaced by a stub that puts the tensors the branch passes -- the ``K[:, ::n_rep]`` head views,
which are not contiguous across heads -- through this library's own argument checks
(``check_attention_args``, with only the CUDA-device requirement lifted) and computes O with
the CPU oracle. The output must equal the reference's own ``q_topk_reference`` branch on the
same inputs (within the attention gate), and a context no longer than k_eff must take the
reference's SDPA fallback without reaching the kernel.

The reference is found through ``REFERENCE_ROOT`` or as a ``reference`` checkout next to this
repository; without it (or without transformers) the test is skipped.
"""
from __future__ import annotations

import dataclasses
import os
import re
import sys

import numpy as np
import pytest
import torch

from golden_io import attention_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_root():
    for cand in (os.environ.get("REFERENCE_ROOT"), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "dcr_attention")):
            return cand
    return None


REF = _reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="the reference checkout is not available")


def _integration_branch() -> str:
    """The Python block of INTEGRATION.md that starts with the q_topk_cuda branch."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    for block in re.findall(r"```python\n(.*?)```", text, flags=re.S):
        if 'axis_source == "q_topk_cuda"' in block:
            return block
    raise AssertionError("INTEGRATION.md has no q_topk_cuda branch")


@pytest.fixture(scope="module")
def ref_modules():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from dcr_attention.models.llama import attention as ref_attn
        from dcr_attention.models.llama import config as ref_cfg
        from transformers import LlamaConfig
        from transformers.models.llama.modeling_llama import LlamaAttention
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"reference not importable here: {e}")
    return ref_attn, ref_cfg, LlamaConfig, LlamaAttention


@pytest.fixture
def hooked(ref_modules, monkeypatch, oracle_mod):
    """The reference with the INTEGRATION.md change applied in memory, and a record of the
    calls that reached the (stubbed) kernel."""
    ref_attn, ref_cfg, LlamaConfig, LlamaAttention = ref_modules
    from dcr_b200 import _lib
    import dcr_b200.kernel.cuda as api
    from dcr_b200.kernel.cuda import topk_axis

    # "q_topk_cuda" accepted by the validator (config.py:113-117): validated like the
    # Triton source otherwise
    orig_post = ref_cfg.DCRLlamaConfig.__post_init__

    def post_init(self):
        if self.axis_source == "q_topk_cuda":
            dataclasses.replace(self, axis_source="q_topk_triton")
            return
        orig_post(self)

    monkeypatch.setattr(ref_cfg.DCRLlamaConfig, "__post_init__", post_init)

    # the branch of INTEGRATION.md, placed where attention.py:805 computes k_eff
    body = "\n".join("    " + ln[8:] if ln.startswith("        ") else ln
                     for ln in _integration_branch().splitlines())
    src = ("def _dcr_forward(self, Q, K, V):\n"
           "    B, H, _, D = Q.shape\n"
           "    N_kv = K.shape[2]\n"
           "    k_eff = adaptive_k_window(k_window_min=self.cfg.k_window, n_kv=N_kv,\n"
           "                              coverage_floor=self.cfg.coverage_floor)\n"
           + body + "\n"
           "    return _orig_dcr_forward(self, Q, K, V)\n")
    ns = {"adaptive_k_window": ref_attn.adaptive_k_window,
          "_orig_dcr_forward": ref_attn.DCRLlamaAttention._dcr_forward, "torch": torch}
    exec(compile(src, "INTEGRATION.md q_topk_cuda branch", "exec"), ns)
    monkeypatch.setattr(ref_attn.DCRLlamaAttention, "_dcr_forward", ns["_dcr_forward"])

    calls = []

    def stub(Q, K_cache, V_cache, k_eff, *, eps=1e-12, out=None, workspace_buf=None):
        # this library's checks on the branch's own tensors (CPU: device check lifted)
        monkeypatch.setattr(_lib, "require_cuda", lambda *t: None)
        B, H, H_kv, N, dt, ksb, ksh, vsb, vsh = topk_axis.check_attention_args(
            Q, K_cache, V_cache, k_eff)
        calls.append({"shape": (B, H, H_kv, N), "k_eff": int(k_eff), "k_strides": (ksb, ksh),
                      "k_contiguous": K_cache.is_contiguous(), "dtype": Q.dtype})
        name = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[Q.dtype]
        bits = (lambda t: t.contiguous().numpy() if t.dtype == torch.float32
                else t.contiguous().view(torch.int16).numpy().view(np.uint16))
        O = oracle_mod.decode(bits(Q), bits(K_cache), bits(V_cache), name, int(k_eff), eps)[3]
        return torch.from_numpy(O).to(Q.dtype)

    monkeypatch.setattr(api, "topk_qaxis_attention", stub)
    return ref_attn, ref_cfg, LlamaConfig, LlamaAttention, calls


def _module(ref, axis_source, H=8, H_kv=2):
    ref_attn, ref_cfg, LlamaConfig, LlamaAttention = ref[:4]
    hf = LlamaConfig(hidden_size=H * 64, num_attention_heads=H, num_key_value_heads=H_kv,
                     head_dim=64, intermediate_size=128, num_hidden_layers=1)
    base = LlamaAttention(hf, layer_idx=0)
    cfg = ref_cfg.DCRLlamaConfig(axis_source=axis_source, T_dispatch=0)
    return ref_attn.DCRLlamaAttention(base, cfg)


def _decode_inputs(B, H, H_kv, N, dtype, seed):
    """Q [B, H, 1, D] and K, V after the reference's repeat_kv ([B, H, N, D])."""
    from dcr_b200.synthetic import make_decode_inputs
    Q, K, V = make_decode_inputs(B, H, H_kv, N, dtype=dtype, seed=seed)
    rep = H // H_kv
    return (Q[:, :, None], K.repeat_interleave(rep, dim=1), V.repeat_interleave(rep, dim=1))


def test_validator_accepts_the_new_axis_source(hooked):
    ref_cfg = hooked[1]
    assert ref_cfg.DCRLlamaConfig(axis_source="q_topk_cuda").axis_source == "q_topk_cuda"
    with pytest.raises(ValueError):
        ref_cfg.DCRLlamaConfig(axis_source="q_topk_cuda", k_window=3)  # still validated
    with pytest.raises(ValueError):
        ref_cfg.DCRLlamaConfig(axis_source="no_such_source")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_branch_matches_the_reference_path(hooked, dtype):
    calls = hooked[4]
    B, H, H_kv, N = 2, 8, 2, 1500
    Q, K, V = _decode_inputs(B, H, H_kv, N, dtype, seed=3)
    cuda_mod = _module(hooked, "q_topk_cuda")
    with torch.no_grad():
        O = cuda_mod._dcr_forward(Q, K, V)
    assert O.shape == (B, H, 1, 64) and O.dtype == dtype
    assert len(calls) == 1
    c = calls[0]
    k_eff = hooked[0].adaptive_k_window(k_window_min=64, n_kv=N, coverage_floor=0.15)
    assert c["shape"] == (B, H, H_kv, N) and c["k_eff"] == k_eff and c["dtype"] == dtype
    # the branch passes K[:, ::n_rep]: a view whose head stride skips the repeated heads
    assert not c["k_contiguous"] and c["k_strides"] == (H * N * 64, (H // H_kv) * N * 64)
    # the reference's own M1 path on the same inputs (it computes in bf16)
    ref_mod = _module(hooked, "q_topk_reference")
    with torch.no_grad():
        O_ref = ref_mod._dcr_forward(Q.to(torch.bfloat16), K.to(torch.bfloat16),
                                     V.to(torch.bfloat16))
    if dtype == torch.bfloat16:
        ok, stats = attention_close(O.squeeze(2).float().numpy(),
                                    O_ref.squeeze(2).float().numpy(), got_rounded_to="bf16")
        assert ok, stats
    else:  # fp16 keeps more mantissa than the reference's bf16 cast: compare loosely
        d = (O.float() - O_ref.float()).abs().max().item()
        assert d < 2e-2, d


def test_short_context_takes_the_sdpa_fallback(hooked):
    calls = hooked[4]
    B, H, H_kv, N = 1, 8, 2, 64  # k_eff = max(64, 0.15 N) = 64 >= N: the reference uses SDPA
    Q, K, V = _decode_inputs(B, H, H_kv, N, torch.bfloat16, seed=4)
    mod = _module(hooked, "q_topk_cuda")
    with torch.no_grad():
        O = mod._dcr_forward(Q, K, V)
    assert calls == []
    assert O.shape == (B, H, 1, 64)
    dense = torch.nn.functional.scaled_dot_product_attention(Q.float(), K.float(), V.float())
    assert (O.float() - dense).abs().max().item() < 2e-2
