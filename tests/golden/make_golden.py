"""Generate the golden vectors under tests/golden/ by running the REFERENCE itself.

Run in the build container, where the reference (Seqev/dcr-attention_v3) is importable:

    REFERENCE_ROOT=/path/to/dcr-attention_v3 python tests/golden/make_golden.py

For every case in cases.py it rebuilds the seeded inputs and runs the reference's oracle
step functions (dcr_attention/kernel/qaxis_topk_reference.py):
``_compute_u_Q`` (:42), ``_compute_projection_scores`` (:58), ``_select_topk_indices``
(:91), ``_gather_kv`` (:111) + ``_fused_softmax_attention`` (:148), and for bf16 cases
also the public ``topk_qaxis_attention_reference`` (:200). It stores, per case:

* ``u``        fp32 [B, H, 64]
* ``scores``   bf16 bits [B*H, N]
* ``idx``      int32 [B*H, k] (ascending)
* ``O_ref``    bf16 bits [B, H, 64]: the reference's own pipeline. ``_gather_kv`` writes
               into bf16 buffers, so for fp16/fp32 inputs the attention runs on
               bf16-rounded rows.
* ``O_native`` bf16 bits [B, H, 64]: same steps, but the gather keeps the stored dtype
               (what the CUDA kernels compute for fp16/fp32). Equal to O_ref for bf16.
* ``O_f32``    fp32 [B, H, 64]: O_native before its final rounding. Produced by the same
               reference function with its output-cast constant (``_BF16``, :35) set to
               float32 for the call, so the attention arithmetic is the reference's own.
* ``meta``     JSON: shape, dtype, seed, kind, the input SHA-256, the reference's git/
               torch versions.

Only the reference's outputs are stored; inputs are rebuilt from the seeds (torch's CPU
generator is deterministic for a given torch version) and checked against the SHA-256.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, _HERE)
from cases import CASES, build_inputs, fixture_path, input_sha256  # noqa: E402

REF = os.environ.get("REFERENCE_ROOT")


def _reference_root() -> str:
    """The reference checkout to import: REFERENCE_ROOT is required (no default path)."""
    if not REF or not os.path.isdir(os.path.join(REF, "dcr_attention")):
        raise SystemExit("set REFERENCE_ROOT to a checkout of Seqev/dcr-attention_v3 "
                         "(the directory that holds the dcr_attention package)")
    return REF


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    sys.path.insert(0, _reference_root())
    from dcr_attention.kernel import qaxis_topk_reference as R  # noqa: E402

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, (B, H, H_kv, N, k, dt, seed, kind) in CASES.items():
        Q, K, V = build_inputs(name)
        sha = input_sha256(Q, K, V)
        u = R._compute_u_Q(Q, 1e-12)
        scores = R._compute_projection_scores(K, u)
        idx = R._select_topk_indices(scores, k)
        K_sel, V_sel = R._gather_kv(K, V, idx)          # bf16 buffers (reference behaviour)
        O_ref = R._fused_softmax_attention(K_sel, V_sel, Q)
        # dtype-preserving gather (restated from _gather_kv without the bf16 buffer)
        G = H // H_kv
        hk = torch.arange(H) // G
        bi = torch.arange(B)[:, None, None]
        K_nat = K[bi, hk[None, :, None], idx]
        V_nat = V[bi, hk[None, :, None], idx]
        O_nat = R._fused_softmax_attention(K_nat, V_nat, Q)
        saved = R._BF16
        try:
            R._BF16 = torch.float32
            O_f32 = R._fused_softmax_attention(K_nat, V_nat, Q)
        finally:
            R._BF16 = saved
        assert O_f32.dtype == torch.float32 and torch.equal(O_f32.to(torch.bfloat16), O_nat)
        if dt == "bf16":
            O_pub = R.topk_qaxis_attention_reference(Q, K, V, k)
            assert torch.equal(O_pub, O_ref), name
            assert torch.equal(O_nat, O_ref), name
        meta = dict(name=name, B=B, H=H, H_kv=H_kv, N=N, k=k, dtype=dt, seed=seed, kind=kind,
                    input_sha256=sha, torch=torch.__version__,
                    reference="Seqev/dcr-attention_v3 dcr_attention/kernel/qaxis_topk_reference.py")
        np.savez_compressed(
            fixture_path(name),
            meta=np.array(json.dumps(meta)),
            u=u.numpy().astype(np.float32),
            scores=_bits(scores).reshape(B * H, N),
            idx=idx.numpy().astype(np.int32).reshape(B * H, k),
            O_ref=_bits(O_ref),
            O_native=_bits(O_nat),
            O_f32=O_f32.numpy().astype(np.float32),
        )
        print(f"{name}: {os.path.getsize(fixture_path(name)) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
