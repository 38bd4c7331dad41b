"""dcr_b200 — B200-native (sm_100a) sparse top-K decode attention for DCR-Attention.

A from-scratch CUDA implementation of the per-step sparse decode attention of
Seqev/dcr-attention_v3, behind that project's kernel API:

* ``dcr_b200.kernel.cuda.topk_axis``       - ``topk_qaxis_select``, ``topk_qaxis_attention``
* ``dcr_b200.kernel.cuda.topk_axis_pass1`` - ``topk_pass1_projection``
* ``dcr_b200.kernel.cuda.topk_axis_pass2`` - ``topk_pass2_select``
* ``dcr_b200.kernel.cuda.fused_attn``      - ``fused_topk_attention``
* ``dcr_b200.models.llama.adaptive``       - ``adaptive_k_window``

Beyond the reference's API:

* ``dcr_b200.kernel.cuda.projected`` - projected-score mode (rank-16 keys written at append)
* ``dcr_b200.kv_cache``              - ``StaticKVCache``: preallocated K/V/KP, in-place append
* ``dcr_b200.sharded``               - the decode step over several GPUs (KV-head split;
  sequence split with an exact global top-K over NCCL or NVLink peer memory)

The compute runs in ``libdcr_b200.so`` (C ABI: ``include/dcr_b200.h``); there is no CPU
fallback.
"""
__version__ = "0.1.0"
