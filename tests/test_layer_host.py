"""Host-side pieces of the decode layer (CPU): the Llama-3 RoPE frequency table against
transformers' own implementation, and the KV-head-parallel weight slicing."""
from __future__ import annotations

import pytest
import torch


def test_llama3_inv_freq_matches_transformers():
    transformers = pytest.importorskip("transformers")
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import _compute_llama3_parameters

    from dcr_b200.models.llama.attention import llama3_inv_freq
    cfg = LlamaConfig(hidden_size=2048, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=64, max_position_embeddings=131072,
                      rope_theta=500000.0,
                      rope_scaling={"rope_type": "llama3", "factor": 32.0,
                                    "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                    "original_max_position_embeddings": 8192})
    ref, scale = _compute_llama3_parameters(cfg, device=torch.device("cpu"))
    assert scale == 1.0
    assert torch.equal(llama3_inv_freq(), ref.float())


def test_kv_head_parallel_slices_cover_the_layer():
    from dcr_b200.models.llama.attention import DCRDecodeAttention, KVHeadParallelDecodeAttention
    full = DCRDecodeAttention(256, 8, 4, dtype=torch.float32, device="cpu")
    shards = [KVHeadParallelDecodeAttention(256, 8, 4, world=2, rank=r, dtype=torch.float32,
                                            device="cpu").load_shard(full) for r in range(2)]
    assert torch.equal(torch.cat([s.q_proj.weight for s in shards]), full.q_proj.weight)
    assert torch.equal(torch.cat([s.k_proj.weight for s in shards]), full.k_proj.weight)
    assert torch.equal(torch.cat([s.o_proj.weight for s in shards], dim=1), full.o_proj.weight)
    assert shards[1].H == 4 and shards[1].H_kv == 2
