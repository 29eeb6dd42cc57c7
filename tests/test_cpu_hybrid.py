"""Qwen3.5 hybrid checkpoints through the library's load plan (l0b_model_shard_plan, no device): where the
Gated DeltaNet tensors and the gated q_proj of a hybrid model go (LlmLayerWeights.Load,
L/LlmLayerWeights.cs:110-212) and what the plan refuses."""
from __future__ import annotations

import numpy as np
import pytest

import hf_tiny


def _cfg(lz, **kw):
    return lz.model_config(**(hf_tiny.hybrid_model_config_kwargs(hf_tiny.HYBRID["qwen3_5"]) | kw))


def test_hybrid_plan_places_linear_and_gated_attention_tensors(lz):
    c = hf_tiny.HYBRID["qwen3_5"]
    cfg = _cfg(lz)
    w = hf_tiny.hybrid_weights(c, 7)
    hv, dk, dv = c["lin_v_heads"], c["lin_k_dim"], c["lin_v_dim"]
    cd, vd = 2 * c["lin_k_heads"] * dk + hv * dv, hv * dv
    rows = {}
    for name, v in w.items():
        sp = lz.shard_plan(cfg, name)
        assert sp.full_rows * sp.full_cols == v.size, name
        if sp.kind == lz.ShardPlan.MATRIX and sp.slot == lz.ShardPlan.LIN_IN:
            rows[name.rsplit(".", 2)[-2]] = (sp.dst_row, sp.rows)
    # [qkv; z; b; a] stacked in one matrix, in that order.
    assert rows == {"in_proj_qkv": (0, cd), "in_proj_z": (cd, vd), "in_proj_b": (cd + vd, hv),
                    "in_proj_a": (cd + vd + hv, hv)}
    sp = lz.shard_plan(cfg, "model.layers.1.self_attn.q_proj.weight")
    qd = c["heads"] * c["head_dim"]
    assert (sp.kind, sp.slot, sp.full_rows, sp.rows, sp.dst_row) == (lz.ShardPlan.QUERY_GATE, lz.ShardPlan.QKV,
                                                                     2 * qd, qd, 0)
    sp = lz.shard_plan(cfg, "model.layers.0.linear_attn.conv1d.weight")
    assert (sp.kind, sp.slot, sp.cols) == (lz.ShardPlan.VECTOR, lz.ShardPlan.LIN_CONV, cd * c["lin_conv"])
    sp = lz.shard_plan(cfg, "model.layers.2.linear_attn.out_proj.weight")
    assert (sp.slot, sp.full_rows, sp.full_cols) == (lz.ShardPlan.LIN_OUT, c["hidden"], vd)


def test_hybrid_plan_refusals(lz):
    cfg = _cfg(lz)
    # Attention tensors on a linear layer, DeltaNet tensors on a full-attention layer.
    for name in ("model.layers.0.self_attn.q_proj.weight", "model.layers.1.linear_attn.A_log"):
        with pytest.raises(lz.InvalidDataException):
            lz.shard_plan(cfg, name)
    # Hybrid models run on one GPU.
    with pytest.raises(lz.NotSupportedException):
        lz.shard_plan(_cfg(lz, tp_size=2, tp_rank=0), "model.layers.0.mlp.up_proj.weight")


def test_model_config_mirror_matches_the_c_struct(lz):
    """levelzero.ModelConfig mirrors l0b_model_config field for field: l0b_model_config_init writes
    exactly sizeof(ModelConfig) bytes (a canary right after it survives) and its defaults land on the
    fields that carry them."""
    import ctypes as C

    n = C.sizeof(lz.ModelConfig)
    buf = (C.c_uint8 * (n + 64))(*([0xA5] * (n + 64)))
    cfg = lz.ModelConfig.from_buffer(buf)
    lz.check(lz.load_library().l0b_model_config_init(C.byref(cfg)))
    assert bytes(buf[n:]) == b"\xa5" * 64
    assert cfg.max_position_embeddings == 2048 and cfg.rope_truncate == 1 and cfg.partial_rotary_factor == 1.0
    assert cfg.linear_layer_mask == 0 and cfg.attention_output_gate == 0 and cfg.rms_norm_offset == 0.0
