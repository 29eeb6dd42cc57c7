"""Tiny seeded decoder configs and weights shared by the golden generator and the tests.

Weights come from numpy's PCG64 uniform stream (stable across numpy versions), scaled to a small
range, in Hugging Face tensor names and [out, in] order.
"""
from __future__ import annotations

import numpy as np

TINY = {
    "qwen2": dict(model_type="qwen2", hidden=128, inter=256, layers=2, heads=2, kv_heads=1, head_dim=64, vocab=512,
                  theta=1000000.0, eps=1e-6, bias=True, qk_norm=False, tie=True, rope=None, max_pos=4096),
    "llama3": dict(model_type="llama", hidden=256, inter=512, layers=2, heads=4, kv_heads=2, head_dim=64, vocab=384,
                   theta=500000.0, eps=1e-5, bias=False, qk_norm=False, tie=False,
                   rope={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                         "original_max_position_embeddings": 64}, max_pos=4096),
    "qwen3": dict(model_type="qwen3", hidden=256, inter=384, layers=2, heads=2, kv_heads=1, head_dim=128, vocab=320,
                  theta=1000000.0, eps=1e-6, bias=False, qk_norm=True, tie=False, rope=None, max_pos=4096),
}

# Qwen3.5-style hybrid decoder: Gated DeltaNet (linear attention) layers between full-attention layers with a
# sigmoid output gate carried in q_proj, QK-norm, partial rotary and (1 + w) RMSNorm weights. Kept apart from
# TINY: the CUDA model host runs the standard decoders only; the oracle runs this one.
HYBRID = {
    "qwen3_5": dict(model_type="qwen3_5_text", hidden=128, inter=256, layers=4, heads=2, kv_heads=1, head_dim=64,
                    vocab=256, theta=1000000.0, eps=1e-6, partial_rotary=0.25, max_pos=4096,
                    layer_types=["linear_attention", "full_attention", "linear_attention", "full_attention"],
                    lin_k_heads=1, lin_v_heads=2, lin_k_dim=128, lin_v_dim=128, lin_conv=4),
}

PROMPT_LEN = 12
GREEDY_NEW = 16


def weights(cfg: dict, seed: int, scale: float = 0.08) -> dict[str, np.ndarray]:
    rng = np.random.Generator(np.random.PCG64(seed))

    def u(*shape, s=scale):
        return ((rng.random(shape, dtype=np.float64) * 2 - 1) * s).astype(np.float32)

    H, I, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    qd, kd = cfg["heads"] * hd, cfg["kv_heads"] * hd
    w = {"model.embed_tokens.weight": u(cfg["vocab"], H, s=0.5)}
    for i in range(cfg["layers"]):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = (1.0 + u(H, s=0.1)).astype(np.float32)
        w[p + "post_attention_layernorm.weight"] = (1.0 + u(H, s=0.1)).astype(np.float32)
        w[p + "self_attn.q_proj.weight"] = u(qd, H)
        w[p + "self_attn.k_proj.weight"] = u(kd, H)
        w[p + "self_attn.v_proj.weight"] = u(kd, H)
        w[p + "self_attn.o_proj.weight"] = u(H, qd)
        if cfg["bias"]:
            w[p + "self_attn.q_proj.bias"] = u(qd, s=0.1)
            w[p + "self_attn.k_proj.bias"] = u(kd, s=0.1)
            w[p + "self_attn.v_proj.bias"] = u(kd, s=0.1)
        if cfg["qk_norm"]:
            w[p + "self_attn.q_norm.weight"] = (1.0 + u(hd, s=0.1)).astype(np.float32)
            w[p + "self_attn.k_norm.weight"] = (1.0 + u(hd, s=0.1)).astype(np.float32)
        w[p + "mlp.gate_proj.weight"] = u(I, H)
        w[p + "mlp.up_proj.weight"] = u(I, H)
        w[p + "mlp.down_proj.weight"] = u(H, I)
    w["model.norm.weight"] = (1.0 + u(H, s=0.1)).astype(np.float32)
    if not cfg["tie"]:
        w["lm_head.weight"] = u(cfg["vocab"], H)
    return w


def prompt(cfg: dict, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed + 1000))
    return rng.integers(0, cfg["vocab"], PROMPT_LEN).astype(np.int32)


def oracle_config(cfg: dict, wdtype: int = 0, group: int = 0, kv_dtype: int = 0) -> dict:
    """Keyword arguments of oracle.OracleModel for a tiny config."""
    rope = cfg["rope"] or {}
    kind = {"linear": 1, "yarn": 2, "llama3": 3}.get(rope.get("rope_type", "default"), 0)
    return dict(hidden=cfg["hidden"], inter=cfg["inter"], layers=cfg["layers"], heads=cfg["heads"],
                kv_heads=cfg["kv_heads"], head_dim=cfg["head_dim"], vocab=cfg["vocab"], max_pos=cfg["max_pos"],
                eps=cfg["eps"], theta=cfg["theta"], tie=int(cfg["tie"]), bias=int(cfg["bias"]),
                qk_norm=int(cfg["qk_norm"]), rope_type=kind, rope_factor=rope.get("factor", 1.0),
                rope_original_max=rope.get("original_max_position_embeddings", 0),
                rope_low=rope.get("low_freq_factor", 1.0), rope_high=rope.get("high_freq_factor", 4.0),
                rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0, wdtype=wdtype, group=group,
                kv_dtype=kv_dtype)


def model_config_kwargs(cfg: dict, kv_dtype: int = 0, q8_group: int = 0) -> dict:
    """Keyword arguments of levelzero.model_config for a tiny config."""
    rope = cfg["rope"] or {}
    return dict(hidden_size=cfg["hidden"], intermediate_size=cfg["inter"], num_layers=cfg["layers"],
                num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"], head_dim=cfg["head_dim"],
                vocab_size=cfg["vocab"], max_position_embeddings=cfg["max_pos"], rms_norm_eps=cfg["eps"],
                rope_theta=cfg["theta"], tie_word_embeddings=int(cfg["tie"]), attention_bias=int(cfg["bias"]),
                qk_norm=int(cfg["qk_norm"]), rope_type=rope.get("rope_type", "default"),
                rope_factor=rope.get("factor", 1.0),
                rope_original_max_position=rope.get("original_max_position_embeddings", 0),
                rope_low_freq_factor=rope.get("low_freq_factor", 1.0),
                rope_high_freq_factor=rope.get("high_freq_factor", 4.0), kv_dtype=kv_dtype, q8_group=q8_group)


def hybrid_weights(cfg: dict, seed: int, scale: float = 0.08) -> dict[str, np.ndarray]:
    """HF-named tensors of a HYBRID config. The four (1 + w) norms (input, post-attention, final, q/k) hold
    small deltas around 0; the gated norm of a linear layer holds its weight itself (around 1)."""
    rng = np.random.Generator(np.random.PCG64(seed))

    def u(*shape, s=scale):
        return ((rng.random(shape, dtype=np.float64) * 2 - 1) * s).astype(np.float32)

    H, I, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    qd, kd = cfg["heads"] * hd, cfg["kv_heads"] * hd
    hk, hv, dk, dv = cfg["lin_k_heads"], cfg["lin_v_heads"], cfg["lin_k_dim"], cfg["lin_v_dim"]
    conv = 2 * hk * dk + hv * dv
    w = {"model.embed_tokens.weight": u(cfg["vocab"], H, s=0.5)}
    for i, kind in enumerate(cfg["layer_types"]):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = u(H, s=0.1)
        w[p + "post_attention_layernorm.weight"] = u(H, s=0.1)
        if kind == "linear_attention":
            lp = p + "linear_attn."
            w[lp + "in_proj_qkv.weight"] = u(conv, H)
            w[lp + "in_proj_z.weight"] = u(hv * dv, H)
            w[lp + "in_proj_b.weight"] = u(hv, H, s=0.5)
            w[lp + "in_proj_a.weight"] = u(hv, H, s=0.5)
            w[lp + "conv1d.weight"] = u(conv, 1, cfg["lin_conv"], s=0.3)
            w[lp + "A_log"] = np.log(1 + 15 * rng.random(hv)).astype(np.float32)
            w[lp + "dt_bias"] = u(hv, s=0.3)
            w[lp + "norm.weight"] = (1.0 + u(dv, s=0.1)).astype(np.float32)
            w[lp + "out_proj.weight"] = u(H, hv * dv)
        else:
            w[p + "self_attn.q_proj.weight"] = u(2 * qd, H)  # per head: query rows, then gate rows
            w[p + "self_attn.k_proj.weight"] = u(kd, H)
            w[p + "self_attn.v_proj.weight"] = u(kd, H)
            w[p + "self_attn.o_proj.weight"] = u(H, qd)
            w[p + "self_attn.q_norm.weight"] = u(hd, s=0.1)
            w[p + "self_attn.k_norm.weight"] = u(hd, s=0.1)
        w[p + "mlp.gate_proj.weight"] = u(I, H)
        w[p + "mlp.up_proj.weight"] = u(I, H)
        w[p + "mlp.down_proj.weight"] = u(H, I)
    w["model.norm.weight"] = u(H, s=0.1)
    w["lm_head.weight"] = u(cfg["vocab"], H)
    return w


def hybrid_oracle_config(cfg: dict, wdtype: int = 0, group: int = 0, kv_dtype: int = 0) -> dict:
    """Keyword arguments of oracle.OracleModel for a HYBRID config."""
    mask = sum(1 << i for i, k in enumerate(cfg["layer_types"]) if k == "linear_attention")
    return dict(hidden=cfg["hidden"], inter=cfg["inter"], layers=cfg["layers"], heads=cfg["heads"],
                kv_heads=cfg["kv_heads"], head_dim=cfg["head_dim"], vocab=cfg["vocab"], max_pos=cfg["max_pos"],
                eps=cfg["eps"], theta=cfg["theta"], tie=0, bias=0, qk_norm=1, rope_type=0, rope_factor=1.0,
                rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, wdtype=wdtype, group=group,
                kv_dtype=kv_dtype, linear_mask=mask, lin_k_heads=cfg["lin_k_heads"], lin_v_heads=cfg["lin_v_heads"],
                lin_k_dim=cfg["lin_k_dim"], lin_v_dim=cfg["lin_v_dim"], lin_conv=cfg["lin_conv"], attn_gate=1,
                norm_offset=1.0, partial_rotary=cfg["partial_rotary"])


def hybrid_model_config_kwargs(cfg: dict, kv_dtype: int = 0, q8_group: int = 0) -> dict:
    """Keyword arguments of levelzero.model_config for a HYBRID config."""
    mask = sum(1 << i for i, k in enumerate(cfg["layer_types"]) if k == "linear_attention")
    return dict(hidden_size=cfg["hidden"], intermediate_size=cfg["inter"], num_layers=cfg["layers"],
                num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"], head_dim=cfg["head_dim"],
                vocab_size=cfg["vocab"], max_position_embeddings=cfg["max_pos"], rms_norm_eps=cfg["eps"],
                rope_theta=cfg["theta"], tie_word_embeddings=0, attention_bias=0, qk_norm=1,
                partial_rotary_factor=cfg["partial_rotary"], kv_dtype=kv_dtype, q8_group=q8_group,
                linear_layer_mask=mask, linear_num_key_heads=cfg["lin_k_heads"],
                linear_num_value_heads=cfg["lin_v_heads"], linear_key_head_dim=cfg["lin_k_dim"],
                linear_value_head_dim=cfg["lin_v_dim"], linear_conv_kernel=cfg["lin_conv"], attention_output_gate=1,
                rms_norm_offset=1.0)
