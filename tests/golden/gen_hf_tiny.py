"""Generates tests/golden/hf_tiny.json: logits and greedy tokens of tiny seeded decoders from Hugging Face
transformers in float32 with eager attention -- the method the reference uses for its own goldens
(T/golden/gen_layer_golden.py:28-78, T/golden/gen_generation_golden.py). The weights are rebuilt in the
tests from tests/hf_tiny.py with the same seed, so the fixture holds outputs only.

With --hybrid it writes tests/golden/hf_tiny_hybrid.json instead: the Qwen3.5-style hybrid decoder of
hf_tiny.HYBRID (Gated DeltaNet and gated full-attention layers) from transformers' Qwen3_5ForCausalLM.

Usage: python tests/golden/gen_hf_tiny.py [--hybrid]
"""
from __future__ import annotations

import base64
import json
import sys
from pathlib import Path

import numpy as np
import torch
from transformers import LlamaConfig, LlamaForCausalLM, Qwen2Config, Qwen2ForCausalLM, Qwen3Config, Qwen3ForCausalLM

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import hf_tiny  # noqa: E402

OUT = Path(__file__).resolve().parent / "hf_tiny.json"
OUT_HYBRID = Path(__file__).resolve().parent / "hf_tiny_hybrid.json"
SEED = 7


def build(name: str, cfg: dict):
    common = dict(hidden_size=cfg["hidden"], intermediate_size=cfg["inter"], num_hidden_layers=cfg["layers"],
                  num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"], head_dim=cfg["head_dim"],
                  vocab_size=cfg["vocab"], max_position_embeddings=cfg["max_pos"], rms_norm_eps=cfg["eps"],
                  tie_word_embeddings=cfg["tie"], hidden_act="silu", attn_implementation="eager")
    params = {"rope_theta": cfg["theta"]}
    params.update(cfg["rope"] or {"rope_type": "default"})
    if cfg["model_type"] == "qwen2":
        model = Qwen2ForCausalLM(Qwen2Config(rope_parameters=params, use_sliding_window=False, **common))
    elif cfg["model_type"] == "llama":
        model = LlamaForCausalLM(LlamaConfig(rope_parameters=params, attention_bias=False, mlp_bias=False, **common))
    else:
        model = Qwen3ForCausalLM(Qwen3Config(rope_parameters=params, attention_bias=False, **common))
    w = hf_tiny.weights(cfg, SEED)
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    if cfg["tie"]:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing
    return model.float().eval()


def build_hybrid(cfg: dict):
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    conf = Qwen3_5TextConfig(
        hidden_size=cfg["hidden"], intermediate_size=cfg["inter"], num_hidden_layers=cfg["layers"],
        num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"], head_dim=cfg["head_dim"],
        vocab_size=cfg["vocab"], max_position_embeddings=cfg["max_pos"], rms_norm_eps=cfg["eps"],
        tie_word_embeddings=False, hidden_act="silu", attention_bias=False, layer_types=cfg["layer_types"],
        linear_num_key_heads=cfg["lin_k_heads"], linear_num_value_heads=cfg["lin_v_heads"],
        linear_key_head_dim=cfg["lin_k_dim"], linear_value_head_dim=cfg["lin_v_dim"],
        linear_conv_kernel_dim=cfg["lin_conv"], attn_implementation="eager",
        rope_parameters={"rope_theta": cfg["theta"], "partial_rotary_factor": cfg["partial_rotary"],
                         "rope_type": "default"})
    model = Qwen3_5ForCausalLM(conf)
    sd = {k: torch.from_numpy(v) for k, v in hf_tiny.hybrid_weights(cfg, SEED).items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing
    return model.float().eval()


def enc(a: np.ndarray) -> str:
    return base64.b64encode(np.ascontiguousarray(a, "<f4").tobytes()).decode("ascii")


def main() -> None:
    torch.manual_seed(0)
    hybrid = "--hybrid" in sys.argv[1:]
    doc = {"seed": SEED, "generator": "transformers " + __import__("transformers").__version__, "models": {}}
    for name, cfg in (hf_tiny.HYBRID if hybrid else hf_tiny.TINY).items():
        model = build_hybrid(cfg) if hybrid else build(name, cfg)
        ids = hf_tiny.prompt(cfg, SEED)
        with torch.no_grad():
            logits = model(torch.from_numpy(ids[None].astype(np.int64)), use_cache=False).logits[0].numpy()
            gen = model.generate(torch.from_numpy(ids[None].astype(np.int64)), max_new_tokens=hf_tiny.GREEDY_NEW,
                                 do_sample=False, min_new_tokens=hf_tiny.GREEDY_NEW)[0, len(ids):].tolist()
        doc["models"][name] = {"prompt": ids.tolist(), "logits": enc(logits), "shape": list(logits.shape),
                               "greedy": gen}
        print(name, logits.shape, gen[:8])
    out = OUT_HYBRID if hybrid else OUT
    out.write_text(json.dumps(doc))
    print("wrote", out, out.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
