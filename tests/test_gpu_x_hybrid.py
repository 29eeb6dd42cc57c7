"""The model host on a Qwen3.5-style hybrid decoder (hf_tiny.HYBRID: Gated DeltaNet layers between
full-attention layers whose q_proj carries a sigmoid output gate, QK-norm, partial rotary, (1 + w) norms)
against transformers' Qwen3_5ForCausalLM fp32 (tests/golden/hf_tiny_hybrid.json) and against the CPU
oracle: the reference op sequence of LlmDecoderLayer.Forward / MixFull / MixLinear
(L/LlmDecoderLayer.cs:129-397) with the load rules of LlmLayerWeights.Load (L/LlmLayerWeights.cs:110-297)."""
from __future__ import annotations

import base64
import json
from pathlib import Path

import numpy as np
import pytest

import hf_tiny

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "hf_tiny_hybrid.json"


def _golden():
    doc = json.loads(GOLDEN.read_text())
    g = doc["models"]["qwen3_5"]
    logits = np.frombuffer(base64.b64decode(g["logits"]), "<f4").reshape(g["shape"])
    return doc["seed"], np.array(g["prompt"], np.int32), logits, g["greedy"]


def _model(lz, device, suite, seed, max_seq=128):
    cfg = hf_tiny.HYBRID["qwen3_5"]
    mc = lz.model_config(**hf_tiny.hybrid_model_config_kwargs(cfg, kv_dtype=lz.F32))
    model = lz.LlmModel(device, suite, mc, max_seq, "float32")
    for k, v in hf_tiny.hybrid_weights(cfg, seed).items():
        model.set_tensor(k, v)
    return model


def test_hybrid_model_matches_transformers(lz, device, suite):
    seed, prompt, logits_hf, greedy_hf = _golden()
    with _model(lz, device, suite, seed) as model:
        for t, tok in enumerate(prompt):
            lg = model.ComputeLogits(int(tok), t)
            err = float(np.abs(lg - logits_hf[t]).max())
            assert err < 1e-3 + 1e-3 * float(np.abs(logits_hf[t]).max()), f"position {t}: max err {err}"
        assert model.GenerateGreedy(prompt, len(greedy_hf)) == greedy_hf
        last = model.Prefill(prompt)
        assert float(np.abs(last - logits_hf[-1]).max()) < 2e-3


def test_hybrid_long_prefill_matches_oracle(lz, orc, device, suite):
    """A 40-token prompt as one chunk (the token-parallel conv and the chunked / scanned recurrence), then
    decode steps that continue the DeltaNet state, against the oracle."""
    seed = _golden()[0]
    cfg = hf_tiny.HYBRID["qwen3_5"]
    prompt = np.random.default_rng(11).integers(0, cfg["vocab"], 40).astype(np.int32)
    om = orc.OracleModel(hf_tiny.hybrid_oracle_config(cfg), 128)
    for k, v in hf_tiny.hybrid_weights(cfg, seed).items():
        om.set_tensor(k, v)
    want = om.forward(prompt, np.arange(prompt.size), last_only=True)
    with _model(lz, device, suite, seed) as model:
        got = model.Prefill(prompt)
        assert float(np.abs(got - want).max()) < 1e-3 + 1e-3 * float(np.abs(want).max())
        tok = int(np.argmax(got))
        for p in range(prompt.size, prompt.size + 4):
            w = om.step(tok, p)
            g = model.Decode(tok)
            assert float(np.abs(g - w).max()) < 1e-3 + 1e-3 * float(np.abs(w).max()), f"step at {p}"
            tok = int(np.argmax(w))
    om.close()
