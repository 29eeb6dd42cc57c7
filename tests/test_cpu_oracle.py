"""CPU tests: the oracle against the reference's known answers and golden vectors, the host-side logic
of the library, and its exported C ABI. No GPU is used here."""
from __future__ import annotations

import base64
import ctypes as C
import json
import re
from pathlib import Path

import numpy as np
import pytest

import hf_tiny

GOLDEN = Path(__file__).resolve().parent / "golden"
HEADER = Path(__file__).resolve().parents[1] / "include" / "l0b200.h"
ROPE_KIND = {"linear": 1, "yarn": 2, "llama3": 3}


def rope_cases():
    doc = json.loads((GOLDEN / "rope_tables.json").read_text())
    return doc["cases"]


def rope_args(case):
    s = case["scaling"] or {}
    return dict(dim=case["head_dim"], theta=case["theta"], max_pos=case["max_position_embeddings"],
                rope_type=ROPE_KIND.get(s.get("rope_type"), 0), factor=s.get("factor", 1.0),
                original_max=s.get("original_max_position_embeddings", 0), low=s.get("low_freq_factor", 1.0),
                high=s.get("high_freq_factor", 4.0), beta_fast=s.get("beta_fast", 32.0),
                beta_slow=s.get("beta_slow", 1.0), attention_factor=s.get("attention_factor", 0.0))


# --------------------------------------------------------------------------------------------
# RoPE tables: T/RopeFrequenciesTests.cs:25-47 (rel 1e-5) and T/RopeLlama3Tests.cs:8-38
# --------------------------------------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(rope_cases()))
def test_oracle_rope_tables_match_golden(orc, name):
    case = rope_cases()[name]
    inv, att = orc.rope_frequencies(**rope_args(case))
    want = np.array(case["inv_freq"])
    assert len(inv) == len(want)
    np.testing.assert_allclose(inv, want, rtol=1e-5, atol=1e-12)
    assert att == pytest.approx(case["attention_factor"], abs=1e-5)


@pytest.mark.parametrize("name", sorted(rope_cases()))
def test_library_rope_tables_match_golden(lz, name):
    case = rope_cases()[name]
    a = rope_args(case)
    cfg = lz.model_config(head_dim=a["dim"], rope_theta=a["theta"], max_position_embeddings=a["max_pos"],
                          rope_type=a["rope_type"], rope_factor=a["factor"], rope_original_max_position=a["original_max"],
                          rope_low_freq_factor=a["low"], rope_high_freq_factor=a["high"], rope_beta_fast=a["beta_fast"],
                          rope_beta_slow=a["beta_slow"], rope_attention_factor=a["attention_factor"])
    inv, att = lz.rope_frequencies(cfg)
    np.testing.assert_allclose(inv, np.array(case["inv_freq"]), rtol=1e-5, atol=1e-12)
    assert att == pytest.approx(case["attention_factor"], abs=1e-5)


def test_rope_unknown_type_is_not_supported(lz):
    cfg = lz.model_config(head_dim=16, rope_type=7)
    with pytest.raises(lz.NotSupportedException):
        lz.rope_frequencies(cfg)


def test_rope_linear_divides_every_frequency(orc):
    plain, _ = orc.rope_frequencies(16, 10000.0, 2048)
    lin, att = orc.rope_frequencies(16, 10000.0, 2048, rope_type=orc.ROPE_LINEAR, factor=4.0)
    assert att == 1.0
    np.testing.assert_allclose(lin, plain / 4, rtol=1e-6)


def test_rope_yarn_factor_one_is_unscaled(orc):
    plain, _ = orc.rope_frequencies(16, 10000.0, 2048)
    yarn, att = orc.rope_frequencies(16, 10000.0, 2048, rope_type=orc.ROPE_YARN, factor=1.0)
    assert att == 1.0
    np.testing.assert_array_equal(plain, yarn)


# --------------------------------------------------------------------------------------------
# Linear layers: T/LlmMatrixTests.cs:47-130, T/LlmMatrixInt8Tests.cs:45-119
# --------------------------------------------------------------------------------------------

def test_gemv_known_answer_both_layouts(orc):
    hf = np.arange(1, 9, dtype=np.float32).reshape(4, 2)  # [out=4, in=2]
    x = np.array([[1.0, 10.0]], np.float32)
    np.testing.assert_array_equal(orc.gemv_out_in(x, hf, orc.F32)[0], [21, 43, 65, 87])
    np.testing.assert_array_equal(orc.gemv_in_out(x, np.ascontiguousarray(hf.T), half=False)[0], [21, 43, 65, 87])
    halves = np.ascontiguousarray(hf.T).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(orc.gemv_in_out(x, halves, half=True)[0], [21, 43, 65, 87])
    np.testing.assert_array_equal(orc.gemv_out_in(x, hf.astype(np.float16).view(np.uint16), orc.F16)[0],
                                  [21, 43, 65, 87])


@pytest.mark.parametrize("out_dim,in_dim", [(64, 48), (30, 17)])
def test_gemv_matches_double_loop(orc, out_dim, in_dim):
    rng = np.random.default_rng(out_dim + in_dim)
    w = ((rng.random((in_dim, out_dim)) * 2 - 1) * 0.1).astype(np.float32)  # [in, out]
    x = ((rng.random(in_dim) * 2 - 1)).astype(np.float32)
    y = orc.gemv_in_out(x[None], w, half=False)[0]
    want = (x.astype(np.float64) @ w.astype(np.float64))
    assert np.max(np.abs(y - want)) < 1e-4


@pytest.mark.parametrize("rows", [1, 5])
def test_int8_projection_error_bound(orc, rows):
    rng = np.random.default_rng(3)
    hf = ((rng.random((96, 160)) * 2 - 1) * 0.2).astype(np.float32)
    x = ((rng.random((rows, 160)) * 2 - 1) * 1.5).astype(np.float32)
    q, s = orc.q8_quantize(hf, 32)
    y = orc.gemv_out_in(x, q, orc.I8, s, 32)
    truth = x.astype(np.float64) @ hf.T.astype(np.float64)
    rel = np.sqrt(np.sum((y - truth) ** 2) / np.sum(truth ** 2))
    assert rel < 0.02, rel


def test_int8_size_rule():
    # SizeInBytes of an int8 matrix: N*K bytes + K/32*N halves (L/LlmMatrix.cs:29-31).
    n, k = 64, 96
    assert n * k + k // 32 * n * 2 == 6528


@pytest.mark.parametrize("n,k,group", [(8, 64, 32), (16, 896, 896), (5, 96, 32), (12, 160, 160)])
def test_host_quantizer_matches_oracle_bit_exact(lz, orc, n, k, group):
    rng = np.random.default_rng(n * k + group)
    hf = ((rng.random((n, k)) * 2 - 1) * 0.3).astype(np.float32)
    hf[0, :group] = 0.0                      # an all-zero group: scale 0, codes 0
    hf[1, :4] = [0.5, -0.5, 1.5, -2.5]       # values that land on .5 after scaling test ties-to-even
    q_lib, s_lib = lz.q8_quantize_out_in(hf, group)
    q_orc, s_orc = orc.q8_quantize(hf, group)
    np.testing.assert_array_equal(q_lib, q_orc)
    np.testing.assert_array_equal(s_lib.view(np.uint16), s_orc)
    assert np.all(np.abs(q_lib.astype(int)) <= 127)
    # Dequantisation indexing: value(o, i) = q[o, i] * s[o, i // group].
    deq = q_lib.astype(np.float32) * np.repeat(s_lib.astype(np.float32), group, axis=1)
    assert np.max(np.abs(deq - hf)) <= np.max(s_lib.astype(np.float32)) * 0.5 + 1e-7


def test_f16_and_bf16_conversions_match_numpy(orc):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        (rng.standard_normal(20000) * 10).astype(np.float32),
        (rng.standard_normal(2000) * 1e-5).astype(np.float32),   # half subnormals
        np.array([65504, 65519, 65520, 70000, -0.0, 0.0, 2 ** -24, 2 ** -25, 3 * 2 ** -26, np.inf, -np.inf],
                 np.float32),
    ])
    L = orc.lib()
    got = np.array([L.orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    np.testing.assert_array_equal(got, vals.astype(np.float16).view(np.uint16))
    back = np.array([L.orc_f16_to_f32(int(h)) for h in got[:3000]], np.float32)
    np.testing.assert_array_equal(back, vals[:3000].astype(np.float16).astype(np.float32))
    bf = np.array([L.orc_f32_to_bf16(float(v)) for v in vals[:3000]], np.uint16)
    import torch
    want = torch.from_numpy(vals[:3000]).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(bf, want)


# --------------------------------------------------------------------------------------------
# Synthetic weight generator (restated in the oracle; the GPU test checks device == oracle)
# --------------------------------------------------------------------------------------------

def _splitmix(x):
    m = (1 << 64) - 1
    x = (x + 0x9E3779B97F4A7C15) & m
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
    return x ^ (x >> 31)


def test_synth_generator_matches_python_restatement(orc):
    seed, tid = 1234, 1002
    stream = _splitmix(seed ^ ((tid * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)))
    got8 = orc.synth_fill(64, orc.I8, seed, tid, 2, 0.0)
    got = orc.synth_fill(64, orc.F32, seed, tid, 0, 0.02)
    for i in range(64):
        bits = _splitmix((stream + i * 0xD1B54A32D192ED03) & ((1 << 64) - 1))
        assert got8[i] == (bits % 255) - 127
        s = (bits & 0xFFFF) + ((bits >> 16) & 0xFFFF) + ((bits >> 32) & 0xFFFF) + (bits >> 48)
        u = np.float32(s) * np.float32(1.0 / 65536.0)
        v = np.float32(np.float32(u - np.float32(2.0)) * np.float32(1.7320508)) * np.float32(0.02)
        assert got[i] == v


def test_synth_normal_statistics(orc):
    x = orc.synth_fill(200000, orc.F32, 1, 77, 0, 0.02)
    assert abs(float(x.mean())) < 2e-4
    assert float(x.std()) == pytest.approx(0.02, rel=0.01)


# --------------------------------------------------------------------------------------------
# Whole decoder: the oracle against Hugging Face transformers fp32 eager
# --------------------------------------------------------------------------------------------

def _hf_golden(name):
    doc = json.loads((GOLDEN / "hf_tiny.json").read_text())
    m = doc["models"][name]
    logits = np.frombuffer(base64.b64decode(m["logits"]), "<f4").reshape(m["shape"])
    return doc["seed"], np.array(m["prompt"], np.int32), logits, m["greedy"]


@pytest.mark.parametrize("name", sorted(hf_tiny.TINY))
def test_oracle_model_matches_transformers(orc, name):
    cfg = hf_tiny.TINY[name]
    seed, prompt, logits_hf, greedy_hf = _hf_golden(name)
    m = orc.OracleModel(hf_tiny.oracle_config(cfg), 64)
    for k, v in hf_tiny.weights(cfg, seed).items():
        m.set_tensor(k, v)
    for t, tok in enumerate(prompt):
        lg = m.step(int(tok), t)
        np.testing.assert_allclose(lg, logits_hf[t], atol=2e-4, rtol=1e-3)
    toks, pos, nxt = [], len(prompt), int(np.argmax(lg))
    for _ in range(len(greedy_hf)):
        toks.append(nxt)
        nxt = int(np.argmax(m.step(nxt, pos)))
        pos += 1
    assert toks == greedy_hf
    m.close()


def test_oracle_hybrid_model_matches_transformers(orc):
    """A Qwen3.5-style hybrid decoder (hf_tiny.HYBRID: Gated DeltaNet layers between full-attention
    layers with the sigmoid output gate in q_proj, QK-norm, partial rotary, (1 + w) norms) in the oracle
    against transformers' Qwen3_5ForCausalLM in fp32 (tests/golden/hf_tiny_hybrid.json): every prompt
    position's logits token by token, the 16 greedy tokens after it, and the prompt as one prefill chunk
    (the linear layers walk the chunk's rows in order from a reset state)."""
    cfg = hf_tiny.HYBRID["qwen3_5"]
    doc = json.loads((GOLDEN / "hf_tiny_hybrid.json").read_text())
    g = doc["models"]["qwen3_5"]
    logits_hf = np.frombuffer(base64.b64decode(g["logits"]), "<f4").reshape(g["shape"])
    prompt = np.array(g["prompt"], np.int32)
    assert np.array_equal(prompt, hf_tiny.prompt(cfg, doc["seed"]))
    w = hf_tiny.hybrid_weights(cfg, doc["seed"])
    m = orc.OracleModel(hf_tiny.hybrid_oracle_config(cfg), 64, batch=2)
    for k, v in w.items():
        m.set_tensor(k, v)
    for t, tok in enumerate(prompt):
        lg = m.step(int(tok), t)
        np.testing.assert_allclose(lg, logits_hf[t], atol=2e-4, rtol=1e-3)
    toks, pos, nxt = [], len(prompt), int(np.argmax(lg))
    for _ in range(len(g["greedy"])):
        toks.append(nxt)
        nxt = int(np.argmax(m.step(nxt, pos)))
        pos += 1
    assert toks == g["greedy"]
    # The whole prompt as one chunk of sequence 1 (state reset at position 0, rows in order).
    chunk = m.forward(prompt, np.arange(prompt.size), np.ones(prompt.size, np.int32))
    np.testing.assert_allclose(chunk, logits_hf, atol=2e-4, rtol=1e-3)
    m.close()


def test_oracle_hybrid_rejects_attention_names_on_linear_layers(orc):
    cfg = hf_tiny.HYBRID["qwen3_5"]
    m = orc.OracleModel(hf_tiny.hybrid_oracle_config(cfg), 8)
    with pytest.raises(Exception):
        m.set_tensor("model.layers.0.self_attn.k_proj.weight", np.zeros((64, 128), np.float32))
    m.close()


# --------------------------------------------------------------------------------------------
# Gated DeltaNet: the oracle against transformers' torch reference functions (Qwen3.5)
# --------------------------------------------------------------------------------------------

def test_oracle_gated_delta_matches_transformers(orc):
    import torch
    from transformers.models.qwen3_5 import modeling_qwen3_5 as q35

    rng = np.random.default_rng(5)
    hk, hv, dk, dv, T, K = 2, 4, 64, 64, 9, 4
    conv_dim = 2 * hk * dk + hv * dv
    x = rng.standard_normal((T, conv_dim)).astype(np.float32)
    w = (rng.standard_normal((conv_dim, K)) * 0.5).astype(np.float32)
    z = rng.standard_normal((T, hv * dv)).astype(np.float32)
    b = rng.standard_normal((T, hv)).astype(np.float32)
    a = rng.standard_normal((T, hv)).astype(np.float32)
    a_log = np.log(rng.uniform(1, 16, hv)).astype(np.float32)
    dt_bias = rng.standard_normal(hv).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    # Oracle: conv (zero history) then the recurrence from a zero state.
    state_c = np.zeros((conv_dim, K - 1), np.float32)
    conv = np.zeros_like(x)
    orc.lib().orc_causal_conv(x, state_c, w, conv, conv_dim, K, T)
    S = np.zeros((hv, dk, dv), np.float32)
    out = np.zeros((T, hv * dv), np.float32)
    orc.lib().orc_gated_delta(conv, z, b, a, a_log, dt_bias, norm_w, S, out, hk, hv, dk, dv, T, 1e-6)
    # transformers: F.silu(conv1d) then torch_recurrent_gated_delta_rule and the gated norm.
    xt = torch.from_numpy(x).T[None]
    ref_conv = torch.nn.functional.silu(torch.nn.functional.conv1d(
        torch.nn.functional.pad(xt, (K - 1, 0)), torch.from_numpy(w)[:, None], groups=conv_dim))[0].T
    np.testing.assert_allclose(conv, ref_conv.numpy(), atol=1e-5, rtol=1e-5)
    q, k, v = torch.split(ref_conv[None], [hk * dk, hk * dk, hv * dv], dim=-1)
    q = q.reshape(1, T, hk, dk).repeat_interleave(hv // hk, dim=2)
    k = k.reshape(1, T, hk, dk).repeat_interleave(hv // hk, dim=2)
    v = v.reshape(1, T, hv, dv)
    beta = torch.from_numpy(b)[None].sigmoid()
    g = -torch.from_numpy(a_log).exp() * torch.nn.functional.softplus(torch.from_numpy(a)[None] +
                                                                       torch.from_numpy(dt_bias))
    core, last = q35.torch_recurrent_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=None,
                                                      output_final_state=True, use_qk_l2norm_in_kernel=True)
    norm = q35.Qwen3_5RMSNormGated(dv, eps=1e-6)
    norm.weight.data = torch.from_numpy(norm_w)
    ref = norm(core.reshape(-1, dv), torch.from_numpy(z).reshape(-1, dv)).reshape(T, hv * dv)
    np.testing.assert_allclose(out, ref.detach().numpy(), atol=2e-4, rtol=2e-3)
    np.testing.assert_allclose(S, last[0].numpy(), atol=2e-5, rtol=1e-4)
    # Chunked HF prefill gives the same state (the recurrence is order-exact in the oracle).
    core_c, last_c = q35.torch_chunk_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=None,
                                                      output_final_state=True, use_qk_l2norm_in_kernel=True)
    np.testing.assert_allclose(S, last_c[0].numpy(), atol=1e-4, rtol=1e-3)


# --------------------------------------------------------------------------------------------
# The library: exports, host rules and failure without a GPU
# --------------------------------------------------------------------------------------------

def header_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"L0B_API\s+[^;(]*?\b(l0b_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lz):
    syms = header_symbols()
    assert len(syms) > 60
    lib = C.CDLL(str(lz.LIB_PATH))
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_static_shape_rules(lz):
    L = lz.load_library()
    assert L.l0b_gemv_supports(896) and not L.l0b_gemv_supports(30)
    assert L.l0b_gemv_q8_supports(4864, 896) and not L.l0b_gemv_q8_supports(64, 50)
    assert not L.l0b_gemv_q8_supports(30, 64)
    assert L.l0b_gemv_q8_group_size() == 32
    assert L.l0b_gemv_max_rows() >= 8


def test_config_defaults_follow_hf_parse(lz):
    cfg = lz.model_config()
    assert cfg.max_position_embeddings == 2048
    assert cfg.rms_norm_eps == pytest.approx(1e-6)
    assert cfg.rope_theta == 10000.0
    assert cfg.kv_dtype == lz.F32 and cfg.q8_group == 32 and cfg.tp_size == 1


def test_no_device_is_reported_without_gpu(lz):
    if lz.LevelZeroRuntime.IsAvailable():
        pytest.skip("a GPU is present")
    with pytest.raises(lz.NoDeviceError):
        lz.ComputeDevice(0)


def test_quantizer_rejects_bad_shapes(lz):
    with pytest.raises(lz.ArgumentException):
        lz.q8_quantize_out_in(np.zeros((4, 50), np.float32), 32)


# ----------------------------------------------------------------------------------------------
# The oracle's fp32 timing GEMM and its batched forward (prefill chunks, decode batches)
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("m,n,k,wdtype,group", [(1, 97, 896, 3, 0), (13, 64, 896, 3, 32), (7, 33, 72, 1, 0),
                                                 (5, 10, 19, 0, 0), (30, 65, 256, 2, 0)])
def test_gemm_fast_matches_double_accumulation(orc, m, n, k, wdtype, group):
    rng = np.random.default_rng(m * 1000 + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    s = None
    if wdtype == orc.I8:
        w = rng.integers(-127, 128, (n, k)).astype(np.int8)
        g = group or k
        s = orc.f16_bits(rng.uniform(1e-3, 2e-2, n * (k // g)).astype(np.float32)).reshape(n, k // g)
    elif wdtype == orc.F32:
        w = rng.standard_normal((n, k)).astype(np.float32)
    else:
        wf = rng.standard_normal((n, k)).astype(np.float32)
        w = (orc.f16_bits(wf) if wdtype == orc.F16 else (wf.view(np.uint32) >> 16).astype(np.uint16)).reshape(n, k)
    exact = orc.gemv_out_in(x, w, wdtype, s, group)
    fast = orc.gemm_fast(x, w, wdtype, s, group)
    assert np.abs(fast - exact).max() <= 1e-5 * np.abs(exact).max()


def _tiny_oracle(orc, name, batch):
    cfg = hf_tiny.TINY[name]
    om = orc.OracleModel(hf_tiny.oracle_config(cfg, orc.F32, 0, orc.F16), 32, batch)
    for key, v in hf_tiny.weights(cfg, 7).items():
        om.set_tensor(key, v)
    return om, hf_tiny.prompt(cfg, 7)


@pytest.mark.parametrize("name", ["qwen2", "llama3", "qwen3"])
def test_oracle_prefill_chunk_equals_token_steps(orc, name):
    """IngestPrompt as one causal chunk equals one Step per token, bit for bit in double accumulation
    (the reference's chunked-prefill == sequential test, T/Qwen25PrefillTests.cs:41-75)."""
    a, prompt = _tiny_oracle(orc, name, 1)
    for t, tok in enumerate(prompt[:9]):
        want = a.step(int(tok), t)
    b, _ = _tiny_oracle(orc, name, 3)
    got = b.prefill(prompt[:9], seq=2)
    np.testing.assert_array_equal(got, want)
    ka, va = a.read_kv(1, 0, 9, a.kv_dim)
    kb, vb = b.read_kv(1, 0, 9, b.kv_dim, seq=2)
    np.testing.assert_array_equal(ka, kb)
    np.testing.assert_array_equal(va, vb)
    c, _ = _tiny_oracle(orc, name, 1)
    c.set_fast(True)
    np.testing.assert_allclose(c.prefill(prompt[:9]), want, rtol=0, atol=1e-4 * np.abs(want).max())
    for m in (a, b, c):
        m.close()


def test_oracle_decode_batch_equals_separate_sequences(orc):
    """StepBatch: rows of different sequences, each at its own position, equal separate single steps."""
    om, prompt = _tiny_oracle(orc, "qwen2", 2)
    om.prefill(prompt[:5], seq=0)
    om.prefill(prompt[3:10], seq=1)
    got = om.forward([11, 12], [5, 7], [0, 1])
    for seq, (p, off) in enumerate(((prompt[:5], 5), (prompt[3:10], 7))):
        ref, _ = _tiny_oracle(orc, "qwen2", 1)
        ref.prefill(p)
        np.testing.assert_array_equal(got[seq], ref.step(11 + seq, off))
        ref.close()
    # A context written from outside (another prefill's K/V rows) is what the next step attends to.
    other, _ = _tiny_oracle(orc, "qwen2", 1)
    for layer in range(hf_tiny.TINY["qwen2"]["layers"]):
        k, v = om.read_kv(layer, 0, 7, om.kv_dim, seq=1)
        other.write_kv(layer, 0, k, v)
    np.testing.assert_array_equal(other.step(12, 7), got[1])
    om.close()
    other.close()


def test_config2_weights_amplify_rounding(orc):
    """Config 2's synthetic int8 weights amplify rounding differences: four layers of config-2 width
    in the oracle's fp32 build and in its double build (each projection agreeing to ~1e-7 relative)
    already disagree by more than the elementwise max-abs 1e-2 + rel 1e-2 bar on part of the logits,
    while staying within 1e-2 of the logit range. This is why the full-depth config-2 GPU tests hold the
    elementwise bar on the decisive (top) logits and the range-relative bar on the rest. (A 32-token
    prompt: the spread grows with the number of attended positions.)"""
    cfg = dict(hidden=3584, inter=18944, layers=4, heads=28, kv_heads=4, head_dim=128, vocab=152064, max_pos=32768,
               eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
               rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0,
               wdtype=orc.I8, group=0, kv_dtype=orc.F16)
    prompt = np.random.default_rng(2).integers(0, 152064, 32).astype(np.int32)
    out = []
    for fast in (False, True):
        om = orc.OracleModel(cfg, 34)
        om.init_synthetic(2, 0.02, 1e-3, 2e-2)
        om.set_fast(fast)
        out.append(om.prefill(prompt))
        om.close()
    exact, fast = out
    err = np.abs(fast.astype(np.float64) - exact)
    assert (err > 1e-2 + 1e-2 * np.abs(exact)).sum() > 0
    assert err.max() <= 1e-2 * np.abs(exact).max()


def test_block_int8_matches_blocked_index():
    """levelzero.block_int8 puts element (r, c) of a row-major int8 [N, K] matrix at byte
    ((r / 16) * (K / 512) + c / 512) * 16 * 512 + (r % 16) * 512 + c % 512: the blocked layout the
    library's GEMVs and GEMM address (blocked_index in csrc/gemv.cuh)."""
    from l0llm_b200 import levelzero as lz

    rng = np.random.default_rng(0)
    n, k = 48, 1536
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    b = lz.block_int8(q).reshape(-1)
    r, c = np.meshgrid(np.arange(n), np.arange(k), indexing="ij")
    idx = ((r // 16) * (k // 512) + c // 512) * 16 * 512 + (r % 16) * 512 + c % 512
    assert np.array_equal(b[idx], q)
    with pytest.raises(ValueError):
        lz.block_int8(q[:40])
