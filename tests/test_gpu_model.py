"""GPU parity of the decoder host (LlmModel mirror) against Hugging Face goldens and the CPU oracle.

Mirrors the reference's model-level tests on synthetic weights: per-step logits against HF fp32 eager
(T/Qwen25LayerGoldenTests.cs method), greedy token agreement (T/Qwen25GenerationGoldenTests.cs), chunked
prefill == token-by-token within 2e-3 with the KV cache checked through the next step
(T/Qwen25PrefillTests.cs:41-89), and restarts from position 0.
"""
from __future__ import annotations

import base64
import json
from pathlib import Path

import numpy as np
import pytest

import hf_tiny

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def hf_golden(name):
    doc = json.loads((GOLDEN / "hf_tiny.json").read_text())
    m = doc["models"][name]
    logits = np.frombuffer(base64.b64decode(m["logits"]), "<f4").reshape(m["shape"])
    return doc["seed"], np.array(m["prompt"], np.int32), logits, m["greedy"]


def make_model(lz, device, suite, name, precision="float32", kv="f32", max_seq=256, q8_group=0, seed=None):
    cfg = hf_tiny.TINY[name]
    kvc = {"f32": lz.F32, "f16": lz.F16, "bf16": lz.BF16}[kv]
    mc = lz.model_config(**hf_tiny.model_config_kwargs(cfg, kv_dtype=kvc, q8_group=q8_group))
    model = lz.LlmModel(device, suite, mc, max_seq, precision)
    gseed = hf_golden(name)[0] if seed is None else seed
    for k, v in hf_tiny.weights(cfg, gseed).items():
        model.set_tensor(k, v)
    return model


def oracle_model(orc, name, wdtype=0, group=0, kv=0, max_seq=256):
    cfg = hf_tiny.TINY[name]
    m = orc.OracleModel(hf_tiny.oracle_config(cfg, wdtype, group, kv), max_seq)
    for k, v in hf_tiny.weights(cfg, hf_golden(name)[0]).items():
        m.set_tensor(k, v)
    return m


def max_diff(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("name", sorted(hf_tiny.TINY))
def test_logits_and_greedy_match_transformers(lz, device, suite, name, fused):
    seed, prompt, logits_hf, greedy_hf = hf_golden(name)
    with make_model(lz, device, suite, name) as model:
        model.set_fused(fused)
        for t, tok in enumerate(prompt):
            lg = model.ComputeLogits(int(tok), t)
            assert max_diff(lg, logits_hf[t]) < 1e-3 + 1e-3 * float(np.abs(logits_hf[t]).max())
        assert model.GenerateGreedy(prompt, len(greedy_hf)) == greedy_hf
        batched = model.Prefill(prompt)
        assert max_diff(batched, logits_hf[-1]) < 2e-3


@pytest.mark.parametrize("precision,wdtype,group,kv", [("float16", 1, 0, "f16"), ("bfloat16", 2, 0, "bf16"),
                                                         ("int8", 3, 0, "f16"), ("int8", 3, 32, "f32")])
@pytest.mark.parametrize("name", ["qwen2", "llama3"])
def test_reduced_precision_matches_oracle(lz, orc, device, suite, name, precision, wdtype, group, kv):
    seed, prompt, _, _ = hf_golden(name)
    kvo = {"f32": 0, "f16": 1, "bf16": 2}[kv]
    om = oracle_model(orc, name, wdtype, group, kvo)
    with make_model(lz, device, suite, name, precision, kv, q8_group=group) as model:
        for t, tok in enumerate(prompt):
            lg = model.ComputeLogits(int(tok), t)
            want = om.step(int(tok), t)
            assert max_diff(lg, want) < 1e-2 + 1e-2 * float(np.abs(want).max())
        # Greedy continuation from the prompt matches the oracle's greedy tokens.
        toks = model.GenerateGreedy(prompt, 12)
        nxt, pos, ref = int(np.argmax(want)), len(prompt), []
        for _ in range(12):
            ref.append(nxt)
            nxt = int(np.argmax(om.step(nxt, pos)))
            pos += 1
        assert toks == ref
    om.close()


@pytest.mark.parametrize("length", [1, 2, 7, 8, 9, 16, 17, 35, 64, 65, 130, 513, 600])
def test_prefill_matches_token_by_token(lz, device, suite, length):
    rng = np.random.default_rng(length)
    cfg = hf_tiny.TINY["llama3"]
    prompt = rng.integers(0, cfg["vocab"], length).astype(np.int32)
    with make_model(lz, device, suite, "llama3", "float16", "f16", max_seq=max(256, length + 8)) as model:
        seq = None
        for i, tok in enumerate(prompt):
            seq = model.ComputeLogits(int(tok), i)
        nxt = int(np.argmax(seq))
        seq_after = model.ComputeLogits(nxt, length)
        batched = model.Prefill(prompt)
        assert model.Position == length
        batched_after = model.Decode(nxt)
        assert int(np.argmax(batched)) == nxt
        assert max_diff(seq, batched) < 2e-3
        assert int(np.argmax(seq_after)) == int(np.argmax(batched_after))
        assert max_diff(seq_after, batched_after) < 2e-3


@pytest.mark.parametrize("precision,kv", [("float16", "f16"), ("bfloat16", "bf16"), ("int8", "f16")])
@pytest.mark.parametrize("name", ["qwen2", "llama3"])
def test_prefill_tensor_core_gemm_matches_gemv(lz, device, suite, name, precision, kv):
    """Prefill chunks of >= 16 rows run their projections on the tcgen05 GEMM with the activations split
    into hi + lo 16-bit halves (int8: per-row scales, bytes converted to f16 in shared memory); the
    logits agree with the GEMV-only prefill up to f32 summation order."""
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, hf_tiny.TINY[name]["vocab"], 600).astype(np.int32)  # chunks of 512 and 88
    with make_model(lz, device, suite, name, precision, kv, max_seq=640) as model:
        model.set_gemm_rows(0)
        want = model.Prefill(prompt)
        want_next = model.Decode(int(np.argmax(want)))
        model.set_gemm_rows(16)
        got = model.Prefill(prompt)
        got_next = model.Decode(int(np.argmax(got)))
    assert int(np.argmax(got)) == int(np.argmax(want))
    assert max_diff(got, want) < 2e-3
    assert max_diff(got_next, want_next) < 2e-3


def test_prefill_restarts_from_position_zero(lz, device, suite):
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 384, 20).astype(np.int32)
    with make_model(lz, device, suite, "llama3", "int8", "f16") as model:
        first = model.Prefill(prompt[:12])
        model.Prefill(prompt)
        again = model.Prefill(prompt[:12])
        assert model.Position == 12
        assert max_diff(first, again) < 1e-4


def test_kv_cache_matches_oracle(lz, orc, device, suite):
    _, prompt, _, _ = hf_golden("qwen2")
    om = oracle_model(orc, "qwen2", 1, 0, 1)
    with make_model(lz, device, suite, "qwen2", "float16", "f16") as model:
        model.Prefill(prompt)
        for t, tok in enumerate(prompt):
            om.step(int(tok), t)
        kvd = hf_tiny.TINY["qwen2"]["kv_heads"] * hf_tiny.TINY["qwen2"]["head_dim"]
        for layer in range(2):
            k, v = model.read_kv(layer, 0, len(prompt))
            ko, vo = om.read_kv(layer, 0, len(prompt), kvd)
            assert max_diff(k, ko) < 2e-3 * (1 + np.abs(ko).max())
            assert max_diff(v, vo) < 2e-3 * (1 + np.abs(vo).max())
    om.close()


def test_device_greedy_matches_host_greedy_and_reuses_one_graph(lz, device, suite):
    _, prompt, _, _ = hf_golden("llama3")
    with make_model(lz, device, suite, "llama3", "int8", "f16") as model:
        host = model.GenerateGreedy(prompt, 24)
        model.Prefill(prompt)
        first = int(host[0])
        built0, reused0, _ = device.graph_stats()
        dev = model.decode_greedy_device(23)
        built, reused, _ = device.graph_stats()
        assert [first] + dev.tolist() == host
        assert built - built0 <= 1 and reused - reused0 >= 22
        assert model.Position == len(prompt) + 23


@pytest.mark.parametrize("name", ["qwen2", "qwen3"])
def test_fused_and_reference_sequence_agree(lz, device, suite, name):
    """The fused decoder layer against the one-op-per-reference-call sequence (qwen3: with QK-norm)."""
    _, prompt, _, _ = hf_golden(name)
    outs = []
    for fused in (True, False):
        with make_model(lz, device, suite, name, "int8", "f16") as model:
            model.set_fused(fused)
            outs.append((model.Prefill(prompt), model.Decode(7), model.GenerateGreedy(prompt, 10)))
    assert max_diff(outs[0][0], outs[1][0]) < 1e-3
    assert max_diff(outs[0][1], outs[1][1]) < 1e-3
    assert outs[0][2] == outs[1][2]


def test_unrecorded_probe_mode_matches(lz, device, suite):
    _, prompt, _, _ = hf_golden("llama3")
    with make_model(lz, device, suite, "llama3", "float16", "f16") as model:
        a = model.Prefill(prompt)
        model.set_recording(False)
        b = model.Prefill(prompt)
    assert max_diff(a, b) < 1e-5


def test_float16_rejects_out_of_range_values(lz, device, suite):
    cfg = hf_tiny.TINY["llama3"]
    with lz.LlmModel(device, suite, lz.model_config(**hf_tiny.model_config_kwargs(cfg)), 64, "float16") as model:
        bad = np.zeros((cfg["heads"] * cfg["head_dim"], cfg["hidden"]), np.float32)
        bad[0, 0] = 70000.0
        with pytest.raises(lz.InvalidDataException):
            model.set_tensor("model.layers.0.self_attn.q_proj.weight", bad)
        with pytest.raises(lz.InvalidDataException):
            model.set_tensor("model.layers.9.mlp.up_proj.weight", bad)


def test_decode_past_cache_end_is_rejected(lz, device, suite):
    cfg = hf_tiny.TINY["llama3"]
    with lz.LlmModel(device, suite, lz.model_config(**hf_tiny.model_config_kwargs(cfg)), 4, "float16") as model:
        model.init_synthetic(3)
        model.Prefill(np.array([1, 2, 3], np.int32))
        model.Decode(4)
        with pytest.raises(lz.InvalidOperationException):
            model.Decode(5)
        with pytest.raises(lz.ArgumentOutOfRangeException):
            model.ComputeLogits(cfg["vocab"], 0)


# ----------------------------------------------------------------------------------------------
# BASELINE configurations at full width
# ----------------------------------------------------------------------------------------------

QWEN05B = dict(hidden_size=896, intermediate_size=4864, num_layers=24, num_attention_heads=14, num_key_value_heads=2,
               head_dim=64, vocab_size=151936, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
               tie_word_embeddings=1, attention_bias=1)
ORC05B = dict(hidden=896, inter=4864, layers=24, heads=14, kv_heads=2, head_dim=64, vocab=151936, max_pos=32768,
              eps=1e-6, theta=1e6, tie=1, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
              rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0)


def _greedy_oracle(om, prompt, steps):
    lg = None
    for t, tok in enumerate(prompt):
        lg = om.step(int(tok), t, want_logits=(t == len(prompt) - 1))
    out, pos, margins = [], len(prompt), []
    for _ in range(steps):
        top2 = np.partition(lg, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        nxt = int(np.argmax(lg))
        out.append(nxt)
        lg = om.step(nxt, pos)
        pos += 1
    return out, margins


@pytest.mark.parametrize("ksplit", [1, 0])
def test_int8_blocked_gate_up_prefill_and_decode_against_oracle(lz, orc, device, suite, ksplit):
    """Int8 per-row weights at hidden 1024 / inter 2048: every projection, [gate; up] included, is stored in
    the blocked layout (few row tiles), so the prompt runs the tcgen05 GEMM's SwiGLU epilogue over blocked
    weights and the decode steps the k-split GEMV with gate / up tiles paired (ksplit 1) or the
    register-streamed GEMV (ksplit 0). Logits of the prompt and of each decode step against the oracle."""
    cfgd = dict(hidden_size=1024, intermediate_size=2048, num_layers=2, num_attention_heads=8, num_key_value_heads=2,
                head_dim=128, vocab_size=4096, max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6,
                attention_bias=1, q8_group=0)
    orcd = dict(hidden=1024, inter=2048, layers=2, heads=8, kv_heads=2, head_dim=128, vocab=4096, max_pos=4096,
                eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
                rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0,
                wdtype=orc.I8, group=0, kv_dtype=orc.F16)
    prompt = np.random.default_rng(7).integers(0, 4096, 40).astype(np.int32)
    lib = lz.load_library()
    lib.l0b_set_gemv_ksplit(ksplit)
    try:
        with lz.LlmModel(device, suite, lz.model_config(kv_dtype=lz.F16, **cfgd), 64, "int8") as model:
            model.init_synthetic(3, 0.02, 2e-4, 1e-3)  # int8 weights of std ~0.04: a well-conditioned decoder
            got = [model.Prefill(prompt)]
            toks = [int(np.argmax(got[0]))]
            for _ in range(4):
                got.append(model.Decode(toks[-1]))
                toks.append(int(np.argmax(got[-1])))
    finally:
        lib.l0b_set_gemv_ksplit(1)
    om = orc.OracleModel(orcd, 64)
    om.init_synthetic(3, 0.02, 2e-4, 1e-3)
    want = None
    for t, tok in enumerate(prompt):
        want = om.step(int(tok), t, want_logits=(t == len(prompt) - 1))
    wants = [want]
    for i, tok in enumerate(toks[:-1]):
        wants.append(om.step(tok, len(prompt) + i))
    om.close()
    for i, (g, w) in enumerate(zip(got, wants)):
        err = np.abs(g.astype(np.float64) - w)
        assert np.all(err <= 1e-2 + 1e-2 * np.abs(w)), f"step {i}: max err {err.max():.3e}"


def test_config1_qwen05b_fp16_greedy_64_steps(lz, orc, device, suite):
    """Config 1: Qwen2.5-0.5B shape, fp16 weights N(0, 0.02) seed 1, 128-token prompt, greedy decode."""
    steps = 64
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 151936, 128).astype(np.int32)
    mc = lz.model_config(kv_dtype=lz.F16, **QWEN05B)
    with lz.LlmModel(device, suite, mc, 256, "float16") as model:
        model.init_synthetic(1, 0.02)
        got = model.GenerateGreedy(prompt, steps)
    om = orc.OracleModel(dict(ORC05B, wdtype=orc.F16, group=0, kv_dtype=orc.F16), 256)
    om.init_synthetic(1, 0.02)
    want, margins = _greedy_oracle(om, prompt, steps)
    om.close()
    # Token-exact, except where the oracle's top-2 logits are closer than the fp16 tolerance.
    for i, (g, w) in enumerate(zip(got, want)):
        if g != w:
            assert margins[i] < 1e-2, f"step {i}: {g} != {w} with margin {margins[i]}"
            break


@pytest.mark.parametrize("blocked_path", ["ksplit", "register", "bulk"])
def test_config2_qwen7b_int8_shape_two_layers(lz, orc, device, suite, blocked_path):
    """Config 2 widths (hidden 3584, 28/4 heads, inter 18944, vocab 152064), int8 per-channel weights with
    fp16 scales U[1e-3, 2e-2], fp16 KV; two layers so the oracle finishes in seconds. The decode steps run
    the blocked projections (q/k/v, o_proj: 7 blocks per row; down: 37) on the k-split GEMV, or with it
    off on the register GEMV (short rows) and the bulk GEMV (down), or on the bulk GEMV for all three."""
    lib = lz.load_library()
    lib.l0b_set_gemv_ksplit(1 if blocked_path == "ksplit" else 0)
    lib.l0b_set_gemv_bulk_short_rows(1 if blocked_path == "bulk" else 0)
    try:
        _config2_two_layers(lz, orc, device, suite)
    finally:
        lib.l0b_set_gemv_ksplit(1)
        lib.l0b_set_gemv_bulk_short_rows(0)


def _config2_two_layers(lz, orc, device, suite):
    cfgd = dict(hidden_size=3584, intermediate_size=18944, num_layers=2, num_attention_heads=28,
                num_key_value_heads=4, head_dim=128, vocab_size=152064, max_position_embeddings=32768,
                rms_norm_eps=1e-6, rope_theta=1e6, attention_bias=1, q8_group=0)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, 152064, 16).astype(np.int32)
    with lz.LlmModel(device, suite, lz.model_config(kv_dtype=lz.F16, **cfgd), 64, "int8") as model:
        model.init_synthetic(2, 0.02, 1e-3, 2e-2)
        logits = model.Prefill(prompt)
        toks = model.GenerateGreedy(prompt, 8)
    om = orc.OracleModel(dict(hidden=3584, inter=18944, layers=2, heads=28, kv_heads=4, head_dim=128, vocab=152064,
                              max_pos=32768, eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0,
                              rope_factor=1.0, rope_original_max=0, rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0,
                              rope_beta_slow=1.0, rope_attention=0.0, wdtype=orc.I8, group=0, kv_dtype=orc.F16), 64)
    om.init_synthetic(2, 0.02, 1e-3, 2e-2)
    want_toks, margins = _greedy_oracle(om, prompt, 8)
    om.close()
    om2 = orc.OracleModel(dict(hidden=3584, inter=18944, layers=2, heads=28, kv_heads=4, head_dim=128, vocab=152064,
                               max_pos=32768, eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0,
                               rope_factor=1.0, rope_original_max=0, rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0,
                               rope_beta_slow=1.0, rope_attention=0.0, wdtype=orc.I8, group=0, kv_dtype=orc.F16), 64)
    om2.init_synthetic(2, 0.02, 1e-3, 2e-2)
    want = None
    for t, tok in enumerate(prompt):
        want = om2.step(int(tok), t, want_logits=(t == len(prompt) - 1))
    om2.close()
    assert max_diff(logits, want) < 1e-2 + 1e-2 * float(np.abs(want).max())
    for i, (g, w) in enumerate(zip(toks, want_toks)):
        if g != w:
            assert margins[i] < 1e-2 * max(1.0, float(np.abs(want).max())), f"step {i}"
            break


# ----------------------------------------------------------------------------------------------
# Per-stage parity (the Probe stages of LlmDecoderLayer, T/Qwen25LayerGoldenTests.cs method) and the
# uploaded weight storage
# ----------------------------------------------------------------------------------------------

@pytest.mark.parametrize("name,precision,wdtype,kv", [("llama3", "float32", 0, "f32"), ("qwen2", "float16", 1, "f16"),
                                                      ("qwen3", "float32", 0, "f32"), ("qwen2", "int8", 3, "f16")])
def test_probe_stages_match_oracle(lz, orc, device, suite, name, precision, wdtype, kv):
    _, prompt, _, _ = hf_golden(name)
    kvo = {"f32": 0, "f16": 1, "bf16": 2}[kv]
    om = oracle_model(orc, name, wdtype, 0, kvo)
    got, want = [], []
    with make_model(lz, device, suite, name, precision, kv) as model:
        model.Probe = lambda layer, stage, v: got.append((layer, stage, v))
        om.set_probe(lambda layer, stage, v: want.append((layer, stage, v)))
        for t, tok in enumerate(prompt[:3]):
            model.ComputeLogits(int(tok), t)
            om.step(int(tok), t)
    om.close()
    assert [g[:2] for g in got] == [w[:2] for w in want]
    for (layer, stage, a), (_, _, b) in zip(got, want):
        err = max_diff(a, b)
        assert err <= 1e-3 + 1e-3 * float(np.abs(b).max()), f"layer {layer} stage {stage}: max diff {err}"


@pytest.mark.parametrize("precision", ["float32", "float16", "bfloat16", "int8"])
def test_uploaded_weights_match_hf_tensors(lz, device, suite, precision):
    import torch

    name = "llama3"
    cfg = hf_tiny.TINY[name]
    w = hf_tiny.weights(cfg, hf_golden(name)[0])
    with make_model(lz, device, suite, name, precision, "f32", q8_group=32 if precision == "int8" else 0) as model:
        p = "model.layers.1."
        stacks = {0: ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"], 1: ["self_attn.o_proj"],
                  2: ["mlp.gate_proj", "mlp.up_proj"], 3: ["mlp.down_proj"]}
        for kind, names in stacks.items():
            full = np.concatenate([w[p + n + ".weight"] for n in names])
            if precision == "int8":
                q = model.read_weight(1, kind, np.int8, full.size).reshape(full.shape)
                s = model.read_weight(1, kind + 4, np.float16, full.shape[0] * (full.shape[1] // 32))
                qw, sw = lz.q8_quantize_out_in(full, 32)
                np.testing.assert_array_equal(q, qw)
                np.testing.assert_array_equal(s, sw.ravel())
            elif precision == "float32":
                np.testing.assert_array_equal(model.read_weight(1, kind, np.float32, full.size), full.ravel())
            elif precision == "float16":
                np.testing.assert_array_equal(model.read_weight(1, kind, np.float16, full.size),
                                              full.ravel().astype(np.float16))
            else:
                want = torch.from_numpy(full.ravel()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
                np.testing.assert_array_equal(model.read_weight(1, kind, np.uint16, full.size), want)


@pytest.mark.parametrize("precision", ["float32", "float16", "bfloat16", "int8"])
@pytest.mark.parametrize("raw", ["bf16", "f16"])
def test_raw_16bit_upload_matches_f32_upload(lz, device, suite, precision, raw):
    """l0b_model_set_tensor_raw uploads a checkpoint's 16-bit payload and converts it on the device; the
    stored weights and the logits equal those of uploading the same values widened to f32 on the host."""
    import torch

    name = "llama3"
    cfg = hf_tiny.TINY[name]
    w = hf_tiny.weights(cfg, 11)
    tdt = torch.bfloat16 if raw == "bf16" else torch.float16
    bits = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(tdt).view(torch.int16).numpy().view(np.uint16)
            for k, v in w.items()}
    wide = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(tdt).to(torch.float32).numpy()
            for k, v in w.items()}
    prompt = hf_tiny.prompt(cfg, 11)[:6]
    out = []
    for use_raw in (True, False):
        mc = lz.model_config(**hf_tiny.model_config_kwargs(cfg, kv_dtype=lz.F32, q8_group=0))
        with lz.LlmModel(device, suite, mc, 32, precision) as model:
            for k in w:
                if use_raw:
                    model.set_tensor_raw(k, bits[k], lz.BF16 if raw == "bf16" else lz.F16)
                else:
                    model.set_tensor(k, wide[k])
            dt = {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16, "int8": np.int8}[precision]
            n = model.read_weight(0, 2, dt, 2 * cfg["inter"] * cfg["hidden"])
            out.append((model.Prefill(prompt), n))
    np.testing.assert_array_equal(out[0][1], out[1][1])
    np.testing.assert_array_equal(out[0][0], out[1][0])


def test_raw_bf16_outside_half_range_is_rejected_for_float16(lz, device, suite):
    cfg = hf_tiny.TINY["llama3"]
    mc = lz.model_config(**hf_tiny.model_config_kwargs(cfg, kv_dtype=lz.F32, q8_group=0))
    big = np.full((cfg["inter"], cfg["hidden"]), 0x4780, np.uint16)  # bf16 65536
    with lz.LlmModel(device, suite, mc, 8, "float16") as model:
        with pytest.raises(lz.InvalidDataException):
            model.set_tensor_raw("model.layers.0.mlp.up_proj.weight", big, lz.BF16)
