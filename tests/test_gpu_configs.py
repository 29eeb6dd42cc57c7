"""BASELINE configurations at full size against the CPU oracle (the method of
T/Qwen25GenerationGoldenTests.cs:100-178 and T/Qwen25PrefillTests.cs:41-75 on seeded synthetic weights).

logits within max-abs 1e-2 and relative 1e-2 of the oracle, elementwise
(|got - want| <= 1e-2 + 1e-2 * |want|), and greedy token ids equal for 64 steps. Logits are compared
teacher-forced (both sides are fed the oracle's greedy tokens), so every step is checked even where a
near-tie could send the two free-running greedy sequences apart; the free-running device greedy path
(the benchmarked one) must then reproduce the oracle's tokens, a difference being allowed only at a
step whose top-2 oracle logits are closer than the logit tolerance allows to order.

The oracle ingests long prompts with its fp32-accumulate GEMM (relative error ~1e-6 per projection)
and decodes single sequences in double accumulation.

Config 1 (fp16 weights N(0, 0.02)) is well conditioned: the oracle's own fp32 build agrees with its
double build to ~1e-4 on logits of ~3, so every logit is held to the elementwise bar. Config 2's
synthetic int8 weights (codes uniform in +-127 times scales up to 0.02: weights of std ~0.8) are not:
activations reach ~1e7 and attention scores ~1e3, so attention is nearly one-hot and a 1e-7 relative
perturbation of any projection grows, through near-ties between attended positions, to ~1e-3 of the
logit range (tests/test_cpu_oracle.py::test_config2_weights_amplify_rounding shows the oracle's fp32
and double builds failing the elementwise bar against each other; over 64 decode steps they differ by
3.4e-4 of the range at the median and 4.3e-3 at worst after a 128-token prompt, and by 1.9e-4 at the
median but 7.2e-2 at worst after a 32-token prompt, where fewer attended positions make a flipped
near-tie weigh more). A full-depth config-2 comparison therefore holds: every greedy token
(teacher-forced argmax and the free-running device decode) equal to the oracle's unless the oracle's
top-2 margin is inside the step's measured error; the per-step maximum error at a median of <= 2e-3 of
the logit range; and no step above 0.15 of it (twice the oracle's own worst spread).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2

CFG2 = dict(hidden_size=3584, intermediate_size=18944, num_layers=28, num_attention_heads=28, num_key_value_heads=4,
            head_dim=128, vocab_size=152064, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
            attention_bias=1, q8_group=0)
ORC2 = dict(hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128, vocab=152064, max_pos=32768,
            eps=1e-6, theta=1e6, tie=0, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
            rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0)


def assert_logits(got: np.ndarray, want: np.ndarray, what: str) -> None:
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} logits outside max-abs {ATOL} + rel {RTOL}; "
                           f"worst abs err {err.max():.3e} at |want| {float(np.abs(want).ravel()[err.argmax()]):.3e}")


def assert_logits_top(got: np.ndarray, want: np.ndarray, what: str, top: int = 64) -> None:
    """The elementwise bar on the oracle's `top` largest logits of each row, 1e-2 of the logit range on
    every logit."""
    got2, want2 = np.atleast_2d(got), np.atleast_2d(want)
    for r in range(want2.shape[0]):
        idx = np.argpartition(want2[r], -top)[-top:]
        assert_logits(got2[r, idx], want2[r, idx], f"{what} (row {r}, top {top})")
        err = float(np.abs(got2[r].astype(np.float64) - want2[r]).max())
        scale = float(np.abs(want2[r]).max())
        assert err <= 1e-2 * scale, f"{what} (row {r}): max abs err {err:.3e} > 1e-2 of the logit range {scale:.3e}"


def tie_margin(logits: np.ndarray) -> tuple[float, float]:
    """(top1 - top2, the gap under which the tolerance cannot order the two)."""
    top2 = np.partition(logits, -2)[-2:]
    return float(top2[1] - top2[0]), 2 * (ATOL + RTOL * float(np.abs(top2[1])))


def check_free_running(got_tokens, want_tokens, want_logits, what):
    """Token ids equal until a step whose oracle top-2 is a near-tie (after which contexts differ)."""
    for i, (g, w) in enumerate(zip(got_tokens, want_tokens)):
        if g != w:
            margin, allowed = tie_margin(want_logits[i])
            assert margin < allowed, f"{what}: step {i} token {g} != {w}, oracle margin {margin:.3e} >= {allowed:.3e}"
            return i
    return len(want_tokens)


QWEN05B = dict(hidden_size=896, intermediate_size=4864, num_layers=24, num_attention_heads=14, num_key_value_heads=2,
               head_dim=64, vocab_size=151936, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6,
               tie_word_embeddings=1, attention_bias=1)
ORC05B = dict(hidden=896, inter=4864, layers=24, heads=14, kv_heads=2, head_dim=64, vocab=151936, max_pos=32768,
              eps=1e-6, theta=1e6, tie=1, bias=1, qk_norm=0, rope_type=0, rope_factor=1.0, rope_original_max=0,
              rope_low=1.0, rope_high=4.0, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_attention=0.0)


def test_config1_full_size_logits_every_step(lz, orc, device, suite):
    """Config 1 exactly (Qwen2.5-0.5B shape, fp16 N(0, 0.02) seed 1, 128-token prompt): the prompt's
    logits and 64 teacher-forced decode steps, every logit within max-abs 1e-2 + rel 1e-2, then the
    device greedy decode against the oracle's greedy tokens."""
    steps, plen = 64, 128
    prompt = np.random.default_rng(1).integers(0, 151936, plen).astype(np.int32)
    om = orc.OracleModel(dict(ORC05B, wdtype=orc.F16, group=0, kv_dtype=orc.F16), plen + steps + 1)
    om.init_synthetic(1, 0.02)
    want = [om.prefill(prompt)]
    toks = [int(np.argmax(want[0]))]
    for i in range(steps):
        want.append(om.step(toks[-1], plen + i))
        toks.append(int(np.argmax(want[-1])))
    om.close()
    with lz.LlmModel(device, suite, lz.model_config(kv_dtype=lz.F16, **QWEN05B), plen + steps + 1, "float16") as model:
        model.init_synthetic(1, 0.02)
        assert_logits(model.Prefill(prompt), want[0], "prefill")
        for i in range(steps):
            assert_logits(model.Decode(toks[i]), want[i + 1], f"decode step {i}")
        first = int(np.argmax(model.Prefill(prompt)))
        dev = [first] + model.decode_greedy_device(steps).tolist()
    check_free_running(dev, toks, want, "device greedy")


def config2_check(got_rows, want_rows, tf_tokens, dev_tokens, oracle_tokens, what):
    """The full-depth config-2 criteria above, over rows of (GPU logits, oracle logits) per step."""
    rel, first_mismatch = [], None
    for i, (g, w) in enumerate(zip(got_rows, want_rows)):
        err = np.abs(g.astype(np.float64) - w)
        scale = float(np.abs(w).max())
        rel.append(float(err.max()) / scale)
        top = np.argpartition(w, -64)[-64:]
        margin, _ = tie_margin(w)
        if tf_tokens[i] != oracle_tokens[i]:
            assert margin < 2 * float(err[top].max()), (
                f"{what} step {i}: argmax {tf_tokens[i]} != {oracle_tokens[i]} with margin {margin:.3e} "
                f"outside the step's error {float(err[top].max()):.3e}")
        if first_mismatch is None and dev_tokens[i] != oracle_tokens[i]:
            first_mismatch = i
            assert margin < 2 * float(err[top].max()), (
                f"{what} device greedy step {i}: {dev_tokens[i]} != {oracle_tokens[i]} with margin {margin:.3e}")
    med, worst = float(np.median(rel)), max(rel)
    assert med <= 2e-3, f"{what}: median per-step max error {med:.3e} of the logit range (> 2e-3)"
    assert worst <= 0.15, f"{what}: a step's max error reached {worst:.3e} of the logit range (> 0.15)"
    return med, worst, first_mismatch


def test_config2_full_depth_bs1_512_prompt_64_greedy_steps(lz, orc, device, suite):
    """Config 2 exactly: 28 layers, int8 per-channel weights (fp16 scales U[1e-3, 2e-2]), fp16 KV, a
    512-token uniform-random prompt, 64 greedy decode steps at batch 1 (teacher-forced logits, then the
    free-running device greedy decode that the benchmark times)."""
    steps, plen = 64, 512
    prompt = np.random.default_rng(2).integers(0, 152064, plen).astype(np.int32)
    om = orc.OracleModel(dict(ORC2, wdtype=orc.I8, group=0, kv_dtype=orc.F16), plen + steps + 1)
    om.init_synthetic(2, 0.02, 1e-3, 2e-2)
    om.set_fast(True)
    want = [om.prefill(prompt)]
    om.set_fast(False)
    toks = [int(np.argmax(want[0]))]
    for i in range(steps):
        want.append(om.step(toks[-1], plen + i))
        toks.append(int(np.argmax(want[-1])))
    om.close()
    with lz.LlmModel(device, suite, lz.model_config(kv_dtype=lz.F16, **CFG2), plen + steps + 1, "int8") as model:
        model.init_synthetic(2, 0.02, 1e-3, 2e-2)
        got = [model.Prefill(prompt)]
        for i in range(steps):
            got.append(model.Decode(toks[i]))
        first = int(np.argmax(model.Prefill(prompt)))
        dev = [first] + model.decode_greedy_device(steps).tolist()
    tf = [int(np.argmax(g)) for g in got]
    med, worst, mismatch = config2_check(got, want, tf, dev, toks, "config 2 bs1")
    print(f"config 2 bs1: median {med:.2e}, worst {worst:.2e} of the logit range; "
          f"device greedy tokens equal for {steps if mismatch is None else mismatch} of {steps} steps")


def test_config2_full_depth_bs16_against_oracle(lz, orc, device, suite):
    """Config 2 at batch 16 on the batched path (tcgen05 kind::i8 GEMM for the projections): 16
    sequences with their own 32-token prompts, 64 batched decode steps teacher-forced with the oracle's
    tokens (every sequence's logits against the oracle's batched forward), then the free-running
    device-resident batched greedy decode against the oracle's tokens."""
    bs, plen, steps = 16, 32, 64
    rng = np.random.default_rng(22)
    prompts = rng.integers(0, 152064, (bs, plen)).astype(np.int32)
    om = orc.OracleModel(dict(ORC2, wdtype=orc.I8, group=0, kv_dtype=orc.F16), plen + steps + 1, bs)
    om.init_synthetic(2, 0.02, 1e-3, 2e-2)
    om.set_fast(True)
    mc = lz.model_config(kv_dtype=lz.F16, max_batch=bs, **CFG2)
    got_rows, want_rows, tf_rows = [[] for _ in range(bs)], [[] for _ in range(bs)], [[] for _ in range(bs)]
    with lz.LlmModel(device, suite, mc, plen + steps + 1, "int8") as model:
        model.init_synthetic(2, 0.02, 1e-3, 2e-2)
        toks = []
        first = []
        for s in range(bs):
            w = om.prefill(prompts[s], seq=s)
            g = model.PrefillSequence(s, prompts[s])
            got_rows[s].append(g)
            want_rows[s].append(w)
            first.append(int(np.argmax(w)))
        toks.append(np.array(first, np.int32))
        for i in range(steps):
            pos = np.full(bs, plen + i, np.int32)
            want = om.forward(toks[-1], pos, np.arange(bs, dtype=np.int32))
            got = model.DecodeBatch(toks[-1], pos)
            for s in range(bs):
                got_rows[s].append(got[s])
                want_rows[s].append(want[s])
            toks.append(np.argmax(want, axis=1).astype(np.int32))
        for s in range(bs):
            model.PrefillSequence(s, prompts[s], want_logits=False)
        dev = model.decode_greedy_device_batch(steps, bs)
    om.close()
    for s in range(bs):
        oracle_s = [int(t[s]) for t in toks]
        dev_s = [int(np.argmax(got_rows[s][0]))] + dev[:, s].tolist()
        tf_s = [int(np.argmax(g)) for g in got_rows[s]]
        config2_check(got_rows[s], want_rows[s], tf_s, dev_s, oracle_s, f"config 2 bs16 sequence {s}")
