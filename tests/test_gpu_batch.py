"""Batched decoding of independent sequences (cfg.max_batch > 1) against the same sequences decoded alone.

Each sequence owns one KV-cache row. Prefill fills row `seq`; a batched step decodes rows 0..count-1 at
their own positions. The reference has no multi-sequence decode (its engine serialises requests), so
the check is consistency: sequence b decoded in a batch must give the logits and greedy tokens it gets
when decoded alone by a single-sequence model with the same weights.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=256, intermediate_size=640, num_layers=2, num_attention_heads=8, num_key_value_heads=2,
           head_dim=64, vocab_size=1000, max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6,
           attention_bias=1, q8_group=0)


def _model(lz, device, suite, batch, precision):
    cfg = lz.model_config(kv_dtype=lz.F16, max_batch=batch, **CFG)
    m = lz.LlmModel(device, suite, cfg, 96, precision)
    m.init_synthetic(7, 0.02, 1e-3, 2e-2) if precision == "int8" else m.init_synthetic(7, 0.05, 0.0, 0.0)
    return m


def _prompts(n):
    rng = np.random.default_rng(11)
    return [rng.integers(0, CFG["vocab_size"], 3 + (7 * i) % 61).astype(np.int32) for i in range(n)]


@pytest.mark.parametrize("precision", ["int8", "float16"])
@pytest.mark.parametrize("batch", [5, 16])
def test_batched_logits_match_single_sequences(lz, device, suite, precision, batch):
    prompts = _prompts(batch)
    with _model(lz, device, suite, batch, precision) as mb:
        first = [mb.PrefillSequence(s, p) for s, p in enumerate(prompts)]
        assert [mb.SequencePosition(s) for s in range(batch)] == [len(p) for p in prompts]
        toks = np.array([int(np.argmax(f)) for f in first], np.int32)
        pos = np.array([len(p) for p in prompts], np.int32)
        got = mb.DecodeBatch(toks, pos)
    with _model(lz, device, suite, 1, precision) as ms:
        for s, p in enumerate(prompts):
            want0 = ms.Prefill(p)
            np.testing.assert_allclose(first[s], want0, rtol=1e-4, atol=1e-4 * np.abs(want0).max())
            want = ms.Decode(int(toks[s]))
            scale = np.abs(want).max()
            err = np.abs(got[s] - want).max()
            assert err <= 2e-3 * scale, f"sequence {s}: max err {err} (scale {scale})"


@pytest.mark.parametrize("batch", [4, 12])
def test_batched_device_greedy_matches_single(lz, device, suite, batch):
    """Batch 12 runs its projections and the LM head's argmax on the tensor-core GEMM (8+ rows)."""
    steps = 6
    prompts = _prompts(batch)
    with _model(lz, device, suite, batch, "int8") as mb:
        for s, p in enumerate(prompts):
            mb.PrefillSequence(s, p, want_logits=False)
        got = mb.decode_greedy_device_batch(steps, batch)
        assert [mb.SequencePosition(s) for s in range(batch)] == [len(p) + steps for p in prompts]
    with _model(lz, device, suite, 1, "int8") as ms:
        for s, p in enumerate(prompts):
            ms.Prefill(p)
            want = ms.decode_greedy_device(steps)
            np.testing.assert_array_equal(got[:, s], want)


def test_batched_rejects_out_of_range(lz, device, suite):
    with _model(lz, device, suite, 2, "int8") as mb:
        with pytest.raises(lz.ArgumentOutOfRangeException):
            mb.PrefillSequence(2, np.array([1, 2], np.int32))
        with pytest.raises(lz.ArgumentOutOfRangeException):
            mb.DecodeBatch(np.array([1, 2, 3], np.int32), np.array([0, 0, 0], np.int32))


def test_fork_sequence_on_device(lz, device, suite):
    """ForkSequence copies a sequence's KV rows and its next-token state device to device (the
    reference's CaptureState / RestoreState go through host arrays): forked rows then decode exactly as
    the source, both through DecodeBatch and the device-resident greedy loop."""
    a = _prompts(3)[2]
    b = a.copy()
    b[5:] = (b[5:] + 1) % CFG["vocab_size"]  # shares a's first 5 tokens only
    with _model(lz, device, suite, 3, "int8") as mb:
        mb.PrefillSequence(0, a, want_logits=False)
        mb.PrefillSequence(1, b, want_logits=False)
        mb.ForkSequence(0, 1, 5)  # the first 5 rows are shared: only the tail is copied
        mb.ForkSequence(0, 2, 0)
        assert [mb.SequencePosition(s) for s in range(3)] == [len(a)] * 3
        got = mb.DecodeBatch(np.full(3, 7, np.int32), np.full(3, len(a), np.int32))
        np.testing.assert_array_equal(got[0], got[1])
        np.testing.assert_array_equal(got[0], got[2])
        toks = mb.decode_greedy_device_batch(4, 3)
        np.testing.assert_array_equal(toks[:, 0], toks[:, 1])
        np.testing.assert_array_equal(toks[:, 0], toks[:, 2])
        with pytest.raises(lz.ArgumentException):
            mb.ForkSequence(1, 1, 0)
        with pytest.raises(lz.ArgumentOutOfRangeException):
            mb.ForkSequence(0, 3, 0)


def test_sequence0_length_is_one_value_across_single_and_batched_calls(lz, device, suite):
    """Decode on sequence 0 advances the length the batched calls check: a batched device decode that
    would run past the cache after single-sequence decodes is refused, not written past the rows."""
    prompts = _prompts(2)
    with _model(lz, device, suite, 2, "int8") as mb:
        mb.PrefillSequence(1, prompts[1], want_logits=False)
        mb.Prefill(np.arange(80, dtype=np.int32))
        for t in range(10):
            mb.Decode(t)
        assert mb.Position == 90 and mb.SequencePosition(0) == 90
        with pytest.raises(lz.InvalidOperationException):
            mb.decode_greedy_device_batch(7, 1)  # 90 + 7 > 96 rows
        toks = mb.decode_greedy_device_batch(6, 1)
        assert toks.shape == (6, 1) and mb.Position == 96 and mb.SequencePosition(0) == 96


def test_single_sequence_step_keeps_other_rows_device_state(lz, device, suite):
    """A one-token step of sequence 0 writes only row 0's token and position: rows prefilled before it
    still continue from their own device state in a later batched greedy decode."""
    steps = 5
    prompts = _prompts(3)
    with _model(lz, device, suite, 3, "int8") as mb:
        mb.PrefillSequence(1, prompts[1], want_logits=False)
        mb.PrefillSequence(2, prompts[2], want_logits=False)
        mb.Prefill(np.array([5], np.int32))  # a one-token prompt of sequence 0 runs as a Step
        got = mb.decode_greedy_device_batch(steps, 3)
    with _model(lz, device, suite, 1, "int8") as ms:
        for s, p in ((0, np.array([5], np.int32)), (1, prompts[1]), (2, prompts[2])):
            ms.Prefill(p)
            np.testing.assert_array_equal(got[:, s], ms.decode_greedy_device(steps))
