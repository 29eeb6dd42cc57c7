"""Device sampling (LlmSampler.Sample, src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) against the
CPU oracle: the op on seeded logits with the same uniform draw, and the model's device-resident sampled
decode against the host path (Prefill / Decode logits through the C ABI, sampled by the oracle with the
documented per-position draw)."""
from __future__ import annotations

import numpy as np
import pytest

import hf_tiny

pytestmark = pytest.mark.gpu

CASES = [  # temperature, top_p, top_k, penalty
    (0.7, 0.9, 40, 1.1), (1.0, 1.0, 1024, 1.0), (0.3, 0.5, 5, 1.3), (1.5, 0.95, 200, 1.0), (0.0, 0.9, 40, 1.1),
    (2.0, 0.0, 1000, 0.8), (0.9, 0.999, 1, 1.2), (0.8, 0.2, 700, 1.1),
]


@pytest.mark.parametrize("vocab", [1000, 152064])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sampler_op_matches_oracle(lz, orc, device, suite, vocab, case):
    T, top_p, top_k, pen = CASES[case]
    rng = np.random.default_rng(vocab + 17 * case)
    with lz.SharedBuffer(device, lz.F32, vocab) as lb, lz.SharedBuffer(device, lz.I32, 64) as cb, \
            lz.SharedBuffer(device, lz.I32, 1) as ob:
        for trial in range(5):
            logits = (rng.standard_normal(vocab) * rng.uniform(0.5, 8.0)).astype(np.float32)
            ctx = np.concatenate([rng.integers(0, vocab, 40), np.argsort(logits)[-8:]]).astype(np.int32)
            u = float(rng.random())
            lb.Write(logits)
            cb.Write(ctx)
            suite.Sampler.Execute(device, lb, vocab, cb, ctx.size, T, top_p, top_k, pen, u, ob)
            got = int(ob.ToArray()[0])
            want = orc.sampler(logits, ctx, T, top_p, top_k, pen, u)
            assert got == want, (case, vocab, trial)


def test_sampler_op_usable_vocab_and_ties(lz, orc, device, suite):
    """vocab below the buffer length (the tokenizer's usable ids); exact ties order by index."""
    logits = np.zeros(4096, np.float32)
    logits[[5, 9, 700, 3000]] = 4.0
    logits[4000] = 9.0  # beyond the usable vocab: never chosen
    with lz.SharedBuffer.from_array(device, logits) as lb, lz.SharedBuffer(device, lz.I32, 1) as ob:
        for u in [0.0, 0.3, 0.6, 0.9, 0.999]:
            suite.Sampler.Execute(device, lb, 3500, None, 0, 1.0, 1.0, 3, 1.0, u, ob)
            got = int(ob.ToArray()[0])
            assert got == orc.sampler(logits[:3500], None, 1.0, 1.0, 3, 1.0, u)
            assert got in (5, 9, 700)
        suite.Sampler.Execute(device, lb, 3500, None, 0, 0.0, 1.0, 3, 1.0, 0.5, ob)
        assert int(ob.ToArray()[0]) == 5


def test_sampler_op_rejects_unsupported_top_k(lz, device, suite):
    with lz.SharedBuffer(device, lz.F32, 5000) as lb, lz.SharedBuffer(device, lz.I32, 1) as ob:
        with pytest.raises(lz.NotSupportedException):
            suite.Sampler.Execute(device, lb, 5000, None, 0, 0.7, 0.9, 0, 1.0, 0.5, ob)
        with pytest.raises(lz.NotSupportedException):
            suite.Sampler.Execute(device, lb, 5000, None, 0, 0.7, 0.9, 2000, 1.0, 0.5, ob)


@pytest.mark.parametrize("precision,kv", [("float16", "f16"), ("int8", "f16")])
def test_model_device_sampled_decode_matches_host_path(lz, orc, device, suite, precision, kv):
    from test_gpu_model import make_model

    T, top_p, top_k, pen, seed, steps = 0.9, 0.92, 50, 1.15, 20260, 12
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, hf_tiny.TINY["llama3"]["vocab"], 23).astype(np.int32)
    with make_model(lz, device, suite, "llama3", precision, kv) as m:
        m.Prefill(prompt)
        first = m.sample_logits(T, top_p, top_k, pen, seed, prompt)
        dev = [first] + m.decode_sample_device(steps, T, top_p, top_k, pen, seed).tolist()
        assert m.Position == prompt.size + steps
    with make_model(lz, device, suite, "llama3", precision, kv) as m:
        logits = m.Prefill(prompt)
        ctx = prompt.tolist()
        host = []
        for i in range(steps + 1):
            pos = prompt.size + i  # position of the token being drawn
            tok = orc.sampler(logits, ctx, T, top_p, top_k, pen, orc.sample_uniform(seed, pos))
            host.append(tok)
            ctx.append(tok)
            if i < steps:
                logits = m.Decode(tok)
    assert dev == host
