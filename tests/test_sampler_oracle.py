"""The CPU oracle of LlmSampler.Sample (src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) against a
second, line-by-line Python restatement of the same C# method.

The reference ships no tests or golden vectors for the sampler, so its parity is pinned here: the C
restatement (the checker of the device sampler) must pick the same token as this independent
restatement for every case, including duplicate context ids, negative logits under the penalty, top-k
beyond the vocabulary, disabled top-k / top-p and greedy temperatures.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle.oracle as orc


def ref_sample(logits, temperature, top_p, top_k, penalty, context, u):
    """LlmSampler.Sample with the draw u in place of Random.NextDouble(); float steps in float32, the
    probabilities in double, the sort descending by probability with ties by index."""
    c = np.array(logits, np.float32)
    V = c.size
    if penalty != 1.0 and context:
        pen = np.float32(penalty)
        for t in set(context):
            if 0 <= t < V:
                l = c[t]
                c[t] = np.float32(l / pen) if l >= 0.0 else np.float32(l * pen)
    if temperature <= 0.0:
        best = 0
        for i in range(1, V):
            if c[i] > c[best]:
                best = i
        return best
    c = (c / np.float32(temperature)).astype(np.float32)
    mx = c.max()
    probs = [math.exp(float(np.float32(ci - mx))) for ci in c]
    s = 0.0
    for p in probs:
        s += p
    probs = [p / s for p in probs]
    order = sorted(range(V), key=lambda i: (-probs[i], i))
    if 0 < top_k < len(order):
        order = order[:top_k]
    tp = float(np.float32(top_p))
    if 0.0 < tp < 1.0:
        cum, keep = 0.0, 0
        for i in order:
            cum += probs[i]
            keep += 1
            if cum >= tp:
                break
        order = order[:keep]
    fs = 0.0
    for i in order:
        fs += probs[i]
    if fs <= 0.0:
        return order[0]
    r = u * fs
    cur = 0.0
    for i in order:
        cur += probs[i]
        if r <= cur:
            return i
    return order[-1]


CASES = [  # temperature, top_p, top_k, penalty
    (0.7, 0.9, 40, 1.1), (1.0, 1.0, 0, 1.0), (0.3, 0.5, 5, 1.3), (1.5, 0.95, 200, 1.0), (0.0, 0.9, 40, 1.1),
    (-1.0, 0.9, 40, 1.0), (2.0, 0.0, 0, 0.8), (0.9, 0.999, 1, 1.2), (0.8, 0.2, 5000, 1.1),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("vocab", [7, 300, 2000])
def test_oracle_sampler_matches_restatement(case, vocab):
    T, top_p, top_k, pen = CASES[case]
    rng = np.random.default_rng(vocab * 31 + case)
    for trial in range(6):
        logits = (rng.standard_normal(vocab) * rng.uniform(0.5, 6.0)).astype(np.float32)
        ctx = rng.integers(0, vocab, rng.integers(0, 12)).tolist() + [int(np.argmax(logits))] * (trial % 2)
        u = float(rng.random())
        want = ref_sample(logits, T, top_p, top_k, pen, ctx, u)
        got = orc.sampler(logits, ctx, T, top_p, top_k, pen, u)
        assert got == want, (case, vocab, trial)


def test_oracle_sampler_known_answers():
    # Greedy takes the first maximum; the penalty divides positive logits and multiplies negative ones.
    lg = np.array([1.0, 3.0, 3.0, -2.0], np.float32)
    assert orc.sampler(lg, None, 0.0, 0.9, 40, 1.0, 0.5) == 1
    assert orc.sampler(lg, [1], 0.0, 0.9, 40, 2.0, 0.5) == 2
    assert orc.sampler(np.array([-1.0, -1.5], np.float32), [0], 0.0, 1.0, 0, 2.0, 0.0) == 1
    # With T = 1 the probabilities of [ln 1, ln 3] are 0.25 / 0.75, sorted as (1, 0): u < 0.75 picks 1.
    lg = np.log(np.array([1.0, 3.0], np.float32)).astype(np.float32)
    assert orc.sampler(lg, None, 1.0, 1.0, 0, 1.0, 0.70) == 1
    assert orc.sampler(lg, None, 1.0, 1.0, 0, 1.0, 0.80) == 0
    # top_p = 0.5 keeps only the 0.75 token; top_k = 1 likewise.
    assert orc.sampler(lg, None, 1.0, 0.5, 0, 1.0, 0.99) == 1
    assert orc.sampler(lg, None, 1.0, 1.0, 1, 1.0, 0.99) == 1


def test_sample_uniform_is_the_documented_hash():
    def mix(x):
        m = (1 << 64) - 1
        x = (x + 0x9E3779B97F4A7C15) & m
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
        return x ^ (x >> 31)

    for seed, p in [(0, 0), (7, 3), (123456789, 4095)]:
        h = mix(seed ^ (((p + 1) * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)))
        assert orc.sample_uniform(seed, p) == (h >> 11) / float(1 << 53)
