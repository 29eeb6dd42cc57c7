"""Bookkeeping of the continuous-batching engine (l0llm_b200/engine.py) against a fake model on CPU.

The fake keeps per-row token histories and answers greedy steps with a deterministic function of the
history, so a request's tokens depend only on its own prompt: run through the engine (rows shared,
freed rows refilled by moving the last row) they must equal the same request run alone.
"""
from __future__ import annotations

import numpy as np
import pytest

from l0llm_b200.engine import BatchEngine

V = 97


def next_token(hist):
    return (sum((i + 1) * t for i, t in enumerate(hist)) * 31 + len(hist)) % V


class FakeModel:
    def __init__(self, rows, max_seq):
        self.rows = [None] * rows
        self.max_seq = max_seq
        self.forks = 0

    def PrefillSequence(self, seq, prompt_ids, want_logits=True):
        hist = [int(t) for t in prompt_ids]
        tok = next_token(hist)
        self.rows[seq] = hist + [tok]  # history incl. the pending input token
        logits = np.zeros(V, np.float32)
        logits[tok] = 1.0
        return logits

    def decode_greedy_device_batch(self, steps, count):
        out = np.zeros((steps, count), np.int32)
        for s in range(steps):
            for r in range(count):
                h = self.rows[r]
                assert h is not None and len(h) <= self.max_seq, "decoded an empty or full row"
                tok = next_token(h)
                h.append(tok)
                out[s, r] = tok
        return out

    def ForkSequence(self, src, dst, base):
        assert src != dst and base == 0
        self.rows[dst] = list(self.rows[src])
        self.forks += 1


def alone(prompt, max_new, stops, max_seq):
    hist = [int(t) for t in prompt]
    toks = []
    while True:
        tok = next_token(hist)
        toks.append(tok)
        hist.append(tok)
        if len(toks) >= max_new or tok in stops or len(prompt) + len(toks) >= max_seq:
            return toks


@pytest.mark.parametrize("max_batch", [1, 2, 3, 5])
def test_engine_matches_requests_run_alone(max_batch):
    rng = np.random.default_rng(max_batch)
    max_seq = 60
    m = FakeModel(max_batch, max_seq)
    eng = BatchEngine(m, max_batch, max_seq)
    reqs = []
    for i in range(9):
        prompt = rng.integers(0, V, rng.integers(1, 20)).astype(np.int32)
        max_new = int(rng.integers(1, 30))
        stops = {int(rng.integers(0, V))} if i % 3 == 0 else set()
        reqs.append((eng.submit(prompt, max_new, stops), prompt, max_new, stops))
    # Late arrivals join while others run.
    for _ in range(3):
        eng.step()
    prompt = rng.integers(0, V, 50).astype(np.int32)
    reqs.append((eng.submit(prompt, 40), prompt, 40, set()))  # stops at the cache end
    got = eng.run()
    for rid, prompt, max_new, stops in reqs:
        assert got[rid] == alone(prompt, max_new, stops, max_seq), rid
    assert eng.pending == 0 and eng.active == 0
    if max_batch > 1:
        assert m.forks > 0


def test_engine_rejects_bad_requests():
    eng = BatchEngine(FakeModel(2, 16), 2, 16)
    with pytest.raises(ValueError):
        eng.submit([], 4)
    with pytest.raises(ValueError):
        eng.submit([1, 2], 0)
    with pytest.raises(ValueError):
        eng.submit(list(range(16)), 4)
