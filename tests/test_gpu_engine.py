"""The continuous-batching engine (l0llm_b200/engine.py) on a real multi-sequence model: requests that
share the model's KV-cache rows, join late and free rows mid-run (moved with the device-side fork) give
the tokens that single-sequence greedy generation gives for each prompt alone."""
from __future__ import annotations

import numpy as np
import pytest

import hf_tiny
from l0llm_b200.engine import BatchEngine

pytestmark = pytest.mark.gpu


def test_engine_matches_single_sequence_greedy(lz, device, suite):
    from test_gpu_model import make_model

    max_seq, batch = 96, 3
    cfg = hf_tiny.TINY["llama3"]
    rng = np.random.default_rng(12)
    reqs = [(rng.integers(0, cfg["vocab"], int(rng.integers(2, 30))).astype(np.int32), int(rng.integers(1, 20)))
            for _ in range(7)]
    with make_model(lz, device, suite, "llama3", "int8", "f16", max_seq=max_seq) as single:
        want = [list(single.GenerateGreedy(p, n)) for p, n in reqs]
    kw = hf_tiny.model_config_kwargs(cfg, kv_dtype=lz.F16, q8_group=0)
    mc = lz.model_config(max_batch=batch, **kw)
    with lz.LlmModel(device, suite, mc, max_seq, "int8") as model:
        from test_gpu_model import hf_golden

        for k, v in hf_tiny.weights(cfg, hf_golden("llama3")[0]).items():
            model.set_tensor(k, v)
        eng = BatchEngine(model, batch, max_seq)
        ids = [eng.submit(p, n) for p, n in reqs[:5]]
        eng.step()
        eng.step()
        ids += [eng.submit(p, n) for p, n in reqs[5:]]  # late arrivals
        got = eng.run()
    for i, rid in enumerate(ids):
        assert got[rid] == want[i], f"request {i}"
