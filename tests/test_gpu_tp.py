"""Tensor parallelism over 2 GPUs (NCCL) against the same model on one GPU.

Two ranks, one process each, build the model with tp_size = 2: q/k/v, gate/up and lm_head column-split,
o_proj/down row-split with their partial sums all-reduced before the residual add, attention head-split,
the vocab-sharded argmax keys max-reduced. Rank 0 compares the prefill logits and the device greedy
tokens with a tp_size = 1 model of the same synthetic weights on its own GPU.
"""
from __future__ import annotations

import multiprocessing as mp

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden_size=512, intermediate_size=1024, num_layers=2, num_attention_heads=8, num_key_value_heads=2,
           head_dim=64, vocab_size=2048, max_position_embeddings=4096, rms_norm_eps=1e-5, rope_theta=5e5,
           attention_bias=0, q8_group=0)
STEPS = 6


def _rank(rank, world, idq, precision, q):
    try:
        from l0llm_b200 import levelzero as lz

        # Rank 0 makes the id, so every rank bootstraps with the same NCCL build.
        if rank == 0:
            uid = lz.Communicator.unique_id()
            for _ in range(world - 1):
                idq.put(uid)
        else:
            uid = idq.get(timeout=60)
        import sys

        def note(msg):  # shown with the test's captured output if it fails
            print(f"rank {rank}: {msg}", file=sys.stderr, flush=True)

        dev = lz.ComputeDevice(rank)
        suite = lz.LlmKernelSuite.Create(dev)
        note("device ready")
        prompt = np.random.default_rng(4).integers(0, CFG["vocab_size"], 20).astype(np.int32)
        out = {}
        with lz.Communicator(dev, uid, world, rank) as comm:
            note("communicator ready")
            cfg = lz.model_config(kv_dtype=lz.F16, tp_size=world, tp_rank=rank, **CFG)
            with lz.LlmModel(dev, suite, cfg, 64, precision, comm=comm) as m:
                m.init_synthetic(4, 0.05, 1e-3, 2e-2)
                out["logits"] = m.Prefill(prompt)
                note("prefill done")
                out["tokens"] = m.decode_greedy_device(STEPS)
                note("decode done")
        if rank == 0:
            cfg1 = lz.model_config(kv_dtype=lz.F16, **CFG)
            with lz.LlmModel(dev, suite, cfg1, 64, precision) as m1:
                m1.init_synthetic(4, 0.05, 1e-3, 2e-2)
                out["ref_logits"] = m1.Prefill(prompt)
                out["ref_tokens"] = m1.decode_greedy_device(STEPS)
        suite.Dispose()
        dev.Dispose()
        q.put((rank, out, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("precision", ["bfloat16", "int8"])
def test_tensor_parallel_two_gpus_match_single(lz, device, precision):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q, idq = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, idq, precision, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, out, err = q.get(timeout=150)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = out
    finally:
        for p in procs:
            p.join(timeout=20)
            if p.is_alive():
                p.kill()
    r0, r1 = results[0], results[1]
    # Both ranks see the gathered full-vocabulary logits and the same greedy tokens.
    np.testing.assert_array_equal(r0["logits"], r1["logits"])
    np.testing.assert_array_equal(r0["tokens"], r1["tokens"])
    want = r0["ref_logits"]
    err = np.abs(r0["logits"] - want).max()
    assert err <= 2e-3 * np.abs(want).max(), f"max err {err}"
    np.testing.assert_array_equal(r0["tokens"], r0["ref_tokens"])
