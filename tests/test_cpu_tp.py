"""The tensor-parallel split of a decoder layer, checked on CPU with two gloo ranks.

Mirrors the library's sharding (l0llm_b200/csrc/model.cu, resolve / init_synthetic and the fused layer):
rank r keeps q rows [r*QD/tp, ...), k and v rows [r*KD/tp, ...) (whole heads, so each rank's query
heads keep their own KV head), gate and up rows [r*I/tp, ...), lm_head rows [r*V/tp, ...); o_proj and
down keep all rows but columns [r*QD/tp, ...) and [r*I/tp, ...), and their partial products are summed
over the ranks before the residual add; the greedy token is the largest (value, -index) key over the
ranks' vocab shards. The layer computed this way must equal the unsplit layer.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

H, I, NH, NKV, HD, V = 64, 96, 8, 2, 8, 128


def _weights():
    rng = np.random.default_rng(3)
    w = {k: rng.standard_normal(s).astype(np.float64) * 0.2 for k, s in
         dict(q=(NH * HD, H), k=(NKV * HD, H), v=(NKV * HD, H), o=(H, NH * HD), gate=(I, H), up=(I, H),
              down=(H, I), lm=(V, H)).items()}
    x = rng.standard_normal(H)
    return w, x


def _rms(x):
    return x / np.sqrt(np.mean(x * x) + 1e-6)


def _layer(w, x, heads, kv_heads):
    """One decode position (attention over itself only: softmax of one score = 1, output = v)."""
    q = w["q"] @ _rms(x)
    v = w["v"] @ _rms(x)
    g = heads // kv_heads
    attn = np.concatenate([v[(h // g) * HD:(h // g + 1) * HD] for h in range(heads)])
    assert q.shape[0] == heads * HD
    return attn


def _full():
    w, x = _weights()
    h = x + w["o"] @ _layer(w, x, NH, NKV)
    gu_in = _rms(h)
    a = w["gate"] @ gu_in
    h = h + w["down"] @ (a / (1 + np.exp(-a)) * (w["up"] @ gu_in))
    logits = w["lm"] @ _rms(h)
    return h, int(np.argmax(logits))


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w, x = _weights()
    qd, kd, i_, v_ = NH * HD // world, NKV * HD // world, I // world, V // world
    sh = dict(q=w["q"][rank * qd:(rank + 1) * qd], k=w["k"][rank * kd:(rank + 1) * kd],
              v=w["v"][rank * kd:(rank + 1) * kd], o=w["o"][:, rank * qd:(rank + 1) * qd],
              gate=w["gate"][rank * i_:(rank + 1) * i_], up=w["up"][rank * i_:(rank + 1) * i_],
              down=w["down"][:, rank * i_:(rank + 1) * i_], lm=w["lm"][rank * v_:(rank + 1) * v_])
    part = torch.from_numpy(sh["o"] @ _layer(sh, x, NH // world, NKV // world))
    dist.all_reduce(part)
    h = x + part.numpy()
    gu_in = _rms(h)
    a = sh["gate"] @ gu_in
    part = torch.from_numpy(sh["down"] @ (a / (1 + np.exp(-a)) * (sh["up"] @ gu_in)))
    dist.all_reduce(part)
    h = h + part.numpy()
    logits = sh["lm"] @ _rms(h)
    local = int(np.argmax(logits))
    # (value, -global index) as one comparable key: the reduction takes the maximum.
    key = torch.tensor([float(logits[local]), -float(rank * v_ + local)], dtype=torch.float64)
    keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(keys, key)
    best = max((float(k[0]), float(k[1])) for k in keys)
    out[rank] = (h.copy(), int(-best[1]))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_split_matches_full_layer(world):
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = tmp.get_context("spawn").Manager()
    out = mgr.dict()
    tmp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    h_full, tok_full = _full()
    for r in range(world):
        h, tok = out[r]
        np.testing.assert_allclose(h, h_full, rtol=1e-12, atol=1e-12)
        assert tok == tok_full
