"""The tensor-parallel split of a decoder layer, checked on CPU with gloo ranks.

Each rank places the checkpoint tensors where the library's own plan puts them (l0b_model_shard_plan,
the arithmetic l0b_model_set_tensor follows: l0llm_b200/csrc/model.cu shard_plan): it builds its stacked
[q; k; v] and [gate; up] matrices and its q/k/v bias from the plans' rows, columns and destination rows,
runs one decode position of the layer the way the fused layer does (o_proj and down as row-split partial
products summed over the ranks before the residual add), and picks the greedy token as the largest
(value, -index) key over the ranks' vocab shards. The result must equal the unsplit layer.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

H, I, NH, NKV, HD, V = 64, 96, 8, 4, 8, 128
NAMES = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"] + [
    f"model.layers.0.{n}" for n in (
        "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
        "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight", "self_attn.q_proj.bias",
        "self_attn.k_proj.bias", "self_attn.v_proj.bias", "mlp.gate_proj.weight", "mlp.up_proj.weight",
        "mlp.down_proj.weight")]


def _cfg(lz, world=1, rank=0):
    return lz.model_config(hidden_size=H, intermediate_size=I, num_layers=1, num_attention_heads=NH,
                           num_key_value_heads=NKV, head_dim=HD, vocab_size=V, attention_bias=1, tp_size=world,
                           tp_rank=rank)


def _weights():
    rng = np.random.default_rng(3)
    p = "model.layers.0."
    shapes = {p + "self_attn.q_proj.weight": (NH * HD, H), p + "self_attn.k_proj.weight": (NKV * HD, H),
              p + "self_attn.v_proj.weight": (NKV * HD, H), p + "self_attn.o_proj.weight": (H, NH * HD),
              p + "self_attn.q_proj.bias": (NH * HD,), p + "self_attn.k_proj.bias": (NKV * HD,),
              p + "self_attn.v_proj.bias": (NKV * HD,), p + "mlp.gate_proj.weight": (I, H),
              p + "mlp.up_proj.weight": (I, H), p + "mlp.down_proj.weight": (H, I), "lm_head.weight": (V, H),
              "model.embed_tokens.weight": (V, H)}
    w = {k: rng.standard_normal(s) * 0.2 for k, s in shapes.items()}
    for k in ("model.norm.weight", p + "input_layernorm.weight", p + "post_attention_layernorm.weight"):
        w[k] = 1 + 0.1 * rng.standard_normal(H)
    return w, rng.standard_normal(H)


def _rms(x, w):
    return x / np.sqrt(np.mean(x * x) + 1e-6) * w


def _attention_block(qkv, bias, o, w, x, heads, kv_heads):
    """One decode position at position 0 (attention over itself only: softmax of one score = 1, so each
    query head's output is its KV head's value). o_proj / down / lm_head give this rank's partials."""
    p = "model.layers.0."
    y = qkv @ _rms(x, w[p + "input_layernorm.weight"]) + bias
    qd, kd = heads * HD, kv_heads * HD
    v = y[qd + kd:qd + 2 * kd]
    g = heads // kv_heads
    attn = np.concatenate([v[(h // g) * HD:(h // g + 1) * HD] for h in range(heads)])
    return o @ attn


def _mlp(gate_up, down, w, h, inter):
    a = gate_up @ _rms(h, w["model.layers.0.post_attention_layernorm.weight"])
    return down @ (a[:inter] / (1 + np.exp(-a[:inter])) * a[inter:])


def _full(w, x):
    p = "model.layers.0."
    qkv = np.concatenate([w[p + f"self_attn.{n}_proj.weight"] for n in "qkv"])
    bias = np.concatenate([w[p + f"self_attn.{n}_proj.bias"] for n in "qkv"])
    h = x + _attention_block(qkv, bias, w[p + "self_attn.o_proj.weight"], w, x, NH, NKV)
    gu = np.concatenate([w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]])
    h = h + _mlp(gu, w[p + "mlp.down_proj.weight"], w, h, I)
    logits = w["lm_head.weight"] @ _rms(h, w["model.norm.weight"])
    return h, int(np.argmax(logits))


def _shards(lz, cfg, w):
    """This rank's tensors assembled from the library's shard plans."""
    world = max(cfg.tp_size, 1)
    qd, kd, inter = NH * HD // world, NKV * HD // world, I // world
    mats = {lz.ShardPlan.QKV: np.zeros((qd + 2 * kd, H)), lz.ShardPlan.GATE_UP: np.zeros((2 * inter, H))}
    bias = np.zeros(qd + 2 * kd)
    out = {}
    for name in NAMES:
        sp = lz.shard_plan(cfg, name)
        part = sp.take(w[name])
        if sp.kind == lz.ShardPlan.MATRIX and sp.slot in mats:
            mats[sp.slot][sp.dst_row:sp.dst_row + sp.rows] = part
        elif sp.kind == lz.ShardPlan.VECTOR and sp.slot == lz.ShardPlan.QKV_BIAS:
            bias[sp.dst_row:sp.dst_row + sp.cols] = part.reshape(-1)
        else:
            out[name] = part.reshape(-1) if sp.kind == lz.ShardPlan.VECTOR else part
    out["qkv"], out["gate_up"], out["qkv_bias"] = mats[lz.ShardPlan.QKV], mats[lz.ShardPlan.GATE_UP], bias
    return out


def _worker(rank, world, port, out):
    import sys

    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parents[1]))
    from l0llm_b200 import levelzero as lz

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w, x = _weights()
    cfg = _cfg(lz, world, rank)
    s = _shards(lz, cfg, w)
    for k in ("model.norm.weight", "model.layers.0.input_layernorm.weight",
              "model.layers.0.post_attention_layernorm.weight"):
        w[k] = s[k]  # replicated: the plan keeps the whole vector
    p = "model.layers.0."
    inter = I // world
    part = torch.from_numpy(_attention_block(s["qkv"], s["qkv_bias"], s[p + "self_attn.o_proj.weight"], w, x,
                                             NH // world, NKV // world))
    dist.all_reduce(part)
    h = x + part.numpy()
    part = torch.from_numpy(_mlp(s["gate_up"], s[p + "mlp.down_proj.weight"], w, h, inter))
    dist.all_reduce(part)
    h = h + part.numpy()
    logits = s["lm_head.weight"] @ _rms(h, w["model.norm.weight"])
    local = int(np.argmax(logits))
    head = lz.shard_plan(cfg, "lm_head.weight")
    # (value, -global index) as one comparable key: the reduction takes the maximum.
    key = torch.tensor([float(logits[local]), -float(head.row0 + local)], dtype=torch.float64)
    keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(keys, key)
    best = max((float(k[0]), float(k[1])) for k in keys)
    out[rank] = (h.copy(), int(-best[1]), s["model.embed_tokens.weight"].shape)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_split_matches_full_layer(world):
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mgr = tmp.get_context("spawn").Manager()
    out = mgr.dict()
    tmp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    w, x = _weights()
    h_full, tok_full = _full(w, x)
    for r in range(world):
        h, tok, emb_shape = out[r]
        np.testing.assert_allclose(h, h_full, rtol=1e-12, atol=1e-12)
        assert tok == tok_full
        assert emb_shape == (V, H)  # the embedding table is replicated


def test_shard_plan_covers_each_output_once():
    """Over the ranks, the plans of every split tensor tile it exactly once (rows for column splits,
    columns for row splits), and optional tensors the config does not use are refused."""
    from l0llm_b200 import levelzero as lz

    w, _ = _weights()
    for world in (1, 2, 4):
        for name in NAMES:
            seen = np.zeros(w[name].shape if w.get(name) is not None else (H,), int).reshape(
                lz.shard_plan(_cfg(lz, world, 0), name).full_rows, -1)
            for r in range(world):
                sp = lz.shard_plan(_cfg(lz, world, r), name)
                seen[sp.row0:sp.row0 + sp.rows, sp.col0:sp.col0 + sp.cols] += 1
            want = 1 if "embed" in name or "norm" in name else None
            if want is None:
                assert (seen == 1).all(), f"{name} at tp {world}"
            else:
                assert (seen == world).all(), f"{name} at tp {world}: replicated"
    cfg = lz.model_config(hidden_size=H, intermediate_size=I, num_layers=1, num_attention_heads=NH,
                          num_key_value_heads=NKV, head_dim=HD, vocab_size=V, attention_bias=0)
    with pytest.raises(lz.InvalidDataException):
        lz.shard_plan(cfg, "model.layers.0.self_attn.q_proj.bias")
    with pytest.raises(lz.InvalidDataException):
        lz.shard_plan(cfg, "model.layers.1.mlp.up_proj.weight")
    with pytest.raises(lz.NotSupportedException):
        lz.shard_plan(_cfg(lz, 3, 0), "lm_head.weight")
