"""Both decode GEMV kernels (tensor-core mma.sync streaming and fp32-FMA streaming) against the oracle.

The tensor-core kernel splits each activation into two f16 halves (hi + residual), so its result must
stay within fp32-accumulation distance of the fp64 oracle, far tighter than a plain f16 activation
would allow. Shapes cover a single piece of K (K = 64, most warps idle), K not a multiple of the
eight-warp stride (896), the long down-projection row (18944), row counts that leave partial 16-row
tiles, and 1..16 activation rows (one, two or four B-column groups). Row counts whose activations do not
fit one CTA's shared memory run split-K across a thread-block cluster, which also exchanges the fused
RMSNorm's sums of squares between the ranks.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["mma", "fma", "bulk"])
def path(request, lz):
    """mma: register-streamed tensor-core GEMV; fma: fp32 FMA; bulk: the TMA-streamed tensor-core GEMV
    for one activation row (other row counts fall back to mma)."""
    lib = lz.load_library()
    lib.l0b_set_gemv_tensor_cores(0 if request.param == "fma" else 1)
    lib.l0b_set_gemv_bulk(1 if request.param == "bulk" else 0)  # mma: the register-streamed kernel only
    yield request.param
    lib.l0b_set_gemv_tensor_cores(1)
    lib.l0b_set_gemv_bulk(1)


def _weights(lz, orc, wkind, hf, k):
    import torch

    if wkind == "f16":
        w = hf.astype(np.float16)
        return w, w.view(np.uint16), orc.F16, lz.F16, None, 0
    if wkind == "bf16":
        w = torch.from_numpy(hf).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        return w, w, orc.BF16, lz.BF16, None, 0
    q, s = lz.q8_quantize_out_in(hf, k)
    return q, q, orc.I8, lz.I8, s, k


@pytest.mark.parametrize("wkind", ["f16", "bf16", "i8c"])
@pytest.mark.parametrize("n,k", [(40, 64), (1000, 896), (4608, 3584), (3584, 18944), (17, 128)])
@pytest.mark.parametrize("m", [1, 2, 5, 8, 13, 16])
def test_gemv_paths_store(lz, orc, device, suite, path, wkind, n, k, m):
    rng = np.random.default_rng(n + 3 * k + m)
    hf = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
    x = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    w_dev, w_orc, wdt, dt, scales, group = _weights(lz, orc, wkind, hf, k)
    want = orc.gemv_out_in(x, w_orc, wdt, None if scales is None else scales.view(np.uint16), group) + bias
    with lz.SharedBuffer.from_array(device, w_dev, dt) as W, lz.SharedBuffer.from_array(device, x) as xb, \
            lz.SharedBuffer.from_array(device, bias) as bb, lz.SharedBuffer(device, lz.F32, m * n) as y:
        sb = lz.SharedBuffer.from_array(device, scales) if scales is not None else None
        suite.linear(device, m, n, k, xb, W, sb, group, bb, y)
        got = y.ToArray().reshape(m, n)
        if sb is not None:
            sb.Dispose()
    # bf16 activations split in two keep ~16 bits; f16 pairs keep ~22.
    tol = 2e-4 if wkind == "bf16" else 2e-5
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= tol * scale, f"{path}: max err {err} vs scale {scale}"


@pytest.mark.parametrize("fill", [1, 2, 4, 8])
@pytest.mark.parametrize("wkind", ["bf16", "i8c"])
@pytest.mark.parametrize("n,k,m", [(1280, 8192, 1), (1280, 8192, 3), (200, 8192, 1), (1024, 4096, 2)])
def test_gemv_fill_split(lz, orc, device, suite, fill, wkind, n, k, m):
    """Projections with fewer 16-row tiles than SMs split K across a cluster only to fill idle SMs (the
    q/k/v shard of an 8-way tensor-parallel 70B layer is 80 tiles over K = 8192): every split count
    gives the oracle's result."""
    lib = lz.load_library()
    rng = np.random.default_rng(n + k + m + fill)
    hf = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
    x = (rng.standard_normal((m, k)) * 2).astype(np.float32)
    w_dev, w_orc, wdt, dt, scales, group = _weights(lz, orc, wkind, hf, k)
    want = orc.gemv_out_in(x, w_orc, wdt, None if scales is None else scales.view(np.uint16), group)
    lib.l0b_set_gemv_fill_split(fill)
    try:
        with lz.SharedBuffer.from_array(device, w_dev, dt) as W, lz.SharedBuffer.from_array(device, x) as xb, \
                lz.SharedBuffer(device, lz.F32, m * n) as y:
            sb = lz.SharedBuffer.from_array(device, scales) if scales is not None else None
            suite.linear(device, m, n, k, xb, W, sb, group, None, y)
            got = y.ToArray().reshape(m, n)
            if sb is not None:
                sb.Dispose()
    finally:
        lib.l0b_set_gemv_fill_split(2)
    tol = 2e-4 if wkind == "bf16" else 2e-5
    assert np.abs(got - want).max() <= tol * np.abs(want).max()


@pytest.mark.parametrize("wkind", ["f16", "i8c"])
@pytest.mark.parametrize("H,inter", [(896, 4864), (896, 100), (3584, 1000)])
@pytest.mark.parametrize("m", [1, 3, 8, 16])
def test_gemv_paths_norm_swiglu(lz, orc, device, suite, path, wkind, H, inter, m):
    rng = np.random.default_rng(inter + m + H)
    x = (rng.standard_normal((m, H)) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    hf = ((rng.random((2 * inter, H)) * 2 - 1) * 0.05).astype(np.float32)
    _, normed = orc.rmsnorm(x, nw, 1e-6)
    w_dev, w_orc, wdt, dt, scales, group = _weights(lz, orc, wkind, hf, H)
    y = orc.gemv_out_in(normed, w_orc, wdt, None if scales is None else scales.view(np.uint16), group)
    g, u = y[:, :inter], y[:, inter:]
    want = g / (1 + np.exp(-g.astype(np.float64))) * u
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, w_dev, dt) as W, \
            lz.SharedBuffer.from_array(device, nw) as nb, lz.SharedBuffer(device, lz.F32, m * inter) as ob:
        sb = lz.SharedBuffer.from_array(device, scales) if scales is not None else None
        suite.linear_fused(device, m, 2 * inter, H, xb, W, sb, group, nb, 1e-6, suite.EPI_SWIGLU, None, ob)
        got = ob.ToArray().reshape(m, inter)
        if sb is not None:
            sb.Dispose()
    err = np.abs(got - want)
    assert np.all(err <= 1e-4 + 1e-4 * np.abs(want)), f"{path}: max err {err.max()}"


@pytest.mark.parametrize("m", [1, 2, 9, 16])
def test_gemv_paths_accumulate_down_projection(lz, orc, device, suite, path, m):
    rng = np.random.default_rng(90 + m)
    H, I = 3584, 18944
    hidden = rng.standard_normal((m, H)).astype(np.float32)
    x = rng.standard_normal((m, I)).astype(np.float32)
    hf = ((rng.random((H, I)) * 2 - 1) * 0.02).astype(np.float32)
    q, s = lz.q8_quantize_out_in(hf, I)
    want = hidden + orc.gemv_out_in(x, q, orc.I8, s.view(np.uint16), I)
    with lz.SharedBuffer.from_array(device, hidden) as hb, lz.SharedBuffer.from_array(device, x) as xb, \
            lz.SharedBuffer.from_array(device, q) as W, lz.SharedBuffer.from_array(device, s) as S:
        suite.linear_fused(device, m, H, I, xb, W, S, I, None, 0.0, suite.EPI_ACCUM, None, hb)
        got = hb.ToArray().reshape(m, H)
    err = np.abs(got - want)
    assert np.all(err <= 2e-4 + 1e-5 * np.abs(want)), f"{path}: max err {err.max()}"


def test_gemv_paths_one_hot_reads_weights_exactly(lz, device, suite, path):
    """x = e_c reads column c of the dequantised weights back bit-exactly on both kernels."""
    rng = np.random.default_rng(5)
    n, k = 272, 1024
    hf = ((rng.random((n, k)) * 2 - 1) * 0.3).astype(np.float32)
    q, s = lz.q8_quantize_out_in(hf, k)
    cols = [0, 15, 16, 63, 64, 511, 512, 1023]
    x = np.zeros((len(cols), k), np.float32)
    for r, c in enumerate(cols):
        x[r, c] = 1.0
    with lz.SharedBuffer.from_array(device, q) as W, lz.SharedBuffer.from_array(device, s) as S, \
            lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer(device, lz.F32, len(cols) * n) as y:
        suite.linear(device, len(cols), n, k, xb, W, S, k, None, y)
        got = y.ToArray().reshape(len(cols), n)
    sf = s.astype(np.float32)
    for r, c in enumerate(cols):
        np.testing.assert_array_equal(got[r], q[:, c].astype(np.float32) * sf[:, 0])


@pytest.fixture
def bulk(lz):
    lib = lz.load_library()
    lib.l0b_set_gemv_bulk(1)
    yield


@pytest.mark.parametrize("n,k,epi", [(20003, 896, "store"), (19000, 3584, "accum")])
def test_gemv_bulk_many_tiles(lz, orc, device, suite, bulk, n, k, epi):
    """The whole-tile bulk kernel serves one-row int8 projections with at least 8 tiles per SM: a partial
    last tile, the store and residual-add epilogues, against the oracle."""
    rng = np.random.default_rng(n + k)
    hf = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
    x = (rng.standard_normal((1, k)) * 2).astype(np.float32)
    base = rng.standard_normal((1, n)).astype(np.float32)
    q, s = lz.q8_quantize_out_in(hf, k)
    want = orc.gemv_out_in(x, q, orc.I8, s.view(np.uint16), k)
    if epi == "accum":
        want = want + base
    with lz.SharedBuffer.from_array(device, q) as W, lz.SharedBuffer.from_array(device, s) as S, \
            lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, base) as ob:
        suite.linear_fused(device, 1, n, k, xb, W, S, k, None, 0.0,
                           suite.EPI_ACCUM if epi == "accum" else suite.EPI_STORE, None, ob)
        got = ob.ToArray().reshape(1, n)
    err = np.abs(got - want)
    assert np.all(err <= 1e-4 + 1e-5 * np.abs(want)), f"max err {err.max()}"


def test_gemv_bulk_norm_swiglu_many_tiles(lz, orc, device, suite, bulk):
    rng = np.random.default_rng(77)
    H, inter = 3584, 9500  # 1188 SwiGLU tiles, the last one partial
    x = (rng.standard_normal((1, H)) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    hf = ((rng.random((2 * inter, H)) * 2 - 1) * 0.05).astype(np.float32)
    _, normed = orc.rmsnorm(x, nw, 1e-6)
    q, s = lz.q8_quantize_out_in(hf, H)
    y = orc.gemv_out_in(normed, q, orc.I8, s.view(np.uint16), H)
    g, u = y[:, :inter], y[:, inter:]
    want = g / (1 + np.exp(-g.astype(np.float64))) * u
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, q) as W, \
            lz.SharedBuffer.from_array(device, s) as S, lz.SharedBuffer.from_array(device, nw) as nb, \
            lz.SharedBuffer(device, lz.F32, inter) as ob:
        suite.linear_fused(device, 1, 2 * inter, H, xb, W, S, H, nb, 1e-6, suite.EPI_SWIGLU, None, ob)
        got = ob.ToArray().reshape(1, inter)
    err = np.abs(got - want)
    assert np.all(err <= 1e-4 + 1e-4 * np.abs(want)), f"max err {err.max()}"


def test_gemv_bulk_model_matches_register_path(lz, device, suite):
    """Config-2 widths, two layers: greedy decode with the bulk kernel on the gate/up projections and the
    152,064-row LM head (argmax epilogue) gives the register path's tokens and logits."""
    cfgd = dict(hidden_size=3584, intermediate_size=18944, num_layers=2, num_attention_heads=28,
                num_key_value_heads=4, head_dim=128, vocab_size=152064, max_position_embeddings=32768,
                rms_norm_eps=1e-6, rope_theta=1e6, attention_bias=1, q8_group=0)
    prompt = np.random.default_rng(2).integers(0, 152064, 16).astype(np.int32)
    lib = lz.load_library()
    out = {}
    for on in (0, 1):
        lib.l0b_set_gemv_bulk(on)
        try:
            with lz.LlmModel(device, suite, lz.model_config(kv_dtype=lz.F16, **cfgd), 64, "int8") as model:
                model.init_synthetic(2, 0.02, 1e-3, 2e-2)
                model.Prefill(prompt)
                toks = model.decode_greedy_device(6)
                out[on] = (toks, model.Decode(int(toks[-1])))
        finally:
            lib.l0b_set_gemv_bulk(1)
    np.testing.assert_array_equal(out[0][0], out[1][0])
    scale = float(np.abs(out[0][1]).max())
    assert float(np.abs(out[0][1] - out[1][1]).max()) <= 1e-4 * scale


CFG2_W = dict(hidden_size=3584, intermediate_size=18944, num_attention_heads=28, num_key_value_heads=4, head_dim=128,
              vocab_size=152064, max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1e6, attention_bias=1,
              q8_group=0)


def test_blocked_layout_model_matches_row_major(lz, device, suite):
    """q/k/v, o_proj and down of config-2 widths are stored in the blocked layout ([N/16][K/512][16][512]):
    the same model built row-major gives the same prefill logits (tcgen05 GEMM, 4-D tensor map), the same
    one-row decode (bulk GEMV over units of contiguous blocks, with the two-CTA tile fixup), the same
    batch-5 decode (register-streamed GEMV, blocked addressing) and batch-12 decode (tcgen05 GEMM)."""
    lib = lz.load_library()
    prompts = [np.random.default_rng(40 + s).integers(0, 152064, 9 + 3 * s).astype(np.int32) for s in range(12)]
    out = {}
    for blocked in (1, 0):
        lib.l0b_set_weight_blocking(blocked)
        try:
            mc = lz.model_config(kv_dtype=lz.F16, num_layers=2, max_batch=12, **CFG2_W)
            with lz.LlmModel(device, suite, mc, 96, "int8") as model:
                model.init_synthetic(2, 0.02, 1e-3, 2e-2)
                r = {"prefill": model.Prefill(prompts[0]), "greedy": model.decode_greedy_device(6)}
                firsts = [model.PrefillSequence(s, p) for s, p in enumerate(prompts)]
                toks = np.array([int(np.argmax(f)) for f in firsts], np.int32)
                pos = np.array([len(p) for p in prompts], np.int32)
                r["batch5"] = model.DecodeBatch(toks[:5], pos[:5])
                for s, p in enumerate(prompts):
                    model.PrefillSequence(s, p, want_logits=False)
                r["batch12"] = model.DecodeBatch(toks, pos)
                r["o_proj"] = model.read_weight(1, 1, np.int8, 3584 * 3584)
                out[blocked] = r
        finally:
            lib.l0b_set_weight_blocking(1)
    a, b = out[1], out[0]
    np.testing.assert_array_equal(a["greedy"], b["greedy"])
    np.testing.assert_array_equal(a["o_proj"], b["o_proj"])
    for key in ("prefill", "batch5", "batch12"):
        scale = float(np.abs(b[key]).max())
        err = float(np.abs(a[key] - b[key]).max())
        assert err <= 1e-4 * scale, f"{key}: blocked vs row-major max err {err} (scale {scale})"


def test_blocked_layout_set_tensor_round_trip(lz, device, suite):
    """Uploaded HF tensors land in the blocked layout and read back in [out, in] order as the host
    quantizer's codes; the stacked q/k/v rows keep their offsets."""
    mc = lz.model_config(kv_dtype=lz.F16, num_layers=1, **CFG2_W)
    rng = np.random.default_rng(9)
    with lz.LlmModel(device, suite, mc, 8, "int8") as model:
        want = {}
        for name, (n, k) in {"self_attn.q_proj": (3584, 3584), "self_attn.k_proj": (512, 3584),
                             "self_attn.v_proj": (512, 3584), "self_attn.o_proj": (3584, 3584),
                             "mlp.down_proj": (3584, 18944)}.items():
            hf = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
            model.set_tensor(f"model.layers.0.{name}.weight", hf)
            want[name] = lz.q8_quantize_out_in(hf, k)
        qkv = np.concatenate([want[n][0] for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")])
        np.testing.assert_array_equal(model.read_weight(0, 0, np.int8, qkv.size).reshape(qkv.shape), qkv)
        np.testing.assert_array_equal(model.read_weight(0, 1, np.int8, 3584 * 3584).reshape(3584, 3584),
                                      want["self_attn.o_proj"][0])
        np.testing.assert_array_equal(model.read_weight(0, 3, np.int8, 3584 * 18944).reshape(3584, 18944),
                                      want["mlp.down_proj"][0])


@pytest.mark.parametrize("m", [1, 3])
@pytest.mark.parametrize("case", ["down", "qkv", "gate_up"])
def test_linear_fused_blocked_weights(lz, orc, device, suite, case, m):
    """l0b_linear_fused with L0B_EPI_BLOCKED_WEIGHTS: int8 weights handed over in the blocked layout
    [N/16][K/512][16][512] give the oracle's result for the row-major bytes. One row runs the k-split GEMV
    (down: 37 k blocks x 4 tile groups, residual add; q/k/v: 7 x 21, RMSNorm prologue + bias; [gate; up]
    with SwiGLU); three rows the register-streamed GEMV with blocked addressing. Two calls in a row check
    that the k-split scratch (row sums, group counters) is left at zero."""
    rng = np.random.default_rng({"down": 11, "qkv": 12, "gate_up": 13}[case] + m)
    if case == "down":
        n, k, epi, norm, bias = 3584, 18944, suite.EPI_ACCUM, False, False
    elif case == "qkv":
        n, k, epi, norm, bias = 4608, 3584, suite.EPI_STORE, True, True
    else:
        n, k, epi, norm, bias = 2 * 1024, 4096, suite.EPI_SWIGLU, True, False
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    s = rng.uniform(1e-3, 2e-2, n).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    bv = (rng.standard_normal(n) * 0.1).astype(np.float32)
    xin = orc.rmsnorm(x, nw, 1e-6)[1] if norm else x
    y = orc.gemv_out_in(xin, q, orc.I8, s.view(np.uint16), k)
    out_cols = n // 2 if epi == suite.EPI_SWIGLU else n
    base = rng.standard_normal((m, out_cols)).astype(np.float32)
    if epi == suite.EPI_ACCUM:
        want = base + y
    elif epi == suite.EPI_SWIGLU:
        g, u = y[:, :n // 2], y[:, n // 2:]
        want = g / (1 + np.exp(-g.astype(np.float64))) * u
    else:
        want = y + (bv if bias else 0)
    with lz.SharedBuffer.from_array(device, lz.block_int8(q)) as W, lz.SharedBuffer.from_array(device, s) as S, \
            lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, nw) as nb, \
            lz.SharedBuffer.from_array(device, bv) as bb, lz.SharedBuffer(device, lz.F32, m * out_cols) as ob:
        for _ in range(2):
            ob.Write(base.reshape(-1))
            suite.linear_fused(device, m, n, k, xb, W, S, k, nb if norm else None, 1e-6,
                               epi | suite.EPI_BLOCKED_WEIGHTS, bb if bias else None, ob)
            got = ob.ToArray().reshape(m, out_cols)
            err = np.abs(got - want)
            scale = np.abs(want).max()
            assert np.all(err <= 2e-5 * scale + 1e-5 * np.abs(want)), f"{case} m={m}: max err {err.max()} ({scale})"


def test_linear_fused_blocked_weights_rejects_bad_shapes(lz, device, suite):
    """The blocked flag needs int8 with one scale per row, N % 16 == 0 and K % 512 == 0."""
    with lz.SharedBuffer(device, lz.I8, 40 * 512) as W, lz.SharedBuffer(device, lz.F16, 40) as S, \
            lz.SharedBuffer(device, lz.F32, 512) as xb, lz.SharedBuffer(device, lz.F32, 40) as ob:
        with pytest.raises(lz.ArgumentException):
            suite.linear_fused(device, 1, 40, 512, xb, W, S, 512, None, 0.0,
                               suite.EPI_STORE | suite.EPI_BLOCKED_WEIGHTS, None, ob)


@pytest.mark.parametrize("wkind", ["bf16", "i8c"])
@pytest.mark.parametrize("m", [1, 8])
def test_linear_shared_equals_separate_projections(lz, orc, device, suite, wkind, m):
    """ProjectShared over stacked weights (l0b_linear_shared): the Gated DeltaNet in-projections of
    config 3 (qkv 8192, z 4096, b 32, a 32 rows over K = 2048) as one launch give the oracle's result for
    each projection, with a bias on one of them, and the same values as four separate l0b_linear calls."""
    rng = np.random.default_rng(31 + m)
    K, rows = 2048, [8192, 4096, 32, 32]
    hf = ((rng.random((sum(rows), K)) * 2 - 1) * 0.05).astype(np.float32)
    x = rng.standard_normal((m, K)).astype(np.float32)
    bias = (rng.standard_normal(rows[1]) * 0.1).astype(np.float32)
    w_dev, w_orc, wdt, dt, scales, group = _weights(lz, orc, wkind, hf, K)
    want = orc.gemv_out_in(x, w_orc, wdt, None if scales is None else scales.view(np.uint16), group)
    edges = np.cumsum([0] + rows)
    with lz.SharedBuffer.from_array(device, w_dev, dt) as W, lz.SharedBuffer.from_array(device, x) as xb, \
            lz.SharedBuffer.from_array(device, bias) as bb:
        sb = lz.SharedBuffer.from_array(device, scales) if scales is not None else None
        outs = [lz.SharedBuffer(device, lz.F32, m * r) for r in rows]
        suite.linear_shared(device, m, K, xb, W, sb, group, rows, outs, [None, bb, None, None])
        got = [o.ToArray().reshape(m, r) for o, r in zip(outs, rows)]
        tol = 2e-4 if wkind == "bf16" else 2e-5
        for i, r in enumerate(rows):
            w_i = want[:, edges[i]:edges[i + 1]] + (bias if i == 1 else 0)
            err = np.abs(got[i] - w_i).max()
            assert err <= tol * max(np.abs(w_i).max(), 1e-3), f"projection {i}: max err {err}"
        # Separate calls over the same rows (views of W) give the same values.
        wv = w_dev.reshape(sum(rows), K)
        for i, r in enumerate(rows):
            with lz.SharedBuffer.from_array(device, np.ascontiguousarray(wv[edges[i]:edges[i + 1]]), dt) as Wi, \
                    lz.SharedBuffer(device, lz.F32, m * r) as yi:
                si = lz.SharedBuffer.from_array(device, np.ascontiguousarray(scales[edges[i]:edges[i + 1]])) \
                    if scales is not None else None
                suite.linear(device, m, r, K, xb, Wi, si, group, bb if i == 1 else None, yi)
                sep = yi.ToArray().reshape(m, r)
                if si is not None:
                    si.Dispose()
            err = np.abs(sep - got[i]).max()
            assert err <= tol * max(np.abs(sep).max(), 1e-3), f"projection {i}: shared vs separate {err}"
        for o in outs:
            o.Dispose()
        if sb is not None:
            sb.Dispose()
