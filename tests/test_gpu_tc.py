"""GPU parity of the tcgen05 tensor-core GEMM (prefill linear layers) against the CPU oracle.

The GEMM multiplies activations rounded to the weight's 16-bit format, so the oracle is fed the same
rounded activations; what remains is accumulation order (fp32 in TMEM vs fp64), held to 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _round16(x, fmt):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    return (t.to(torch.bfloat16) if fmt == "bf16" else t.to(torch.float16)).to(torch.float32).numpy()


def _wbits(w, fmt):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(w, np.float32))
    return (t.to(torch.bfloat16) if fmt == "bf16" else t.to(torch.float16)).view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k", [(64, 256, 896), (130, 4608, 3584), (17, 384, 512), (512, 1000, 1024),
                                   (256, 3584, 3584), (1, 128, 64)])
@pytest.mark.parametrize("epi", ["store", "accum"])
def test_tc_gemm_store_accum(lz, orc, device, suite, fmt, m, n, k, epi):
    rng = np.random.default_rng(m * 3 + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    base = rng.standard_normal((m, n)).astype(np.float32)
    wb = _wbits(w, fmt)
    want = orc.gemv_out_in(_round16(x, fmt), wb, orc.BF16 if fmt == "bf16" else orc.F16) + bias
    if epi == "accum":
        want = want + base
    code = lz.BF16 if fmt == "bf16" else lz.F16
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, wb, code) as W, \
            lz.SharedBuffer.from_array(device, bias) as bb, lz.SharedBuffer.from_array(device, base) as ob:
        lz.check(lz.load_library().l0b_linear_tc(suite.handle, device.handle, m, n, k, xb.handle, W.handle, None,
                                                  0.0, 1 if epi == "accum" else 0, bb.handle, ob.handle))
        got = ob.ToArray().reshape(m, n)
    err = np.abs(got - want)
    assert np.all(err <= 1e-3 + 1e-3 * np.abs(want)), f"max err {err.max()}"


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("m", [5, 128, 300])
def test_tc_gemm_norm_swiglu(lz, orc, device, suite, fmt, m):
    rng = np.random.default_rng(m)
    H, I = 896, 4864
    x = rng.standard_normal((m, H)).astype(np.float32) * 2
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    w = ((rng.random((2 * I, H)) * 2 - 1) * 0.05).astype(np.float32)
    _, normed = orc.rmsnorm(x, nw, 1e-6)
    wb = _wbits(w, fmt)
    y = orc.gemv_out_in(_round16(normed, fmt), wb, orc.BF16 if fmt == "bf16" else orc.F16)
    g, u = y[:, :I], y[:, I:]
    want = g / (1 + np.exp(-g.astype(np.float64))) * u
    code = lz.BF16 if fmt == "bf16" else lz.F16
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, wb, code) as W, \
            lz.SharedBuffer.from_array(device, nw) as nb, lz.SharedBuffer(device, lz.F32, m * I) as ob:
        lz.check(lz.load_library().l0b_linear_tc(suite.handle, device.handle, m, 2 * I, H, xb.handle, W.handle,
                                                  nb.handle, 1e-6, 2, None, ob.handle))
        got = ob.ToArray().reshape(m, I)
    # The norm runs before the 16-bit rounding on both sides; a few elements may round differently.
    err = np.abs(got - want)
    assert np.all(err <= 2e-3 + 2e-2 * np.abs(want)), f"max err {err.max()}"
    assert np.median(err) < 1e-3


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k,epi", [(64, 512, 896, 0), (100, 4608, 3584, 1), (17, 384, 200, 0), (1, 128, 64, 1)])
def test_tc_gemm_f32_activations(lz, orc, device, suite, fmt, m, n, k, epi):
    """Split activations (x = hi + lo in the weight's 16-bit format, rows scaled by powers of two): the
    result is the product of the UNROUNDED f32 rows with the 16-bit weights. Row magnitudes span 2^+-17,
    beyond f16's range without the row scale; K = 200 leaves a zero-padded partial K tile."""
    rng = np.random.default_rng(m * 7 + n + k)
    x = (rng.standard_normal((m, k)) * np.exp2(rng.uniform(-17, 17, (m, 1)))).astype(np.float32)
    w = ((rng.random((n, k)) * 2 - 1) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    base = rng.standard_normal((m, n)).astype(np.float32)
    wb = _wbits(w, fmt)
    w16 = _round16(w, fmt).astype(np.float64)
    want = x.astype(np.float64) @ w16.T + bias
    if epi == 1:
        want = want + base
    # hi + lo keeps 16 (bf16) or 22 (f16) bits of each x; fp32 accumulation over K adds ~sqrt(K) ulps.
    bound = np.abs(x).astype(np.float64) @ np.abs(w16).T
    code = lz.BF16 if fmt == "bf16" else lz.F16
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, wb, code) as W, \
            lz.SharedBuffer.from_array(device, bias) as bb, lz.SharedBuffer.from_array(device, base) as ob:
        lz.check(lz.load_library().l0b_linear_tc(suite.handle, device.handle, m, n, k, xb.handle, W.handle, None,
                                                  0.0, epi | lz.LlmKernelSuite.EPI_F32_ACTIVATIONS, bb.handle,
                                                  ob.handle))
        got = ob.ToArray().reshape(m, n)
    err = np.abs(got - want)
    assert np.all(err <= 3e-5 * bound + 1e-6 * np.abs(want) + 1e-6), f"max err {err.max()}"


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
def test_tc_gemm_f32_activations_norm_swiglu(lz, orc, device, suite, fmt):
    rng = np.random.default_rng(11)
    m, H, I = 48, 896, 4864
    x = rng.standard_normal((m, H)).astype(np.float32) * 2
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    w = ((rng.random((2 * I, H)) * 2 - 1) * 0.05).astype(np.float32)
    _, normed = orc.rmsnorm(x, nw, 1e-6)
    wb = _wbits(w, fmt)
    y = np.asarray(normed, np.float64) @ _round16(w, fmt).astype(np.float64).T
    g, u = y[:, :I], y[:, I:]
    want = g / (1 + np.exp(-g)) * u
    code = lz.BF16 if fmt == "bf16" else lz.F16
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, wb, code) as W, \
            lz.SharedBuffer.from_array(device, nw) as nb, lz.SharedBuffer(device, lz.F32, m * I) as ob:
        lz.check(lz.load_library().l0b_linear_tc(suite.handle, device.handle, m, 2 * I, H, xb.handle, W.handle,
                                                  nb.handle, 1e-6, 2 | lz.LlmKernelSuite.EPI_F32_ACTIVATIONS, None,
                                                  ob.handle))
        got = ob.ToArray().reshape(m, I)
    # Twenty times tighter than the rounded-activation bound of test_tc_gemm_norm_swiglu.
    err = np.abs(got - want)
    assert np.all(err <= 1e-4 + 1e-3 * np.abs(want)), f"max err {err.max()}"


def _q8_rows(rng, n, k):
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    q[:, 0] = -128  # the full int8 range converts exactly
    s16 = (rng.random(n) * 2e-3 + 1e-4).astype(np.float16)
    return q, s16


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("m,n,k,epi", [(64, 512, 896, 0), (100, 4608, 3584, 1), (17, 384, 208, 0), (300, 256, 512, 1),
                                       (8, 640, 3584, 1), (5, 256, 208, 0), (16, 3584, 18944, 1)])
def test_tc_gemm_int8_row_scales(lz, device, suite, split, m, n, k, epi):
    """int8 weights with one f16 scale per row on the integer MMA (kind::i8): the activations go in as four
    int8 digits of x * 2^s (~27 bits of each token's largest value, with or without the f32 flag), the
    s32 sums are exact, so against the f64 product only the digit rounding and the final f32 rounding
    remain. K = 208 leaves a partial 128-k stage; K = 18944 checks the s32 range."""
    rng = np.random.default_rng(m + n * 3 + k)
    x = (rng.standard_normal((m, k)) * np.exp2(rng.uniform(-8, 8, (m, 1)))).astype(np.float32)
    q, s16 = _q8_rows(rng, n, k)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    base = rng.standard_normal((m, n)).astype(np.float32)
    xa = x.astype(np.float64)
    sc = s16.astype(np.float64)
    want = (xa @ q.astype(np.float64).T) * sc + bias
    if epi == 1:
        want = want + base
    bound = (np.abs(xa) @ np.abs(q.astype(np.float64)).T) * sc
    flag = lz.LlmKernelSuite.EPI_F32_ACTIVATIONS if split else 0
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, q, lz.I8) as W, \
            lz.SharedBuffer.from_array(device, s16.view(np.uint16), lz.F16) as S, \
            lz.SharedBuffer.from_array(device, bias) as bb, lz.SharedBuffer.from_array(device, base) as ob:
        lz.check(lz.load_library().l0b_linear_tc_scaled(suite.handle, device.handle, m, n, k, xb.handle, W.handle,
                                                         S.handle, k, None, 0.0, epi | flag, bb.handle, ob.handle))
        got = ob.ToArray().reshape(m, n)
    err = np.abs(got - want)
    assert np.all(err <= 1e-5 * bound + 1e-6 * np.abs(want) + 1e-6), f"max err {err.max()}"


def test_tc_gemm_int8_norm_swiglu(lz, orc, device, suite):
    rng = np.random.default_rng(21)
    m, H, I = 48, 896, 4864
    x = rng.standard_normal((m, H)).astype(np.float32) * 2
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    q, s16 = _q8_rows(rng, 2 * I, H)
    _, normed = orc.rmsnorm(x, nw, 1e-6)
    y = (np.asarray(normed, np.float64) @ q.astype(np.float64).T) * s16.astype(np.float64)
    g, u = y[:, :I], y[:, I:]
    want = g / (1 + np.exp(-g)) * u
    with lz.SharedBuffer.from_array(device, x) as xb, lz.SharedBuffer.from_array(device, q, lz.I8) as W, \
            lz.SharedBuffer.from_array(device, s16.view(np.uint16), lz.F16) as S, \
            lz.SharedBuffer.from_array(device, nw) as nb, lz.SharedBuffer(device, lz.F32, m * I) as ob:
        lz.check(lz.load_library().l0b_linear_tc_scaled(suite.handle, device.handle, m, 2 * I, H, xb.handle,
                                                         W.handle, S.handle, 0, nb.handle, 1e-6,
                                                         2 | lz.LlmKernelSuite.EPI_F32_ACTIVATIONS, None, ob.handle))
        got = ob.ToArray().reshape(m, I)
    err = np.abs(got - want)
    assert np.all(err <= 1e-4 + 1e-3 * np.abs(want)), f"max err {err.max()}"


def test_tc_gemm_int8_refuses_group_scales(lz, device, suite):
    with lz.SharedBuffer(device, lz.F32, 64 * 128) as xb, lz.SharedBuffer(device, lz.I8, 128 * 128) as W, \
            lz.SharedBuffer(device, lz.F16, 128 * 4) as S, lz.SharedBuffer(device, lz.F32, 64 * 128) as ob:
        st = lz.load_library().l0b_linear_tc_scaled(suite.handle, device.handle, 64, 128, 128, xb.handle, W.handle,
                                                     S.handle, 32, None, 0.0, 0, None, ob.handle)
    assert st != 0


def test_tc_gemm_reports_no_timeouts(lz, device):
    import ctypes as C

    code = C.c_int32()
    lz.check(lz.load_library().l0b_device_error_status(device.handle, C.byref(code)))
    assert code.value == 0
