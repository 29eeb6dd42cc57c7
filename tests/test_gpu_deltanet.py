"""Gated DeltaNet (Qwen3.5 linear attention) at the BASELINE config-3 shape against the CPU oracle.

Config 3: hidden 2048, 16 key heads and 32 value heads of dim 128, conv kernel 4; beta = sigmoid(N(0,1)),
per-step decay exp(-softplus(N(0,1))) (A_log = 0, dt_bias = 0), q and k L2-normalised inside the op.
The recurrence runs in chunks of 64 tokens (WY form) for prefill calls and token by token for decode;
both are checked against the oracle's token-by-token restatement in double (orc_gated_delta), output
and final state, including a nonzero starting state and chunks cut short by the token count. The whole
MixLinear layer (L/LlmDecoderLayer.cs:381-397: projections, causal conv, recurrence with its gated norm,
out_proj) is checked as a 512-token prefill followed by decode steps carrying the state.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng


def _buf(lz, device, arr):
    return lz.SharedBuffer.from_array(device, np.ascontiguousarray(arr))


def _close(got, want, tol, what):
    err = float(np.abs(got.astype(np.float64) - want).max())
    scale = float(np.abs(want).max())
    assert err <= tol * max(scale, 1.0), f"{what}: max abs err {err:.3e} (scale {scale:.3e}, tol {tol})"


def _inputs(rng, hk, hv, dk, dv, tokens, config3=True):
    conv_dim = 2 * hk * dk + hv * dv
    conv = rng.standard_normal((tokens, conv_dim)).astype(np.float32)
    z = rng.standard_normal((tokens, hv * dv)).astype(np.float32)
    b = rng.standard_normal((tokens, hv)).astype(np.float32)
    a = rng.standard_normal((tokens, hv)).astype(np.float32)
    if config3:
        a_log = np.zeros(hv, np.float32)
        dt = np.zeros(hv, np.float32)
    else:
        a_log = np.log(rng.uniform(1, 16, hv)).astype(np.float32)
        dt = rng.standard_normal(hv).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    S0 = (rng.standard_normal((hv, dk, dv)) * 0.1).astype(np.float32)
    return conv, z, b, a, a_log, dt, nw, S0


@pytest.fixture(params=["chunked", "scan"])
def gdn_path(request, lz):
    lib = lz.load_library()
    lib.l0b_set_gated_delta_chunked(1 if request.param == "chunked" else 0)
    yield request.param
    lib.l0b_set_gated_delta_chunked(1)


@pytest.mark.parametrize("hk,hv,dk,dv,tokens,config3", [(16, 32, 128, 128, 4096, True), (2, 4, 128, 128, 200, False),
                                                        (4, 8, 64, 64, 65, False), (4, 8, 128, 128, 16, True),
                                                        (2, 4, 64, 64, 127, True)])
def test_gated_delta_prefill_against_oracle(lz, orc, device, suite, gdn_path, hk, hv, dk, dv, tokens, config3):
    rng = RNG(tokens + 7 * hv)
    conv, z, b, a, a_log, dt, nw, S0 = _inputs(rng, hk, hv, dk, dv, tokens, config3)
    S_o = S0.copy()
    out_o = np.zeros((tokens, hv * dv), np.float32)
    orc.lib().orc_gated_delta(conv, z, b, a, a_log, dt, nw, S_o, out_o, hk, hv, dk, dv, tokens, 1e-6)
    with _buf(lz, device, conv) as cb, _buf(lz, device, z) as zb, _buf(lz, device, b) as bb, \
            _buf(lz, device, a) as ab, _buf(lz, device, a_log) as alb, _buf(lz, device, dt) as dtb, \
            _buf(lz, device, nw) as nwb, _buf(lz, device, S0) as sb, \
            lz.SharedBuffer(device, lz.F32, tokens * hv * dv) as ob:
        suite.GatedDelta.ExecuteGrouped(device, cb, zb, bb, ab, alb, dtb, nwb, sb, ob, hk, hv, dk, dv, tokens, 1e-6)
        got = ob.ToArray().reshape(tokens, -1)
        S = sb.ToArray().reshape(hv, dk, dv)
    _close(got, out_o, 1e-3, f"{gdn_path} output")
    _close(S, S_o, 1e-3, f"{gdn_path} final state")


def test_chunked_prefill_then_decode_continues_the_state(lz, orc, device, suite):
    """A chunked 300-token prefill hands its state to 3 single-token decode calls, as LlmModel does
    (prefill chunk, then Step), matching the oracle fed the 303 tokens one by one."""
    hk, hv, dk, dv, pre, dec = 16, 32, 128, 128, 300, 3
    rng = RNG(5)
    tokens = pre + dec
    conv, z, b, a, a_log, dt, nw, S0 = _inputs(rng, hk, hv, dk, dv, tokens)
    S_o = S0.copy()
    out_o = np.zeros((tokens, hv * dv), np.float32)
    orc.lib().orc_gated_delta(conv, z, b, a, a_log, dt, nw, S_o, out_o, hk, hv, dk, dv, tokens, 1e-6)
    outs = []
    with _buf(lz, device, a_log) as alb, _buf(lz, device, dt) as dtb, _buf(lz, device, nw) as nwb, \
            _buf(lz, device, S0) as sb:
        for lo, hi in [(0, pre)] + [(pre + i, pre + i + 1) for i in range(dec)]:
            n = hi - lo
            with _buf(lz, device, conv[lo:hi]) as cb, _buf(lz, device, z[lo:hi]) as zb, \
                    _buf(lz, device, b[lo:hi]) as bb, _buf(lz, device, a[lo:hi]) as ab, \
                    lz.SharedBuffer(device, lz.F32, n * hv * dv) as ob:
                suite.GatedDelta.ExecuteGrouped(device, cb, zb, bb, ab, alb, dtb, nwb, sb, ob, hk, hv, dk, dv, n, 1e-6)
                outs.append(ob.ToArray().reshape(n, -1))
        S = sb.ToArray().reshape(hv, dk, dv)
    _close(np.concatenate(outs), out_o, 1e-3, "prefill + decode output")
    _close(S, S_o, 1e-3, "final state")


def _bf16(x):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(
        np.uint16)


def test_mix_linear_layer_against_oracle(lz, orc, device, suite):
    """MixLinear at the config-3 width: bf16 in-projections (qkv, z, b, a) of the layer input, causal conv +
    SiLU with its window, the gated delta recurrence with the gated RMSNorm, bf16 out_proj; a 512-token
    prefill from a reset state, then 4 decode tokens, outputs [tokens, hidden] against the oracle."""
    H, HK, HV, DK, DV, KC = 2048, 16, 32, 128, 128, 4
    CONV, ZD = 2 * HK * DK + HV * DV, HV * DV
    pre, dec = 512, 4
    T = pre + dec
    rng = RNG(3)
    x = rng.standard_normal((T, H)).astype(np.float32)
    wq, wz, wb, wa, wo = (_bf16(rng.standard_normal(s) * 0.02) for s in
                          ((CONV, H), (ZD, H), (HV, H), (HV, H), (H, ZD)))
    conv_w = (rng.standard_normal((CONV, KC)) * 0.3).astype(np.float32)
    a_log = np.zeros(HV, np.float32)
    dt = np.zeros(HV, np.float32)
    nw = (1 + 0.1 * rng.standard_normal(DV)).astype(np.float32)
    # Oracle: the same op chain.
    qkv_o = orc.gemm_fast(x, wq, orc.BF16)
    z_o = orc.gemm_fast(x, wz, orc.BF16)
    b_o = orc.gemv_out_in(x, wb, orc.BF16)
    a_o = orc.gemv_out_in(x, wa, orc.BF16)
    hist = np.zeros((CONV, KC - 1), np.float32)
    conv_o = np.zeros_like(qkv_o)
    orc.lib().orc_causal_conv(qkv_o, hist, conv_w, conv_o, CONV, KC, T)
    S_o = np.zeros((HV, DK, DV), np.float32)
    mixed = np.zeros((T, ZD), np.float32)
    orc.lib().orc_gated_delta(conv_o, z_o, b_o, a_o, a_log, dt, nw, S_o, mixed, HK, HV, DK, DV, T, 1e-6)
    y_o = orc.gemm_fast(mixed, wo, orc.BF16)
    got = []
    def bbuf(w):
        return lz.SharedBuffer.from_array(device, w, lz.BF16)

    with bbuf(wq) as Wq, bbuf(wz) as Wz, bbuf(wb) as Wb, bbuf(wa) as Wa, bbuf(wo) as Wo, _buf(lz, device, conv_w) as cw, \
            _buf(lz, device, a_log) as alb, _buf(lz, device, dt) as dtb, _buf(lz, device, nw) as nwb, \
            lz.SharedBuffer(device, lz.F32, HV * DK * DV) as S, lz.SharedBuffer(device, lz.F32, CONV * (KC - 1)) as hb:
        for lo, hi in [(0, pre)] + [(pre + i, pre + i + 1) for i in range(dec)]:
            n = hi - lo
            with _buf(lz, device, x[lo:hi]) as xb, lz.SharedBuffer(device, lz.F32, n * CONV) as qkv, \
                    lz.SharedBuffer(device, lz.F32, n * ZD) as zb, lz.SharedBuffer(device, lz.F32, n * HV) as bb, \
                    lz.SharedBuffer(device, lz.F32, n * HV) as ab, lz.SharedBuffer(device, lz.F32, n * CONV) as cb, \
                    lz.SharedBuffer(device, lz.F32, n * ZD) as ob, lz.SharedBuffer(device, lz.F32, n * H) as yb:
                suite.linear(device, n, CONV, H, xb, Wq, None, 0, None, qkv)
                suite.linear(device, n, ZD, H, xb, Wz, None, 0, None, zb)
                suite.linear(device, n, HV, H, xb, Wb, None, 0, None, bb)
                suite.linear(device, n, HV, H, xb, Wa, None, 0, None, ab)
                suite.CausalConv.Execute(device, qkv, hb, cw, cb, CONV, KC, n)
                suite.GatedDelta.ExecuteGrouped(device, cb, zb, bb, ab, alb, dtb, nwb, S, ob, HK, HV, DK, DV, n, 1e-6)
                suite.linear(device, n, H, ZD, ob, Wo, None, 0, None, yb)
                got.append(yb.ToArray().reshape(n, H))
    got = np.concatenate(got)
    _close(got[:pre], y_o[:pre], 2e-3, "prefill output")
    _close(got[pre:], y_o[pre:], 2e-3, "decode outputs")


def test_batched_decode_equals_per_sequence_and_fork(lz, device, suite):
    """The batched decode ops (one launch for all sequences) give each sequence exactly what the
    single-sequence ops give it; a forked sequence (conv window and recurrent state copied on the device)
    then decodes exactly as its source."""
    hk, hv, dk, dv, kc, bs, steps = 16, 32, 128, 128, 4, 5, 3
    conv_dim = 2 * hk * dk + hv * dv
    rng = RNG(11)
    conv_w = (rng.standard_normal((conv_dim, kc)) * 0.3).astype(np.float32)
    a_log = np.zeros(hv, np.float32)
    dt = np.zeros(hv, np.float32)
    nw = (1 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    hist0 = rng.standard_normal((bs, conv_dim, kc - 1)).astype(np.float32)
    S0 = (rng.standard_normal((bs, hv, dk, dv)) * 0.1).astype(np.float32)
    xs = rng.standard_normal((steps, bs, conv_dim)).astype(np.float32)
    zs = rng.standard_normal((steps, bs, hv * dv)).astype(np.float32)
    bb_ = rng.standard_normal((steps, bs, hv)).astype(np.float32)
    aa_ = rng.standard_normal((steps, bs, hv)).astype(np.float32)
    with _buf(lz, device, conv_w) as cw, _buf(lz, device, a_log) as alb, _buf(lz, device, dt) as dtb, \
            _buf(lz, device, nw) as nwb, _buf(lz, device, hist0) as H, _buf(lz, device, S0) as S:
        batched = []
        for t in range(steps):
            with _buf(lz, device, xs[t]) as xb, _buf(lz, device, zs[t]) as zb, _buf(lz, device, bb_[t]) as bb, \
                    _buf(lz, device, aa_[t]) as ab, lz.SharedBuffer(device, lz.F32, bs * conv_dim) as cb, \
                    lz.SharedBuffer(device, lz.F32, bs * hv * dv) as ob:
                suite.CausalConv.ExecuteBatch(device, xb, H, cw, cb, conv_dim, kc, bs)
                suite.GatedDelta.ExecuteBatch(device, cb, zb, bb, ab, alb, dtb, nwb, S, ob, hk, hv, dk, dv, bs, 1e-6)
                batched.append(ob.ToArray().reshape(bs, -1))
        S_b, H_b = S.ToArray().reshape(S0.shape), H.ToArray().reshape(hist0.shape)
        # Fork sequence 1 onto 3, then one more batched step with equal inputs for both.
        suite.GatedDelta.ForkState(device, H, S, conv_dim, kc, hv, dk, dv, 1, 3)
        x1 = np.repeat(xs[0][1:2], bs, 0)
        z1 = np.repeat(zs[0][1:2], bs, 0)
        with _buf(lz, device, x1) as xb, _buf(lz, device, z1) as zb, _buf(lz, device, np.repeat(bb_[0][1:2], bs, 0)) as bb, \
                _buf(lz, device, np.repeat(aa_[0][1:2], bs, 0)) as ab, \
                lz.SharedBuffer(device, lz.F32, bs * conv_dim) as cb, lz.SharedBuffer(device, lz.F32, bs * hv * dv) as ob:
            suite.CausalConv.ExecuteBatch(device, xb, H, cw, cb, conv_dim, kc, bs)
            suite.GatedDelta.ExecuteBatch(device, cb, zb, bb, ab, alb, dtb, nwb, S, ob, hk, hv, dk, dv, bs, 1e-6)
            after = ob.ToArray().reshape(bs, -1)
        np.testing.assert_array_equal(after[1], after[3])
        for q in range(bs):
            with _buf(lz, device, hist0[q]) as H1, _buf(lz, device, S0[q]) as S1:
                for t in range(steps):
                    with _buf(lz, device, xs[t][q]) as xb, _buf(lz, device, zs[t][q]) as zb, \
                            _buf(lz, device, bb_[t][q]) as bb, _buf(lz, device, aa_[t][q]) as ab, \
                            lz.SharedBuffer(device, lz.F32, conv_dim) as cb, \
                            lz.SharedBuffer(device, lz.F32, hv * dv) as ob:
                        suite.CausalConv.Execute(device, xb, H1, cw, cb, conv_dim, kc, 1)
                        suite.GatedDelta.ExecuteGrouped(device, cb, zb, bb, ab, alb, dtb, nwb, S1, ob, hk, hv, dk, dv,
                                                        1, 1e-6)
                        np.testing.assert_array_equal(ob.ToArray(), batched[t][q])
                np.testing.assert_array_equal(S1.ToArray().reshape(S0.shape[1:]), S_b[q])
                np.testing.assert_array_equal(H1.ToArray().reshape(hist0.shape[1:]), H_b[q])
