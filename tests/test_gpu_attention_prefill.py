"""Prefill attention (Attention.ExecutePrefill, L/LlmDecoderLayer.cs:369-371) on the tensor-core kernel
against the oracle and against the scalar kernel.

The tensor-core kernel takes f16 / bf16 caches: queries and probabilities enter the MMA as hi + lo
16-bit halves against exact 16-bit keys and values, so its results stay within fp32-accumulation
distance of the oracle's double-precision softmax. Cases: both head dims, the config-2 (28 / 4 heads)
and config-4 (64 / 8) GQA shapes, chunks that continue a cache (pos0 > 0), partial 64-row tiles and
a 2048-token chunk.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["mma", "scalar"])
def kernel(request, lz):
    lib = lz.load_library()
    lib.l0b_set_attention_prefill_tensor_cores(1 if request.param == "mma" else 0)
    yield request.param
    lib.l0b_set_attention_prefill_tensor_cores(1)


def _bits(x, dt):
    import torch

    if dt == "f16":
        return x.astype(np.float16).view(np.uint16)
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(
        np.uint16)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("hd,nh,nkv,pos0,tokens", [(128, 28, 4, 0, 512), (128, 28, 4, 300, 77), (64, 14, 2, 5, 130),
                                                   (128, 64, 8, 0, 2048), (64, 8, 8, 63, 2), (128, 8, 1, 1000, 65)])
def test_prefill_attention_against_oracle(lz, orc, device, suite, kernel, dt, hd, nh, nkv, pos0, tokens):
    if tokens == 2048 and kernel == "scalar":
        pytest.skip("the scalar kernel at 2048 rows is the slow reference path; covered at smaller sizes")
    rng = np.random.default_rng(hd + nh + pos0 + tokens)
    kvd = nkv * hd
    max_seq = pos0 + tokens + 3
    kc = rng.standard_normal((max_seq, kvd)).astype(np.float32)
    vc = rng.standard_normal((max_seq, kvd)).astype(np.float32)
    q = (rng.standard_normal((tokens, nh * hd)) * 0.5).astype(np.float32)
    kb_, vb_ = _bits(kc, dt), _bits(vc, dt)
    want = orc.attention(q, kb_, vb_, orc.F16 if dt == "f16" else orc.BF16, hd, nh, nkv, pos0, tokens)
    ldt = lz.F16 if dt == "f16" else lz.BF16
    with lz.SharedBuffer.from_array(device, q) as qb, lz.SharedBuffer.from_array(device, kb_, ldt) as kb, \
            lz.SharedBuffer.from_array(device, vb_, ldt) as vb, lz.SharedBuffer(device, lz.F32, tokens * nh * hd) as ob:
        suite.Attention.ExecutePrefill(device, qb, kb, vb, ob, hd, nh, nkv, pos0, tokens, max_seq)
        got = ob.ToArray().reshape(tokens, -1)
    err = np.abs(got - want)
    assert err.max() <= 2e-5 + 2e-4 * np.abs(want).max(), f"max err {err.max()}"
