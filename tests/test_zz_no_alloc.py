"""The allocation-free decode attention entry point (l0b_attention_decode_noalloc).

It exists for callers that cannot let a call allocate device memory (a server that plans all of HBM
at start-up, code running while another runtime owns the allocator, a host that must not block in
cudaMalloc mid-step). Its scratch is a fixed array inside the library, so two calls in a row must both
agree with the regular entry point (l0b_attention_execute) and with the CPU oracle's attention
(oracle/l0b_oracle.c orc_attention), the second call reusing what the first left in that scratch.
Kept in its own file so a run that stops at the first failure has run every other test first.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(lz, stream, q, kc, vc, cache_dtype, out, hd, nh, nkv, seq, max_seq):
    L = lz.load_library()
    fn = L.l0b_attention_decode_noalloc
    fn.restype = C.c_int32
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_int32,
                   C.c_int32, C.c_int32, C.c_int32]
    lz.check(fn(stream, C.c_void_p(q.Pointer), C.c_void_p(kc.Pointer), C.c_void_p(vc.Pointer), cache_dtype,
                C.c_void_p(out.Pointer), hd, nh, nkv, seq, max_seq))


def test_noalloc_attention_matches_regular_entry_twice(lz, device, suite):
    from oracle import oracle as orc

    stream = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(device.handle, C.byref(stream)))
    hd, nh, nkv, max_seq = 128, 28, 4, 4096
    for call, seq in enumerate((3000, 1777)):
        rng = np.random.default_rng(100 + call)
        kc = rng.standard_normal((max_seq, nkv * hd)).astype(np.float16)
        vc = rng.standard_normal((max_seq, nkv * hd)).astype(np.float16)
        q = (rng.standard_normal(nh * hd) * 0.3).astype(np.float32)
        with lz.SharedBuffer.from_array(device, q) as qb, lz.SharedBuffer.from_array(device, kc) as kb, \
                lz.SharedBuffer.from_array(device, vc) as vb, lz.SharedBuffer(device, lz.F32, nh * hd) as want, \
                lz.SharedBuffer(device, lz.F32, nh * hd) as got:
            suite.Attention.Execute(device, qb, kb, vb, want, hd, nh, nkv, seq, max_seq)
            _noalloc(lz, stream, qb, kb, vb, lz.F16, got, hd, nh, nkv, seq, max_seq)
            device.Synchronize()
            a, b = got.ToArray(), want.ToArray()
        np.testing.assert_allclose(a, b, atol=1e-4, rtol=1e-3)
        ref = orc.attention(q[None, :], kc.view(np.uint16), vc.view(np.uint16), orc.F16, hd, nh, nkv, seq - 1, 1)[0]
        np.testing.assert_allclose(a, ref, atol=1e-4, rtol=1e-3)


def test_noalloc_rejects_sizes_beyond_its_scratch(lz, device):
    stream = C.c_void_p()
    lz.check(lz.load_library().l0b_device_stream(device.handle, C.byref(stream)))
    with lz.SharedBuffer(device, lz.F32, 128) as b:
        with pytest.raises(lz.ArgumentOutOfRangeException):
            # 16384 heads x 130 floats per split exceed the 1,048,576-float scratch.
            _noalloc(lz, stream, b, b, b, lz.F32, b, 128, 16384, 1, 1, 1)
