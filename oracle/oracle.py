"""ctypes wrapper of the CPU oracle (liboracle.so). TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and reference arms, as the
checker of the CUDA backend. See l0b_oracle.h for what each function restates and what pins it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

F32, F16, BF16, I8 = 0, 1, 2, 3
ROPE_DEFAULT, ROPE_LINEAR, ROPE_YARN, ROPE_LLAMA3 = 0, 1, 2, 3

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")


def build() -> Path:
    """Compiles liboracle.so with the committed Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


class OrcConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("inter", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
        ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("max_pos", C.c_int),
        ("eps", C.c_float), ("theta", C.c_double), ("tie", C.c_int), ("bias", C.c_int), ("qk_norm", C.c_int),
        ("rope_type", C.c_int), ("rope_factor", C.c_double), ("rope_original_max", C.c_int),
        ("rope_low", C.c_double), ("rope_high", C.c_double), ("rope_beta_fast", C.c_double),
        ("rope_beta_slow", C.c_double), ("rope_attention", C.c_double),
        ("wdtype", C.c_int), ("group", C.c_int), ("kv_dtype", C.c_int),
        ("linear_mask", C.c_uint64), ("lin_k_heads", C.c_int), ("lin_v_heads", C.c_int), ("lin_k_dim", C.c_int),
        ("lin_v_dim", C.c_int), ("lin_conv", C.c_int), ("attn_gate", C.c_int), ("norm_offset", C.c_float),
        ("partial_rotary", C.c_double),
    ]


_lib = None
PROBE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_float), C.c_int64)


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = C.CDLL(str(LIB_PATH))
    vp = C.c_void_p
    L.orc_f32_to_f16.restype = C.c_uint16
    L.orc_f32_to_f16.argtypes = [C.c_float]
    L.orc_f16_to_f32.restype = C.c_float
    L.orc_f16_to_f32.argtypes = [C.c_uint16]
    L.orc_f32_to_bf16.restype = C.c_uint16
    L.orc_f32_to_bf16.argtypes = [C.c_float]
    L.orc_gemv_out_in.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, C.c_int, vp, vp, C.c_int, _f32p]
    L.orc_gemv_in_out.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, C.c_int, vp, _f32p]
    L.orc_q8_quantize.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _i8p, _u16p]
    L.orc_rmsnorm.argtypes = [_f32p, vp, _f32p, _f32p, C.c_float, C.c_int, C.c_int, C.c_int]
    L.orc_bias_add.argtypes = [_f32p, _f32p, C.c_int, C.c_int]
    L.orc_swiglu.argtypes = [_f32p, _f32p, C.c_int64]
    L.orc_add.argtypes = [_f32p, _f32p, C.c_int64]
    L.orc_sigmoid_gate.argtypes = [_f32p, _f32p, C.c_int64]
    L.orc_embedding.argtypes = [_i32p, vp, C.c_int, _f32p, C.c_int, C.c_int64]
    L.orc_rope_frequencies.restype = C.c_int
    L.orc_rope_frequencies.argtypes = [C.c_int, C.c_double, C.c_int, C.c_int, C.c_double, C.c_int, C.c_double,
                                       C.c_double, C.c_double, C.c_double, C.c_double, C.c_double, C.c_double,
                                       C.c_int, _f32p, C.POINTER(C.c_float)]
    L.orc_rope.argtypes = [_f32p, _f32p, _i32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int]
    L.orc_kv_store.argtypes = [_f32p, _f32p, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int]
    L.orc_attention.argtypes = [_f32p, vp, vp, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    L.orc_argmax.restype = C.c_int
    L.orc_argmax.argtypes = [_f32p, C.c_int]
    L.orc_sample.restype = C.c_int
    L.orc_sample.argtypes = [_f32p, C.c_int, C.c_float, C.c_float]
    L.orc_sampler.restype = C.c_int
    L.orc_sampler.argtypes = [_f32p, C.c_int, vp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, C.c_double]
    L.orc_sample_uniform.restype = C.c_double
    L.orc_sample_uniform.argtypes = [C.c_uint64, C.c_int]
    L.orc_tensor_stream.restype = C.c_uint64
    L.orc_tensor_stream.argtypes = [C.c_uint64, C.c_uint64]
    L.orc_synth_fill.argtypes = [vp, C.c_int, C.c_int64, C.c_uint64, C.c_int, C.c_float, C.c_float, C.c_int64,
                                 C.c_int64, C.c_int64, C.c_int64]
    L.orc_causal_conv.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]
    L.orc_gated_delta.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_float]
    L.orc_gemm_fast.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, C.c_int, vp, vp, C.c_int, _f32p]
    L.orc_model_create.restype = vp
    L.orc_model_create.argtypes = [C.POINTER(OrcConfig), C.c_int]
    L.orc_model_create_batch.restype = vp
    L.orc_model_create_batch.argtypes = [C.POINTER(OrcConfig), C.c_int, C.c_int]
    L.orc_model_set_fast.argtypes = [vp, C.c_int]
    L.orc_model_forward.restype = C.c_int
    L.orc_model_forward.argtypes = [vp, C.c_int, _i32p, _i32p, vp, vp, C.c_int]
    L.orc_model_read_kv_seq.restype = C.c_int
    L.orc_model_read_kv_seq.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
    L.orc_model_write_kv_seq.restype = C.c_int
    L.orc_model_write_kv_seq.argtypes = [vp, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
    L.orc_model_free.argtypes = [vp]
    L.orc_model_init_synthetic.argtypes = [vp, C.c_uint64, C.c_float, C.c_float, C.c_float]
    L.orc_model_set_tensor.restype = C.c_int
    L.orc_model_set_tensor.argtypes = [vp, C.c_char_p, _f32p, C.c_int64]
    L.orc_model_step.restype = C.c_int
    L.orc_model_step.argtypes = [vp, C.c_int, C.c_int, vp]
    L.orc_model_set_layer_limit.argtypes = [vp, C.c_int]
    L.orc_model_read_kv.restype = C.c_int
    L.orc_model_read_kv.argtypes = [vp, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
    L.orc_model_set_probe.argtypes = [vp, PROBE_FN, vp]
    L.orc_num_threads.restype = C.c_int
    L.orc_set_num_threads.argtypes = [C.c_int]
    _lib = L
    return L


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits with the oracle's own round-to-nearest-even conversion."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    L = lib()
    return np.array([L.orc_f32_to_f16(float(v)) for v in x], np.uint16)


def sampler(logits: np.ndarray, ctx, temperature: float, top_p: float, top_k: int, penalty: float, u: float) -> int:
    """LlmSampler.Sample (src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) with the draw u given."""
    lg = np.ascontiguousarray(logits, np.float32)
    c = None if ctx is None or len(ctx) == 0 else np.ascontiguousarray(ctx, np.int32)
    return lib().orc_sampler(lg, lg.size, _ptr(c), 0 if c is None else c.size, temperature, top_p, top_k, penalty, u)


def sample_uniform(seed: int, p: int) -> float:
    """The device sampled decode's draw for the token at position p."""
    return lib().orc_sample_uniform(seed, p)


def gemv_out_in(x: np.ndarray, w: np.ndarray, wdtype: int, scales: np.ndarray | None = None,
                group: int = 0) -> np.ndarray:
    """y = x @ W^T for W [N, K] stored as f32 / f16 bits / bf16 bits / int8 (+ f16-bit scales)."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    lib().orc_gemv_out_in(M, N, K, x.reshape(M, K), wdtype, _ptr(np.ascontiguousarray(w)),
                          _ptr(None if scales is None else np.ascontiguousarray(scales)), group, y)
    return y


def gemm_fast(x: np.ndarray, w: np.ndarray, wdtype: int, scales: np.ndarray | None = None,
              group: int = 0) -> np.ndarray:
    """gemv_out_in accumulated in fp32 with FMA (the timing build)."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = w.shape[0]
    y = np.zeros((M, N), np.float32)
    lib().orc_gemm_fast(M, N, K, x.reshape(M, K), wdtype, _ptr(np.ascontiguousarray(w)),
                        _ptr(None if scales is None else np.ascontiguousarray(scales)), group, y)
    return y


def gemv_in_out(x: np.ndarray, w: np.ndarray, half: bool) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.reshape(-1, x.shape[-1]).shape
    N = w.shape[1]
    y = np.zeros((M, N), np.float32)
    lib().orc_gemv_in_out(M, N, K, x.reshape(M, K), 1 if half else 0, _ptr(np.ascontiguousarray(w)), y)
    return y


def q8_quantize(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    g = group if group > 0 else K
    q = np.zeros((N, K), np.int8)
    s = np.zeros((N, K // g), np.uint16)
    lib().orc_q8_quantize(w, N, K, g, q, s)
    return q, s


def rmsnorm(x, w, eps, res=None):
    x = np.array(x, np.float32, copy=True)
    rows, width = x.reshape(-1, w.shape[0]).shape
    out = np.zeros_like(x)
    r = None if res is None else np.ascontiguousarray(res, np.float32)
    lib().orc_rmsnorm(x, _ptr(r), np.ascontiguousarray(w, np.float32), out, eps, width, rows, 0 if res is None else 1)
    return x, out


def rope_frequencies(dim, theta, max_pos, rope_type=ROPE_DEFAULT, factor=1.0, original_max=0, low=1.0, high=4.0,
                     beta_fast=32.0, beta_slow=1.0, attention_factor=0.0, mscale=0.0, mscale_all_dim=0.0,
                     truncate=True):
    out = np.zeros(dim // 2, np.float32)
    att = C.c_float(0)
    n = lib().orc_rope_frequencies(dim, theta, max_pos, rope_type, factor, original_max, low, high, beta_fast,
                                   beta_slow, attention_factor, mscale, mscale_all_dim, 1 if truncate else 0, out,
                                   C.byref(att))
    return out[:n], float(att.value)


def rope(q, k, positions, inv_freq, hd, nh, nkv, attn_scale=1.0, rot=None):
    q = np.array(q, np.float32, copy=True)
    k = np.array(k, np.float32, copy=True)
    pos = np.ascontiguousarray(positions, np.int32)
    rot = rot or hd
    lib().orc_rope(q, k, pos, np.ascontiguousarray(inv_freq, np.float32), hd, nh, nkv, attn_scale, rot, len(pos))
    return q, k


def attention(q, kc, vc, cache_dtype, hd, nh, nkv, pos0, tokens):
    out = np.zeros((tokens, nh * hd), np.float32)
    lib().orc_attention(np.ascontiguousarray(q, np.float32), _ptr(np.ascontiguousarray(kc)),
                        _ptr(np.ascontiguousarray(vc)), cache_dtype, out, hd, nh, nkv, pos0, tokens)
    return out


def synth_fill(count, dtype, seed, tensor_id, mode, a, b=0.0, row_len=0, full_len=0, row0=0, col0=0):
    np_dt = {F32: np.float32, F16: np.uint16, BF16: np.uint16, I8: np.int8}[dtype]
    out = np.zeros(count, np_dt)
    L = lib()
    L.orc_synth_fill(_ptr(out), dtype, count, L.orc_tensor_stream(seed, tensor_id), mode, a, b, row_len, full_len,
                     row0, col0)
    return out


class OracleModel:
    """The whole decoder on the CPU, one token per step (LlmModel.Step semantics)."""

    def __init__(self, cfg: dict, max_seq: int, batch: int = 1):
        c = OrcConfig()
        for k, v in cfg.items():
            setattr(c, k, v)
        self.cfg = cfg
        self._h = lib().orc_model_create_batch(C.byref(c), max_seq, batch)
        if not self._h:
            raise MemoryError("oracle model allocation failed")
        self.vocab = cfg["vocab"]
        self.kv_dim = cfg["kv_heads"] * cfg["head_dim"]

    def set_fast(self, fast: bool):
        """fp32-accumulate projections (timing build, relative error ~1e-6) instead of double."""
        lib().orc_model_set_fast(self._h, 1 if fast else 0)

    def forward(self, tokens, positions, seqs=None, last_only: bool = False) -> np.ndarray:
        """Rows of (token, position, sequence) at once: a causal prefill chunk or a decode batch."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        sq = None if seqs is None else np.ascontiguousarray(seqs, np.int32)
        logits = np.zeros((1 if last_only else t.size, self.vocab), np.float32)
        rc = lib().orc_model_forward(self._h, t.size, t, p, _ptr(sq), _ptr(logits), 1 if last_only else 0)
        if rc != 0:
            raise ValueError(f"oracle forward failed ({rc})")
        return logits[0] if last_only else logits

    def prefill(self, prompt, seq: int = 0, chunk: int = 512) -> np.ndarray:
        """LlmModel.Prefill of sequence `seq` from position 0; the last position's logits."""
        prompt = np.asarray(prompt, np.int32)
        lg = None
        for s0 in range(0, prompt.size, chunk):
            part = prompt[s0:s0 + chunk]
            last = s0 + part.size == prompt.size
            lg = self.forward(part, np.arange(s0, s0 + part.size), np.full(part.size, seq), last_only=True)
        return lg

    def write_kv(self, layer: int, row0: int, keys: np.ndarray, values: np.ndarray, seq: int = 0):
        k = np.ascontiguousarray(keys, np.float32).reshape(-1, self.kv_dim)
        v = np.ascontiguousarray(values, np.float32).reshape(-1, self.kv_dim)
        if lib().orc_model_write_kv_seq(self._h, layer, seq, row0, k.shape[0], k, v) != 0:
            raise ValueError("oracle write_kv failed")

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def init_synthetic(self, seed: int, std: float, scale_lo: float = 1e-3, scale_hi: float = 2e-2):
        lib().orc_model_init_synthetic(self._h, seed, std, scale_lo, scale_hi)

    def set_tensor(self, name: str, data: np.ndarray):
        d = np.ascontiguousarray(data, np.float32).ravel()
        rc = lib().orc_model_set_tensor(self._h, name.encode(), d, d.size)
        if rc != 0:
            raise ValueError(f"oracle rejected tensor {name} ({rc})")

    def step(self, token: int, position: int, want_logits: bool = True) -> np.ndarray | None:
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        rc = lib().orc_model_step(self._h, token, position, _ptr(logits))
        if rc != 0:
            raise ValueError("oracle step failed")
        return logits

    def set_probe(self, fn):
        """fn(layer, stage, values) after each stage of each layer; None removes it."""
        if fn is None:
            self._probe = None
            lib().orc_model_set_probe(self._h, PROBE_FN(), None)
            return
        self._probe = PROBE_FN(lambda _u, layer, stage, vals, n: fn(layer, stage.decode(),
                                                                        np.ctypeslib.as_array(vals, (n,)).copy()))
        lib().orc_model_set_probe(self._h, self._probe, None)

    def set_layer_limit(self, n: int):
        lib().orc_model_set_layer_limit(self._h, n)

    def read_kv(self, layer: int, row0: int, rows: int, kv_dim: int, seq: int = 0):
        k = np.zeros(rows * kv_dim, np.float32)
        v = np.zeros(rows * kv_dim, np.float32)
        lib().orc_model_read_kv_seq(self._h, layer, seq, row0, rows, k, v)
        return k.reshape(rows, kv_dim), v.reshape(rows, kv_dim)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(n)


if __name__ == "__main__":
    print(build())
    os.environ.setdefault("OMP_NUM_THREADS", "1")
