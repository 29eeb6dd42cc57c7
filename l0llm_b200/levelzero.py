"""Python mirror of the reference's kernel surface, bound to libl0b200.so through ctypes.

Names follow the C# types the l0llm decoder calls (LevelZero.NET 2.0.0): LevelZeroRuntime,
ComputeDevice, SharedBuffer, LlmKernelSuite with its ops (suite.Gemv.Execute(...), ...), and the
model host LlmModel. Errors raise the exception types the reference throws. There is no CPU fallback:
every op runs on the sm_100 device through the native library, and importing this module without the
built library raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libl0b200.so"

F32, F16, BF16, I8, I32, U8 = 0, 1, 2, 3, 4, 5
NP_DTYPE = {F32: np.float32, F16: np.float16, BF16: np.uint16, I8: np.int8, I32: np.int32, U8: np.uint8}
PRECISION = {"auto": 0, "float32": 1, "float16": 2, "int8": 3, "bfloat16": 4}
ROPE_TYPES = {"default": 0, "linear": 1, "yarn": 2, "llama3": 3}


class L0bError(RuntimeError):
    status = -1


class ArgumentException(L0bError, ValueError):
    status = 1


class ArgumentOutOfRangeException(ArgumentException):
    status = 2


class NotSupportedException(L0bError):
    status = 3


class InvalidOperationException(L0bError):
    status = 4


class InvalidDataException(L0bError):
    status = 5


class CudaError(L0bError):
    status = 6


class OutOfMemoryError(L0bError, MemoryError):
    status = 7


class NoDeviceError(L0bError):
    status = 8


class DeviceTimeoutError(L0bError):
    status = 9


class NcclError(L0bError):
    status = 10


_ERRORS = {c.status: c for c in (ArgumentException, ArgumentOutOfRangeException, NotSupportedException,
                                  InvalidOperationException, InvalidDataException, CudaError, OutOfMemoryError,
                                  NoDeviceError, DeviceTimeoutError, NcclError)}


class ModelConfig(C.Structure):
    """l0b_model_config: the HfModelConfig fields the decoder reads."""

    _fields_ = [
        ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32), ("num_layers", C.c_int32),
        ("num_attention_heads", C.c_int32), ("num_key_value_heads", C.c_int32), ("head_dim", C.c_int32),
        ("vocab_size", C.c_int32), ("max_position_embeddings", C.c_int32), ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_double), ("tie_word_embeddings", C.c_int32), ("attention_bias", C.c_int32),
        ("qk_norm", C.c_int32), ("rope_type", C.c_int32), ("rope_factor", C.c_double),
        ("rope_original_max_position", C.c_int32), ("rope_low_freq_factor", C.c_double),
        ("rope_high_freq_factor", C.c_double), ("rope_beta_fast", C.c_double), ("rope_beta_slow", C.c_double),
        ("rope_attention_factor", C.c_double), ("rope_mscale", C.c_double), ("rope_mscale_all_dim", C.c_double),
        ("rope_truncate", C.c_int32), ("partial_rotary_factor", C.c_double), ("kv_dtype", C.c_int32),
        ("q8_group", C.c_int32), ("tp_size", C.c_int32), ("tp_rank", C.c_int32), ("max_batch", C.c_int32),
        ("linear_layer_mask", C.c_uint64), ("linear_num_key_heads", C.c_int32),
        ("linear_num_value_heads", C.c_int32), ("linear_key_head_dim", C.c_int32),
        ("linear_value_head_dim", C.c_int32), ("linear_conv_kernel", C.c_int32),
        ("attention_output_gate", C.c_int32), ("rms_norm_offset", C.c_float),
    ]


_lib: C.CDLL | None = None
PROBE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int32, C.c_char_p, C.POINTER(C.c_float), C.c_int64)


def load_library() -> C.CDLL:
    """Loads libl0b200.so (built by l0llm_b200.build); raises when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m l0llm_b200.build` "
                          "(there is no CPU fallback)")
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float
    pp = C.POINTER(C.c_void_p)
    sigs = {
        "l0b_last_error": (C.c_char_p, []),
        "l0b_version": (i32, []),
        "l0b_kernel_launch_count": (i64, []),
        "l0b_runtime_is_available": (i32, [C.POINTER(i32)]),
        "l0b_device_count": (i32, [C.POINTER(i32)]),
        "l0b_device_info": (i32, [i32, C.c_char_p, i32, C.POINTER(i32), C.POINTER(i64)]),
        "l0b_device_create": (i32, [i32, pp]),
        "l0b_device_free": (i32, [vp]),
        "l0b_device_begin_recording": (i32, [vp]),
        "l0b_device_end_recording": (i32, [vp]),
        "l0b_device_abort_recording": (i32, [vp]),
        "l0b_device_is_recording": (i32, [vp, C.POINTER(i32)]),
        "l0b_device_synchronize": (i32, [vp]),
        "l0b_device_stream": (i32, [vp, pp]),
        "l0b_device_graph_stats": (i32, [vp, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
        "l0b_device_set_pdl": (i32, [vp, i32]),
        "l0b_buffer_alloc": (i32, [vp, i32, i64, pp]),
        "l0b_buffer_alloc_from": (i32, [vp, i32, i64, vp, pp]),
        "l0b_buffer_view": (i32, [vp, i64, i64, pp]),
        "l0b_buffer_free": (i32, [vp]),
        "l0b_buffer_write": (i32, [vp, i64, vp, i64]),
        "l0b_buffer_read": (i32, [vp, i64, vp, i64]),
        "l0b_buffer_copy": (i32, [vp, i64, vp, i64, i64]),
        "l0b_buffer_zero": (i32, [vp]),
        "l0b_buffer_count": (i32, [vp, C.POINTER(i64)]),
        "l0b_buffer_dtype": (i32, [vp, C.POINTER(i32)]),
        "l0b_buffer_device_ptr": (i32, [vp, pp]),
        "l0b_suite_create": (i32, [vp, pp]),
        "l0b_suite_free": (i32, [vp]),
        "l0b_suite_has_q8": (i32, [vp]),
        "l0b_suite_ensure_q8_scratch": (i32, [vp, i32, i32]),
        "l0b_suite_q8_scratch_rows": (i32, [vp]),
        "l0b_gemv_supports": (i32, [i32]),
        "l0b_gemv_max_rows": (i32, []),
        "l0b_gemv_q8_supports": (i32, [i32, i32]),
        "l0b_gemv_q8_group_size": (i32, []),
        "l0b_q8_quantize_out_in": (i32, [vp, i32, i32, i32, vp, vp]),
        "l0b_q8_quantize_device": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "l0b_embedding_execute": (i32, [vp, vp, vp, vp, vp, i32, i32]),
        "l0b_rmsnorm_execute": (i32, [vp, vp, vp, vp, vp, vp, f32, i32, i32, i32]),
        "l0b_gemv_execute": (i32, [vp, vp, i32, i32, vp, vp, vp]),
        "l0b_gemv_execute_rows": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "l0b_gemm_execute": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "l0b_gemv_q8_quantize": (i32, [vp, vp, i32, i32, vp]),
        "l0b_gemv_q8_execute": (i32, [vp, vp, i32, i32, vp, vp, vp]),
        "l0b_gemv_q8_execute_rows": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "l0b_bias_add_execute": (i32, [vp, vp, vp, vp, i32, i32]),
        "l0b_rope_execute": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, f32, i32]),
        "l0b_rope_execute_with_frequencies": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, f32, i32, i32]),
        "l0b_kv_cache_store_execute": (i32, [vp, vp, vp, vp, vp, vp, i32, i32]),
        "l0b_kv_cache_store_execute_rows": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32]),
        "l0b_attention_execute": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32]),
        "l0b_attention_execute_prefill": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32]),
        "l0b_sigmoid_gate_execute": (i32, [vp, vp, vp, vp, i32]),
        "l0b_swiglu_execute": (i32, [vp, vp, vp, vp, i32]),
        "l0b_add_execute": (i32, [vp, vp, vp, vp, i32]),
        "l0b_copy_execute": (i32, [vp, vp, vp, vp, i32, i32]),
        "l0b_sampling_execute": (i32, [vp, vp, vp, vp, f32, f32, i32]),
        "l0b_causal_conv_execute": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32]),
        "l0b_gated_delta_execute": (i32, [vp, vp] + [vp] * 9 + [i32, i32, i32, i32, f32]),
        "l0b_gated_delta_execute_grouped": (i32, [vp, vp] + [vp] * 9 + [i32, i32, i32, i32, i32, f32]),
        "l0b_causal_conv_execute_batch": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32]),
        "l0b_gated_delta_execute_batch": (i32, [vp, vp] + [vp] * 9 + [i32, i32, i32, i32, i32, f32]),
        "l0b_linear_state_fork": (i32, [vp, vp, vp, vp] + [i32] * 7),
        "l0b_set_gated_delta_chunked": (i32, [i32]),
        "l0b_set_weight_blocking": (i32, [i32]),
        "l0b_linear": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, vp]),
        "l0b_gemv_w8a16_raw": (i32, [vp, i32, i32, i32, vp, i32, vp, vp, i32, vp, i32]),
        "l0b_linear_fused": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, f32, i32, vp, vp]),
        "l0b_linear_tc": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, f32, i32, vp, vp]),
        "l0b_linear_tc_scaled": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, f32, i32, vp, vp]),
        "l0b_tc_set_max_splits": (i32, [i32]),
        "l0b_set_gemv_bulk": (i32, [i32]),
        "l0b_set_gemv_fill_split": (i32, [i32]),
        "l0b_set_gemv_bulk_short_rows": (i32, [i32]),
        "l0b_set_gemv_ksplit": (i32, [i32]),
        "l0b_set_gemv_ksplit_stages": (i32, [i32]),
        "l0b_set_l2_prefetch": (i32, [i32]),
        "l0b_set_gemv_bulk_stages": (i32, [i32]),
        "l0b_set_attention_cluster16": (i32, [i32]),
        "l0b_set_attention_decode_tensor_cores": (i32, [i32]),
        "l0b_comm_set_fused_allreduce": (i32, [i32]),
        "l0b_sample_execute": (i32, [vp, vp, vp, i32, vp, i32, f32, f32, i32, f32, C.c_double, vp]),
        "l0b_model_sample_logits": (i32, [vp, f32, f32, i32, f32, C.c_uint64, vp, i32, C.POINTER(i32)]),
        "l0b_model_decode_sample_device": (i32, [vp, i32, f32, f32, i32, f32, C.c_uint64, vp]),
        "l0b_model_fork_sequence": (i32, [vp, i32, i32, i32]),
        "l0b_device_error_status": (i32, [vp, C.POINTER(i32)]),
        "l0b_set_gemv_tensor_cores": (i32, [i32]),
        "l0b_comm_unique_id": (i32, [vp, i32]),
        "l0b_comm_create": (i32, [vp, vp, i32, i32, i32, pp]),
        "l0b_comm_free": (i32, [vp]),
        "l0b_comm_allreduce": (i32, [vp, vp, i64]),
        "l0b_model_prefill_sequence": (i32, [vp, i32, vp, i32, vp]),
        "l0b_model_decode_batch": (i32, [vp, vp, vp, i32, vp]),
        "l0b_model_decode_greedy_device_batch": (i32, [vp, i32, i32, vp]),
        "l0b_model_sequence_position": (i32, [vp, i32, C.POINTER(i32)]),
        "l0b_attention_decode_noalloc": (i32, [vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32]),
        "l0b_model_config_init": (i32, [C.POINTER(ModelConfig)]),
        "l0b_linear_shared": (i32, [vp, vp, i32, i32, vp, vp, vp, i32, i32, vp, vp, vp]),
        "l0b_model_shard_plan": (i32, [C.POINTER(ModelConfig), C.c_char_p, vp]),
        "l0b_rope_frequencies": (i32, [C.POINTER(ModelConfig), vp, i32, C.POINTER(i32), C.POINTER(f32)]),
        "l0b_model_create": (i32, [vp, vp, C.POINTER(ModelConfig), i32, i32, vp, pp]),
        "l0b_model_free": (i32, [vp]),
        "l0b_model_set_tensor": (i32, [vp, C.c_char_p, vp, i64]),
        "l0b_model_init_synthetic": (i32, [vp, C.c_uint64, f32, f32, f32]),
        "l0b_model_set_tensor_raw": (i32, [vp, C.c_char_p, vp, i32, i64]),
        "l0b_model_prefill": (i32, [vp, vp, i32, vp]),
        "l0b_model_decode": (i32, [vp, i32, vp]),
        "l0b_model_compute_logits": (i32, [vp, i32, i32, vp]),
        "l0b_model_generate_greedy": (i32, [vp, vp, i32, i32, vp, i32, vp, C.POINTER(i32)]),
        "l0b_model_position": (i32, [vp, C.POINTER(i32)]),
        "l0b_model_reset_sequence": (i32, [vp]),
        "l0b_model_projection_bytes": (i32, [vp, C.POINTER(i64)]),
        "l0b_model_decode_greedy_device": (i32, [vp, i32, vp]),
        "l0b_model_set_recording": (i32, [vp, i32]),
        "l0b_model_set_fused": (i32, [vp, i32]),
        "l0b_model_set_gemm_rows": (i32, [vp, i32]),
        "l0b_model_read_kv": (i32, [vp, i32, i32, i32, vp, vp]),
        "l0b_model_set_probe": (i32, [vp, PROBE_FN, vp]),
        "l0b_model_read_weight": (i32, [vp, i32, i32, vp, i64]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int) -> None:
    if status != 0:
        msg = load_library().l0b_last_error().decode(errors="replace")
        raise _ERRORS.get(status, L0bError)(msg or f"status {status}")


def _p(arr: np.ndarray | None):
    return None if arr is None else arr.ctypes.data_as(C.c_void_p)


def _h(obj):
    return None if obj is None else obj.handle


# -------------------------------------------------------------------------------------------------
# Runtime, device, buffers
# -------------------------------------------------------------------------------------------------

class LevelZeroRuntime:
    @staticmethod
    def IsAvailable() -> bool:
        v = C.c_int32(0)
        check(load_library().l0b_runtime_is_available(C.byref(v)))
        return bool(v.value)

    @staticmethod
    def GetDefaultDevice() -> "ComputeDevice":
        return ComputeDevice(0)

    @staticmethod
    def GetDevice(index: int) -> "ComputeDevice":
        return ComputeDevice(index)

    @staticmethod
    def EnumerateDevices() -> list[tuple[int, str]]:
        n = C.c_int32(0)
        check(load_library().l0b_device_count(C.byref(n)))
        out = []
        for i in range(n.value):
            name = C.create_string_buffer(256)
            check(load_library().l0b_device_info(i, name, 256, None, None))
            out.append((i, name.value.decode()))
        return out


class ComputeDevice:
    def __init__(self, index: int = 0):
        h = C.c_void_p()
        check(load_library().l0b_device_create(index, C.byref(h)))
        self.handle = h
        self.index = index

    def AllocShared(self, dtype_or_data, count: int | None = None) -> "SharedBuffer":
        """AllocShared<T>(count) with a dtype code, or AllocShared(T[] data) with a numpy array."""
        if isinstance(dtype_or_data, np.ndarray):
            return SharedBuffer.from_array(self, dtype_or_data)
        return SharedBuffer(self, dtype_or_data, count)

    def BeginRecording(self):
        check(load_library().l0b_device_begin_recording(self.handle))

    def EndRecording(self):
        check(load_library().l0b_device_end_recording(self.handle))

    def AbortRecording(self):
        check(load_library().l0b_device_abort_recording(self.handle))

    @property
    def IsRecording(self) -> bool:
        v = C.c_int32()
        check(load_library().l0b_device_is_recording(self.handle, C.byref(v)))
        return bool(v.value)

    def Synchronize(self):
        check(load_library().l0b_device_synchronize(self.handle))

    def graph_stats(self) -> tuple[int, int, int]:
        b, r, u = C.c_int64(), C.c_int64(), C.c_int64()
        check(load_library().l0b_device_graph_stats(self.handle, C.byref(b), C.byref(r), C.byref(u)))
        return b.value, r.value, u.value

    def set_pdl(self, enabled: bool):
        check(load_library().l0b_device_set_pdl(self.handle, 1 if enabled else 0))

    def Dispose(self):
        if self.handle:
            load_library().l0b_device_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


class SharedBuffer:
    def __init__(self, device: ComputeDevice, dtype: int, count: int, _handle=None):
        self.device = device
        self.dtype = dtype
        self.Count = int(count)
        if _handle is None:
            h = C.c_void_p()
            check(load_library().l0b_buffer_alloc(device.handle, dtype, self.Count, C.byref(h)))
            _handle = h
        self.handle = _handle

    def View(self, offset: int, count: int) -> "SharedBuffer":
        """Elements [offset, offset + count) of this buffer (no copy, owns nothing; must not outlive it)."""
        h = C.c_void_p()
        check(load_library().l0b_buffer_view(self.handle, offset, count, C.byref(h)))
        return SharedBuffer(self.device, self.dtype, count, _handle=h)

    @classmethod
    def from_array(cls, device: ComputeDevice, data: np.ndarray, dtype: int | None = None) -> "SharedBuffer":
        if dtype is None:
            dtype = {np.dtype(np.float32): F32, np.dtype(np.float16): F16, np.dtype(np.int8): I8,
                     np.dtype(np.int32): I32, np.dtype(np.uint8): U8, np.dtype(np.uint16): BF16}[data.dtype]
        b = cls(device, dtype, np.asarray(data).size)
        b.Write(data)
        return b

    def Write(self, data: np.ndarray, offset: int = 0):
        want = np.dtype(NP_DTYPE[self.dtype])
        data = np.asarray(data)
        if self.dtype in (F16, BF16) and data.dtype != want and data.dtype.itemsize == 2 and data.dtype.kind in "ui":
            # 16-bit payloads given as raw bits (uint16 / int16): reinterpret, never convert.
            data = np.ascontiguousarray(data).view(want)
        arr = np.ascontiguousarray(data, want).ravel()
        check(load_library().l0b_buffer_write(self.handle, offset, _p(arr), arr.size))

    def ToArray(self, offset: int = 0, count: int | None = None) -> np.ndarray:
        n = self.Count - offset if count is None else count
        out = np.zeros(n, NP_DTYPE[self.dtype])
        check(load_library().l0b_buffer_read(self.handle, offset, _p(out), n))
        return out

    def Zero(self):
        check(load_library().l0b_buffer_zero(self.handle))

    @property
    def Pointer(self) -> int:
        p = C.c_void_p()
        check(load_library().l0b_buffer_device_ptr(self.handle, C.byref(p)))
        return p.value or 0

    def Dispose(self):
        if self.handle:
            load_library().l0b_buffer_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


# -------------------------------------------------------------------------------------------------
# Kernel suite
# -------------------------------------------------------------------------------------------------

class _Op:
    def __init__(self, suite: "LlmKernelSuite"):
        self.suite = suite
        self.L = load_library()

    def _s(self):
        return self.suite.handle


class _Embedding(_Op):
    def Execute(self, dev, ids, table, out, h, count):
        check(self.L.l0b_embedding_execute(self._s(), dev.handle, ids.handle, table.handle, out.handle, h, count))


class _RMSNorm(_Op):
    def Execute(self, dev, x, res, w, out, eps, width, rows, addResidual):
        check(self.L.l0b_rmsnorm_execute(self._s(), dev.handle, x.handle, _h(res), w.handle, out.handle, eps, width,
                                         rows, 1 if addResidual else 0))


class _Gemv(_Op):
    @staticmethod
    def Supports(n: int) -> bool:
        return bool(load_library().l0b_gemv_supports(n))

    @staticmethod
    def MaxRows() -> int:
        return load_library().l0b_gemv_max_rows()

    def Execute(self, dev, N, K, x, W, y):
        check(self.L.l0b_gemv_execute(self._s(), dev.handle, N, K, x.handle, W.handle, y.handle))

    def ExecuteRows(self, dev, M, N, K, x, W, y):
        check(self.L.l0b_gemv_execute_rows(self._s(), dev.handle, M, N, K, x.handle, W.handle, y.handle))


class _Gemm(_Op):
    def Execute(self, dev, M, N, K, A, B, Cb):
        check(self.L.l0b_gemm_execute(self._s(), dev.handle, M, N, K, A.handle, B.handle, Cb.handle))


class _GemvQ8(_Op):
    GroupSize = 32

    @staticmethod
    def Supports(n: int, k: int) -> bool:
        return bool(load_library().l0b_gemv_q8_supports(n, k))

    def Quantize(self, dev, rows, K, x, scratch=None):
        check(self.L.l0b_gemv_q8_quantize(self._s(), dev.handle, rows, K, x.handle))

    def Execute(self, dev, N, K, scratch, words, scales, y):
        check(self.L.l0b_gemv_q8_execute(self._s(), dev.handle, N, K, words.handle, scales.handle, y.handle))

    def ExecuteRows(self, dev, M, N, K, scratch, words, scales, y):
        check(self.L.l0b_gemv_q8_execute_rows(self._s(), dev.handle, M, N, K, words.handle, scales.handle, y.handle))


class _BiasAdd(_Op):
    def Execute(self, dev, x, b, width, rows):
        check(self.L.l0b_bias_add_execute(self._s(), dev.handle, x.handle, b.handle, width, rows))


class _RoPE(_Op):
    def Execute(self, dev, q, k, positions, hd, nH, nKv, theta, tokens):
        check(self.L.l0b_rope_execute(self._s(), dev.handle, q.handle, k.handle, positions.handle, hd, nH, nKv, theta,
                                      tokens))

    def ExecuteWithFrequencies(self, dev, q, k, positions, invFreq, hd, nH, nKv, attnScale, tokens, rotaryDim):
        check(self.L.l0b_rope_execute_with_frequencies(self._s(), dev.handle, q.handle, k.handle, positions.handle,
                                                       invFreq.handle, hd, nH, nKv, attnScale, tokens, rotaryDim))


class _KvCacheStore(_Op):
    def Execute(self, dev, k, v, Kc, Vc, pos0, kvDim):
        check(self.L.l0b_kv_cache_store_execute(self._s(), dev.handle, k.handle, v.handle, Kc.handle, Vc.handle, pos0,
                                                kvDim))

    def ExecuteRows(self, dev, k, v, Kc, Vc, pos0, kvDim, tokens):
        check(self.L.l0b_kv_cache_store_execute_rows(self._s(), dev.handle, k.handle, v.handle, Kc.handle, Vc.handle,
                                                     pos0, kvDim, tokens))


class _Attention(_Op):
    def Execute(self, dev, q, Kc, Vc, out, hd, nH, nKv, seqLen, maxSeq):
        check(self.L.l0b_attention_execute(self._s(), dev.handle, q.handle, Kc.handle, Vc.handle, out.handle, hd, nH,
                                           nKv, seqLen, maxSeq))

    def ExecutePrefill(self, dev, q, Kc, Vc, out, hd, nH, nKv, pos0, tokens, maxSeq):
        check(self.L.l0b_attention_execute_prefill(self._s(), dev.handle, q.handle, Kc.handle, Vc.handle, out.handle,
                                                   hd, nH, nKv, pos0, tokens, maxSeq))


class _Unary(_Op):
    def __init__(self, suite, fn):
        super().__init__(suite)
        self.fn = getattr(self.L, fn)

    def Execute(self, dev, a, b, n):
        check(self.fn(self._s(), dev.handle, a.handle, b.handle, n))


class _Copy(_Op):
    def Execute(self, dev, src, dst, offset, n):
        check(self.L.l0b_copy_execute(self._s(), dev.handle, src.handle, dst.handle, offset, n))


class _Sampling(_Op):
    def Execute(self, dev, logits, sampled, temperature, randomVal, vocab):
        check(self.L.l0b_sampling_execute(self._s(), dev.handle, logits.handle, sampled.handle, temperature,
                                          randomVal, vocab))


class _Sampler(_Op):
    """LlmSampler.Sample on the device: the token goes to `out` (i32 [1])."""

    def Execute(self, dev, logits, vocab, context, n_context, temperature, top_p, top_k, repetition_penalty,
                random_value, out):
        check(self.L.l0b_sample_execute(self._s(), dev.handle, logits.handle, vocab,
                                        context.handle if context is not None else None, n_context, temperature,
                                        top_p, top_k, repetition_penalty, random_value, out.handle))


class _CausalConv(_Op):
    def Execute(self, dev, qkv, convState, convW, out, convDim, k, tokens):
        check(self.L.l0b_causal_conv_execute(self._s(), dev.handle, qkv.handle, convState.handle, convW.handle,
                                             out.handle, convDim, k, tokens))


    def ExecuteBatch(self, dev, qkv, convStates, convW, out, convDim, k, batch):
        """One token of each of `batch` sequences (rows of qkv/out, windows of convStates)."""
        check(self.L.l0b_causal_conv_execute_batch(self._s(), dev.handle, qkv.handle, convStates.handle, convW.handle,
                                                   out.handle, convDim, k, batch))


class _GatedDelta(_Op):
    def Execute(self, dev, conv, z, b, a, A_log, dt_bias, normW, S, out, Hv, dk, dv, tokens, eps):
        check(self.L.l0b_gated_delta_execute(self._s(), dev.handle, conv.handle, z.handle, b.handle, a.handle,
                                             A_log.handle, dt_bias.handle, normW.handle, S.handle, out.handle, Hv, dk,
                                             dv, tokens, eps))

    def ExecuteGrouped(self, dev, conv, z, b, a, A_log, dt_bias, normW, S, out, Hk, Hv, dk, dv, tokens, eps):
        check(self.L.l0b_gated_delta_execute_grouped(self._s(), dev.handle, conv.handle, z.handle, b.handle, a.handle,
                                                     A_log.handle, dt_bias.handle, normW.handle, S.handle, out.handle,
                                                     Hk, Hv, dk, dv, tokens, eps))

    def ExecuteBatch(self, dev, conv, z, b, a, A_log, dt_bias, normW, states, out, Hk, Hv, dk, dv, batch, eps):
        """One token of each of `batch` sequences, states [batch, Hv, dk, dv]."""
        check(self.L.l0b_gated_delta_execute_batch(self._s(), dev.handle, conv.handle, z.handle, b.handle, a.handle,
                                                   A_log.handle, dt_bias.handle, normW.handle, states.handle,
                                                   out.handle, Hk, Hv, dk, dv, batch, eps))

    def ForkState(self, dev, convStates, states, convDim, k, Hv, dk, dv, src, dst):
        """Sequence dst's conv window and recurrent state become device copies of sequence src's."""
        check(self.L.l0b_linear_state_fork(self._s(), dev.handle, convStates.handle, states.handle, convDim, k, Hv, dk,
                                           dv, src, dst))


class LlmKernelSuite:
    """LlmKernelSuite.Create(device): the op objects the reference decoder calls."""

    def __init__(self, device: ComputeDevice):
        h = C.c_void_p()
        check(load_library().l0b_suite_create(device.handle, C.byref(h)))
        self.handle = h
        self.device = device
        self.Embedding = _Embedding(self)
        self.RMSNorm = _RMSNorm(self)
        self.Gemv = _Gemv(self)
        self.Gemm = _Gemm(self)
        self.GemvQ8 = _GemvQ8(self)
        self.BiasAdd = _BiasAdd(self)
        self.RoPE = _RoPE(self)
        self.KvCacheStore = _KvCacheStore(self)
        self.Attention = _Attention(self)
        self.SigmoidGate = _Unary(self, "l0b_sigmoid_gate_execute")
        self.SwiGLU = _Unary(self, "l0b_swiglu_execute")
        self.Add = _Unary(self, "l0b_add_execute")
        self.Copy = _Copy(self)
        self.Sampling = _Sampling(self)
        self.Sampler = _Sampler(self)
        self.CausalConv = _CausalConv(self)
        self.GatedDelta = _GatedDelta(self)

    @classmethod
    def Create(cls, device: ComputeDevice) -> "LlmKernelSuite":
        return cls(device)

    def EnsureQ8Scratch(self, device, rows: int, width: int):
        check(load_library().l0b_suite_ensure_q8_scratch(self.handle, rows, width))

    @property
    def Q8ScratchRows(self) -> int:
        return load_library().l0b_suite_q8_scratch_rows(self.handle)

    def linear(self, dev, M, N, K, x, W, scales, group, bias, y):
        """Y = X W^T for W in the [out, in] order (f32/f16/bf16/int8 + scales)."""
        check(load_library().l0b_linear(self.handle, dev.handle, M, N, K, x.handle, W.handle, _h(scales), group,
                                        _h(bias), y.handle))

    EPI_STORE, EPI_ACCUM, EPI_SWIGLU = 0, 1, 2
    EPI_F32_ACTIVATIONS = 0x100  # linear_tc only: x enters as hi + lo 16-bit halves
    EPI_BLOCKED_WEIGHTS = 0x200  # linear_fused only: int8 W (one scale per row) in the blocked layout

    def linear_shared(self, dev, M, K, x, W, scales, group, seg_rows, outs, biases=None):
        """ProjectShared over stacked weights W = [W1; W2; ...]: one launch, Y_i = X W_i^T (+ b_i)."""
        n = len(seg_rows)
        rows = (C.c_int32 * n)(*seg_rows)
        ob = (C.c_void_p * n)(*[o.handle for o in outs])
        bb = (C.c_void_p * n)(*[_h(b) for b in biases]) if biases is not None else None
        check(load_library().l0b_linear_shared(self.handle, dev.handle, M, K, x.handle, W.handle, _h(scales), group,
                                               n, rows, bb, ob))

    def linear_fused(self, dev, M, N, K, x, W, scales, group, norm_w, eps, epilogue, bias, out):
        """RMSNorm prologue (norm_w) + projection + store / residual-add / SwiGLU epilogue, one kernel."""
        check(load_library().l0b_linear_fused(self.handle, dev.handle, M, N, K, x.handle, W.handle, _h(scales),
                                              group, _h(norm_w), eps, epilogue, _h(bias), out.handle))

    def Dispose(self):
        if self.handle:
            load_library().l0b_suite_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


WEIGHT_BLOCK = 512  # k per block of the blocked int8 layout


def block_int8(q: np.ndarray) -> np.ndarray:
    """Row-major int8 [N, K] -> the blocked layout [N/16][K/512][16][512] that models keep their q/k/v,
    o_proj and down projections in (the bytes of one 16-row x 512-k block are contiguous). N % 16 == 0 and
    K % 512 == 0. For LlmKernelSuite.linear_fused with EPI_BLOCKED_WEIGHTS."""
    n, k = q.shape
    if n % 16 or k % WEIGHT_BLOCK:
        raise ValueError(f"blocked layout needs N % 16 == 0 and K % {WEIGHT_BLOCK} == 0, got {n} x {k}")
    b = q.reshape(n // 16, 16, k // WEIGHT_BLOCK, WEIGHT_BLOCK).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(b).reshape(n, k)


def q8_quantize_out_in(hf: np.ndarray, group: int = 32) -> tuple[np.ndarray, np.ndarray]:
    """LlmQ8Quantizer.QuantizeOutIn: HF [N, K] fp32 -> (int8 [N, K], fp16 scales [N, K/group])."""
    hf = np.ascontiguousarray(hf, np.float32)
    N, K = hf.shape
    g = group if group > 0 else K
    q = np.zeros((N, K), np.int8)
    s = np.zeros((N, K // g), np.uint16)
    check(load_library().l0b_q8_quantize_out_in(_p(hf), N, K, g, _p(q), _p(s)))
    return q, s.view(np.float16)


def rope_frequencies(cfg: ModelConfig) -> tuple[np.ndarray, float]:
    n = C.c_int32()
    att = C.c_float()
    check(load_library().l0b_rope_frequencies(C.byref(cfg), None, 0, C.byref(n), C.byref(att)))
    out = np.zeros(n.value, np.float32)
    check(load_library().l0b_rope_frequencies(C.byref(cfg), _p(out), n.value, C.byref(n), C.byref(att)))
    return out, float(att.value)


def kernel_launch_count() -> int:
    return int(load_library().l0b_kernel_launch_count())


# -------------------------------------------------------------------------------------------------
# Model host (LlmModel)
# -------------------------------------------------------------------------------------------------

def model_config(**kw) -> ModelConfig:
    cfg = ModelConfig()
    check(load_library().l0b_model_config_init(C.byref(cfg)))
    for k, v in kw.items():
        if k == "rope_type" and isinstance(v, str):
            v = ROPE_TYPES[v]
        setattr(cfg, k, v)
    return cfg


class ShardPlan(C.Structure):
    """l0b_shard_plan: where l0b_model_set_tensor puts one checkpoint tensor on one tensor-parallel rank."""
    _fields_ = [(n, C.c_int32) for n in ("kind", "layer", "slot", "full_rows", "full_cols", "row0", "rows", "col0",
                                         "cols", "dst_row")]
    MATRIX, VECTOR, EMBEDDING, QUERY_GATE = 0, 1, 2, 3
    QKV, O, GATE_UP, DOWN, LM_HEAD, LIN_IN, LIN_OUT = 0, 1, 2, 3, 4, 5, 6
    IN_NORM, POST_NORM, QKV_BIAS, Q_NORM, K_NORM, FINAL_NORM = 0, 1, 2, 3, 4, 5
    LIN_CONV, LIN_A_LOG, LIN_DT_BIAS, LIN_NORM = 6, 7, 8, 9

    def take(self, full: np.ndarray) -> np.ndarray:
        """This rank's part of the full checkpoint tensor (rows x cols of it)."""
        full = np.asarray(full).reshape(self.full_rows, self.full_cols)
        return full[self.row0:self.row0 + self.rows, self.col0:self.col0 + self.cols]


def shard_plan(cfg: ModelConfig, name: str) -> ShardPlan:
    """The model's tensor-parallel placement of checkpoint tensor `name` for rank cfg.tp_rank of
    cfg.tp_size (host arithmetic; no device needed)."""
    out = ShardPlan()
    check(load_library().l0b_model_shard_plan(C.byref(cfg), name.encode(), C.byref(out)))
    return out


class Communicator:
    """Tensor-parallel communicator (NCCL), one per rank. Rank 0 makes the id with unique_id() and the
    caller hands it to every rank (any channel, e.g. torch.distributed over gloo)."""

    ID_BYTES = 128

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * Communicator.ID_BYTES)()
        check(load_library().l0b_comm_unique_id(buf, Communicator.ID_BYTES))
        return bytes(buf)

    def __init__(self, device: ComputeDevice, uid: bytes, nranks: int, rank: int):
        buf = (C.c_uint8 * len(uid)).from_buffer_copy(uid)
        h = C.c_void_p()
        check(load_library().l0b_comm_create(device.handle, buf, len(uid), nranks, rank, C.byref(h)))
        self.handle = h
        self.nranks, self.rank = nranks, rank

    def AllReduce(self, buf: "SharedBuffer", count: int | None = None):
        check(load_library().l0b_comm_allreduce(self.handle, buf.handle, buf.Count if count is None else count))

    @property
    def UsesPeerAllReduce(self) -> bool:
        """True when this communicator's small all-reduces run over peer memory (IPC-mapped mailboxes)."""
        v = C.c_int32()
        check(load_library().l0b_comm_uses_peer_allreduce(self.handle, C.byref(v)))
        return bool(v.value)

    @staticmethod
    def set_peer_allreduce(enabled: bool):
        """Process-wide: communicators made afterwards use the peer all-reduce (True, default) or NCCL only."""
        check(load_library().l0b_comm_set_peer_allreduce(1 if enabled else 0))

    _fused = True

    @staticmethod
    def set_fused_allreduce(enabled: bool):
        """Process-wide: steps recorded afterwards fold the row-split decode all-reduces into their GEMVs
        (True, default, with peer memory) or run GEMV + all-reduce pairs."""
        check(load_library().l0b_comm_set_fused_allreduce(1 if enabled else 0))
        Communicator._fused = bool(enabled)

    @staticmethod
    def fused_allreduce() -> bool:
        """The setting of set_fused_allreduce (as made through this module)."""
        return Communicator._fused

    def Dispose(self):
        if self.handle:
            load_library().l0b_comm_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()


class LlmModel:
    """LlmModel: prefill / decode / greedy generation on the device."""

    def __init__(self, device: ComputeDevice, suite: LlmKernelSuite, cfg: ModelConfig, max_seq_len: int,
                 precision: str = "auto", comm=None):
        h = C.c_void_p()
        check(load_library().l0b_model_create(device.handle, suite.handle, C.byref(cfg), max_seq_len,
                                              PRECISION[precision], _h(comm) if comm is not None else None,
                                              C.byref(h)))
        self.handle = h
        self.cfg = cfg
        self.vocab = cfg.vocab_size  # under TP the logits are gathered to the full vocabulary
        self.MaxSeqLen = max_seq_len

    def set_tensor_raw(self, name: str, bits: np.ndarray, dtype: int):
        """Uploads the 16-bit payload (F16 or BF16 bits as uint16) of a checkpoint tensor as is."""
        d = np.ascontiguousarray(bits).view(np.uint16).ravel()
        check(load_library().l0b_model_set_tensor_raw(self.handle, name.encode(), _p(d), dtype, d.size))

    def init_synthetic(self, seed: int, std: float = 0.02, scale_lo: float = 1e-3, scale_hi: float = 2e-2):
        check(load_library().l0b_model_init_synthetic(self.handle, seed, std, scale_lo, scale_hi))

    def set_tensor(self, name: str, data: np.ndarray):
        d = np.ascontiguousarray(data, np.float32).ravel()
        check(load_library().l0b_model_set_tensor(self.handle, name.encode(), _p(d), d.size))

    def Prefill(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.zeros(self.vocab, np.float32)
        check(load_library().l0b_model_prefill(self.handle, _p(ids), ids.size, _p(logits)))
        return logits

    def Decode(self, token: int, logits: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros(self.vocab, np.float32) if logits is None else logits
        check(load_library().l0b_model_decode(self.handle, int(token), _p(out)))
        return out

    def ComputeLogits(self, token: int, position: int) -> np.ndarray:
        logits = np.zeros(self.vocab, np.float32)
        check(load_library().l0b_model_compute_logits(self.handle, int(token), int(position), _p(logits)))
        return logits

    def GenerateGreedy(self, ids, max_new: int, stop_ids=()) -> list[int]:
        ids = np.ascontiguousarray(ids, np.int32)
        stops = np.ascontiguousarray(list(stop_ids) or [0], np.int32)
        out = np.zeros(max(1, max_new), np.int32)
        n = C.c_int32()
        check(load_library().l0b_model_generate_greedy(self.handle, _p(ids), ids.size, max_new, _p(stops),
                                                       len(stop_ids), _p(out), C.byref(n)))
        return out[: n.value].tolist()

    def decode_greedy_device(self, steps: int) -> np.ndarray:
        out = np.zeros(max(1, steps), np.int32)
        check(load_library().l0b_model_decode_greedy_device(self.handle, steps, _p(out)))
        return out[:steps]

    def ForkSequence(self, src: int, dst: int, base_position: int = 0):
        """Sequence dst becomes a device-side copy of sequence src (KV rows from base_position on)."""
        check(load_library().l0b_model_fork_sequence(self.handle, src, dst, base_position))

    # Device sampling (LlmSampler.Sample on the GPU; no logits readback).
    def sample_logits(self, temperature: float, top_p: float, top_k: int, repetition_penalty: float, seed: int,
                      context) -> int:
        """Samples the next token from the last step's logits; it becomes the next input token."""
        ctx = np.ascontiguousarray(context if context is not None else [], np.int32)
        tok = C.c_int32()
        check(load_library().l0b_model_sample_logits(self.handle, temperature, top_p, top_k, repetition_penalty,
                                                     seed, _p(ctx) if ctx.size else None, ctx.size, C.byref(tok)))
        return tok.value

    def decode_sample_device(self, steps: int, temperature: float, top_p: float, top_k: int,
                             repetition_penalty: float, seed: int) -> np.ndarray:
        """`steps` device-resident decode steps, each sampling the next token (draws seeded by position)."""
        out = np.zeros(max(1, steps), np.int32)
        check(load_library().l0b_model_decode_sample_device(self.handle, steps, temperature, top_p, top_k,
                                                            repetition_penalty, seed, _p(out)))
        return out[:steps]

    # Batched sequences (cfg.max_batch > 1): sequence `seq` owns KV-cache row seq.
    def PrefillSequence(self, seq: int, prompt_ids, want_logits: bool = True) -> np.ndarray | None:
        ids = np.ascontiguousarray(prompt_ids, np.int32)
        logits = np.zeros(self.vocab, np.float32) if want_logits else None
        check(load_library().l0b_model_prefill_sequence(self.handle, seq, _p(ids), ids.size,
                                                         _p(logits) if logits is not None else None))
        return logits

    def DecodeBatch(self, tokens, positions, want_logits: bool = True) -> np.ndarray | None:
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        logits = np.zeros((t.size, self.vocab), np.float32) if want_logits else None
        check(load_library().l0b_model_decode_batch(self.handle, _p(t), _p(p), t.size,
                                                     _p(logits) if logits is not None else None))
        return logits

    def decode_greedy_device_batch(self, steps: int, count: int) -> np.ndarray:
        out = np.zeros((max(1, steps), count), np.int32)
        check(load_library().l0b_model_decode_greedy_device_batch(self.handle, steps, count, _p(out)))
        return out[:steps]

    def SequencePosition(self, seq: int) -> int:
        v = C.c_int32()
        check(load_library().l0b_model_sequence_position(self.handle, seq, C.byref(v)))
        return v.value

    @property
    def Position(self) -> int:
        v = C.c_int32()
        check(load_library().l0b_model_position(self.handle, C.byref(v)))
        return v.value

    def ResetSequence(self):
        check(load_library().l0b_model_reset_sequence(self.handle))

    @property
    def ProjectionBytes(self) -> int:
        v = C.c_int64()
        check(load_library().l0b_model_projection_bytes(self.handle, C.byref(v)))
        return v.value

    def set_recording(self, on: bool):
        check(load_library().l0b_model_set_recording(self.handle, 1 if on else 0))

    def set_fused(self, on: bool):
        check(load_library().l0b_model_set_fused(self.handle, 1 if on else 0))

    def set_gemm_rows(self, min_rows: int):
        """Projections over >= min_rows rows (16-bit or per-row-scaled int8 weights) use the tcgen05 GEMM
        (0 = GEMV only; default 8)."""
        check(load_library().l0b_model_set_gemm_rows(self.handle, int(min_rows)))

    @property
    def Probe(self):
        return getattr(self, "_probe_py", None)

    @Probe.setter
    def Probe(self, fn):
        """LlmDecoderLayer.Probe: fn(layer, stage, values) after each stage; None removes it."""
        self._probe_py = fn
        if fn is None:
            self._probe_c = None
            check(load_library().l0b_model_set_probe(self.handle, PROBE_FN(), None))
            return
        self._probe_c = PROBE_FN(lambda _u, layer, stage, vals, n: fn(layer, stage.decode(),
                                                                          np.ctypeslib.as_array(vals, (n,)).copy()))
        check(load_library().l0b_model_set_probe(self.handle, self._probe_c, None))

    def read_weight(self, layer: int, kind: int, dtype, count: int) -> np.ndarray:
        out = np.zeros(count, dtype)
        check(load_library().l0b_model_read_weight(self.handle, layer, kind, _p(out), out.nbytes))
        return out

    def read_kv(self, layer: int, row0: int, rows: int) -> tuple[np.ndarray, np.ndarray]:
        kvd = (self.cfg.num_key_value_heads // max(1, self.cfg.tp_size)) * self.cfg.head_dim
        k = np.zeros(rows * kvd, np.float32)
        v = np.zeros(rows * kvd, np.float32)
        check(load_library().l0b_model_read_kv(self.handle, layer, row0, rows, _p(k), _p(v)))
        return k.reshape(rows, kvd), v.reshape(rows, kvd)

    def Dispose(self):
        if self.handle:
            load_library().l0b_model_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Dispose()
