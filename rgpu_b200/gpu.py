"""Python mirror of rtensor's GPU API (crates/rtensor/src/gpu/mod.rs) over the
C ABI of librtgpu.so (include/rtgpu.h).

Names follow the reference: ``Gpu`` (context + op helpers), ``GpuTensor``,
``upload_labels``, ``GpuMlp.from_params / step / forward_only / logits /
last_loss / weights / grads / dispatches_por_passo``.  Where the reference
panics on misuse, these raise ``RtError`` carrying ``rt_last_error()``.

There is no CPU fallback: every compute call goes to a CUDA kernel in
librtgpu.so, and importing the library fails loudly when it is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librtgpu.so")

RT_OK, RT_ERR_INVALID, RT_ERR_CUDA, RT_ERR_NCCL, RT_ERR_OOM, RT_ERR_DEVICE_TIMEOUT, RT_ERR_UNSUPPORTED = range(7)
RT_F32, RT_BF16, RT_U32 = 0, 1, 2
RT_NN, RT_NT, RT_TN = 0, 1, 2
RT_EPI_NONE, RT_EPI_BIAS, RT_EPI_BIAS_RELU, RT_EPI_RELU_MASK = 0, 1, 2, 3
RT_OPT_NONE, RT_OPT_SGD, RT_OPT_ADAM = 0, 1, 2
RT_ACT_SPLIT, RT_ACT_BF16 = 0, 1

_DTYPES = {"f32": RT_F32, "float32": RT_F32, "bf16": RT_BF16, "bfloat16": RT_BF16, "u32": RT_U32}
_OPTS = {"none": RT_OPT_NONE, "sgd": RT_OPT_SGD, "adam": RT_OPT_ADAM}
_ACTS = {"split": RT_ACT_SPLIT, "bf16": RT_ACT_BF16}


class RtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[rt status {code}] {msg}")
        self.code = code


class GemmArgs(C.Structure):
    _fields_ = [
        ("layout", C.c_int), ("in_dtype", C.c_int), ("out_dtype", C.c_int),
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64),
        ("a", C.c_void_p), ("lda", C.c_int64),
        ("b", C.c_void_p), ("ldb", C.c_int64),
        ("c", C.c_void_p), ("ldc", C.c_int64),
        ("epilogue", C.c_int), ("bias", C.c_void_p),
        ("mask", C.c_void_p), ("ldmask", C.c_int64),
        ("split_k", C.c_int), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("a_lo", C.c_void_p), ("c_lo", C.c_void_p),
    ]


class MlpConfig(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int), ("dims", C.POINTER(C.c_int64)), ("batch", C.c_int64),
        ("global_batch", C.c_int64), ("dtype", C.c_int), ("optimizer", C.c_int),
        ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
        ("activations", C.c_int),
    ]


_lib = None

# (name, restype, argtypes)
_SIGS = [
    ("rt_last_error", C.c_char_p, []),
    ("rt_abi_version", C.c_int, []),
    ("rt_ctx_create", C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    ("rt_ctx_destroy", C.c_int, [C.c_void_p]),
    ("rt_ctx_info", C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    ("rt_ctx_sync", C.c_int, [C.c_void_p]),
    ("rt_ctx_selftest_timeout", C.c_int, [C.c_void_p]),
    ("rt_ctx_stream", C.c_void_p, [C.c_void_p]),
    ("rt_ctx_set_stream", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_ctx_set_fast_gemm", C.c_int, [C.c_void_p, C.c_int]),
    ("rt_ctx_set_f32_tensor", C.c_int, [C.c_void_p, C.c_int]),
    ("rt_ctx_set_l2_group", C.c_int, [C.c_void_p, C.c_int]),
    ("rt_ctx_launch_count", C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    ("rt_host_alloc", C.c_int, [C.c_size_t, C.POINTER(C.c_void_p)]),
    ("rt_host_free", C.c_int, [C.c_void_p]),
    ("rt_tensor_zeros", C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int64), C.POINTER(C.c_void_p)]),
    ("rt_tensor_upload", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_int64),
                                   C.POINTER(C.c_void_p)]),
    ("rt_upload_labels", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    ("rt_tensor_download", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    ("rt_tensor_wrap", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int64), C.c_int64,
                                 C.POINTER(C.c_void_p)]),
    ("rt_tensor_free", C.c_int, [C.c_void_p]),
    ("rt_tensor_ptr", C.c_void_p, [C.c_void_p]),
    ("rt_tensor_dims", C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    ("rt_matmul", C.c_int, [C.c_void_p] * 4),
    ("rt_matmul_at_b", C.c_int, [C.c_void_p] * 4),
    ("rt_matmul_a_bt", C.c_int, [C.c_void_p] * 4),
    ("rt_matmul_bias", C.c_int, [C.c_void_p] * 5 + [C.c_int]),
    ("rt_matmul_split_k", C.c_int, [C.c_void_p] * 5 + [C.c_int, C.c_int]),
    ("rt_matmul_split_k_noalloc", C.c_int, [C.c_void_p] * 4 + [C.c_int, C.c_int]),
    ("rt_split_k_static_capacity", C.c_int64, []),
    ("rt_split_k_suggest", C.c_int, [C.c_int64, C.c_int64, C.c_int64]),
    ("rt_split_k_workspace", C.c_int64, [C.c_int64, C.c_int64, C.c_int]),
    ("rt_gemm", C.c_int, [C.c_void_p, C.POINTER(GemmArgs)]),
    ("rt_gemm_workspace_size", C.c_size_t, [C.c_void_p, C.POINTER(GemmArgs)]),
    ("rt_bias_add", C.c_int, [C.c_void_p] * 3),
    ("rt_relu", C.c_int, [C.c_void_p] * 3),
    ("rt_relu_bwd", C.c_int, [C.c_void_p] * 3),
    ("rt_softmax_xent", C.c_int, [C.c_void_p] * 5 + [C.c_float]),
    ("rt_colsum", C.c_int, [C.c_void_p] * 4),
    ("rt_adam", C.c_int, [C.c_void_p] * 5 + [C.c_float] * 4 + [C.c_int]),
    ("rt_sgd", C.c_int, [C.c_void_p] * 3 + [C.c_float]),
    ("rt_cast", C.c_int, [C.c_void_p] * 3),
    ("rt_mlp_create", C.c_int, [C.c_void_p, C.POINTER(MlpConfig), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                C.POINTER(C.c_void_p)]),
    ("rt_mlp_destroy", C.c_int, [C.c_void_p]),
    ("rt_mlp_step", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    ("rt_mlp_step_host", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_mlp_forward_only", C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    ("rt_mlp_forward_host", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    ("rt_mlp_logits", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_mlp_last_loss", C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    ("rt_mlp_global_loss", C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    ("rt_mlp_weights", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_mlp_grads", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_mlp_set_weights", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_mlp_state_size", C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    ("rt_mlp_save_state", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    ("rt_mlp_load_state", C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    ("rt_mlp_dispatches_per_step", C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    ("rt_mlp_enable_timing", C.c_int, [C.c_void_p, C.c_int]),
    ("rt_mlp_op_count", C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    ("rt_mlp_op_time", C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_double),
                                 C.POINTER(C.c_float)]),
    ("rt_mlp_set_comm", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_mlp_comm_mode", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_plan_ld", C.c_int64, [C.c_int64]),
    ("rt_plan_dw_chunks", C.c_int, [C.c_int, C.c_int64, C.c_int64, C.c_int, C.c_int]),
    ("rt_plan_chunk_row", C.c_int64, [C.c_int64, C.c_int, C.c_int]),
    ("rt_plan_shard_slice", C.c_int64, [C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int,
                                        C.POINTER(C.c_int64)]),
    ("rt_param_create", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(C.c_void_p)]),
    ("rt_param_destroy", C.c_int, [C.c_void_p]),
    ("rt_param_read", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_param_write", C.c_int, [C.c_void_p, C.c_void_p]),
    ("rt_param_value", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_tape_create", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_tape_destroy", C.c_int, [C.c_void_p]),
    ("rt_tape_len", C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    ("rt_tape_constant", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_param_watch", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_matmul", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_add", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_relu", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_softmax_cross_entropy", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_binary", C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]),
    ("rt_var_unary", C.c_int, [C.c_void_p, C.c_int, C.c_float, C.POINTER(C.c_void_p)]),
    ("rt_var_sum", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_mean", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_softmax", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_loss_mse", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_loss_mae", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_loss_bce", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_accuracy", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_float)]),
    ("rt_var_value", C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_var_item", C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    ("rt_var_backward", C.c_int, [C.c_void_p]),
    ("rt_grads_of", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_sgd_step", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_float]),
    ("rt_adam_create", C.c_int, [C.c_void_p, C.c_float, C.c_float, C.c_float, C.c_float, C.POINTER(C.c_void_p)]),
    ("rt_adam_destroy", C.c_int, [C.c_void_p]),
    ("rt_adam_step", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_sgd_create", C.c_int, [C.c_void_p, C.c_float, C.c_float, C.POINTER(C.c_void_p)]),
    ("rt_sgd_destroy", C.c_int, [C.c_void_p]),
    ("rt_sgd_state_step", C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    ("rt_comm_unique_id", C.c_int, [C.c_void_p]),
    ("rt_comm_init", C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    ("rt_comm_destroy", C.c_int, [C.c_void_p]),
    ("rt_comm_allreduce_f32", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64]),
]


def lib():
    """Load librtgpu.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C rgpu_b200/csrc` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return [name for name, _, _ in _SIGS]


def _check(code: int):
    if code != RT_OK:
        raise RtError(code, lib().rt_last_error().decode(errors="replace"))


def _dt(dtype) -> int:
    if isinstance(dtype, int):
        return dtype
    return _DTYPES[str(dtype)]


def _shape_arr(shape):
    return (C.c_int64 * len(shape))(*[int(s) for s in shape])


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    rounding = ((b >> 16) & 1) + 0x7FFF
    return ((b + rounding) >> 16).astype(np.uint16)


class GpuTensor:
    """A device tensor (GpuTensor, gpu/mod.rs:191-209)."""

    def __init__(self, gpu: "Gpu", handle: int, owned: bool = True, dtype: int = RT_F32):
        self.gpu = gpu
        self.dtype_code = dtype
        self.handle = C.c_void_p(handle)
        self._owned = owned
        r, c, ld = C.c_int64(), C.c_int64(), C.c_int64()
        _check(lib().rt_tensor_dims(self.handle, C.byref(r), C.byref(c), C.byref(ld)))
        self.rows, self.cols, self.ld = r.value, c.value, ld.value

    @property
    def shape(self):
        return (self.rows, self.cols)

    def __len__(self):
        return self.rows * self.cols

    @property
    def ptr(self) -> int:
        return lib().rt_tensor_ptr(self.handle)

    def free(self):
        if self.handle and self.handle.value:
            # A tensor outliving its context is released with the context's
            # device memory; freeing it after rt_ctx_destroy would touch a
            # destroyed context.
            if self.gpu.alive():
                lib().rt_tensor_free(self.handle)
            self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Gpu:
    """CUDA context on one B200 (Gpu, gpu/mod.rs:224-1287)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().rt_ctx_create(device, C.byref(h)))
        self.handle = h
        self.device = device

    def alive(self) -> bool:
        return bool(self.handle and self.handle.value)

    def close(self):
        if self.alive():
            lib().rt_ctx_destroy(self.handle)
            self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- context
    def info(self) -> str:
        buf = C.create_string_buffer(256)
        _check(lib().rt_ctx_info(self.handle, buf, 256))
        return buf.value.decode()

    def sync(self):
        _check(lib().rt_ctx_sync(self.handle))

    def selftest_timeout(self):
        """Enqueue the device-timeout self-test (rt_ctx_selftest_timeout): the
        next sync raises RtError with RT_ERR_DEVICE_TIMEOUT."""
        _check(lib().rt_ctx_selftest_timeout(self.handle))

    def stream(self) -> int:
        return lib().rt_ctx_stream(self.handle)

    def set_stream(self, stream_ptr: int | None):
        _check(lib().rt_ctx_set_stream(self.handle, stream_ptr))

    def set_fast_gemm(self, on: bool):
        _check(lib().rt_ctx_set_fast_gemm(self.handle, int(bool(on))))

    def set_f32_tensor(self, on: bool):
        """f32 GEMMs as 3xTF32 on the tensor cores (True) or on the SIMT kernel."""
        _check(lib().rt_ctx_set_f32_tensor(self.handle, int(bool(on))))

    def set_grupo_l2(self, group: int):
        _check(lib().rt_ctx_set_l2_group(self.handle, int(group)))

    def launch_count(self) -> int:
        v = C.c_uint64()
        _check(lib().rt_ctx_launch_count(self.handle, C.byref(v)))
        return v.value

    # --- buffers
    def zeros(self, shape, dtype="f32") -> GpuTensor:
        h = C.c_void_p()
        _check(lib().rt_tensor_zeros(self.handle, _dt(dtype), len(shape), _shape_arr(shape), C.byref(h)))
        return GpuTensor(self, h.value, dtype=_dt(dtype))

    def upload(self, t: np.ndarray, dtype="f32") -> GpuTensor:
        a = np.ascontiguousarray(t, np.float32)
        shape = a.shape if a.ndim in (1, 2) else (a.size,)
        h = C.c_void_p()
        _check(lib().rt_tensor_upload(self.handle, _dt(dtype), a.ctypes.data, len(shape), _shape_arr(shape),
                                      C.byref(h)))
        return GpuTensor(self, h.value, dtype=_dt(dtype))

    def wrap(self, device_ptr: int, shape, dtype="f32", ld: int = 0) -> GpuTensor:
        h = C.c_void_p()
        _check(lib().rt_tensor_wrap(self.handle, device_ptr, _dt(dtype), len(shape), _shape_arr(shape), ld,
                                    C.byref(h)))
        return GpuTensor(self, h.value, owned=False, dtype=_dt(dtype))

    def download(self, t: GpuTensor) -> np.ndarray:
        out = np.empty((t.rows, t.cols), np.float32)
        _check(lib().rt_tensor_download(self.handle, t.handle, out.ctypes.data))
        return out

    # --- ops (gpu/mod.rs:685-953)
    def matmul(self, a, b, c):
        _check(lib().rt_matmul(self.handle, a.handle, b.handle, c.handle))

    def matmul_at_b(self, a, b, c):
        _check(lib().rt_matmul_at_b(self.handle, a.handle, b.handle, c.handle))

    def matmul_a_bt(self, a, b, c):
        _check(lib().rt_matmul_a_bt(self.handle, a.handle, b.handle, c.handle))

    def matmul_bias(self, a, b, c, bias, relu: bool):
        _check(lib().rt_matmul_bias(self.handle, a.handle, b.handle, c.handle, bias.handle, int(relu)))

    def split_k(self, a, b, c, partials, slices: int, transposed: bool):
        _check(lib().rt_matmul_split_k(self.handle, a.handle, b.handle, c.handle, partials.handle, slices,
                                       int(transposed)))

    def split_k_noalloc(self, a, b, c, slices: int, transposed: bool):
        """Split-K GEMM with the partial sums in the library's built-in scratch
        array: no device allocation, for callers that may not allocate (e.g.
        during CUDA graph capture).  Calls overlapping on the GPU race on the
        shared scratch; slices*m*n must fit split_k_static_capacity()."""
        _check(lib().rt_matmul_split_k_noalloc(self.handle, a.handle, b.handle, c.handle, slices, int(transposed)))

    @staticmethod
    def split_k_static_capacity() -> int:
        return lib().rt_split_k_static_capacity()

    @staticmethod
    def fatias_sugeridas(m: int, n: int, k: int) -> int:
        return lib().rt_split_k_suggest(m, n, k)

    def bias_add(self, z, b):
        _check(lib().rt_bias_add(self.handle, z.handle, b.handle))

    def relu(self, x, y):
        _check(lib().rt_relu(self.handle, x.handle, y.handle))

    def relu_bwd(self, a, dz):
        _check(lib().rt_relu_bwd(self.handle, a.handle, dz.handle))

    def softmax_xent(self, logits, labels, delta, loss, scale=None):
        s = (1.0 / logits.rows) if scale is None else scale
        _check(lib().rt_softmax_xent(self.handle, logits.handle, labels.handle, delta.handle, loss.handle, s))

    def colsum(self, src, dst, scratch=None):
        _check(lib().rt_colsum(self.handle, src.handle, dst.handle, scratch.handle if scratch else None))

    def adam(self, theta, m, v, g, lr, t, beta1=0.9, beta2=0.999, eps=1e-8):
        _check(lib().rt_adam(self.handle, theta.handle, m.handle, v.handle, g.handle, lr, beta1, beta2, eps, t))

    def sgd(self, theta, g, lr):
        _check(lib().rt_sgd(self.handle, theta.handle, g.handle, lr))

    def cast(self, src, dst):
        _check(lib().rt_cast(self.handle, src.handle, dst.handle))

    def gemm(self, args: GemmArgs):
        _check(lib().rt_gemm(self.handle, C.byref(args)))

    def gemm_workspace_size(self, args: GemmArgs) -> int:
        return lib().rt_gemm_workspace_size(self.handle, C.byref(args))


def upload_labels(gpu: Gpu, labels) -> GpuTensor:
    """upload_labels (gpu/mod.rs:1671-1675)."""
    lab = np.ascontiguousarray(labels, np.uint32)
    h = C.c_void_p()
    _check(lib().rt_upload_labels(gpu.handle, lab.ctypes.data, lab.size, C.byref(h)))
    return GpuTensor(gpu, h.value, dtype=RT_U32)


class Comm:
    """NCCL communicator (new; the reference has no data parallelism)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_ubyte * 128)()
        _check(lib().rt_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, gpu: Gpu, rank: int, world: int, uid: bytes):
        assert len(uid) == 128
        buf = (C.c_ubyte * 128)(*uid)
        h = C.c_void_p()
        _check(lib().rt_comm_init(gpu.handle, rank, world, buf, C.byref(h)))
        self.handle = h
        self.gpu = gpu

    def allreduce_(self, dev_ptr: int, count: int):
        _check(lib().rt_comm_allreduce_f32(self.handle, dev_ptr, count))

    def close(self):
        if self.handle and self.handle.value and self.gpu.alive():
            lib().rt_comm_destroy(self.handle)
            self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GpuMlp:
    """Whole-step plan for a ReLU MLP + softmax-CE (GpuMlp, gpu/mod.rs:1289-1562)."""

    def __init__(self, gpu: Gpu, handle, dims, batch, dtype):
        self.gpu = gpu
        self.handle = handle
        self.dims = list(dims)
        self.lote = batch
        self.dtype = dtype
        self._comm = None

    @classmethod
    def from_params(cls, gpu: Gpu, params, batch: int, lr: float, *, dtype="f32", optimizer="adam",
                    global_batch: int | None = None, beta1=0.9, beta2=0.999, eps=1e-8,
                    activations="split") -> "GpuMlp":
        """params = [W1, b1, W2, b2, ...] as Sequential::params() returns them
        (nn.rs:190-192); W_l is [d_l, d_{l+1}], b_l is [1, d_{l+1}].
        ``activations`` (bf16 plans): "split" keeps each hidden activation as a
        bf16 hi + lo pair for the next forward GEMM (the default, within the
        2e-2 parity bar), "bf16" rounds it once (faster forward, hidden-layer
        gradients 2e-2 .. 8e-2 from the f32 reference)."""
        assert len(params) % 2 == 0 and params, "expected (W, b) pairs"
        ws = [np.ascontiguousarray(params[i], np.float32) for i in range(0, len(params), 2)]
        bs = [np.ascontiguousarray(params[i], np.float32).ravel() for i in range(1, len(params), 2)]
        dims = [ws[0].shape[0]] + [w.shape[1] for w in ws]
        for l, w in enumerate(ws):
            assert w.shape == (dims[l], dims[l + 1]), "inconsistent layer shapes"
        dims_arr = (C.c_int64 * len(dims))(*dims)
        cfg = MlpConfig(len(ws), dims_arr, batch, global_batch or 0, _dt(dtype), _OPTS[optimizer], lr, beta1,
                        beta2, eps, _ACTS[activations])
        wp = (C.c_void_p * len(ws))(*[w.ctypes.data for w in ws])
        bp = (C.c_void_p * len(bs))(*[b.ctypes.data for b in bs])
        h = C.c_void_p()
        _check(lib().rt_mlp_create(gpu.handle, C.byref(cfg), wp, bp, C.byref(h)))
        m = cls(gpu, h, dims, batch, _dt(dtype))
        m._keep = (ws, bs, dims_arr)
        return m

    def close(self):
        if self.handle and self.handle.value and self.gpu.alive():
            lib().rt_mlp_destroy(self.handle)
            self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, x: GpuTensor, labels: GpuTensor):
        """GpuMlp::step (gpu/mod.rs:1499-1511): x, labels already on the device."""
        if x.rows * x.cols != self.lote * self.dims[0]:
            raise RtError(RT_ERR_INVALID, f"batch of {x.rows * x.cols} elements, plan built for "
                                          f"{self.lote * self.dims[0]}")
        if x.ld != x.cols:
            raise RtError(RT_ERR_INVALID, "step input must be packed (ld == cols)")
        dt = RT_BF16 if _is_bf16(x) else RT_F32
        _check(lib().rt_mlp_step(self.handle, x.ptr, dt, labels.ptr))

    def step_ptr(self, x_ptr: int, x_dtype, labels_ptr: int):
        _check(lib().rt_mlp_step(self.handle, x_ptr, _dt(x_dtype), labels_ptr))

    def step_host(self, x: np.ndarray, labels: np.ndarray, loss_rows_out: np.ndarray | None = None,
                  x_dtype="f32"):
        """One step from host buffers (copies inside); x is f32, or uint16 bf16 bits with x_dtype='bf16'."""
        out = None if loss_rows_out is None else loss_rows_out.ctypes.data
        _check(lib().rt_mlp_step_host(self.handle, x.ctypes.data, _dt(x_dtype), labels.ctypes.data, out))

    def step_host_ptr(self, x_ptr: int, x_dtype, labels_ptr: int, loss_ptr: int | None):
        _check(lib().rt_mlp_step_host(self.handle, x_ptr, _dt(x_dtype), labels_ptr, loss_ptr))

    def forward_only(self, x: GpuTensor):
        dt = RT_BF16 if _is_bf16(x) else RT_F32
        _check(lib().rt_mlp_forward_only(self.handle, x.ptr, dt))

    def forward_only_ptr(self, x_ptr: int, x_dtype):
        _check(lib().rt_mlp_forward_only(self.handle, x_ptr, _dt(x_dtype)))

    def forward_host(self, x: np.ndarray, logits_out: np.ndarray | None = None) -> np.ndarray | None:
        """forward_only + logits from a host array (f32); the logits land in
        `logits_out` ([batch, classes] f32) after the call, which syncs."""
        xa = np.ascontiguousarray(x, np.float32)
        assert xa.shape == (self.lote, self.dims[0])
        out = logits_out if logits_out is not None else np.empty((self.lote, self.dims[-1]), np.float32)
        _check(lib().rt_mlp_forward_host(self.handle, xa.ctypes.data, RT_F32, out.ctypes.data))
        self.gpu.sync()
        return out

    def forward_host_ptr(self, x_ptr: int, x_dtype, logits_ptr: int | None):
        """Asynchronous forward_host on raw (pinned) host pointers."""
        _check(lib().rt_mlp_forward_host(self.handle, x_ptr, _dt(x_dtype), logits_ptr))

    def logits(self) -> np.ndarray:
        out = np.empty((self.lote, self.dims[-1]), np.float32)
        _check(lib().rt_mlp_logits(self.handle, out.ctypes.data))
        return out

    def last_loss(self) -> float:
        v = C.c_float()
        _check(lib().rt_mlp_last_loss(self.handle, C.byref(v)))
        return v.value

    def global_loss(self) -> float:
        """Mean loss of the last step over the global batch (all ranks'
        rows, summed in global row order); collective under a communicator."""
        v = C.c_float()
        _check(lib().rt_mlp_global_loss(self.handle, C.byref(v)))
        return v.value

    def weights(self):
        out = []
        for l in range(len(self.dims) - 1):
            w = np.empty((self.dims[l], self.dims[l + 1]), np.float32)
            b = np.empty((1, self.dims[l + 1]), np.float32)
            _check(lib().rt_mlp_weights(self.handle, l, w.ctypes.data, b.ctypes.data))
            out += [w, b]
        return out

    def grads(self):
        out = []
        for l in range(len(self.dims) - 1):
            w = np.empty((self.dims[l], self.dims[l + 1]), np.float32)
            b = np.empty((1, self.dims[l + 1]), np.float32)
            _check(lib().rt_mlp_grads(self.handle, l, w.ctypes.data, b.ctypes.data))
            out += [w, b]
        return out

    def set_weights(self, layer: int, w: np.ndarray | None, b: np.ndarray | None):
        w = None if w is None else np.ascontiguousarray(w, np.float32)
        b = None if b is None else np.ascontiguousarray(b, np.float32)
        _check(lib().rt_mlp_set_weights(self.handle, layer, None if w is None else w.ctypes.data,
                                        None if b is None else b.ctypes.data))

    def save_state(self) -> bytes:
        """Checkpoint of the training state: f32 weights and biases, Adam
        moments and step count (the rt_mlp_state_header layout)."""
        n = C.c_size_t()
        _check(lib().rt_mlp_state_size(self.handle, C.byref(n)))
        buf = np.empty(n.value, np.uint8)
        _check(lib().rt_mlp_save_state(self.handle, buf.ctypes.data, n.value))
        return buf.tobytes()

    def load_state(self, state: bytes):
        """Resume from save_state()'s bytes (same layer dims and optimiser)."""
        buf = np.frombuffer(state, np.uint8)
        _check(lib().rt_mlp_load_state(self.handle, buf.ctypes.data, buf.nbytes))

    def save(self, path: str):
        with open(path, "wb") as f:
            f.write(self.save_state())

    def load(self, path: str):
        with open(path, "rb") as f:
            self.load_state(f.read())

    def batch_size(self) -> int:
        return self.lote

    def dispatches_per_step(self) -> int:
        v = C.c_int()
        _check(lib().rt_mlp_dispatches_per_step(self.handle, C.byref(v)))
        return v.value

    dispatches_por_passo = dispatches_per_step

    def enable_timing(self, on: bool = True):
        _check(lib().rt_mlp_enable_timing(self.handle, int(on)))

    def op_times(self):
        """[(label, flops, ms)] of the last timed step (Gpu::perfilar, gpu/mod.rs:1245-1286)."""
        n = C.c_int()
        _check(lib().rt_mlp_op_count(self.handle, C.byref(n)))
        out = []
        for i in range(n.value):
            lab, fl, ms = C.c_char_p(), C.c_double(), C.c_float()
            _check(lib().rt_mlp_op_time(self.handle, i, C.byref(lab), C.byref(fl), C.byref(ms)))
            out.append((lab.value.decode(), fl.value, ms.value))
        return out

    def set_comm(self, comm: Comm | None):
        self._comm = comm
        _check(lib().rt_mlp_set_comm(self.handle, comm.handle if comm else None))

    def comm_mode(self) -> str:
        """How gradients are summed: "none", "allreduce", "allreduce_bf16",
        "sharded_opt" (NCCL reduce-scatter, sliced update, weight all-gather),
        "sharded_p2p" (the same, the reduce-scatter done by the dW GEMMs over
        peer memory) or "sharded_ce" (gradient pieces and updated weights
        moved by copy-engine copies between mapped buffers)."""
        v = C.c_int()
        _check(lib().rt_mlp_comm_mode(self.handle, C.byref(v)))
        return ("none", "allreduce", "allreduce_bf16", "sharded_opt", "sharded_p2p", "sharded_ce")[v.value]


def plan_layout(layer: int, d: int, units: int, world: int = 1, rank: int = 0, data_parallel: bool = True,
                fused_update: bool = False):
    """The plan's data-parallel layout of one layer, from the library's own
    rules (host only, no device): the [d+1, ld] block's leading dimension, and
    per dW chunk its rows [r0, r1) and this rank's flat weight slice
    (offset, length) under the sharded optimiser."""
    L = lib()
    ld = int(L.rt_plan_ld(units))
    chunks = int(L.rt_plan_dw_chunks(layer, d, units, int(data_parallel), int(fused_update)))
    out = []
    for c in range(chunks):
        r0 = int(L.rt_plan_chunk_row(d + 1, chunks, c))
        r1 = int(L.rt_plan_chunk_row(d + 1, chunks, c + 1))
        off = C.c_int64(0)
        n = int(L.rt_plan_shard_slice(d, units, r0, r1, world, rank, C.byref(off)))
        if n < 0:
            raise RtError(RT_ERR_INVALID, "rt_plan_shard_slice: bad arguments")
        out.append((r0, r1, int(off.value), n))
    return ld, out


def _is_bf16(t: GpuTensor) -> bool:
    return t.dtype_code == RT_BF16
