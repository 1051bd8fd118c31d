"""CPU oracle: ctypes binding of the C++ restatement of rtensor's CPU backend.

TEST INFRASTRUCTURE.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import this
package.  The product library (``rgpu_b200``) never does: it is the checker,
not the thing measured or shipped.

Reference: MMMejias39/RGPU, crates/rtensor/src/{rng,tensor,ops,tape,nn,
losses,optim}.rs.  Each wrapped symbol cites its reference function in
``oracle/rtensor_cpu.h``.  Parity pin: tests/test_oracle.py re-runs the
known-answer tests and the central-difference gradient checks of
crates/rtensor/tests/autodiff.rs against this restatement.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = C.POINTER(C.c_float)
_u32p = C.POINTER(C.c_uint32)
_u64p = C.POINTER(C.c_uint64)
_szp = C.POINTER(C.c_size_t)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.or_rng_seed.restype = C.c_uint64
        L.or_rng_seed.argtypes = [C.c_uint64]
        for name in ("or_rng_uniform", "or_rng_normal"):
            getattr(L, name).argtypes = [_u64p, _f32p, C.c_size_t]
        L.or_rng_range.argtypes = [_u64p, C.c_float, C.c_float, _f32p, C.c_size_t]
        L.or_rng_below.argtypes = [_u64p, C.c_uint64, _u32p, C.c_size_t]
        L.or_matmul.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]
        L.or_transpose.argtypes = [_f32p, _f32p, C.c_size_t, C.c_size_t]
        L.or_reduce_rows.argtypes = [_f32p, _f32p, C.c_size_t, C.c_size_t]
        L.or_softmax_rows.argtypes = [_f32p, _f32p, C.c_size_t, C.c_size_t]
        L.or_softmax_xent.restype = C.c_float
        L.or_softmax_xent.argtypes = [_f32p, _f32p, C.c_size_t, C.c_size_t, _f32p]
        L.or_one_hot.argtypes = [_u32p, C.c_size_t, C.c_size_t, _f32p]
        L.or_mlp_new.restype = C.c_void_p
        L.or_mlp_new.argtypes = [C.c_int, _szp]
        L.or_mlp_free.argtypes = [C.c_void_p]
        L.or_mlp_set.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
        L.or_mlp_get.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
        L.or_mlp_get_grads.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
        L.or_mlp_get_logits.argtypes = [C.c_void_p, _f32p]
        L.or_mlp_init_glorot.argtypes = [C.c_void_p, _u64p]
        L.or_mlp_init_kaiming.argtypes = [C.c_void_p, _u64p]
        L.or_mlp_train_step.restype = C.c_float
        L.or_mlp_train_step.argtypes = [C.c_void_p, _f32p, _u32p, C.c_size_t, C.c_int,
                                        C.c_float, C.c_int, C.c_int]
        L.or_mlp_set_bf16_emulation.argtypes = [C.c_void_p, C.c_int]
        L.or_mlp_set_rounding.argtypes = [C.c_void_p, C.c_int]
        L.or_mlp_forward.restype = C.c_float
        L.or_mlp_forward.argtypes = [C.c_void_p, _f32p, _u32p, C.c_size_t, C.c_int]
        L.or_adam_update.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_size_t, C.c_float,
                                     C.c_float, C.c_float, C.c_float, C.c_int]
        L.or_sgd_update.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_float, C.c_float]
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def _u(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_u32p)


class Rng:
    """rtensor's xorshift64* generator (rng.rs:1-49)."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(lib().or_rng_seed(seed))

    def uniform(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().or_rng_uniform(C.byref(self.state), _f(out), n)
        return out

    def range(self, lo: float, hi: float, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().or_rng_range(C.byref(self.state), lo, hi, _f(out), n)
        return out

    def normal(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().or_rng_normal(C.byref(self.state), _f(out), n)
        return out

    def below(self, bound: int, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        lib().or_rng_below(C.byref(self.state), bound, _u(out), n)
        return out


def matmul(a: np.ndarray, b: np.ndarray, threads: int = 1) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), np.float32)
    lib().or_matmul(_f(a), _f(b), _f(c), m, k, n, threads)
    return c


def transpose(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    r, c = a.shape
    out = np.empty((c, r), np.float32)
    lib().or_transpose(_f(a), _f(out), r, c)
    return out


def reduce_rows(g: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    n, m = g.shape
    out = np.empty((1, m), np.float32)
    lib().or_reduce_rows(_f(g), _f(out), n, m)
    return out


def softmax_rows(z: np.ndarray) -> np.ndarray:
    z = np.ascontiguousarray(z, np.float32)
    r, c = z.shape
    out = np.empty_like(z)
    lib().or_softmax_rows(_f(z), _f(out), r, c)
    return out


def one_hot(labels, classes: int) -> np.ndarray:
    lab = np.ascontiguousarray(labels, np.uint32)
    out = np.empty((lab.size, classes), np.float32)
    lib().or_one_hot(_u(lab), lab.size, classes, _f(out))
    return out


def softmax_xent(logits: np.ndarray, onehot: np.ndarray):
    """Returns (loss, dlogits) of the softmax_cross_entropy node."""
    z = np.ascontiguousarray(logits, np.float32)
    y = np.ascontiguousarray(onehot, np.float32)
    n, c = z.shape
    d = np.empty_like(z)
    loss = lib().or_softmax_xent(_f(z), _f(y), n, c, _f(d))
    return float(loss), d


def adam_update(theta, m, v, g, lr, t, beta1=0.9, beta2=0.999, eps=1e-8):
    lib().or_adam_update(_f(theta), _f(m), _f(v), _f(np.ascontiguousarray(g, np.float32)),
                         theta.size, lr, beta1, beta2, eps, t)


def sgd_update(theta, g, lr):
    lib().or_sgd_update(_f(theta), None, _f(np.ascontiguousarray(g, np.float32)),
                        theta.size, lr, 0.0)


OPT_NONE, OPT_SGD, OPT_ADAM = 0, 1, 2

# bf16 rounding points of the GPU plan, for Mlp.set_rounding (rtensor_cpu.h).
ROUND_X, ROUND_W, ROUND_ACT, ROUND_DELTA, SPLIT_ACT = 1, 2, 4, 8, 16
# The bf16 plan with single-bf16 activations, and with split (hi + lo) ones.
BF16_PLAIN = ROUND_X | ROUND_W | ROUND_ACT | ROUND_DELTA
BF16_SPLIT = ROUND_X | ROUND_W | ROUND_DELTA | SPLIT_ACT


class Mlp:
    """Sequential of Dense layers (ReLU hidden, Linear output) trained with
    softmax cross-entropy through the tape, as rtensor's CPU path does."""

    def __init__(self, dims):
        self.dims = [int(d) for d in dims]
        self.L = len(self.dims) - 1
        arr = (C.c_size_t * len(self.dims))(*self.dims)
        self._h = lib().or_mlp_new(self.L, arr)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_mlp_free(self._h)
            self._h = None

    def set_bf16_emulation(self, on: bool = True):
        """Round at the bf16 GPU plan's storage points (test-only option, not
        the reference algorithm; see rtensor_cpu.h)."""
        lib().or_mlp_set_bf16_emulation(self._h, int(bool(on)))

    def set_rounding(self, flags: int):
        """Round to bf16 at the chosen storage points (ROUND_* / SPLIT_ACT
        flags; 0 = the plain reference).  Test-only, see rtensor_cpu.h."""
        lib().or_mlp_set_rounding(self._h, int(flags))

    def init_glorot(self, rng: Rng):
        lib().or_mlp_init_glorot(self._h, C.byref(rng.state))

    def init_kaiming(self, rng: Rng):
        lib().or_mlp_init_kaiming(self._h, C.byref(rng.state))

    def set_params(self, params):
        for l in range(self.L):
            w = np.ascontiguousarray(params[2 * l], np.float32)
            b = np.ascontiguousarray(params[2 * l + 1], np.float32)
            lib().or_mlp_set(self._h, l, _f(w), _f(b))

    def params(self):
        out = []
        for l in range(self.L):
            w = np.empty((self.dims[l], self.dims[l + 1]), np.float32)
            b = np.empty((1, self.dims[l + 1]), np.float32)
            lib().or_mlp_get(self._h, l, _f(w), _f(b))
            out += [w, b]
        return out

    def grads(self):
        out = []
        for l in range(self.L):
            w = np.empty((self.dims[l], self.dims[l + 1]), np.float32)
            b = np.empty((1, self.dims[l + 1]), np.float32)
            lib().or_mlp_get_grads(self._h, l, _f(w), _f(b))
            out += [w, b]
        return out

    def logits(self, n):
        out = np.empty((n, self.dims[-1]), np.float32)
        lib().or_mlp_get_logits(self._h, _f(out))
        return out

    def train_step(self, x, labels, optimizer=OPT_NONE, lr=0.0, threads=1, input_grad=True):
        x = np.ascontiguousarray(x, np.float32)
        lab = np.ascontiguousarray(labels, np.uint32)
        return float(lib().or_mlp_train_step(self._h, _f(x), _u(lab), x.shape[0], optimizer,
                                             lr, threads, int(input_grad)))

    def forward(self, x, labels=None, threads=1):
        x = np.ascontiguousarray(x, np.float32)
        lab = None if labels is None else np.ascontiguousarray(labels, np.uint32)
        return float(lib().or_mlp_forward(self._h, _f(x), None if lab is None else _u(lab),
                                          x.shape[0], threads))
