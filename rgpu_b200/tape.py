"""GPU autodiff with rtensor's names (crates/rtensor/src/{tape,ops,losses,nn,optim}.rs):
``Tape``, ``Param``, ``constant``, every ``Var`` op of ops.rs (add, sub, mul,
div with broadcasting, matmul, scale, offset, neg, square, sqrt, exp, ln,
relu, leaky_relu, sigmoid, tanh, sum, mean, softmax), ``backward``,
``Grads.of``, ``losses`` (mse, mae, softmax_cross_entropy,
binary_cross_entropy, one_hot, accuracy), ``Dense`` with every
``Activation``, ``Sequential``, ``Sgd`` (with momentum), ``Adam``.

Values and adjoints stay on the device; every op and the backward sweep only
enqueue kernels of librtgpu.so on the context stream.  Reading a value
(``Var.value()``, ``Var.item()``, ``Param.value()``, ``Grads.of``) is the only
point that waits for the device, as ``Gpu::download`` does in the reference.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .gpu import Gpu, GpuTensor, _check, lib, upload_labels

# rt_binary_op / rt_unary_op (include/rtgpu.h)
ADD, SUB, MUL, DIV = range(4)
SCALE, OFFSET, NEG, SQUARE, SQRT, EXP, LN, RELU, LEAKY_RELU, SIGMOID, TANH = range(11)


class Param:
    """Trainable tensor (tape.rs:76-132).  Shares one device buffer however
    many times it is watched."""

    def __init__(self, gpu: Gpu, value: np.ndarray, name: str = ""):
        v = np.ascontiguousarray(value, np.float32)
        if v.ndim == 1:
            v = v.reshape(1, -1)
        h = C.c_void_p()
        _check(lib().rt_param_create(gpu.handle, v.ctypes.data, v.shape[0], v.shape[1], C.byref(h)))
        self.gpu, self.handle, self.name = gpu, h, name
        self._shape = v.shape

    def shape(self):
        return self._shape

    def value(self) -> np.ndarray:
        out = np.empty(self._shape, np.float32)
        _check(lib().rt_param_read(self.handle, out.ctypes.data))
        return out

    def set(self, value: np.ndarray):
        v = np.ascontiguousarray(value, np.float32).reshape(self._shape)
        _check(lib().rt_param_write(self.handle, v.ctypes.data))

    def watch(self, tape: "Tape") -> "Var":
        h = C.c_void_p()
        _check(lib().rt_param_watch(self.handle, tape.handle, C.byref(h)))
        return Var(tape, h)

    def close(self):
        if self.handle and self.handle.value and self.gpu.alive():
            lib().rt_param_destroy(self.handle)
        self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Tape:
    """Recording of one forward pass (tape.rs:43-67)."""

    def __init__(self, gpu: Gpu):
        h = C.c_void_p()
        _check(lib().rt_tape_create(gpu.handle, C.byref(h)))
        self.gpu, self.handle = gpu, h

    def __len__(self):
        n = C.c_int()
        _check(lib().rt_tape_len(self.handle, C.byref(n)))
        return n.value

    def close(self):
        if self.handle and self.handle.value and self.gpu.alive():
            lib().rt_tape_destroy(self.handle)
        self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def constant(tape: Tape, value) -> "Var":
    """constant (tape.rs:70-73): a leaf that receives no useful gradient."""
    t = value if isinstance(value, GpuTensor) else tape.gpu.upload(np.ascontiguousarray(value, np.float32))
    h = C.c_void_p()
    _check(lib().rt_tape_constant(tape.handle, t.handle, C.byref(h)))
    return Var(tape, h)


def _view(gpu: Gpu, handle: C.c_void_p) -> np.ndarray | None:
    if not handle.value:
        return None
    t = GpuTensor(gpu, handle.value, owned=False)
    try:
        return gpu.download(t)
    finally:
        t.free()


class Var:
    """A node of the graph (tape.rs:136-184); owned by its tape."""

    def __init__(self, tape: Tape, handle: C.c_void_p):
        self.tape, self.handle = tape, handle

    def _op2(self, fn, other: "Var") -> "Var":
        h = C.c_void_p()
        _check(fn(self.handle, other.handle, C.byref(h)))
        return Var(self.tape, h)

    def _bin(self, other: "Var", op: int) -> "Var":
        h = C.c_void_p()
        _check(lib().rt_var_binary(self.handle, other.handle, op, C.byref(h)))
        return Var(self.tape, h)

    def _un(self, op: int, param: float = 0.0) -> "Var":
        h = C.c_void_p()
        _check(lib().rt_var_unary(self.handle, op, float(param), C.byref(h)))
        return Var(self.tape, h)

    def _red(self, fn) -> "Var":
        h = C.c_void_p()
        _check(fn(self.handle, C.byref(h)))
        return Var(self.tape, h)

    def matmul(self, other: "Var") -> "Var":
        return self._op2(lib().rt_var_matmul, other)

    def add(self, other: "Var") -> "Var":
        return self._op2(lib().rt_var_add, other)

    def sub(self, other: "Var") -> "Var":
        return self._bin(other, SUB)

    def mul(self, other: "Var") -> "Var":
        return self._bin(other, MUL)

    def div(self, other: "Var") -> "Var":
        return self._bin(other, DIV)

    def scale(self, k: float) -> "Var":
        return self._un(SCALE, k)

    def offset(self, k: float) -> "Var":
        return self._un(OFFSET, k)

    def neg(self) -> "Var":
        return self._un(NEG)

    def square(self) -> "Var":
        return self._un(SQUARE)

    def sqrt(self) -> "Var":
        return self._un(SQRT)

    def exp(self) -> "Var":
        return self._un(EXP)

    def ln(self) -> "Var":
        return self._un(LN)

    def relu(self) -> "Var":
        h = C.c_void_p()
        _check(lib().rt_var_relu(self.handle, C.byref(h)))
        return Var(self.tape, h)

    def leaky_relu(self, slope: float) -> "Var":
        return self._un(LEAKY_RELU, slope)

    def sigmoid(self) -> "Var":
        return self._un(SIGMOID)

    def tanh(self) -> "Var":
        return self._un(TANH)

    def sum(self) -> "Var":
        return self._red(lib().rt_var_sum)

    def mean(self) -> "Var":
        return self._red(lib().rt_var_mean)

    def softmax(self) -> "Var":
        return self._red(lib().rt_var_softmax)

    __matmul__ = matmul
    __add__ = add
    __sub__ = sub
    __mul__ = mul
    __truediv__ = div
    __neg__ = neg

    def value(self) -> np.ndarray:
        h = C.c_void_p()
        _check(lib().rt_var_value(self.handle, C.byref(h)))
        return _view(self.tape.gpu, h)

    def item(self) -> float:
        v = C.c_float()
        _check(lib().rt_var_item(self.handle, C.byref(v)))
        return v.value

    def backward(self) -> "Grads":
        _check(lib().rt_var_backward(self.handle))
        return Grads(self.tape)


class Grads:
    """Gradients of one backward sweep (tape.rs:232-249)."""

    def __init__(self, tape: Tape):
        self.tape = tape

    def of(self, p: Param) -> np.ndarray | None:
        h = C.c_void_p()
        _check(lib().rt_grads_of(self.tape.handle, p.handle, C.byref(h)))
        return _view(self.tape.gpu, h)


def _target(tape: Tape, target) -> GpuTensor:
    t = target if isinstance(target, GpuTensor) else tape.gpu.upload(np.ascontiguousarray(target, np.float32))
    tape._targets = getattr(tape, "_targets", []) + [t]  # alive as long as the tape
    return t


class losses:  # noqa: N801 - mirrors the rtensor module name
    @staticmethod
    def _loss(fn, pred: Var, target) -> Var:
        t = _target(pred.tape, target)
        h = C.c_void_p()
        _check(fn(pred.handle, t.handle, C.byref(h)))
        return Var(pred.tape, h)

    @staticmethod
    def mse(pred: Var, target) -> Var:
        """losses::mse (losses.rs:31-34)."""
        return losses._loss(lib().rt_loss_mse, pred, target)

    @staticmethod
    def mae(pred: Var, target) -> Var:
        """losses::mae (losses.rs:46-55)."""
        return losses._loss(lib().rt_loss_mae, pred, target)

    @staticmethod
    def binary_cross_entropy(probs: Var, target) -> Var:
        """losses::binary_cross_entropy (losses.rs:143-160)."""
        return losses._loss(lib().rt_loss_bce, probs, target)

    @staticmethod
    def one_hot(labels, classes: int) -> np.ndarray:
        """losses::one_hot (losses.rs:169-175), on the host."""
        out = np.zeros((len(labels), classes), np.float32)
        out[np.arange(len(labels)), np.asarray(labels)] = 1
        return out

    @staticmethod
    def accuracy(gpu: Gpu, logits, labels) -> float:
        """losses::accuracy (losses.rs:181-185) on the device."""
        z = logits if isinstance(logits, GpuTensor) else gpu.upload(np.ascontiguousarray(logits, np.float32))
        lab = labels if isinstance(labels, GpuTensor) else upload_labels(gpu, np.asarray(labels))
        out = C.c_float()
        _check(lib().rt_accuracy(gpu.handle, z.handle, lab.handle, C.byref(out)))
        return out.value

    @staticmethod
    def softmax_cross_entropy(logits: Var, targets) -> Var:
        """losses::softmax_cross_entropy (losses.rs:99-115).  `targets` is the
        one-hot [n, c] matrix of the reference, or integer labels [n]."""
        t = np.asarray(targets)
        labels = t.argmax(1).astype(np.uint32) if t.ndim == 2 else t.astype(np.uint32)
        lab = upload_labels(logits.tape.gpu, labels)
        h = C.c_void_p()
        _check(lib().rt_softmax_cross_entropy(logits.handle, lab.handle, C.byref(h)))
        logits.tape._labels = lab  # keep the device labels alive with the tape
        return Var(logits.tape, h)


def _param_array(params):
    return (C.c_void_p * len(params))(*[p.handle.value for p in params])


class Sgd:
    """Sgd::new / Sgd::with_momentum (optim.rs:64-77)."""

    def __init__(self, lr: float, momentum: float = 0.0, gpu: Gpu | None = None):
        self.lr, self.momentum, self.handle, self.gpu = lr, momentum, C.c_void_p(0), gpu

    @classmethod
    def with_momentum(cls, gpu: Gpu, lr: float, momentum: float) -> "Sgd":
        s = cls(lr, momentum, gpu)
        _check(lib().rt_sgd_create(gpu.handle, lr, momentum, C.byref(s.handle)))
        return s

    def step(self, params, grads: Grads):
        ps = list(params)
        if self.handle.value:
            _check(lib().rt_sgd_state_step(self.handle, len(ps), _param_array(ps), grads.tape.handle))
        else:
            _check(lib().rt_sgd_step(grads.tape.gpu.handle, len(ps), _param_array(ps), grads.tape.handle, self.lr))

    def close(self):
        if self.handle and self.handle.value and self.gpu and self.gpu.alive():
            lib().rt_sgd_destroy(self.handle)
        self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Adam:
    """Adam::new / with_betas (optim.rs:152-160)."""

    def __init__(self, gpu: Gpu, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8):
        h = C.c_void_p()
        _check(lib().rt_adam_create(gpu.handle, lr, beta1, beta2, eps, C.byref(h)))
        self.gpu, self.handle = gpu, h

    def step(self, params, grads: Grads):
        ps = list(params)
        _check(lib().rt_adam_step(self.handle, len(ps), _param_array(ps), grads.tape.handle))

    def close(self):
        if self.handle and self.handle.value and self.gpu.alive():
            lib().rt_adam_destroy(self.handle)
        self.handle = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def activate(z: Var, activation) -> Var:
    """Activation::apply (nn.rs:48-60): "linear", "relu", "sigmoid", "tanh" or
    ("leaky_relu", slope)."""
    if activation == "linear":
        return z
    if activation == "relu":
        return z.relu()
    if activation == "sigmoid":
        return z.sigmoid()
    if activation == "tanh":
        return z.tanh()
    if isinstance(activation, tuple) and activation[0] == "leaky_relu":
        return z.leaky_relu(activation[1])
    raise ValueError(f"unknown activation {activation!r}")


class Dense:
    """Dense layer (nn.rs:108-159): A = phi(X W + 1 b)."""

    def __init__(self, gpu: Gpu, w: np.ndarray, b: np.ndarray | None = None, relu: bool = True,
                 activation=None):
        w = np.ascontiguousarray(w, np.float32)
        self.w = Param(gpu, w, "W")
        self.b = Param(gpu, np.zeros((1, w.shape[1]), np.float32) if b is None else b, "b")
        self.activation = activation if activation is not None else ("relu" if relu else "linear")

    def forward(self, x: Var) -> Var:
        z = x.matmul(self.w.watch(x.tape)).add(self.b.watch(x.tape))
        return activate(z, self.activation)

    def params(self):
        return [self.w, self.b]


class Sequential:
    """Sequential (nn.rs:161-207)."""

    def __init__(self, layers=None):
        self.layers = list(layers or [])

    def add(self, layer) -> "Sequential":
        self.layers.append(layer)
        return self

    def forward(self, x: Var) -> Var:
        for layer in self.layers:
            x = layer.forward(x)
        return x

    def params(self):
        return [p for layer in self.layers for p in layer.params()]

    def predict(self, gpu: Gpu, x: np.ndarray) -> np.ndarray:
        """Sequential::predict (nn.rs:184-188): a forward pass on a fresh tape."""
        tape = Tape(gpu)
        try:
            return self.forward(constant(tape, x)).value()
        finally:
            tape.close()
