"""CPU restatement of rtensor's autodiff tape for the parity tests: TEST
INFRASTRUCTURE ONLY.  Only tests/ import it; the product library never calls
it.

It restates, in numpy float32, the reverse-mode engine and the ops of
crates/rtensor/src:
  tape.rs:43-249     Tape, constant, Param.watch (leaf reuse), Var.backward
                     (one reverse sweep, in-place accumulation), Grads.of
  ops.rs:49-309      add/sub/mul/div with broadcasting, matmul, scale, offset,
                     neg, square, sqrt, exp, ln, relu, leaky_relu, sigmoid,
                     tanh, sum, mean, softmax
  tensor.rs:183-246  zip broadcasting; 399-438 reduce_to; 455-472 softmax_rows;
                     476-492 argmax_rows
  losses.rs:31-185   mse, mae, softmax_cross_entropy, binary_cross_entropy,
                     one_hot, accuracy
  optim.rs:44-198    Sgd (with momentum), Adam
  nn.rs:40-207       Activation, Dense, Sequential
Sums run in the reference's sequential f32 order (np.cumsum); elementwise
arithmetic is IEEE f32 like Rust's.  Transcendentals come from numpy, not
from Rust's libm, so exp/ln/tanh may differ in the last bit.
It is pinned by tests/test_oracle_tape.py on the reference's own known
answers and gradient checks (crates/rtensor/tests/autodiff.rs).
"""
from __future__ import annotations

import numpy as np

F = np.float32


def _f(x) -> np.ndarray:
    return np.asarray(x, dtype=F)


def seq_sum(x: np.ndarray, axis=None) -> np.ndarray:
    """f32 sum in sequential order (Rust's iter().sum(), tensor.rs:272-274)."""
    x = _f(x)
    if axis is None:
        flat = x.reshape(-1)
        return np.cumsum(flat, dtype=F)[-1] if flat.size else F(0)
    return np.take(np.cumsum(x, axis=axis, dtype=F), -1, axis=axis)


def broadcast_shape(a, b):
    """broadcast_shapes (tensor.rs) for rank 2."""
    out = []
    for x, y in zip(a, b):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise ValueError(f"shapes {a} and {b} do not broadcast")
    return tuple(out)


def reduce_to(g: np.ndarray, shape) -> np.ndarray:
    """Tensor::reduce_to (tensor.rs:399-438): sum the broadcast axes."""
    shape = tuple(shape)
    if g.shape == shape:
        return g.copy()
    if shape[0] * shape[1] == 1:
        return _f(seq_sum(g)).reshape(shape)
    out = g
    if shape[0] == 1 and g.shape[0] != 1:
        out = seq_sum(out, axis=0).reshape(1, -1)
    if shape[1] == 1 and g.shape[1] != 1:
        out = seq_sum(out, axis=1).reshape(-1, 1)
    return _f(out)


def softmax_rows(z: np.ndarray) -> np.ndarray:
    """tensor.rs:455-472: exp(z - max) / sequential sum, per row."""
    z = _f(z)
    mx = z.max(axis=1, keepdims=True)
    e = np.exp(z - mx).astype(F)
    return (e / seq_sum(e, axis=1).reshape(-1, 1)).astype(F)


def argmax_rows(z: np.ndarray) -> np.ndarray:
    """tensor.rs:476-492: the first maximum of each row, element 0 first."""
    out = np.zeros(z.shape[0], np.int64)
    for i, row in enumerate(_f(z)):
        best, bv = 0, row[0] if row.size else -np.inf
        for j in range(1, row.size):
            if row[j] > bv:
                best, bv = j, row[j]
        out[i] = best
    return out


class Tape:
    """tape.rs:43-67."""

    def __init__(self):
        self.nodes = []  # (parents, backward(g) -> list of parent adjoints, value)
        self.param_nodes = {}

    def __len__(self):
        return len(self.nodes)

    def push(self, parents, backward, value) -> "Var":
        self.nodes.append((parents, backward, _f(value)))
        return Var(self, len(self.nodes) - 1)


_next_id = [0]


class Param:
    """tape.rs:76-132: a trainable tensor, one leaf per tape."""

    def __init__(self, value, name=""):
        v = _f(value)
        self.value = v.reshape(1, -1).copy() if v.ndim == 1 else v.copy()
        self.name = name
        _next_id[0] += 1
        self.id = _next_id[0]

    def watch(self, tape: Tape) -> "Var":
        if self.id in tape.param_nodes:
            return Var(tape, tape.param_nodes[self.id])
        v = tape.push([], None, self.value)
        tape.param_nodes[self.id] = v.idx
        return v


def constant(tape: Tape, value) -> "Var":
    """tape.rs:70-73."""
    v = _f(value)
    return tape.push([], None, v.reshape(1, -1) if v.ndim == 1 else v)


class Grads:
    """tape.rs:232-249."""

    def __init__(self, tape, grads):
        self.tape, self.grads = tape, grads

    def of(self, p: Param):
        i = self.tape.param_nodes.get(p.id)
        return None if i is None else self.grads.get(i)

    def of_var(self, v: "Var"):
        return self.grads.get(v.idx)


class Var:
    """tape.rs:136-184 and ops.rs:38-309."""

    def __init__(self, tape: Tape, idx: int):
        self.tape, self.idx = tape, idx

    def value(self) -> np.ndarray:
        return self.tape.nodes[self.idx][2]

    @property
    def shape(self):
        return self.value().shape

    def item(self) -> float:
        v = self.value()
        assert v.size == 1
        return float(v.reshape(-1)[0])

    def _unary(self, value, bw) -> "Var":
        return self.tape.push([self.idx], lambda g: [bw(g)], value)

    def _binary(self, other, value, bw) -> "Var":
        return self.tape.push([self.idx, other.idx], bw, value)

    # ops.rs:49-101: broadcasting elementwise ops; adjoints reduced to shape
    def _zip(self, other, f):
        a, b = self.value(), other.value()
        shape = broadcast_shape(a.shape, b.shape)
        return _f(f(np.broadcast_to(a, shape), np.broadcast_to(b, shape))), shape

    def add(self, other):
        sa, sb = self.shape, other.shape
        value, _ = self._zip(other, lambda a, b: a + b)
        return self._binary(other, value, lambda g: [reduce_to(g, sa), reduce_to(g, sb)])

    def sub(self, other):
        sa, sb = self.shape, other.shape
        value, _ = self._zip(other, lambda a, b: a - b)
        return self._binary(other, value, lambda g: [reduce_to(g, sa), reduce_to(-g, sb)])

    def mul(self, other):
        a, b = self.value(), other.value()
        value, shape = self._zip(other, lambda x, y: x * y)
        ab, bb = np.broadcast_to(a, shape), np.broadcast_to(b, shape)
        return self._binary(other, value, lambda g: [reduce_to(_f(g * bb), a.shape), reduce_to(_f(g * ab), b.shape)])

    def div(self, other):
        a, b = self.value(), other.value()
        value, shape = self._zip(other, lambda x, y: x / y)
        ab, bb = np.broadcast_to(a, shape), np.broadcast_to(b, shape)

        def bw(g):
            da = reduce_to(_f(g / bb), a.shape)
            db = reduce_to(_f(-(_f(g * ab) / _f(bb * bb))), b.shape)
            return [da, db]

        return self._binary(other, value, bw)

    def matmul(self, other):
        """ops.rs:125-129 with the C++ restatement of Tensor::matmul and
        Tensor::t (tensor.rs:318-373, 132-155)."""
        from . import matmul as mm, transpose as tr

        a, b = self.value(), other.value()
        value = mm(a, b)
        return self._binary(other, value, lambda g: [mm(_f(g), tr(b)), mm(tr(a), _f(g))])

    # ops.rs:132-227: pointwise
    def scale(self, k):
        k = F(k)
        return self._unary(_f(self.value() * k), lambda g: _f(g * k))

    def offset(self, k):
        return self._unary(_f(self.value() + F(k)), lambda g: g.copy())

    def neg(self):
        return self.scale(-1.0)

    def square(self):
        x = self.value()
        return self._unary(_f(x * x), lambda g: _f(_f(g * x) * F(2)))

    def sqrt(self):
        y = _f(np.sqrt(self.value()))
        return self._unary(y, lambda g: _f(g / _f(y * F(2))))

    def exp(self):
        y = _f(np.exp(self.value()))
        return self._unary(y, lambda g: _f(g * y))

    def ln(self):
        x = self.value()
        return self._unary(_f(np.log(np.maximum(x, F(1e-12)))), lambda g: _f(g / x))

    def relu(self):
        x = self.value()
        return self._unary(_f(np.maximum(x, F(0))), lambda g: _f(g * (x > 0).astype(F)))

    def leaky_relu(self, slope):
        x, s = self.value(), F(slope)
        return self._unary(_f(np.where(x > 0, x, _f(s * x))), lambda g: _f(g * np.where(x > 0, F(1), s)))

    def sigmoid(self):
        y = _f(F(1) / _f(F(1) + _f(np.exp(-self.value()))))
        return self._unary(y, lambda g: _f(g * _f(y * _f(F(1) - y))))

    def tanh(self):
        y = _f(np.tanh(self.value()))
        return self._unary(y, lambda g: _f(g * _f(F(1) - _f(y * y))))

    # ops.rs:239-309: contractions
    def sum(self):
        shape = self.shape
        return self._unary(_f(seq_sum(self.value())).reshape(1, 1), lambda g: np.full(shape, g.reshape(-1)[0], F))

    def mean(self):
        shape, n = self.shape, F(self.value().size)
        value = _f(seq_sum(self.value()) / n).reshape(1, 1)
        return self._unary(value, lambda g: np.full(shape, _f(g.reshape(-1)[0] / n), F))

    def softmax(self):
        s = softmax_rows(self.value())

        def bw(g):
            dot = seq_sum(_f(g * s), axis=1).reshape(-1, 1)
            return _f(s * _f(g - dot))

        return self._unary(s, bw)

    __add__, __sub__, __mul__, __truediv__, __matmul__ = add, sub, mul, div, matmul

    def __neg__(self):
        return self.neg()

    def backward(self) -> Grads:
        """tape.rs:187-229: one reverse sweep from a scalar root."""
        assert self.value().size == 1, "backward() needs a scalar"
        grads = {self.idx: np.ones((1, 1), F)}
        for i in range(self.idx, -1, -1):
            parents, bw, _ = self.tape.nodes[i]
            if bw is None or i not in grads:
                continue
            for p, gp in zip(parents, bw(grads[i])):
                gp = _f(gp)
                grads[p] = gp.copy() if p not in grads else _f(grads[p] + gp)
        return Grads(self.tape, grads)


class losses:  # noqa: N801 - mirrors the rtensor module name
    @staticmethod
    def mse(pred: Var, target) -> Var:
        """losses.rs:31-34."""
        return pred.sub(constant(pred.tape, target)).square().mean()

    @staticmethod
    def mae(pred: Var, target) -> Var:
        """losses.rs:46-55: one node over d = pred - target."""
        d = pred.sub(constant(pred.tape, target))
        dv = d.value()
        sign = np.where(dv >= 0, F(1), F(-1))
        n = F(dv.size)
        value = _f(seq_sum(np.abs(dv)) / n).reshape(1, 1)
        return d._unary(value, lambda g: _f(sign * _f(g.reshape(-1)[0] / n)))

    @staticmethod
    def softmax_cross_entropy(logits: Var, targets) -> Var:
        """losses.rs:99-115 with one-hot targets."""
        y = _f(targets)
        p = softmax_rows(logits.value())
        batch = F(logits.shape[0])
        total = F(0)
        for pv, yv in zip(p.reshape(-1), y.reshape(-1)):
            if yv != 0:
                total = F(total - F(yv * F(np.log(max(pv, F(1e-12))))))
        return logits._unary(_f(total / batch).reshape(1, 1), lambda g: _f(_f(p - y) * _f(g.reshape(-1)[0] / batch)))

    @staticmethod
    def binary_cross_entropy(probs: Var, targets) -> Var:
        """losses.rs:143-160."""
        p, y = probs.value(), _f(targets)
        batch = F(p.size)
        c = np.clip(p, F(1e-7), F(1) - F(1e-7)).astype(F)
        total = F(0)
        for cv, yv in zip(c.reshape(-1), y.reshape(-1)):
            total = F(total - F(F(yv * F(np.log(cv))) + F(F(F(1) - yv) * F(np.log(F(1) - cv)))))
        d = _f(_f(c - y) / _f(c * _f(F(1) - c)))
        return probs._unary(_f(total / batch).reshape(1, 1), lambda g: _f(d * _f(g.reshape(-1)[0] / batch)))

    @staticmethod
    def one_hot(labels, classes) -> np.ndarray:
        """losses.rs:169-175."""
        out = np.zeros((len(labels), classes), F)
        out[np.arange(len(labels)), np.asarray(labels)] = 1
        return out

    @staticmethod
    def accuracy(logits, labels) -> float:
        """losses.rs:181-185."""
        pred = argmax_rows(logits)
        return float(F(np.sum(pred == np.asarray(labels))) / F(len(labels)))


class Sgd:
    """optim.rs:44-116."""

    def __init__(self, lr, momentum=0.0):
        self.lr, self.mu, self.velocity = F(lr), F(momentum), {}

    def step(self, params, grads: Grads):
        for p in params:
            g = grads.of(p)
            if g is None:
                continue
            if self.mu == 0:
                p.value = _f(p.value - _f(g * self.lr))
            else:
                v = self.velocity.get(p.id, np.zeros_like(p.value))
                v = _f(_f(v * self.mu) + _f(g * self.lr))
                self.velocity[p.id] = v
                p.value = _f(p.value - v)


class Adam:
    """optim.rs:140-198: pre-inverted bias corrections, powi as repeated squaring."""

    def __init__(self, lr, beta1=0.9, beta2=0.999, eps=1e-8):
        self.lr, self.b1, self.b2, self.eps = F(lr), F(beta1), F(beta2), F(eps)
        self.t, self.m, self.v = 0, {}, {}

    @staticmethod
    def _powi(b, n):
        r, base = F(1), F(b)
        while n:
            if n & 1:
                r = F(r * base)
            base = F(base * base)
            n >>= 1
        return r

    def step(self, params, grads: Grads):
        self.t += 1
        ic1 = F(F(1) / F(F(1) - self._powi(self.b1, self.t)))
        ic2 = F(F(1) / F(F(1) - self._powi(self.b2, self.t)))
        omb1, omb2 = F(F(1) - self.b1), F(F(1) - self.b2)
        for p in params:
            g = grads.of(p)
            if g is None:
                continue
            m = self.m.get(p.id, np.zeros_like(p.value))
            v = self.v.get(p.id, np.zeros_like(p.value))
            m = _f(_f(m * self.b1) + _f(g * omb1))
            v = _f(_f(v * self.b2) + _f(_f(g * g) * omb2))
            self.m[p.id], self.v[p.id] = m, v
            mh, vh = _f(m * ic1), _f(v * ic2)
            p.value = _f(p.value - _f(_f(mh / _f(_f(np.sqrt(vh)) + self.eps)) * self.lr))


class Dense:
    """nn.rs:108-159: A = act(X W + 1 b)."""

    def __init__(self, w, b=None, activation="linear"):
        w = _f(w)
        self.w = Param(w, "W")
        self.b = Param(np.zeros((1, w.shape[1]), F) if b is None else b, "b")
        self.activation = activation

    def forward(self, x: Var) -> Var:
        z = x.matmul(self.w.watch(x.tape)).add(self.b.watch(x.tape))
        return activate(z, self.activation)

    def params(self):
        return [self.w, self.b]


def activate(z: Var, activation) -> Var:
    """Activation::apply (nn.rs:48-60)."""
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
    raise ValueError(f"unknown activation {activation}")


class Sequential:
    """nn.rs:161-207."""

    def __init__(self, layers=None):
        self.layers = list(layers or [])

    def forward(self, x: Var) -> Var:
        for layer in self.layers:
            x = layer.forward(x)
        return x

    def params(self):
        return [p for layer in self.layers for p in layer.params()]

    def predict(self, x) -> np.ndarray:
        tape = Tape()
        return self.forward(constant(tape, x)).value()


def dense_weights(rng, inputs, units):
    """Dense::new (nn.rs:122-130): W ~ rng.range(-l, l) row-major over
    [inputs, units], l = sqrt(6 / (inputs + units)); `rng` is oracle.Rng."""
    lim = float(np.sqrt(F(6.0) / F(inputs + units)))
    return rng.range(-lim, lim, inputs * units).reshape(inputs, units).astype(F)
