"""The rest of ops.rs / losses.rs on the GPU tape against the tape oracle
(oracle/tape_ref.py), and rtensor's own autodiff tests
(crates/rtensor/tests/autodiff.rs) run on the GPU tape."""
import zlib

import numpy as np
import pytest

import oracle
import rgpu_b200
from oracle import tape_ref as R
from rgpu_b200 import tape as T
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
F = np.float32


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _close(got, want, tol, what):
    assert got.shape == want.shape, (what, got.shape, want.shape)
    e = rel_l2(got, want)
    assert e <= tol, f"{what}: rel L2 {e:.2e} > {tol}"


def _close_sum(got, want, abs_terms, what):
    # A sum taken in another order than the oracle's sequential one: both are
    # within n eps sum|terms| of the exact value, so compare on that scale
    # (elementwise; abs_terms = the sum of the magnitudes of each output's terms).
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    bound = 2e-6 * np.asarray(abs_terms, np.float64) + 1e-30
    worst = np.max(np.abs(got - want) / bound)
    assert worst <= 1.0, f"{what}: {worst:.2f} x the sum-order bound"


def _reduce_abs(c, shape):
    """sum of |c| over the axes broadcast to reach c's shape from `shape` (f64)."""
    c = np.abs(np.asarray(c, np.float64))
    if shape[0] == 1 and c.shape[0] != 1:
        c = c.sum(axis=0, keepdims=True)
    if shape[1] == 1 and c.shape[1] != 1:
        c = c.sum(axis=1, keepdims=True)
    return c


UNARY = [("scale", (1.7,)), ("offset", (-0.3,)), ("neg", ()), ("square", ()), ("sqrt", ()), ("exp", ()), ("ln", ()),
         ("relu", ()), ("leaky_relu", (0.1,)), ("sigmoid", ()), ("tanh", ())]


@pytest.mark.parametrize("name,args", UNARY)
def test_unary_op_value_and_adjoint(gpu, name, args):
    rng = np.random.default_rng(len(name))
    x = rng.standard_normal((37, 53)).astype(F)
    if name in ("sqrt", "ln"):
        x = np.abs(x) + F(0.05)
    w = rng.standard_normal((37, 53)).astype(F)  # upstream adjoint through sum(y * w)
    pg, pc = T.Param(gpu, x), R.Param(x)
    tg, tc = T.Tape(gpu), R.Tape()
    yg = getattr(pg.watch(tg), name)(*args)
    yc = getattr(pc.watch(tc), name)(*args)
    _close(yg.value(), yc.value(), 2e-7 if name in ("scale", "offset", "neg", "square", "relu", "leaky_relu") else 2e-6,
           f"{name} value")
    gg = yg.mul(T.constant(tg, w)).sum().backward().of(pg)
    gc = yc.mul(R.constant(tc, w)).sum().backward().of(pc)
    _close(gg, gc, 2e-6, f"{name} adjoint")


SHAPES = [((33, 47), (33, 47)), ((33, 47), (1, 47)), ((1, 47), (33, 47)), ((33, 47), (33, 1)), ((33, 1), (33, 47)),
          ((33, 47), (1, 1)), ((1, 1), (33, 47)), ((1, 47), (33, 1)), ((1, 1), (1, 1))]


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("sa,sb", SHAPES)
def test_broadcasting_binary_op(gpu, op, sa, sb):
    # value over the broadcast shape, each adjoint reduced back to its operand
    rng = np.random.default_rng(zlib.crc32(repr((op, sa, sb)).encode()))
    a = rng.standard_normal(sa).astype(F)
    b = rng.standard_normal(sb).astype(F)
    if op == "div":
        b = (np.abs(b) + F(0.5)) * np.sign(b + F(1e-3))
    out_shape = R.broadcast_shape(sa, sb)
    w = rng.standard_normal(out_shape).astype(F)
    pa, pb, qa, qb = T.Param(gpu, a), T.Param(gpu, b), R.Param(a), R.Param(b)
    tg, tc = T.Tape(gpu), R.Tape()
    cg = getattr(pa.watch(tg), op)(pb.watch(tg))
    cc = getattr(qa.watch(tc), op)(qb.watch(tc))
    _close(cg.value(), cc.value(), 1e-7, f"{op} value")
    g = cg.mul(T.constant(tg, w)).sum().backward()
    gc = cc.mul(R.constant(tc, w)).sum().backward()
    # a broadcast operand's adjoint is a sum over the broadcast axes
    A, B = np.broadcast_to(a, out_shape).astype(np.float64), np.broadcast_to(b, out_shape).astype(np.float64)
    W = w.astype(np.float64)
    ca = {"add": W, "sub": W, "mul": W * B, "div": W / B}[op]
    cb = {"add": W, "sub": W, "mul": W * A, "div": W * A / (B * B)}[op]
    _close_sum(g.of(pa), gc.of(qa), _reduce_abs(ca, sa), f"{op} adjoint of a")
    _close_sum(g.of(pb), gc.of(qb), _reduce_abs(cb, sb), f"{op} adjoint of b")


def test_shapes_that_do_not_broadcast_are_an_error(gpu):
    t = T.Tape(gpu)
    a = T.constant(t, np.ones((3, 4), F))
    b = T.constant(t, np.ones((2, 4), F))
    with pytest.raises(rgpu_b200.RtError):
        a.sub(b)


@pytest.mark.parametrize("shape", [(1, 1), (7, 300), (513, 129)])
def test_sum_mean_softmax(gpu, shape):
    rng = np.random.default_rng(shape[1])
    x = (rng.standard_normal(shape) * 3).astype(F)
    w = rng.standard_normal(shape).astype(F)
    for name in ("sum", "mean", "softmax"):
        pg, pc = T.Param(gpu, x), R.Param(x)
        tg, tc = T.Tape(gpu), R.Tape()
        yg, yc = getattr(pg.watch(tg), name)(), getattr(pc.watch(tc), name)()
        if name == "softmax":
            _close(yg.value(), yc.value(), 5e-6, f"{name} value")
        else:
            _close_sum(yg.value(), yc.value(), np.abs(x.astype(np.float64)).sum() / (x.size if name == "mean" else 1),
                       f"{name} value")
        lg = yg.mul(T.constant(tg, w[:1, :1] if name != "softmax" else w)).sum()
        lc = yc.mul(R.constant(tc, w[:1, :1] if name != "softmax" else w)).sum()
        _close(lg.backward().of(pg), lc.backward().of(pc), 2e-6, f"{name} adjoint")


@pytest.mark.parametrize("loss", ["mse", "mae", "binary_cross_entropy"])
def test_losses_value_and_adjoint(gpu, loss):
    rng = np.random.default_rng(7)
    if loss == "binary_cross_entropy":
        p = rng.uniform(0.0, 1.0, (64, 3)).astype(F)
        p[0, 0], p[1, 1] = 0.0, 1.0  # the clamp at 1e-7 and 1 - 1e-7
        y = (rng.uniform(0, 1, (64, 3)) > 0.5).astype(F)
    else:
        p = rng.standard_normal((64, 3)).astype(F)
        y = rng.standard_normal((64, 3)).astype(F)
        y[0, 0] = p[0, 0]  # sign(0) = +1 for mae
    pg, pc = T.Param(gpu, p), R.Param(p)
    lg = getattr(T.losses, loss)(pg.watch(T.Tape(gpu)), y)
    lc = getattr(R.losses, loss)(pc.watch(R.Tape()), y)
    if loss == "mse":
        terms = (p.astype(np.float64) - y) ** 2
    elif loss == "mae":
        terms = np.abs(p.astype(np.float64) - y)
    else:
        c = np.clip(p.astype(np.float64), 1e-7, 1 - 1e-7)
        terms = np.abs(y * np.log(c) + (1 - y) * np.log(1 - c))
    _close_sum(lg.item(), lc.item(), terms.sum() / terms.size, f"{loss} value")
    _close(lg.backward().of(pg), lc.backward().of(pc), 2e-6, f"{loss} adjoint")


def test_accuracy_first_argmax_and_nan_rows(gpu):
    z = np.array([[1, 3, 3], [np.nan, 5, 1], [2, np.nan, 9], [-np.inf, -np.inf, -np.inf], [0, 0, 1]], F)
    labels = [1, 0, 2, 0, 1]
    assert T.losses.accuracy(gpu, z, labels) == R.losses.accuracy(z, labels) == float(F(0.8))
    rng = np.random.default_rng(3)
    z = rng.standard_normal((1000, 37)).astype(F)
    labels = rng.integers(0, 37, 1000)
    assert T.losses.accuracy(gpu, z, labels) == R.losses.accuracy(z, labels)


# ------------------------------------------------ autodiff.rs on the GPU tape
def _gpu_model(gpu, seed, spec):
    rng = oracle.Rng(seed)
    return T.Sequential([T.Dense(gpu, R.dense_weights(rng, i, o), None, activation=act) for i, o, act in spec])


def _numeric_check(params, grads, loss_fn):
    # autodiff.rs:6-37: central differences (h = 1e-3) of the GPU forward itself
    for p in params:
        g = grads.of(p)
        v = p.value()
        for i in range(v.size):
            orig = v.flat[i]
            v.flat[i] = orig + F(1e-3)
            p.set(v)
            up = loss_fn()
            v.flat[i] = orig - F(1e-3)
            p.set(v)
            down = loss_fn()
            v.flat[i] = orig
            p.set(v)
            num, ana = (up - down) / (2 * 1e-3), float(g.flat[i])
            assert abs(num - ana) < 2e-2 * (1 + max(abs(ana), abs(num))), (p.name, i, num, ana)


def test_mlp_mse_and_bce_and_softmax_gradients(gpu):
    # autodiff.rs:82-173 on the GPU tape: numeric checks and the oracle's gradients
    cases = [
        (11, [(3, 4, "tanh"), (4, 2, "linear")], np.sin(np.arange(15, dtype=F) * F(0.37)).reshape(5, 3),
         np.cos(np.arange(10, dtype=F) * F(0.21)).reshape(5, 2), "mse"),
        (5, [(2, 5, "sigmoid"), (5, 1, "sigmoid")], np.array([[0, 0], [0, 1], [1, 0], [1, 1]], F),
         np.array([[0], [1], [1], [0]], F), "binary_cross_entropy"),
    ]
    for seed, spec, x, y, loss in cases:
        mg = _gpu_model(gpu, seed, spec)
        rng = oracle.Rng(seed)
        mc = R.Sequential([R.Dense(R.dense_weights(rng, i, o), None, act) for i, o, act in spec])
        f = getattr(T.losses, loss)
        gg = f(mg.forward(T.constant(T.Tape(gpu), x)), y).backward()
        gc = getattr(R.losses, loss)(mc.forward(R.constant(R.Tape(), x)), y).backward()
        for p, q in zip(mg.params(), mc.params()):
            _close(gg.of(p), gc.of(q), 1e-5, f"{loss} gradient vs oracle")
        _numeric_check(mg.params(), gg, lambda: f(mg.forward(T.constant(T.Tape(gpu), x)), y).item())
    # explicit softmax: -mean(y * log softmax(z)) op by op
    mg = _gpu_model(gpu, 31, [(3, 3, "linear")])
    x = np.sin(np.arange(12, dtype=F) * F(0.29)).reshape(4, 3)
    y = T.losses.one_hot([2, 0, 1, 2], 3)

    def loss():
        t = T.Tape(gpu)
        return mg.forward(T.constant(t, x)).softmax().ln().mul(T.constant(t, y)).sum().scale(-0.25)

    _numeric_check(mg.params(), loss().backward(), lambda: loss().item())


def test_gradient_accumulates_when_a_variable_is_reused(gpu):
    # autodiff.rs:175-184
    w = T.Param(gpu, np.array([[1.0, 2.0, 3.0]], F))
    t = T.Tape(gpu)
    v = w.watch(t)
    assert np.array_equal(v.mul(v).add(v).sum().backward().of(w), np.array([[3, 5, 7]], F))


def test_xor_converges_on_the_gpu_tape(gpu):
    # autodiff.rs:186-212: tanh 2->8, sigmoid 8->1, Adam(0.08), 1500 steps
    model = _gpu_model(gpu, 2024, [(2, 8, "tanh"), (8, 1, "sigmoid")])
    x = np.array([[0, 0], [0, 1], [1, 0], [1, 1]], F)
    y = np.array([[0], [1], [1], [0]], F)
    opt = T.Adam(gpu, 0.08)
    xg = gpu.upload(x)
    for _ in range(1500):
        tape = T.Tape(gpu)
        loss = T.losses.binary_cross_entropy(model.forward(T.constant(tape, xg)), y)
        opt.step(model.params(), loss.backward())
    assert loss.item() < 0.05
    assert np.array_equal(model.predict(gpu, x).ravel() > 0.5, y.ravel() > 0.5)


def test_sgd_with_momentum_matches_the_oracle(gpu):
    # autodiff.rs:214-231 with the oracle's trajectory: bit-identical updates
    w, q = T.Param(gpu, np.array([[4.0, -3.0]], F)), R.Param(np.array([[4.0, -3.0]], F))
    opt, ref = T.Sgd.with_momentum(gpu, 0.05, 0.9), R.Sgd(0.05, 0.9)
    start = w.watch(T.Tape(gpu)).square().sum().item()
    for _ in range(60):
        opt.step([w], w.watch(T.Tape(gpu)).square().sum().backward())
        ref.step([q], q.watch(R.Tape()).square().sum().backward())
    assert np.array_equal(w.value(), q.value)
    assert w.watch(T.Tape(gpu)).square().sum().item() < start * 1e-2
