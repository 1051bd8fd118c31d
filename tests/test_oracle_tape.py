"""The tape oracle (oracle/tape_ref.py) pinned on rtensor's own known answers
and gradient checks (crates/rtensor/tests/autodiff.rs), on the CPU."""
import numpy as np

import oracle
from oracle import tape_ref as R

F = np.float32


def test_known_answers():
    # autodiff.rs:40-60
    t = R.Tape()
    a = R.constant(t, np.array([[1, 2, 3], [4, 5, 6]], F))
    b = R.constant(t, np.array([[7, 8], [9, 10], [11, 12]], F))
    assert np.array_equal(a.matmul(b).value(), np.array([[58, 64], [139, 154]], F))
    x = R.constant(t, np.array([[1, 2, 3], [4, 5, 6]], F))
    bias = R.constant(t, np.array([[10, 20, 30]], F))
    assert np.array_equal(x.add(bias).value().ravel(), [11, 22, 33, 14, 25, 36])
    g = np.array([[1, 2, 3], [4, 5, 6]], F)
    assert np.array_equal(R.reduce_to(g, (1, 3)).ravel(), [5, 7, 9])
    assert np.array_equal(R.reduce_to(g, (2, 1)).ravel(), [6, 15])


def test_softmax_rows_normalise_and_stay_finite():
    # autodiff.rs:62-72
    s = R.softmax_rows(np.array([[1, 2, 3], [100, 100, 100]], F))
    assert np.all(np.abs(s.sum(1) - 1) < 1e-5) and np.all(np.isfinite(s))


def test_gradient_accumulates_when_a_variable_is_reused():
    # autodiff.rs:175-184: f(w) = sum(w * w + w) => 2w + 1
    w = R.Param(np.array([[1.0, 2.0, 3.0]], F))
    t = R.Tape()
    v = w.watch(t)
    g = v.mul(v).add(v).sum().backward()
    assert np.array_equal(g.of(w), np.array([[3, 5, 7]], F))


def _numeric_check(params, grads, loss_fn):
    # autodiff.rs:6-37: central differences, h = 1e-3, tol 2e-2 (1 + max|.|)
    for p in params:
        g = grads.of(p)
        for i in range(p.value.size):
            orig = p.value.flat[i]
            p.value.flat[i] = orig + F(1e-3)
            up = loss_fn()
            p.value.flat[i] = orig - F(1e-3)
            down = loss_fn()
            p.value.flat[i] = orig
            num = (up - down) / (2 * 1e-3)
            ana = float(g.flat[i])
            assert abs(num - ana) < 2e-2 * (1 + max(abs(ana), abs(num))), (p.name, i, num, ana)


def _model(seed, spec):
    rng = oracle.Rng(seed)
    return R.Sequential([R.Dense(R.dense_weights(rng, i, o), None, act) for i, o, act in spec])


def test_mlp_with_mse_gradients_match_numeric():
    # autodiff.rs:82-102
    model = _model(11, [(3, 4, "tanh"), (4, 2, "linear")])
    x = np.sin(np.arange(15, dtype=F) * F(0.37)).reshape(5, 3)
    y = np.cos(np.arange(10, dtype=F) * F(0.21)).reshape(5, 2)
    fwd = lambda: R.losses.mse(model.forward(R.constant(R.Tape(), x)), y).item()  # noqa: E731
    grads = R.losses.mse(model.forward(R.constant(R.Tape(), x)), y).backward()
    _numeric_check(model.params(), grads, fwd)


def test_cross_entropy_gradients_match_numeric():
    # autodiff.rs:104-125
    model = _model(23, [(4, 6, "relu"), (6, 3, "linear")])
    x = (np.cos(np.arange(32, dtype=F) * F(0.13)) * F(1.5)).reshape(8, 4)
    y = R.losses.one_hot([0, 1, 2, 1, 0, 2, 2, 0], 3)
    fwd = lambda: R.losses.softmax_cross_entropy(model.forward(R.constant(R.Tape(), x)), y).item()  # noqa: E731
    grads = R.losses.softmax_cross_entropy(model.forward(R.constant(R.Tape(), x)), y).backward()
    _numeric_check(model.params(), grads, fwd)


def test_sigmoid_with_bce_gradients_match_numeric():
    # autodiff.rs:127-148
    model = _model(5, [(2, 5, "sigmoid"), (5, 1, "sigmoid")])
    x = np.array([[0, 0], [0, 1], [1, 0], [1, 1]], F)
    y = np.array([[0], [1], [1], [0]], F)
    fwd = lambda: R.losses.binary_cross_entropy(model.forward(R.constant(R.Tape(), x)), y).item()  # noqa: E731
    grads = R.losses.binary_cross_entropy(model.forward(R.constant(R.Tape(), x)), y).backward()
    _numeric_check(model.params(), grads, fwd)


def test_explicit_softmax_gradients_match_numeric():
    # autodiff.rs:150-173: -mean(y * log softmax(z)) assembled op by op
    model = _model(31, [(3, 3, "linear")])
    x = np.sin(np.arange(12, dtype=F) * F(0.29)).reshape(4, 3)
    y = R.losses.one_hot([2, 0, 1, 2], 3)

    def loss():
        t = R.Tape()
        p = model.forward(R.constant(t, x)).softmax()
        return p.ln().mul(R.constant(t, y)).sum().scale(-0.25)

    _numeric_check(model.params(), loss().backward(), lambda: loss().item())


def test_xor_converges_with_adam():
    # autodiff.rs:186-212
    model = _model(2024, [(2, 8, "tanh"), (8, 1, "sigmoid")])
    x = np.array([[0, 0], [0, 1], [1, 0], [1, 1]], F)
    y = np.array([[0], [1], [1], [0]], F)
    opt = R.Adam(0.08)
    for _ in range(1500):
        loss = R.losses.binary_cross_entropy(model.forward(R.constant(R.Tape(), x)), y)
        last = loss.item()
        opt.step(model.params(), loss.backward())
    assert last < 0.05
    assert np.array_equal(model.predict(x).ravel() > 0.5, y.ravel() > 0.5)


def test_sgd_with_momentum_reduces_the_loss():
    # autodiff.rs:214-231
    w = R.Param(np.array([[4.0, -3.0]], F))
    opt = R.Sgd(0.05, 0.9)
    quad = lambda: w.watch(R.Tape()).square().sum()  # noqa: E731
    start = quad().item()
    for _ in range(60):
        loss = quad()
        opt.step([w], loss.backward())
    assert quad().item() < start * 1e-2


def test_mae_and_accuracy_conventions():
    # losses.rs:46-55 sign(0) = +1; losses.rs:181-185 first arg-max, element 0 first
    t = R.Tape()
    p = R.Param(np.array([[1.0, 2.0, 3.0]], F))
    loss = R.losses.mae(p.watch(t), np.array([[1.0, 0.0, 5.0]], F))
    assert abs(loss.item() - 4.0 / 3.0) < 1e-7
    assert np.array_equal(loss.backward().of(p), np.array([[1, 1, -1]], F) / F(3))
    z = np.array([[1, 3, 3], [np.nan, 5, 1], [2, np.nan, 9], [-np.inf, -np.inf, -np.inf]], F)
    assert list(R.argmax_rows(z)) == [1, 0, 2, 0]
    assert R.losses.accuracy(z, [1, 0, 0, 0]) == 0.75
