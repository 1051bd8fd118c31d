"""Pins the CPU oracle (C++ restatement of rtensor's CPU backend).

The reference cannot be built here (it is Rust and there is no Rust
toolchain), so the restatement is pinned on the reference's own known-answer
tests and central-difference gradient checks
(crates/rtensor/tests/autodiff.rs), plus independent re-derivations of the
Rng and optimiser arithmetic in numpy float32.
"""
import numpy as np

import oracle


def test_matmul_known_answer():
    # autodiff.rs:39-46
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    c = oracle.matmul(a, b)
    assert c.shape == (2, 2)
    assert c.ravel().tolist() == [58.0, 64.0, 139.0, 154.0]


def test_broadcast_add_through_dense_forward():
    # autodiff.rs:48-53: x + 1_n b, exercised through Dense::forward with W = I.
    m = oracle.Mlp([3, 3])
    m.set_params([np.eye(3, dtype=np.float32), np.array([[10, 20, 30]], np.float32)])
    x = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    m.forward(x)
    assert m.logits(2).ravel().tolist() == [11, 22, 33, 14, 25, 36]


def test_reduce_to_rows():
    # autodiff.rs:55-60 ([2,3] -> [1,3])
    g = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    assert oracle.reduce_rows(g).ravel().tolist() == [5.0, 7.0, 9.0]


def test_softmax_rows_stable():
    # autodiff.rs:62-72
    z = np.array([[1, 2, 3], [100, 100, 100]], np.float32)
    s = oracle.softmax_rows(z)
    assert np.all(np.isfinite(s))
    assert np.allclose(s.sum(1), 1.0, atol=1e-5)


def test_transpose_involution():
    # autodiff.rs:74-79, plus a ragged shape that crosses the 32x32 blocking.
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    assert oracle.transpose(a).shape == (3, 2)
    assert np.array_equal(oracle.transpose(oracle.transpose(a)), a)
    r = np.arange(70 * 45, dtype=np.float32).reshape(70, 45)
    assert np.array_equal(oracle.transpose(r), r.T)


def _py_xorshift(seed, count):
    s = seed if seed != 0 else 0x9E3779B97F4A7C15
    mask = (1 << 64) - 1
    out = []
    for _ in range(count):
        s ^= s >> 12
        s ^= (s << 25) & mask
        s ^= s >> 27
        out.append((s * 0x2545F4914F6CDD1D) & mask)
    return out


def test_rng_matches_independent_xorshift64star():
    # rng.rs:12-24, 38-40 re-derived in pure Python.
    raw = _py_xorshift(42, 64)
    u = oracle.Rng(42).uniform(64)
    exp = np.array([(r >> 40) for r in raw], np.float32) / np.float32(1 << 24)
    assert np.array_equal(u, exp)
    below = oracle.Rng(7).below(10, 64)
    assert below.tolist() == [r % 10 for r in _py_xorshift(7, 64)]
    # seed 0 maps to the golden-ratio constant (rng.rs:8-10)
    assert np.array_equal(oracle.Rng(0).uniform(4), oracle.Rng(0x9E3779B97F4A7C15).uniform(4))


def test_rng_normal_moments():
    z = oracle.Rng(2024).normal(200_000)
    assert abs(float(z.mean())) < 0.01
    assert abs(float(z.std()) - 1.0) < 0.01


def _powi(a, b):
    a = np.float32(a)
    r = np.float32(1.0)
    while True:
        if b & 1:
            r = np.float32(r * a)
        b //= 2
        if b == 0:
            break
        a = np.float32(a * a)
    return r


def test_adam_matches_float32_rederivation():
    # optim.rs:163-198, re-derived op by op in numpy float32.
    rng = np.random.default_rng(0)
    n = 1000
    theta = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    th_ref, m_ref, v_ref = theta.copy(), m.copy(), v.copy()
    f = np.float32
    b1, b2, eps, lr = f(0.9), f(0.999), f(1e-8), f(1e-3)
    for t in range(1, 6):
        g = rng.standard_normal(n).astype(np.float32)
        oracle.adam_update(theta, m, v, g, float(lr), t)
        inv_c1 = f(1.0) / (f(1.0) - _powi(b1, t))
        inv_c2 = f(1.0) / (f(1.0) - _powi(b2, t))
        m_ref = m_ref * b1 + g * (f(1.0) - b1)
        v_ref = v_ref * b2 + (g * g) * (f(1.0) - b2)
        th_ref = th_ref - (m_ref * inv_c1 / (np.sqrt(v_ref * inv_c2) + eps)) * lr
    assert np.array_equal(theta, th_ref)
    assert np.array_equal(m, m_ref)
    assert np.array_equal(v, v_ref)


def test_sgd_update():
    theta = np.arange(8, dtype=np.float32)
    g = np.full(8, 2.0, np.float32)
    oracle.sgd_update(theta, g, 0.25)
    assert np.array_equal(theta, np.arange(8, dtype=np.float32) - 0.5)


def test_blocked_matmul_equals_unblocked_order():
    # tensor.rs:345-371: blocking keeps each element's p-ascending order, so the
    # blocked path (k*n > 32768) equals a plain ikj sweep bit for bit, for any
    # thread count.
    rng = np.random.default_rng(1)
    a = rng.standard_normal((37, 300)).astype(np.float32)
    a[a < -1.0] = 0.0  # exercise zero-skip
    b = rng.standard_normal((300, 290)).astype(np.float32)
    c1 = oracle.matmul(a, b, threads=1)
    c4 = oracle.matmul(a, b, threads=4)
    ref = np.zeros((37, 290), np.float32)
    for p in range(300):
        ref += a[:, p:p + 1] * b[p]
    assert np.array_equal(c1, c4)
    assert np.array_equal(c1, ref)


def _numeric_grad_check(dims, seed, x, labels):
    # autodiff.rs:6-37: central differences, h = 1e-3, tol 2e-2 (1 + max|g|).
    m = oracle.Mlp(dims)
    m.init_glorot(oracle.Rng(seed))
    m.train_step(x, labels)
    grads = m.grads()
    params = m.params()
    h = np.float32(1e-3)
    for pi, (p, g) in enumerate(zip(params, grads)):
        flat = p.ravel()
        for i in range(flat.size):
            orig = flat[i]
            flat[i] = orig + h
            m.set_params(params)
            up = m.forward(x, labels)
            flat[i] = orig - h
            m.set_params(params)
            down = m.forward(x, labels)
            flat[i] = orig
            m.set_params(params)
            num = (up - down) / (2 * h)
            ana = g.ravel()[i]
            tol = 2e-2 * (1 + max(abs(ana), abs(num)))
            assert abs(num - ana) < tol, (pi, i, num, ana)


def test_relu_softmax_xent_gradients_match_central_differences():
    # autodiff.rs:104-125: Dense(4,6,Relu), Dense(6,3,Linear), Rng::new(23).
    x = (np.cos(np.arange(32, dtype=np.float32) * np.float32(0.13)) * 1.5).astype(np.float32)
    _numeric_grad_check([4, 6, 3], 23, x.reshape(8, 4), np.array([0, 1, 2, 1, 0, 2, 2, 0], np.uint32))


def test_deeper_relu_mlp_gradients_match_central_differences():
    rng = oracle.Rng(5)
    x = rng.normal(16 * 5).reshape(16, 5)
    _numeric_grad_check([5, 7, 6, 4], 9, x, rng.below(4, 16))


def test_training_trajectory_converges():
    # tests/gpu.rs:99-139 data: x_i = sin(0.37 i), quadrant labels; Adam(0.05).
    N, D, H, C = 64, 8, 16, 4
    x = np.sin(np.arange(N * D, dtype=np.float32) * np.float32(0.37)).astype(np.float32).reshape(N, D)
    labels = ((x[:, 0] > 0).astype(np.uint32) + 2 * (x[:, 1] > 0).astype(np.uint32))
    m = oracle.Mlp([D, H, H, C])
    m.init_glorot(oracle.Rng(7))
    loss = None
    for _ in range(120):
        loss = m.train_step(x, labels, oracle.OPT_ADAM, 0.05)
    assert loss < 0.15
