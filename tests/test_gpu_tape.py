"""The GPU autodiff tape against the CPU oracle's tape.

Mirrors crates/rtensor/tests/autodiff.rs (accumulation when a variable is
reused, gradients of a ReLU MLP with softmax-CE) and tests/gpu.rs:62-139 (one
step of gradients, a 120-step Adam trajectory) on the tape path, where each
op's forward and backward run as kernels of librtgpu.so.
"""
import numpy as np
import pytest

import oracle
import rgpu_b200
from rgpu_b200 import tape as T
from tests.helpers import erro_rel, glorot_model, quadrant_data, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _gpu_model(gpu, params):
    layers = []
    for l in range(0, len(params), 2):
        relu = l + 2 < len(params)
        layers.append(T.Dense(gpu, params[l], params[l + 1], relu=relu))
    return T.Sequential(layers)


def test_tape_mlp_gradients_match_cpu(gpu):
    # gpu.rs:62-97 on the tape: N=64, D=8, H=16, C=4, Rng::new(42).
    x, labels = quadrant_data(64, 8)
    cpu = glorot_model([8, 16, 16, 4], 42)
    model = _gpu_model(gpu, cpu.params())
    tape = T.Tape(gpu)
    loss = T.losses.softmax_cross_entropy(model.forward(T.constant(tape, x)), oracle.one_hot(labels, 4))
    grads = loss.backward()
    loss_cpu = cpu.train_step(x, labels)
    assert abs(loss.item() - loss_cpu) < 1e-5
    for p, g_cpu in zip(model.params(), cpu.grads()):
        g = grads.of(p)
        assert rel_l2(g, g_cpu) <= 1e-4 and erro_rel(g, g_cpu) < 2e-4


def test_tape_adam_trajectory_follows_cpu(gpu):
    # gpu.rs:99-139 on the tape: 120 Adam(0.05) steps, loss within 2e-3 each step.
    x, labels = quadrant_data(64, 8)
    cpu = glorot_model([8, 16, 16, 4], 7)
    model = _gpu_model(gpu, cpu.params())
    opt = T.Adam(gpu, 0.05)
    onehot = oracle.one_hot(labels, 4)
    loss_cpu = None
    for step in range(1, 121):
        loss_cpu = cpu.train_step(x, labels, oracle.OPT_ADAM, 0.05)
        tape = T.Tape(gpu)
        loss = T.losses.softmax_cross_entropy(model.forward(T.constant(tape, x)), onehot)
        grads = loss.backward()
        opt.step(model.params(), grads)
        assert abs(loss.item() - loss_cpu) < 2e-3, f"step {step}"
    for p, w_cpu in zip(model.params(), cpu.params()):
        assert erro_rel(p.value(), w_cpu) < 2e-3
    assert loss_cpu < 0.15


def test_tape_sgd_matches_cpu_update(gpu):
    x, labels = quadrant_data(64, 8)
    cpu = glorot_model([8, 16, 4], 3)
    model = _gpu_model(gpu, cpu.params())
    tape = T.Tape(gpu)
    grads = T.losses.softmax_cross_entropy(model.forward(T.constant(tape, x)), labels).backward()
    T.Sgd(0.1).step(model.params(), grads)
    cpu.train_step(x, labels, oracle.OPT_SGD, 0.1)
    for p, w_cpu in zip(model.params(), cpu.params()):
        assert rel_l2(p.value(), w_cpu) < 1e-6


def test_reused_parameter_accumulates(gpu):
    # autodiff.rs:175-184 in matmul form: W watched twice on one tape shares its
    # leaf (tape.rs:124-131) and receives the sum of both adjoints.
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 3)).astype(np.float32)
    w0 = rng.standard_normal((3, 4)).astype(np.float32)
    labels = np.array([0, 1, 2, 3, 1], np.uint32)
    w = T.Param(gpu, w0)
    # twice-used: logits = x W + x W
    t2 = T.Tape(gpu)
    xv = T.constant(t2, x)
    z = xv.matmul(w.watch(t2)).add(xv.matmul(w.watch(t2)))
    g2 = T.losses.softmax_cross_entropy(z, labels).backward().of(w)
    # reference: logits = x (2W), whose gradient w.r.t. W is twice that w.r.t. 2W
    w2 = T.Param(gpu, 2 * w0)
    t1 = T.Tape(gpu)
    g1 = T.losses.softmax_cross_entropy(T.constant(t1, x).matmul(w2.watch(t1)), labels).backward().of(w2)
    assert np.allclose(g2, 2 * g1, rtol=1e-5, atol=1e-6)


def test_bias_broadcast_either_side_and_unused_param(gpu):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((6, 5)).astype(np.float32)
    b = T.Param(gpu, rng.standard_normal((1, 5)).astype(np.float32))
    unused = T.Param(gpu, np.ones((2, 2), np.float32))
    t = T.Tape(gpu)
    xv = T.constant(t, x)
    left = xv.add(b.watch(t))
    right = b.watch(t).add(xv)
    assert np.array_equal(left.value(), x + b.value())
    assert np.array_equal(right.value(), left.value())
    grads = T.losses.softmax_cross_entropy(left.add(right), np.arange(6) % 5).backward()
    # d/db of (x + b) + (b + x): twice the column sums of dL/dz
    assert grads.of(b).shape == (1, 5)
    assert grads.of(unused) is None


def test_backward_needs_a_scalar_root(gpu):
    t = T.Tape(gpu)
    v = T.constant(t, np.ones((3, 3), np.float32))
    with pytest.raises(rgpu_b200.RtError):
        v.relu().backward()
