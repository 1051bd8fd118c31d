"""Whole-step parity of GpuMlp (the captured CUDA-graph train step) against the
CPU oracle's tape-driven step, on identical seeded inputs and weights.

Mirrors crates/rtensor/tests/gpu.rs:62-213 and adds the BASELINE configs
(config 3 at its full batch of 8192 too), with the north-star tolerances:
relative L2 <= 1e-4 per gradient for f32, <= 2e-2 for bf16 operands.  The
bf16 configs take bf16 inputs and weights, so the plain f32 CPU reference is
given exactly the values the GPU plan starts from.
"""
import numpy as np
import pytest

import oracle
import rgpu_b200
from tests.helpers import baseline_inputs, bf16_baseline_inputs, erro_rel, glorot_model, quadrant_data, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _one_step_parity(gpu, cpu_model, x, labels, dtype, tol_l2, fast=True, opt="none"):
    params = cpu_model.params()
    n = x.shape[0]
    gpu.set_fast_gemm(fast)
    try:
        mlp = rgpu_b200.GpuMlp.from_params(gpu, params, n, 0.0, dtype=dtype, optimizer=opt)
        gx = gpu.upload(x)
        gy = rgpu_b200.upload_labels(gpu, labels)
        mlp.step(gx, gy)
        loss_gpu = mlp.last_loss()
        grads_gpu = mlp.grads()
    finally:
        gpu.set_fast_gemm(True)
    loss_cpu = cpu_model.train_step(x, labels)
    grads_cpu = cpu_model.grads()
    worst = 0.0
    for i, (gc, gg) in enumerate(zip(grads_cpu, grads_gpu)):
        e = rel_l2(gg, gc)
        worst = max(worst, e)
        assert e <= tol_l2, f"param {i} ({'W' if i % 2 == 0 else 'b'}{i // 2 + 1}): rel L2 {e:.3e} > {tol_l2}"
    return loss_cpu, loss_gpu, worst


@pytest.mark.parametrize("fast", [True, False])
def test_gradients_match_cpu(gpu, fast):
    # gpu.rs:62-97: N=64, D=8, H=16, C=4, Rng::new(42).
    x, labels = quadrant_data(64, 8)
    model = glorot_model([8, 16, 16, 4], 42)
    loss_cpu, loss_gpu, _ = _one_step_parity(gpu, model, x, labels, "f32", 1e-4, fast)
    assert abs(loss_cpu - loss_gpu) < 1e-4
    # and the reference's own max-relative metric, 2e-4
    model2 = glorot_model([8, 16, 16, 4], 42)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model2.params(), 64, 0.0, optimizer="none")
    mlp.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
    model2.train_step(x, labels)
    for gc, gg in zip(model2.grads(), mlp.grads()):
        assert erro_rel(gc, gg) < 2e-4


def test_training_follows_cpu_trajectory(gpu):
    # gpu.rs:99-139: 120 Adam(0.05) steps; per-step loss within 2e-3, final
    # weights within 2e-3, converged below 0.15.
    x, labels = quadrant_data(64, 8)
    model = glorot_model([8, 16, 16, 4], 7)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 64, 0.05, optimizer="adam")
    gx, gy = gpu.upload(x), rgpu_b200.upload_labels(gpu, labels)
    loss_cpu = None
    for step in range(1, 121):
        loss_cpu = model.train_step(x, labels, oracle.OPT_ADAM, 0.05)
        mlp.step(gx, gy)
        loss_gpu = mlp.last_loss()
        assert abs(loss_cpu - loss_gpu) < 2e-3, f"step {step}: CPU {loss_cpu:.6f} GPU {loss_gpu:.6f}"
    for i, (wc, wg) in enumerate(zip(model.params(), mlp.weights())):
        assert erro_rel(wc, wg) < 2e-3, f"param {i} diverged"
    assert loss_cpu < 0.15


def test_split_k_training_follows_cpu(gpu):
    # gpu.rs:145-213: batch 512, 8 -> 128 -> 4, where dW of the output layer
    # is K-dominant; 60 Adam steps.
    x, labels = quadrant_data(512, 8)
    model = glorot_model([8, 128, 4], 7)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 512, 0.05, optimizer="adam")
    assert mlp.dispatches_por_passo() > 0
    gx, gy = gpu.upload(x), rgpu_b200.upload_labels(gpu, labels)
    loss_cpu = None
    for step in range(1, 61):
        loss_cpu = model.train_step(x, labels, oracle.OPT_ADAM, 0.05)
        mlp.step(gx, gy)
        assert abs(loss_cpu - mlp.last_loss()) < 2e-3, f"step {step}"
    for wc, wg in zip(model.params(), mlp.weights()):
        assert erro_rel(wc, wg) < 2e-3
    assert loss_cpu < 0.2


def test_config1_f32_batch32_sgd(gpu):
    # 512 -> 1024 -> 1024 -> 10, f32, batch 32, SGD 0.01.
    dims = [512, 1024, 1024, 10]
    model, x, labels = baseline_inputs(dims, 32, 2025)
    _, _, worst = _one_step_parity(gpu, model, x, labels, "f32", 1e-4)
    # after the SGD update the weights must agree too
    model, x, labels = baseline_inputs(dims, 32, 2025)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 32, 0.01, optimizer="sgd")
    mlp.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
    model.train_step(x, labels, oracle.OPT_SGD, 0.01, threads=4)
    for i, (wc, wg) in enumerate(zip(model.params(), mlp.weights())):
        # W = W0 - lr g agrees far inside the gradient bar; b starts at zero,
        # so b = -lr db carries the db gradient's own error (<= 1e-4; the
        # column sum of delta cancels, which magnifies the 3xTF32 error).
        bound = 1e-6 if i % 2 == 0 else 1e-4
        assert rel_l2(wg, wc) < bound, f"param {i}: {rel_l2(wg, wc):.3e}"


def test_config2_f32_batch2048(gpu):
    # same MLP at batch 2048 on one B200, gradients vs CPU.
    dims = [512, 1024, 1024, 10]
    model, x, labels = baseline_inputs(dims, 2048, 2026)
    params = model.params()
    mlp = rgpu_b200.GpuMlp.from_params(gpu, params, 2048, 0.0, optimizer="none")
    mlp.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
    grads_gpu = mlp.grads()
    loss_gpu = mlp.last_loss()
    loss_cpu = model.train_step(x, labels, threads=8)
    for i, (gc, gg) in enumerate(zip(model.grads(), grads_gpu)):
        assert rel_l2(gg, gc) <= 1e-4, f"param {i}: {rel_l2(gg, gc):.3e}"
    assert abs(loss_cpu - loss_gpu) < 1e-4


def _wide_bf16_grads(gpu, dims, n, seed, fast, activations="split", optimizer="none", lr=0.0):
    model, x, labels = bf16_baseline_inputs(dims, n, seed)
    gpu.set_fast_gemm(fast)
    try:
        mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), n, lr, dtype="bf16", optimizer=optimizer,
                                           activations=activations)
        mlp.step(gpu.upload(x, "bf16"), rgpu_b200.upload_labels(gpu, labels))
        grads = mlp.grads()
        loss = mlp.last_loss()
        mlp.close()
    finally:
        gpu.set_fast_gemm(True)
    return model, x, labels, grads, loss


@pytest.mark.parametrize("activations,flags", [("split", oracle.BF16_SPLIT), ("bf16", oracle.BF16_PLAIN)])
def test_bf16_step_logic_tracks_the_rounding_point_oracle(gpu, activations, flags):
    # The bf16 plan's rounding points and step logic, isolated from the
    # tensor cores' accumulation order: the SIMT kernels sum k in the
    # oracle's order, and bf16 x bf16 (or (hi + lo) x bf16) products are exact
    # in f32, so what is left is the softmax-CE kernel's lane-parallel sums,
    # which can move a delta across a bf16 rounding boundary.  Measured
    # <= 4e-4; bound 1e-3.
    dims = [512, 1024, 1024, 1024, 100]
    model, x, labels, grads, _ = _wide_bf16_grads(gpu, dims, 256, 2027, fast=False, activations=activations)
    model.set_rounding(flags)
    model.train_step(x, labels, threads=8, input_grad=False)
    for i, (gc, gg) in enumerate(zip(model.grads(), grads)):
        assert rel_l2(gg, gc) <= 1e-3, f"param {i}: {rel_l2(gg, gc):.3e}"


def test_bf16_wide_mlp_meets_the_bar_at_reduced_batch(gpu):
    # BASELINE config 3's architecture (4096 -> 8192 x3 -> 1000), bf16 inputs
    # and weights, f32 accumulate, on the tensor-core path with split
    # activations (the default), against the plain f32 CPU reference given
    # the same bf16 inputs and weights: every gradient within the north-star
    # 2e-2 (measured <= 5e-3).  With single-bf16 activations the hidden-layer
    # gradients are 2e-2 .. 8e-2 away (ReLU masks flipped by the activation
    # rounding), which is why split activations are the default.
    dims = [4096, 8192, 8192, 8192, 1000]
    model, x, labels, grads_split, loss_split = _wide_bf16_grads(gpu, dims, 64, 2027, fast=True)
    _, _, _, grads_plain, _ = _wide_bf16_grads(gpu, dims, 64, 2027, fast=True, activations="bf16")
    loss_cpu = model.train_step(x, labels, threads=8, input_grad=False)
    gref = model.grads()
    errs = [rel_l2(g, r) for g, r in zip(grads_split, gref)]
    for i, e in enumerate(errs):
        assert e <= 2e-2, f"param {i}: rel L2 {e:.3e} > 2e-2 (all: {[f'{v:.2e}' for v in errs]})"
    assert abs(loss_split - loss_cpu) < 1e-3
    plain = [rel_l2(g, r) for g, r in zip(grads_plain, gref)]
    assert max(plain[:6]) > 2 * max(errs[:6]), (plain, errs)


def test_config3_full_batch_meets_the_bar(gpu):
    # BASELINE config 3 exactly: 4096 -> 8192 -> 8192 -> 8192 -> 1000, bf16
    # inputs/weights with f32 accumulate and f32 masters, Adam(1e-3), batch
    # 8192, X ~ N(0,1), uniform labels, Kaiming init.  One step of the
    # production plan (tensor cores, split activations, Adam fused into the
    # dW GEMMs); its gradients against the plain f32 CPU reference on the
    # same inputs and weights (crates/rtensor/tests/gpu.rs:62-97 is the
    # reference's own GPU-vs-CPU gradient check), all host threads, with the
    # north-star bar of 2e-2 relative L2 for every W and b.
    import os

    dims = [4096, 8192, 8192, 8192, 1000]
    n = 8192
    model, x, labels, grads, loss_gpu = _wide_bf16_grads(gpu, dims, n, 2024 + 3, fast=True, optimizer="adam",
                                                         lr=1e-3)
    loss_cpu = model.train_step(x, labels, threads=os.cpu_count() or 8, input_grad=False)
    errs = [rel_l2(g, r) for g, r in zip(grads, model.grads())]
    print("config 3, batch 8192: grad rel L2 " + " ".join(f"{e:.3e}" for e in errs) +
          f"; loss GPU {loss_gpu:.6f} CPU {loss_cpu:.6f}")
    for i, e in enumerate(errs):
        assert e <= 2e-2, f"param {i} ({'W' if i % 2 == 0 else 'b'}{i // 2}): rel L2 {e:.3e} > 2e-2"
    assert abs(loss_gpu - loss_cpu) < 1e-3


def test_bf16_adam_step_updates_master_and_shadow(gpu):
    # Five Adam steps: after the first, the GEMMs read the bf16 shadow of the
    # updated f32 masters, so the oracle rounds its weights at use as well
    # (the split-activation plan's rounding points).
    dims = [256, 512, 512, 100]
    model, x, labels = bf16_baseline_inputs(dims, 256, 2028)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 256, 1e-3, dtype="bf16", optimizer="adam")
    gx, gy = gpu.upload(x), rgpu_b200.upload_labels(gpu, labels)
    model.set_rounding(oracle.BF16_SPLIT)
    loss_cpu = None
    for _ in range(5):
        loss_cpu = model.train_step(x, labels, oracle.OPT_ADAM, 1e-3, threads=4)
        mlp.step(gx, gy)
    for i, (wc, wg) in enumerate(zip(model.params(), mlp.weights())):
        assert erro_rel(wc, wg) < 2e-2, f"param {i}"
    # loss of the 5th step's forward pass (before its update) on both sides
    assert abs(loss_cpu - mlp.last_loss()) < 2e-2


def test_host_step_equals_device_step(gpu):
    x, labels = quadrant_data(64, 8)
    model = glorot_model([8, 16, 16, 4], 42)
    a = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 64, 0.05, optimizer="adam")
    b = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 64, 0.05, optimizer="adam")
    rows = np.zeros(64, np.float32)
    for _ in range(3):
        a.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
        b.step_host(x, labels, rows)
    gpu.sync()
    for wa, wb in zip(a.weights(), b.weights()):
        assert np.array_equal(wa, wb)
    seq = np.float32(0.0)
    for v in rows:  # mean_all's sequential f32 sum (tensor.rs:279-286)
        seq = np.float32(seq + v)
    assert float(seq / np.float32(64)) == b.last_loss()


def test_forward_only_and_logits(gpu):
    x, labels = quadrant_data(64, 8)
    model = glorot_model([8, 16, 16, 4], 3)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 64, 0.0, optimizer="none")
    mlp.forward_only(gpu.upload(x))
    model.forward(x)
    assert erro_rel(model.logits(64), mlp.logits()) < 1e-5


def _suite_data(n, d, shift=0.0):
    """examples/suite.rs:27-32: x[i, j] = sin(0.01 i + 0.03 j) (+ shift)."""
    i = np.arange(n, dtype=np.float32).reshape(n, 1)
    j = np.arange(d, dtype=np.float32).reshape(1, d)
    return np.sin(i * np.float32(0.01) + j * np.float32(0.03) + np.float32(shift)).astype(np.float32)


@pytest.mark.parametrize("batch", [1, 32, 512, 4096])
def test_inference_at_the_reference_batches(gpu, batch):
    # examples/suite.rs:204-240: MLP 512 -> 1024 -> 1024 -> 10 (f32, Glorot
    # from Rng::new(7)), forward_only at batch 1 / 32 / 512 / 4096 against
    # Sequential::predict.  The forward runs as a captured graph: replaying it
    # on new inputs must give the new logits, and the host-buffer entry point
    # the same logits as the device one.
    dims = [512, 1024, 1024, 10]
    model = glorot_model(dims, 7)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), batch, 0.0, optimizer="none")
    for shift in (0.0, 0.5, 1.25):
        x = _suite_data(batch, dims[0], shift)
        mlp.forward_only(gpu.upload(x))
        got = mlp.logits()
        model.forward(x, threads=4)
        want = model.logits(batch)
        assert erro_rel(want, got) < 1e-5, f"batch {batch} shift {shift}: {erro_rel(want, got):.2e}"
        host = mlp.forward_host(x)
        assert np.array_equal(host, got)
    assert mlp.dispatches_por_passo() > 0


def test_bf16_inference_logits_meet_the_bar(gpu):
    # The wide bf16 model's forward alone (split activations), against the
    # plain f32 reference on the same bf16 inputs and weights.
    dims = [4096, 8192, 8192, 8192, 1000]
    model, x, _ = bf16_baseline_inputs(dims, 128, 31)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 128, 0.0, dtype="bf16", optimizer="none")
    mlp.forward_only(gpu.upload(x, "bf16"))
    model.forward(x, threads=8)
    assert rel_l2(mlp.logits(), model.logits(128)) <= 2e-2


def test_batch_mismatch_is_an_error(gpu):
    model = glorot_model([8, 16, 4], 3)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 64, 0.0)
    x, labels = quadrant_data(32, 8)
    with pytest.raises(rgpu_b200.RtError):
        mlp.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))


def test_timing_records_every_op(gpu):
    dims = [512, 1024, 1024, 10]
    model, x, labels = baseline_inputs(dims, 256, 1)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 256, 0.01, optimizer="sgd")
    mlp.enable_timing(True)
    mlp.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
    gpu.sync()
    ops = mlp.op_times()
    labels_seen = [o[0] for o in ops]
    # one dW GEMM per layer (SGD fused into its epilogue on one GPU), dX for
    # the two upper layers, the forward GEMMs and the softmax-CE
    assert sum(1 for x in labels_seen if x.startswith("dw_gemm")) == 3
    assert labels_seen.count("dx_gemm_relu_mask") == 2
    assert "softmax_xent" in labels_seen
    assert all(ms >= 0 for _, _, ms in ops)


@pytest.mark.parametrize("dtype,opt,lr", [("bf16", "adam", 1e-3), ("f32", "sgd", 0.01), ("f32", "adam", 1e-3)])
def test_checkpoint_resume_is_bit_exact(gpu, tmp_path, dtype, opt, lr):
    # 3 steps, save, resume in a plan built from other weights, 2 more steps:
    # identical (bit for bit) to 5 uninterrupted steps, moments and Adam step
    # count included.
    dims = [256, 512, 512, 10]
    model, x, labels = baseline_inputs(dims, 128, 2030)
    gx, gy = gpu.upload(x), rgpu_b200.upload_labels(gpu, labels)
    ref = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 128, lr, dtype=dtype, optimizer=opt)
    for _ in range(5):
        ref.step(gx, gy)
    want = ref.weights()
    a = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 128, lr, dtype=dtype, optimizer=opt)
    for _ in range(3):
        a.step(gx, gy)
    path = tmp_path / "state.rtms"
    a.save(str(path))
    other, _, _ = baseline_inputs(dims, 128, 99)
    b = rgpu_b200.GpuMlp.from_params(gpu, other.params(), 128, lr, dtype=dtype, optimizer=opt)
    b.load(str(path))
    for wa, wb in zip(a.weights(), b.weights()):
        assert np.array_equal(wa, wb)
    for _ in range(2):
        b.step(gx, gy)
    for i, (w, g) in enumerate(zip(want, b.weights())):
        assert np.array_equal(w, g), f"param {i} differs after resume"
    assert b.save_state() == ref.save_state()


@pytest.mark.parametrize("dtype,opt,lr,batch", [("bf16", "adam", 1e-3, 512), ("f32", "sgd", 0.01, 512),
                                                ("f32", "adam", 1e-3, 512), ("bf16", "adam", 1e-3, 2048)])
def test_fused_update_equals_separate_update(gpu, monkeypatch, dtype, opt, lr, batch):
    # On one device the optimiser runs inside the dW GEMMs' epilogues (dX
    # first, then dW + update); RTGPU_FUSED_OPT=0 runs the dW GEMMs plain and
    # the update as its own kernels on a side stream.  Same arithmetic, same
    # GEMMs: three steps agree bit for bit (weights, gradients, moments, loss).
    # f32 at batch 512 and bf16 at 2048 split the narrow layers' dW GEMMs over
    # k; there the split-K reduce kernel applies the update.
    dims = [256, 512, 384, 10]
    model, x, labels = baseline_inputs(dims, batch, 77)
    gx, gy = gpu.upload(x), rgpu_b200.upload_labels(gpu, labels)
    runs = {}
    for fused in ("0", "1"):
        monkeypatch.setenv("RTGPU_FUSED_OPT", fused)
        mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), batch, lr, dtype=dtype, optimizer=opt)
        mlp.enable_timing(True)
        for _ in range(3):
            mlp.step(gx, gy)
        gpu.sync()
        labels_seen = [o[0] for o in mlp.op_times()]
        runs[fused] = (mlp.weights(), mlp.grads(), mlp.save_state(), mlp.last_loss(), labels_seen)
        mlp.close()
    assert any(lab.startswith("dw_gemm_") for lab in runs["1"][4]), runs["1"][4]
    assert not any(lab.startswith("dw_gemm_") for lab in runs["0"][4]), runs["0"][4]
    for i, (a, b) in enumerate(zip(runs["0"][0], runs["1"][0])):
        assert np.array_equal(a, b), f"weights {i}"
    for i, (a, b) in enumerate(zip(runs["0"][1], runs["1"][1])):
        assert np.array_equal(a, b), f"grads {i}"
    assert runs["0"][2] == runs["1"][2]
    assert runs["0"][3] == runs["1"][3]


def test_checkpoint_rejects_another_architecture(gpu):
    model, x, labels = baseline_inputs([64, 128, 10], 32, 1)
    a = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 32, 1e-3, optimizer="adam")
    state = a.save_state()
    other, _, _ = baseline_inputs([64, 96, 10], 32, 1)
    b = rgpu_b200.GpuMlp.from_params(gpu, other.params(), 32, 1e-3, optimizer="adam")
    with pytest.raises(rgpu_b200.RtError) as e:
        b.load_state(state)
    assert "dims[1]" in str(e.value)
    c = rgpu_b200.GpuMlp.from_params(gpu, model.params(), 32, 1e-3, optimizer="sgd")
    with pytest.raises(rgpu_b200.RtError):
        c.load_state(state)
    with pytest.raises(rgpu_b200.RtError):
        a.load_state(b"\0" * 64)
