"""Host-side logic of data parallelism on CPU ranks (gloo, world size 2):
the per-rank adjoint scaling by 1/n_global followed by a sum over ranks gives
the full-batch gradient, and a 128-byte communicator id travels from rank 0 to
every rank, which is how bench.py hands out the NCCL unique id."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _rank(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # id exchange, as bench.py does it (broadcast of 128 bytes from rank 0)
        uid = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            uid.copy_(torch.arange(128, dtype=torch.uint8))
        dist.broadcast(uid, 0)
        assert torch.equal(uid, torch.arange(128, dtype=torch.uint8))
        # data-parallel gradients of the oracle MLP
        rng = oracle.Rng(11)
        model = oracle.Mlp([6, 12, 5])
        model.init_glorot(rng)
        n = 16
        x = rng.normal(n * 6).reshape(n, 6)
        labels = rng.below(5, n)
        per = n // world
        xs, ls = x[rank * per:(rank + 1) * per], labels[rank * per:(rank + 1) * per]
        model.train_step(xs, ls)
        # the rank's adjoint carries 1/per; rescale to 1/n as the plan's xent does
        grads = [torch.from_numpy(g * (per / n)) for g in model.grads()]
        for g in grads:
            dist.all_reduce(g)
        if rank == 0:
            np.savez(os.path.join(out_dir, "dp.npz"), *[g.numpy() for g in grads])
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_sum_to_full_batch_gradient():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, 29617, d), nprocs=world, start_method="spawn")
        got = np.load(os.path.join(d, "dp.npz"))
        rng = oracle.Rng(11)
        model = oracle.Mlp([6, 12, 5])
        model.init_glorot(rng)
        x = rng.normal(16 * 6).reshape(16, 6)
        labels = rng.below(5, 16)
        model.train_step(x, labels)
        for i, ref in enumerate(model.grads()):
            g = got[f"arr_{i}"]
            assert np.allclose(g, ref, rtol=1e-5, atol=1e-7), i
