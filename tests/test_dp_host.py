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


def _free_port() -> int:
    """A port no other job holds right now (rendezvous on shared machines)."""
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


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
        mp.start_processes(_rank, args=(world, _free_port(), d), nprocs=world, start_method="spawn")
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


def _chunk_row_of(rows, chunks, c):
    # the library's chunk edges (mlp.cu chunk_row_of: chunk starts on 256-row
    # edges, the last chunk takes the rest)
    from rgpu_b200.gpu import lib

    return int(lib().rt_plan_chunk_row(rows, chunks, c))


def test_chunk_edges_follow_the_256_row_rule():
    for rows, chunks in [(8193, 4), (4097, 4), (2049, 2), (513, 2), (1001, 3)]:
        edges = [_chunk_row_of(rows, chunks, c) for c in range(chunks + 1)]
        assert edges[0] == 0 and edges[-1] == rows
        assert all(e % 256 == 0 for e in edges[:-1]) and edges == sorted(edges)


@pytest.mark.parametrize("d,ld,world,chunks", [(4096, 8192, 8, 4), (8192, 1024, 8, 4), (1024, 512, 2, 4),
                                               (512, 192, 2, 2), (2048, 64, 4, 2)])
def test_peer_scatter_layout_is_the_flat_reduce_scatter(d, ld, world, chunks):
    # The peer-memory reduce-scatter (p2p_chunk in tc_common.cuh, dw_gemm_rows
    # and allreduce_rows in mlp.cu), restated: launch row i of chunk [r0, r1)
    # goes to owner o = i // h at
    #   o's buffer [src * q_stride + (r0 // world + i - o * h) * ld + col],
    # h = (e - r0) // world, e = min(r1, d), q_stride = d // world * ld; the
    # owner sums its [r0 // world * ld, + h * ld) window of every source region
    # into g[(r0 + o * h) * ld, + h * ld).  Checked: every (source, row) pair
    # lands on its own row of the owner's buffer, inside the buffer, and the
    # owner's sums cover exactly its flat reduce-scatter slice of each chunk,
    # (e - r0) * ld / world elements from r0 * ld + o * (e - r0) * ld / world.
    rows = d + 1
    q_stride = d // world * ld
    seen = [set() for _ in range(world)]
    for c in range(chunks):
        r0, r1 = _chunk_row_of(rows, chunks, c), _chunk_row_of(rows, chunks, c + 1)
        e = min(r1, d)
        assert (e - r0) % world == 0 and r0 % world == 0
        h = (e - r0) // world
        for src in range(world):
            for i in range(r1 - r0):
                if i >= e - r0:
                    continue  # the bias row stays in the rank's own g (allreduced)
                o = i // h
                off = src * q_stride + (r0 // world + i - o * h) * ld
                assert 0 <= off and off + ld <= world * q_stride == d * ld
                assert off not in seen[o]
                seen[o].add(off)
        for o in range(world):
            # what the owner sums for chunk c, row by row, is rows r0 + o*h ...
            window = [(r0 // world + k) * ld for k in range(h)]
            got_rows = [r0 + o * h + k for k in range(h)]
            flat0 = r0 * ld + o * ((e - r0) * ld // world)
            assert got_rows[0] * ld == flat0 and len(window) * ld == (e - r0) * ld // world
            # ... which is the library's shard slice of owner o (ld == units here)
            import ctypes

            from rgpu_b200.gpu import lib

            off = ctypes.c_int64(0)
            assert lib().rt_plan_shard_slice(d, ld, r0, r1, world, o, ctypes.byref(off)) == len(window) * ld
            assert off.value == flat0
    for o in range(world):
        assert len(seen[o]) == world * d // world  # every source's every owned row, once


def _sharded_rank(rank, world, port, out_dir):
    # The sharded optimiser's update on gloo ranks with the oracle's Adam, on
    # the slices the library itself computes (rgpu_b200.gpu.plan_layout: the
    # leading dimension, the dW chunk rows and each rank's flat slice, from
    # mlp.cu's plan_ld, dw_chunks, chunk_row_of and shard_slice): per chunk of
    # [W; b] rows rank r updates its slice of the summed gradient, the bias row
    # is summed and updated on every rank, and the slices are all-gathered.
    # Path A is the replicated update; both must give the same parameters.
    from rgpu_b200.gpu import plan_layout

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # two chunks where the rows allow it, so that the chunk edges are exercised
    os.environ["RTGPU_DW_CHUNKS"] = "2"
    os.environ["RTGPU_FIRST_LAYER_CHUNKS"] = "2"
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dims, n = [512, 384, 10], 16
        rng = oracle.Rng(5)
        model = oracle.Mlp(dims)
        model.init_glorot(rng)
        x = rng.normal(n * dims[0]).reshape(n, dims[0])
        labels = rng.below(dims[-1], n)
        per = n // world
        model.train_step(x[rank * per:(rank + 1) * per], labels[rank * per:(rank + 1) * per])
        grads = [g * (per / n) for g in model.grads()]
        params = model.params()
        out = {}
        n_chunks = []
        for mode in ("replicated", "sharded"):
            thetas = []
            for l in range(len(dims) - 1):
                d, u = dims[l], dims[l + 1]
                ld, chunks = plan_layout(l, d, u, world, rank, data_parallel=True)
                # the [d+1, ld] parameter block, padding columns zero
                block = np.zeros((d + 1, ld), np.float32)
                block[:d, :u], block[d, :u] = params[2 * l], params[2 * l + 1].ravel()
                theta = block.ravel()
                gblock = np.zeros((d + 1, ld), np.float32)
                gblock[:d, :u], gblock[d, :u] = grads[2 * l], grads[2 * l + 1].ravel()
                g = torch.from_numpy(gblock.ravel().copy())
                dist.all_reduce(g)  # the sum (a reduce-scatter keeps only this rank's slice of it)
                g = g.numpy()
                mm, vv = np.zeros_like(theta), np.zeros_like(theta)
                if mode == "replicated":
                    oracle.adam_update(theta, mm, vv, g, 1e-3, 1)
                else:
                    n_chunks.append(len(chunks))
                    covered = 0
                    for r0, r1, a, piece in chunks:
                        e = min(r1, d)
                        assert piece * world == (e - r0) * ld and a == r0 * ld + rank * piece
                        th, m_, v_ = theta[a:a + piece], mm[a:a + piece], vv[a:a + piece]
                        oracle.adam_update(th, m_, v_, g[a:a + piece], 1e-3, 1)
                        if r1 > d:  # the bias row, replicated
                            b0 = d * ld
                            th, m_, v_ = theta[b0:b0 + ld], mm[b0:b0 + ld], vv[b0:b0 + ld]
                            oracle.adam_update(th, m_, v_, g[b0:b0 + ld], 1e-3, 1)
                        parts = [torch.zeros(piece) for _ in range(world)]
                        dist.all_gather(parts, torch.from_numpy(theta[a:a + piece].copy()))
                        theta[r0 * ld:r0 * ld + world * piece] = torch.cat(parts).numpy()
                        covered += world * piece
                    assert covered == d * ld  # the slices tile the weight rows exactly
                thetas.append(theta)
            out[mode] = np.concatenate(thetas)
        if rank == 0:
            np.savez(os.path.join(out_dir, "sharded.npz"), chunks=np.array(n_chunks), **out)
    finally:
        dist.destroy_process_group()


def test_gloo_sharded_update_equals_replicated_update():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_sharded_rank, args=(world, _free_port(), d), nprocs=world, start_method="spawn")
        got = np.load(os.path.join(d, "sharded.npz"))
        assert list(got["chunks"]) == [2, 1]  # the first layer in two chunks; 385 rows allow one
        assert np.array_equal(got["replicated"], got["sharded"])
