"""Multi-rank partitioning of FA-KLA on CPU: two gloo ranks each compute their
shard (heads, then batch rows) with the oracle, gather, and must reproduce the
single-process result exactly. (The GPU kernels take the same shards; the
partition logic is what this checks.)"""
import os
import socket
import tempfile

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pulsartecture_b200.sharding import batch_shard, head_shard, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    g = torch.Generator().manual_seed(3)
    B, T, H, D = 3, 20, 5, 8
    q = torch.randn(B, T, H * D, generator=g, dtype=torch.float64) / 3
    k = torch.randn(B, T, H * D, generator=g, dtype=torch.float64) / 3
    v = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    W = torch.randn(H * D, H * D, generator=g, dtype=torch.float64) / (H * D) ** 0.5
    b = torch.randn(H * D, generator=g, dtype=torch.float64) / 10
    return q, k, v, W, b, H


def _worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import fakla_oracle as O

    q, k, v, W, b, H = _problem()
    # head shard: all batch rows, heads [h0, h1)
    h0, h1, w_r, b_r = head_shard(W, b, H, world, rank)
    out_h, S_h, z_h = O.prefill(q.numpy(), k.numpy(), v[:, :, h0:h1].contiguous().numpy(), w_r.numpy(), b_r.numpy())
    parts = [None] * world
    dist.all_gather_object(parts, (h0, h1, out_h, S_h, z_h))
    # batch shard: rows [r0, r1), all heads
    r0, r1 = batch_shard(q.shape[0], world, rank)
    out_b, _, _ = O.prefill(q[r0:r1].numpy(), k[r0:r1].numpy(), v[r0:r1].numpy(), W.numpy(), b.numpy())
    bparts = [None] * world
    dist.all_gather_object(bparts, (r0, r1, out_b))
    if rank == 0:
        out = np.concatenate([p[2] for p in sorted(parts, key=lambda p: p[0])], axis=2)
        S = np.concatenate([p[3] for p in sorted(parts, key=lambda p: p[0])], axis=1)
        outb = np.concatenate([p[2] for p in sorted(bparts, key=lambda p: p[0])], axis=0)
        np.savez(os.path.join(outdir, "gathered.npz"), out=out, S=S, outb=outb)
    dist.barrier()
    dist.destroy_process_group()


def test_shard_range_covers_exactly():
    for n in range(0, 20):
        for world in range(1, 9):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [s1 - s0 for s0, s1 in spans]
            assert max(sizes) - min(sizes) <= 1


def test_two_gloo_ranks_reproduce_single_process():
    from oracle import fakla_oracle as O

    O.build()
    q, k, v, W, b, H = _problem()
    ref_out, ref_S, _ = O.prefill(q.numpy(), k.numpy(), v.numpy(), W.numpy(), b.numpy())
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, join=True, start_method="spawn")
        got = np.load(os.path.join(d, "gathered.npz"))
        np.testing.assert_array_equal(got["out"], ref_out)
        np.testing.assert_array_equal(got["S"], ref_S)
        np.testing.assert_array_equal(got["outb"], ref_out)


def _gather_worker(rank, world, port, outdir):
    """The bench's gather of shards (its NCCL path on CUDA tensors; gloo here)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench

    full = torch.arange(4 * 6 * 8, dtype=torch.float32).reshape(4, 6, 8)
    b0, b1 = shard_range(4, world, rank)
    h0, h1 = shard_range(6, world, rank)
    by_batch = bench.gather_cat(full[b0:b1], world, 0)
    by_head = bench.gather_cat(full[:, h0:h1], world, 1)
    if rank == 0:
        same = bench.compare(by_batch, full)
        off = bench.compare(by_head + 1e-3, full)
        np.savez(os.path.join(outdir, "g.npz"), b=by_batch.numpy(), h=by_head.numpy(),
                 same=np.array([same["bit_exact"], same["max_abs"], same["rel_l2"]]),
                 off=np.array([off["bit_exact"], off["max_abs"]]))
    dist.barrier()
    dist.destroy_process_group()


def test_bench_gather_of_batch_and_head_shards():
    full = np.arange(4 * 6 * 8, dtype=np.float32).reshape(4, 6, 8)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gather_worker, args=(2, _free_port(), d), nprocs=2, join=True, start_method="spawn")
        with np.load(os.path.join(d, "g.npz")) as z:
            got = {k: z[k] for k in z.files}
    np.testing.assert_array_equal(got["b"], full)
    np.testing.assert_array_equal(got["h"], full)
    assert got["same"][0] == 1 and got["same"][1] == 0 and got["same"][2] == 0
    assert got["off"][0] == 0 and abs(got["off"][1] - 1e-3) < 1e-4  # fp32 rounding of x + 1e-3
