"""The (batch x head) partition on the CUDA kernels (GPU): two ranks each run
their shard of one prefill problem through fakla_prefill (the C ABI), the
shards are gathered (gloo) and rank 0's assembled result is checked against
the oracle and against the same problem run whole on one GPU.

The ranks are two processes; with one GPU they share it (each rank's kernels
are independent of the other's, nothing waits across processes), with more
each takes its own. Head shards take the matching rows of the feature map and
whole q, k rows (the map mixes all heads of a row), which is the split a
multi-GPU run uses when it divides heads.

T=1000 (a ragged last chunk) with 4 sequences per rank makes each rank's scan
run segmented (segment sums, prefix, one CTA per segment), as the small
per-GPU problems of an 8-GPU split do; a per-(token, head) temperature rides
along, split with its heads or batch rows.
"""
import math
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.helpers import BF16_MAX_ABS, BF16_REL_L2, lpm_params, rel_l2

pytestmark = pytest.mark.gpu

B, T, H, D = 2, 1000, 4, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(21)
    q = (torch.randn(B, T, H * D, generator=g) / math.sqrt(D)).bfloat16()
    k = (torch.randn(B, T, H * D, generator=g) / math.sqrt(D)).bfloat16()
    v = (torch.randn(B, T, H, D, generator=g) / math.sqrt(D)).bfloat16()
    W, b = lpm_params(H * D, H * D, seed=22, dtype=torch.bfloat16)
    tp = (torch.rand(B, T, H, generator=g) + 0.5).bfloat16()
    return q, k, v, W, b, tp


def _prefill(dev, q, k, v, W, b, tp):
    """fakla_prefill through the C ABI; returns (out, S, z) on the host."""
    from pulsartecture_b200 import _lib

    L = _lib.lib()
    Bl, Tl, Hl = v.shape[0], v.shape[1], v.shape[2]
    in_dim = q.shape[-1]
    q, k, v, W, b, tp = (t.to(dev).contiguous() for t in (q, k, v, W, b, tp))
    out = torch.empty(Bl, Tl, Hl, D, device=dev, dtype=torch.bfloat16)
    S = torch.empty(Bl, Hl, D, D, device=dev)
    z = torch.empty(Bl, Hl, D, device=dev)
    ws_bytes = L.fakla_prefill_workspace_bytes(Bl, Tl, in_dim, Hl, D, D, _lib.FAKLA_BF16)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(L.fakla_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), tp.data_ptr(), W.data_ptr(), b.data_ptr(),
                               out.data_ptr(), S.data_ptr(), z.data_ptr(), Bl, Tl, in_dim, Hl, D, D,
                               _lib.FAKLA_BF16, _lib.FAKLA_STATE_OUT, ws.data_ptr(), ws_bytes, stream))
    _lib.check(L.fakla_device_status(stream))
    segmented = L.fakla_attention_workspace_bytes(Bl, Tl, Hl, D, D, _lib.FAKLA_BF16) > 0
    return out.float().cpu().numpy(), S.cpu().numpy(), z.cpu().numpy(), segmented


def _worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from pulsartecture_b200.sharding import batch_shard, head_shard

    dev = torch.device("cuda", rank % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    q, k, v, W, b, tp = _inputs()
    # head shard: every batch row, heads [h0, h1), the matching map rows
    h0, h1, w_r, b_r = head_shard(W, b, H, world, rank)
    oh, Sh, zh, seg_h = _prefill(dev, q, k, v[:, :, h0:h1], w_r, b_r, tp[:, :, h0:h1])
    hparts = [None] * world
    dist.all_gather_object(hparts, (h0, oh, Sh, zh, seg_h))
    # batch shard: rows [r0, r1), every head
    r0, r1 = batch_shard(B, world, rank)
    ob, Sb, zb, seg_b = _prefill(dev, q[r0:r1], k[r0:r1], v[r0:r1], W, b, tp[r0:r1])
    bparts = [None] * world
    dist.all_gather_object(bparts, (r0, ob, Sb, zb, seg_b))
    if rank == 0:
        hp = sorted(hparts, key=lambda p: p[0])
        bp = sorted(bparts, key=lambda p: p[0])
        np.savez(os.path.join(outdir, "gathered.npz"),
                 h_out=np.concatenate([p[1] for p in hp], axis=2),
                 h_S=np.concatenate([p[2] for p in hp], axis=1),
                 h_z=np.concatenate([p[3] for p in hp], axis=1),
                 b_out=np.concatenate([p[1] for p in bp], axis=0),
                 b_S=np.concatenate([p[2] for p in bp], axis=0),
                 b_z=np.concatenate([p[3] for p in bp], axis=0),
                 segmented=np.array([p[4] for p in hp] + [p[4] for p in bp]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_head_and_batch_shards_on_the_kernels(cuda):
    from oracle import fakla_oracle as O

    q, k, v, W, b, tp = _inputs()
    f = lambda t: t.float().numpy()  # noqa: E731
    eo, eS, ez = O.prefill(f(q), f(k), f(v), f(W), f(b), f(tp))
    whole_out, whole_S, whole_z, _ = _prefill(cuda, q, k, v, W, b, tp)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, join=True, start_method="spawn")
        with np.load(os.path.join(d, "gathered.npz")) as npz:
            got = {key: npz[key] for key in npz.files}
    assert got["segmented"].all(), "each rank's 4 sequences should take the segmented scan"
    for tag in ("h", "b"):
        out, S, z = got[f"{tag}_out"], got[f"{tag}_S"], got[f"{tag}_z"]
        # against the oracle (parity bar)
        assert rel_l2(out, eo) < BF16_REL_L2, tag
        assert np.abs(out - eo).max() < BF16_MAX_ABS, tag
        assert rel_l2(S, eS) < BF16_REL_L2 and rel_l2(z, ez) < BF16_REL_L2, tag
        # against the whole problem on one GPU (same kernels; the shards only
        # change how the scan is segmented, i.e. the fp32 summation order)
        assert rel_l2(out, whole_out) < 2e-3, tag
        assert rel_l2(S, whole_S) < 2e-4 and rel_l2(z, whole_z) < 2e-4, tag
