"""The N>1 paths on CPU with gloo ranks (world size 2, and 4 and 8 for the Ulysses layout).

* Ulysses layout contract of hexanima_b200/csrc/sp.cu: pack q|k|v token shards into
  send[c][dst][T/P][D/P] (head group dst), all-to-all, attend over the full sequence on H/P heads,
  all-to-all the output rows back and unpack to [T/P][D] — equals unsharded attention.
* Image-batch data parallelism of bench.py: images split evenly, step time = max over ranks.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import anima as oa


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sp_worker(rank, world, port, T, H, nvalid, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, P = H * 128, world
        Tl, Dl = T // P, D // P
        g = torch.Generator().manual_seed(7)
        qkv_full = torch.randn(T, 3 * D, generator=g)
        qkv = qkv_full[rank * Tl:(rank + 1) * Tl]                         # this rank's token shard
        # pack: send[c][j][i][e] = qkv[i][c*D + j*Dl + e]
        send = qkv.view(Tl, 3, P, Dl).permute(1, 2, 0, 3).contiguous()      # [c][j][i][e]
        recv = torch.empty_like(send)                                       # [c][src j][i][e]
        for c in range(3):
            dist.all_to_all_single(recv[c], send[c])
        q, k, v = (recv[c].reshape(T, H // P, 128) for c in range(3))       # full sequence, local heads
        o = oa.attention(q[None], k[None], v[None], scale=1.0 / math.sqrt(128), nvalid=nvalid)[0]
        ofull = o.reshape(T, Dl).view(P, Tl, Dl).contiguous()              # token block j goes to rank j
        orecv = torch.empty_like(ofull)
        dist.all_to_all_single(orecv, ofull)
        O = orecv.permute(1, 0, 2).reshape(Tl, D)                           # O[i][j*Dl + e] = orecv[j][i][e]
        ref = oa.attention(qkv_full[:, :D].view(1, T, H, 128), qkv_full[:, D:2 * D].view(1, T, H, 128),
                           qkv_full[:, 2 * D:].view(1, T, H, 128), scale=1.0 / math.sqrt(128), nvalid=nvalid)
        ref = ref.reshape(T, D)[rank * Tl:(rank + 1) * Tl]
        out[rank] = float((O - ref).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,H,nvalid", [(2, 64, 4, 64), (2, 128, 6, 100), (4, 128, 24, 120), (8, 256, 24, 250)])
def test_ulysses_exchange_layout_gloo(world, T, H, nvalid):
    """world 4 and 8 with the MOSS head count (24: 6 and 3 heads per rank), as the 4- and 8-GPU bench runs."""
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_sp_worker, args=(world, _free_port(), T, H, nvalid, out), nprocs=world, join=True)
    assert sorted(out.keys()) == list(range(world))
    assert max(out.values()) < 1e-5


def _dp_worker(rank, world, port, batch, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        share = bench.images_per_rank(batch, world)
        t = torch.tensor([0.010 * (rank + 1), 0.5 + rank], dtype=torch.float64)  # per-rank step times
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[rank] = (share, t.tolist())
    finally:
        dist.destroy_process_group()


def test_image_batch_sharding_gloo():
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_dp_worker, args=(2, _free_port(), 8, out), nprocs=2, join=True)
    for r in (0, 1):
        share, t = out[r]
        assert share == 4 and t == [0.020, 1.5]   # every rank sees the slowest rank's times
    import bench
    assert [bench.images_per_rank(8, n) for n in (1, 2, 4, 8)] == [8, 4, 2, 1]
    with pytest.raises(ValueError):
        bench.images_per_rank(8, 3)
