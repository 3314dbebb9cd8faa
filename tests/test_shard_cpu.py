"""Host side of the sharded prefill: the chunk partition and the all-gather pack / unpack, run as
two gloo ranks on the CPU (no kernels)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hierarchicalglobalattention_b200.shard import ShardedPrefill, ShardLayout, prefill_partition, unpack_kv, unpack_summaries


def test_partition_covers_every_chunk_once():
    for S, C, W in [(32768, 64, 8), (1000, 64, 3), (100, 64, 4), (64 * 7 + 5, 64, 2)]:
        parts = prefill_partition(S, C, W)
        N = (S + C - 1) // C
        assert [n for lo, hi in parts for n in range(lo, hi)] == list(range(N))
        per = parts[0][1] - parts[0][0]
        assert all(hi - lo <= per for lo, hi in parts)


def _fill(lay, rank):
    flat = torch.empty(lay.numel)
    for i, t in enumerate(lay.views(flat)):
        t.copy_(torch.arange(t.numel(), dtype=torch.float32).view_as(t) + 1000 * rank + 100000 * i)
    return flat


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lay = ShardLayout(B=2, KVH=3, Dh=4, M=2, rows=8, chunks=2, dtype=torch.float32)
        sp = ShardedPrefill(world, rank)
        send = _fill(lay, rank)
        rs, _ = sp._gather("rs", send[:lay.sum_numel], async_op=False)
        rk, h = sp._gather("rk", send[lay.sum_numel:], async_op=True)
        h.wait()
        ck = torch.empty(lay.B, lay.KVH, world * lay.chunks, lay.Dh)
        gk = torch.empty(lay.B, lay.KVH, world * lay.chunks, lay.M, lay.Dh)
        k = torch.empty(lay.B, lay.KVH, world * lay.rows, lay.Dh)
        v = torch.empty_like(k)
        unpack_summaries(lay, rs, world, ck, gk)
        unpack_kv(lay, rk, world, k, v)
        ok = True
        for r in range(world):
            ref = lay.views(_fill(lay, r))
            ok &= torch.equal(ck[:, :, r * lay.chunks:(r + 1) * lay.chunks], ref[0])
            ok &= torch.equal(gk[:, :, r * lay.chunks:(r + 1) * lay.chunks], ref[1])
            ok &= torch.equal(k[:, :, r * lay.rows:(r + 1) * lay.rows], ref[2])
            ok &= torch.equal(v[:, :, r * lay.rows:(r + 1) * lay.rows], ref[3])
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_gather_and_unpack_two_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    assert out[0] and out[1]
