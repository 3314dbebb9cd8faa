"""Host side of the sharded prefill: the zigzag partition, the send-buffer layout and the
all-gather exchange, run as two gloo ranks on the CPU (no kernels; the unpack is restated here
with torch indexing)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hierarchicalglobalattention_b200.shard import (PIECES, ShardedPrefill, ShardLayout, block_table,
                                                    prefill_partition, rank_rows)


def test_partition_covers_every_chunk_once_and_balances():
    for S, C, W in [(32768, 64, 8), (1000, 64, 3), (100, 64, 4), (64 * 7 + 5, 64, 2), (200, 64, 8)]:
        parts = prefill_partition(S, C, W)
        N = (S + C - 1) // C
        assert sorted(n for blocks in parts for lo, hi in blocks for n in range(lo, hi)) == list(range(N))
        tab = block_table(W)
        assert sorted(tab) == list(range(PIECES * W))
        rows = [sum(hi - lo for lo, hi in rank_rows(S, C, W, r)) for r in range(W)]
        assert sum(rows) == S
    # router work ~ chunk index: zigzag pairs give every rank the same sum
    parts = prefill_partition(32768, 64, 8)
    work = [sum(sum(range(lo, hi)) for lo, hi in blocks) for blocks in parts]
    assert max(work) - min(work) <= 0.01 * max(work)


def unpack_reference(lay, recv, world, rank_elems, offset, rows, row_elems, dst):
    """What hga_shard_unpack does, with torch indexing."""
    tab = block_table(world)
    bk = lay.B * lay.KVH
    d = dst.view(bk, PIECES * world, rows, row_elems)
    for r in range(world):
        for j in range(PIECES):
            src = recv[r * rank_elems + offset + j * bk * rows * row_elems:][:bk * rows * row_elems]
            d[:, tab[r * PIECES + j]] = src.view(bk, rows, row_elems)


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
        nb = PIECES * world
        k = torch.empty(lay.B, lay.KVH, nb * lay.rows, lay.Dh)
        unpack_reference(lay, rk, world, lay.kv_numel, 0, lay.rows, lay.Dh, k)
        ck = torch.empty(lay.B, lay.KVH, nb * lay.chunks, lay.Dh)
        unpack_reference(lay, rs, world, lay.sum_numel, 0, lay.chunks, lay.Dh, ck)
        ok = True
        tab = block_table(world)
        for r in range(world):
            ref = lay.views(_fill(lay, r))
            for j in range(PIECES):
                blk = tab[r * PIECES + j]
                ok &= torch.equal(k[:, :, blk * lay.rows:(blk + 1) * lay.rows], ref[2][j])
                ok &= torch.equal(ck[:, :, blk * lay.chunks:(blk + 1) * lay.chunks], ref[0][j])
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_gather_and_unpack_two_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    assert out[0] and out[1]
