"""Host side of the sequence-sharded batched decode: the partition (contiguous, complete,
balanced), NUMA placement from a fake sysfs tree, and two gloo ranks agreeing on the split
without exchanging data."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hierarchicalglobalattention_b200.decode_shard import (decode_partition, local_cpus_of_pci, parse_cpulist)


def test_partition_even_and_weighted():
    for B, W in [(64, 8), (16, 2), (10, 4), (3, 3), (17, 5)]:
        parts = decode_partition(B, W)
        assert parts[0][0] == 0 and parts[-1][1] == B
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        sizes = [hi - lo for lo, hi in parts]
        assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
    g = torch.Generator().manual_seed(4)
    lens = [int(x) * 64 for x in torch.randint(8192 // 64, 131072 // 64 + 1, (64,), generator=g)]
    parts = decode_partition(64, 8, lens)
    assert parts[0][0] == 0 and parts[-1][1] == 64 and all(hi > lo for lo, hi in parts)
    loads = [sum(lens[lo:hi]) for lo, hi in parts]
    even = [sum(lens[lo:hi]) for lo, hi in decode_partition(64, 8)]
    assert max(loads) <= max(even) and max(loads) <= 1.25 * sum(lens) / 8


def test_numa_cpulist_from_fake_sysfs(tmp_path):
    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    d = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    d.mkdir(parents=True)
    (d / "local_cpulist").write_text("48-95,144-191\n")
    cpus = local_cpus_of_pci("0000:1b:00.0", str(tmp_path))
    assert cpus == set(range(48, 96)) | set(range(144, 192))
    assert local_cpus_of_pci("0000:99:00.0", str(tmp_path)) is None


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B = 13
        lo, hi = decode_partition(B, world)[rank]
        mine = torch.zeros(B, dtype=torch.int64)
        mine[lo:hi] = 1
        dist.all_reduce(mine)          # test-only check: every sequence owned exactly once
        out[rank] = bool((mine == 1).all())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_own_every_sequence_once():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(2, port, out), nprocs=2, join=True)
    assert out[0] and out[1]
