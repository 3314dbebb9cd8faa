"""Batched decode split across GPUs by sequence, with no collective on the data path.

The reference decodes a batch on one device (ExistingModelFineTuning/KvRouter/chunk_router.py:
279-407, one ``RamKVCacheStore`` per model).  Its decode routing and attention are independent per
sequence, so here one process per GPU owns a contiguous range of the batch's sequences, each with
its own ``ChunkRouter`` and store (its pinned cold record allocated while the process runs on the
CPUs of the GPU's NUMA node, so the host-link reads of its decode kernels stay node-local).  Ranks
exchange nothing: each returns the outputs of its own sequences.
"""
from __future__ import annotations

import os
from typing import Callable, List, Optional, Sequence, Set, Tuple

import torch


def decode_partition(batch: int, world: int, weights: Optional[Sequence[float]] = None) -> List[Tuple[int, int]]:
    """Contiguous ranges [lo, hi) of the batch's sequences per rank.  Without ``weights`` the
    ranges differ in size by at most one; with per-sequence ``weights`` (e.g. context lengths, the
    decode cost of a sequence grows with its routed pool) the cut points balance the weight sums
    greedily.  Every rank gets at least one sequence when batch >= world."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if weights is None:
        base, extra = divmod(batch, world)
        out, lo = [], 0
        for r in range(world):
            hi = lo + base + (1 if r < extra else 0)
            out.append((lo, hi))
            lo = hi
        return out
    if len(weights) != batch:
        raise ValueError("one weight per sequence")
    total = float(sum(weights))
    out, lo, acc = [], 0, 0.0
    for r in range(world):
        if r == world - 1:
            out.append((lo, batch))
            break
        target = total * (r + 1) / world
        hi = lo
        # take sequences while the running sum stays closer to the target, leaving one per rank
        while hi < batch - (world - 1 - r) and (hi == lo or abs(acc + weights[hi] - target) <= abs(acc - target)):
            acc += weights[hi]
            hi += 1
        out.append((lo, hi))
        lo = hi
    return out


def parse_cpulist(text: str) -> Set[int]:
    """'0-3,8,10-11' -> {0, 1, 2, 3, 8, 10, 11} (the sysfs cpulist format)."""
    cpus: Set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_local_cpus(device: torch.device, sysfs_root: str = "/sys") -> Optional[Set[int]]:
    """The CPUs of the NUMA node the GPU hangs off (sysfs ``local_cpulist`` of its PCI device), or
    None when unknown."""
    try:
        pr = torch.cuda.get_device_properties(device)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
    except Exception:
        return None
    return local_cpus_of_pci(bus, sysfs_root)


def local_cpus_of_pci(bus: str, sysfs_root: str = "/sys") -> Optional[Set[int]]:
    path = os.path.join(sysfs_root, "bus", "pci", "devices", bus, "local_cpulist")
    try:
        with open(path) as f:
            cpus = parse_cpulist(f.read())
    except OSError:
        return None
    return cpus or None


def bind_host_to_gpu(device: torch.device, sysfs_root: str = "/sys") -> bool:
    """Restrict this process to the CPUs near ``device`` (first-touch placement then puts pinned
    host allocations on that node).  Returns whether an affinity was set."""
    cpus = gpu_local_cpus(device, sysfs_root)
    if not cpus:
        return False
    avail = os.sched_getaffinity(0)
    cpus &= avail
    if not cpus:
        return False
    os.sched_setaffinity(0, cpus)
    return True


class ShardedDecode:
    """One rank's share of a batched decode: sequences [lo, hi) of the global batch.

    ``make_router(batch)`` builds the rank's ChunkRouter over a store sized for its own sequences
    (called after the process is bound to the GPU's NUMA node when ``bind_numa``).  ``seed`` and
    ``decode_step`` take global-batch tensors (or already-sliced ones, ``local=True``) and run on
    the rank's rows only; the outputs are the rank's rows."""

    def __init__(self, world: int, rank: int, batch: int, make_router: Callable[[int], object],
                 device: Optional[torch.device] = None, weights: Optional[Sequence[float]] = None,
                 bind_numa: bool = True) -> None:
        self.world, self.rank = world, rank
        self.lo, self.hi = decode_partition(batch, world, weights)[rank]
        if bind_numa and device is not None and device.type == "cuda":
            bind_host_to_gpu(device)
        self.router = make_router(self.hi - self.lo)

    def rows(self, t: torch.Tensor, local: bool) -> torch.Tensor:
        return t if local else t[self.lo:self.hi]

    def seed(self, layer: int, k_rope, k_raw, v, seq_lens: Optional[Sequence[int]] = None, local: bool = False):
        k_rope, k_raw, v = (self.rows(t, local) for t in (k_rope, k_raw, v))
        if seq_lens is None:
            return self.router.seed(layer, k_rope, k_raw, v)
        lens = list(seq_lens) if local else list(seq_lens[self.lo:self.hi])
        return self.router.seed_mixed(layer, k_rope, k_raw, v, lens)

    def decode_step(self, layer: int, q, k_rope, k_raw, v, seq_pos_host: Sequence[int], local: bool = False):
        """One block per owned sequence at its own position; returns the attention output of the
        owned rows [hi - lo, H, L, Dh]."""
        q, k_rope, k_raw, v = (self.rows(t, local) for t in (q, k_rope, k_raw, v))
        pos = list(seq_pos_host) if local else list(seq_pos_host[self.lo:self.hi])
        seq = torch.tensor(pos, dtype=torch.int32, device=q.device)
        rk = self.router.decode_step(layer, q, k_rope, k_raw, v, seq, pos)
        return rk.attend(q)
