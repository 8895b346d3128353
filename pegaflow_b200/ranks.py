"""One process per GPU: rank setup, shard arithmetic and cross-rank timing.

The transfer path needs no collective: every tensor-parallel rank saves and
loads its own KV heads on its own GPU into its own pool region (the reference
keys them apart by slot = layer*tp_size + tp_rank, pegaflow-core/src/lib.rs:205-219).
Collectives appear only around measurement (a barrier before and after the
timed region, and the max of the ranks' times).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import numpy as np


@dataclass
class Ranks:
    rank: int
    world: int
    local: int
    backend: str | None
    _host_group: object = None

    @classmethod
    def from_env(cls, backend: str | None = None, timeout_s: float = 600.0) -> "Ranks":
        """Read RANK/WORLD_SIZE/LOCAL_RANK (torchrun) and join the group when
        there is more than one rank. backend None picks nccl for GPUs."""
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        local = int(os.environ.get("LOCAL_RANK", str(rank)))
        r = cls(rank, world, local, None)
        if world > 1:
            import torch
            import torch.distributed as dist

            backend = backend or "nccl"
            kw = {}
            if backend == "nccl":
                kw["device_id"] = torch.device(f"cuda:{local}")
            dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)
            r.backend = backend
            # Host-side group for waits while another rank works on a GPU this
            # rank also uses: a rank parked in it runs no kernel.
            r._host_group = (dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
                             if backend != "gloo" else None)
        return r

    def _reduce(self, x: float, op: str) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist

        dev = f"cuda:{self.local}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM}[op])
        return float(t.item())

    def max(self, x: float) -> float:
        return self._reduce(x, "max")

    def min(self, x: float) -> float:
        return -self._reduce(-x, "max")

    def sum(self, x: float) -> float:
        return self._reduce(x, "sum")

    def gather(self, x: float) -> list[float]:
        """Every rank's value, in rank order, on every rank."""
        if self.world == 1:
            return [float(x)]
        import torch
        import torch.distributed as dist

        dev = f"cuda:{self.local}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        dist.all_gather(out, t)
        return [float(v.item()) for v in out]

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def host_barrier(self) -> None:
        """A barrier that waits on the host only (gloo), never in a GPU
        kernel: ranks parked here while rank 0 runs kernels on their GPUs
        (the P/D check) hold no spinning collective kernel there."""
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=getattr(self, "_host_group", None))

    def all_true(self, flag: bool) -> bool:
        """True when `flag` holds on every rank."""
        return self.min(1.0 if flag else 0.0) == 1.0

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def bind_to_gpu_cpus(device: int) -> list[int] | None:
    """Restrict this process to the CPUs NVML reports as local to `device`
    (its NUMA node), so pinned pool pages, which are touched when they are
    allocated, land in the memory next to the GPU's PCIe root. Read-only query
    of the topology; returns the CPU list, or None when it cannot be read."""
    try:
        import pynvml
        import torch

        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = [w * 64 + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1]
        cpus = [c for c in cpus if c in os.sched_getaffinity(0)]
        if cpus:
            os.sched_setaffinity(0, cpus)
            return cpus
    except Exception:
        return None
    return None


def tp_heads(num_heads: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads [lo, hi) owned by TP rank `rank` of `world` (even split)."""
    if num_heads % world:
        raise ValueError(f"{num_heads} KV heads do not split over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def pool_region(pool_bytes: int, rank: int, world: int, align: int = 1 << 21) -> tuple[int, int]:
    """Disjoint [offset, offset+size) of a shared pool for one rank (2 MiB aligned)."""
    per = pool_bytes // world // align * align
    return rank * per, per


def block_lists(num_blocks: int, n: int, rank: int, order: str) -> tuple[np.ndarray, np.ndarray]:
    """Source and destination block ids of one rank, disjoint whenever
    2n <= num_blocks, so restoring into the destinations never overwrites a
    source and the restored blocks can be compared with the sources after
    any number of save/load steps.

    sorted: sources 0..n-1, destinations n..2n-1 (sorted-contiguous runs).
    shuffled: one seeded permutation (seed 3+rank); its first n ids are the
    sources and the next n the destinations."""
    if order == "sorted":
        return np.arange(n), (np.arange(n) + n) % num_blocks
    perm = np.random.default_rng(3 + rank).permutation(num_blocks)
    if 2 * n <= num_blocks:
        return perm[:n], perm[n:2 * n]
    return perm[:n], np.random.default_rng(4 + rank).permutation(num_blocks)[:n]
