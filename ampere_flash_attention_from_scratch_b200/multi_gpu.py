"""Host-side plumbing for running the attention forward on several GPUs of one
node, one process per GPU.

The work is independent per (batch, head) slice, so ranks split the batch into
contiguous ranges and never exchange data on the hot path.  The only
collectives are a barrier around a timed region, a MAX reduction of the
per-rank elapsed time, and (for parity checks) a gather of the outputs to rank
0.  The reference has no multi-GPU code; this module exists for the 1/2/4/8-GPU
measurements and works with the NCCL (GPU) and gloo (CPU tests) backends.
"""

from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankInfo:
    rank: int
    world: int
    local_rank: int


def rank_info_from_env() -> RankInfo:
    """RANK / WORLD_SIZE / LOCAL_RANK as set by torchrun (defaults: a single process)."""
    return RankInfo(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                    int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(batch: int, world: int, rank: int) -> slice:
    """Contiguous batch range of `rank`.  Every rank gets the same count, so the
    per-rank work is identical; the batch must divide by the world size."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")
    if batch % world != 0:
        raise ValueError(f"batch {batch} is not divisible by {world} ranks")
    per = batch // world
    return slice(rank * per, (rank + 1) * per)


def init_process_group(backend: str, info: RankInfo, timeout_s: float = 300.0, device=None) -> None:
    """Initialise the default process group from the torchrun environment
    (MASTER_ADDR / MASTER_PORT) with a short timeout, so a rank that dies or
    never joins makes the others fail instead of waiting forever."""
    if info.world <= 1 or dist.is_initialized():
        return
    kwargs = {"backend": backend, "rank": info.rank, "world_size": info.world,
              "timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kwargs["device_id"] = device
    dist.init_process_group(**kwargs)


def barrier(device=None, timeout_s: float | None = None) -> None:
    """Barrier over all ranks.  With gloo, a monitored barrier: a rank that has
    left raises an error on the others within `timeout_s` instead of hanging."""
    if not dist.is_initialized():
        return
    if dist.get_backend() == "gloo":
        kw = {"timeout": timedelta(seconds=timeout_s)} if timeout_s is not None else {}
        dist.monitored_barrier(**kw)
    elif device is not None:
        dist.barrier(device_ids=[device.index])
    else:
        dist.barrier()


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. elapsed ms) over all ranks; every rank gets it."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(local: torch.Tensor, device=None):
    """Concatenate every rank's batch shard along dim 0 on rank 0 (None elsewhere)."""
    if not dist.is_initialized():
        return local
    world = dist.get_world_size()
    src = (local.to(device) if device is not None else local).contiguous()
    if dist.get_backend() == "nccl":
        parts = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(parts, src)
        return torch.cat(parts, 0) if dist.get_rank() == 0 else None
    parts = [torch.empty_like(src) for _ in range(world)] if dist.get_rank() == 0 else None
    dist.gather(src, gather_list=parts, dst=0)
    return torch.cat(parts, 0) if dist.get_rank() == 0 else None


def destroy() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def gpu_local_cpus(device_index: int):
    """The CPU cores NVML reports as local to CUDA device `device_index` (its
    NUMA node), restricted to the cores this process may run on; None when
    NVML or the device cannot say.  Reads only; changes no GPU setting."""
    try:
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 1) + 63) // 64)
        cpus = {w * 64 + b for w, mask in enumerate(words) for b in range(64) if (mask >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:
        return None


@contextlib.contextmanager
def numa_local(device_index: int):
    """Runs the body with this process bound to the cores local to GPU
    `device_index`, so page-locked host buffers allocated inside land on the
    GPU's NUMA node (copies then do not cross the inter-socket link); the
    previous affinity is restored afterwards.  A no-op where the local cores
    are unknown."""
    before = os.sched_getaffinity(0)
    cpus = gpu_local_cpus(device_index)
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield cpus
    finally:
        os.sched_setaffinity(0, before)
