"""Multi-rank host logic on CPU with the gloo backend (world size 2).

The GPU runs split the batch over ranks with no data-path collective; these
tests cover the same code (ampere_flash_attention_from_scratch_b200.multi_gpu)
with the CPU oracle standing in for the kernel:
* every rank computes its batch shard; the gathered result equals the
  single-process result;
* max_over_ranks returns the largest per-rank value on every rank;
* a rank that leaves before a collective makes the other fail with an error
  within the barrier timeout instead of waiting forever.
"""

import multiprocessing as mp
import os
import socket

import pytest
import torch

from ampere_flash_attention_from_scratch_b200 import multi_gpu
from oracle.attention_oracle import attention_fp32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(11)
    q = torch.randn(4, 64, 2, 32, generator=g).to(torch.float16)
    k = torch.randn(4, 64, 2, 32, generator=g).to(torch.float16)
    v = torch.randn(4, 64, 2, 32, generator=g).to(torch.float16)
    return q, k, v


def _put_and_exit(out_q, msg):
    """Deliver `msg` (flush the queue's feeder thread) and end the process at once."""
    out_q.put(msg)
    out_q.close()
    out_q.join_thread()
    os._exit(0)


def _worker(rank, world, port, mode, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        info = multi_gpu.rank_info_from_env()
        multi_gpu.init_process_group("gloo", info, timeout_s=60.0)
        if mode == "shard":
            q, k, v = _inputs()
            sl = multi_gpu.shard_range(q.shape[0], world, rank)
            local = attention_fp32(q[sl], k[sl], v[sl])
            full = multi_gpu.gather_to_rank0(local)
            mx = multi_gpu.max_over_ranks(10.0 * (rank + 1))
            ok = torch.equal(full, attention_fp32(q, k, v)) if rank == 0 else True
            out_q.put(("ok", ok, mx))
            multi_gpu.destroy()
        elif mode == "leave":
            if rank == 1:
                _put_and_exit(out_q, ("left", None, None))  # leaves without taking part in the barrier
            try:
                multi_gpu.barrier(timeout_s=3.0)
                _put_and_exit(out_q, ("no-error", None, None))
            except Exception as e:  # the expected outcome
                _put_and_exit(out_q, ("error", type(e).__name__, None))
    except Exception as e:  # pragma: no cover - surfaced through the queue
        out_q.put(("exception", repr(e), None))


def _run(mode, world=2, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=timeout) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():  # pragma: no cover
                p.kill()
    return results


def test_shard_range():
    assert multi_gpu.shard_range(16, 4, 2) == slice(8, 12)
    assert multi_gpu.shard_range(16, 1, 0) == slice(0, 16)
    with pytest.raises(ValueError):
        multi_gpu.shard_range(16, 3, 0)
    with pytest.raises(ValueError):
        multi_gpu.shard_range(16, 2, 2)
    covered = sorted(i for r in range(8) for i in range(16)[multi_gpu.shard_range(16, 8, r)])
    assert covered == list(range(16))


def test_two_ranks_shard_gather_and_max():
    res = _run("shard")
    assert all(r[0] == "ok" for r in res), res
    assert all(r[1] for r in res)
    assert all(r[2] == 20.0 for r in res)


def test_rank_leaving_is_detected():
    res = _run("leave")
    kinds = sorted(r[0] for r in res)
    assert kinds == ["error", "left"], res


def test_numa_local_restores_affinity_and_is_a_no_op_without_nvml_device():
    """numa_local() binds only where NVML names the GPU's cores (not on this CPU
    machine) and always restores the process's affinity afterwards."""
    import os

    from ampere_flash_attention_from_scratch_b200 import multi_gpu

    before = os.sched_getaffinity(0)
    assert multi_gpu.gpu_local_cpus(0) is None
    with multi_gpu.numa_local(0) as cpus:
        assert cpus is None and os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before
