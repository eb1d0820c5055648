"""The multi-GPU path on real GPUs: one process per GPU over NCCL, each rank
runs the sm_100a kernel on its batch shard, and the shards gathered on rank 0
equal the single-GPU output bit for bit (batch slices are independent work
items of the same kernel).  Also the max-over-ranks timing reduction.  Skipped
on a box with fewer than two GPUs."""

import multiprocessing as mp
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(21)
    q = torch.randn(4, 1000, 4, 128, generator=g).to(torch.float16)
    k = torch.randn(4, 1000, 4, 128, generator=g).to(torch.float16)
    v = torch.randn(4, 1000, 4, 128, generator=g).to(torch.float16)
    return q, k, v


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import afa_flash_attention_kernels as fa
        from afa_py.afa_config import AFAForwardKernelConfig, DType
        from ampere_flash_attention_from_scratch_b200 import multi_gpu
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        info = multi_gpu.rank_info_from_env()
        multi_gpu.init_process_group("nccl", info, timeout_s=60.0, device=dev)
        q, k, v = _inputs()
        sl = multi_gpu.shard_range(q.shape[0], world, rank)
        cfg = AFAForwardKernelConfig(dtype=DType.FP16, d_head=128)
        local, _ = fa.forward(cfg, q[sl].to(dev), k[sl].to(dev), v[sl].to(dev), None, False)
        causal_local, _ = fa.forward_ext(q[sl].to(dev), k[sl].to(dev), v[sl].to(dev), None, True)
        torch.cuda.synchronize()
        fa.check_status(rank)
        full = multi_gpu.gather_to_rank0(local, dev)
        full_causal = multi_gpu.gather_to_rank0(causal_local, dev)
        mx = multi_gpu.max_over_ranks(10.0 * (rank + 1), dev)
        ok = True
        if rank == 0:
            ref, _ = fa.forward(cfg, q.to(dev), k.to(dev), v.to(dev), None, False)
            ref_c, _ = fa.forward_ext(q.to(dev), k.to(dev), v.to(dev), None, True)
            ok = torch.equal(full, ref) and torch.equal(full_causal, ref_c)
        multi_gpu.barrier(dev)
        multi_gpu.destroy()
        out_q.put(("ok", ok, mx))
    except Exception as e:  # surfaced through the queue
        out_q.put(("exception", repr(e), None))


def test_two_gpus_shard_gather_equals_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=240) for _ in range(2)]
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(r[0] == "ok" for r in res), res
    assert all(r[1] for r in res), res
    assert all(r[2] == 20.0 for r in res), res
