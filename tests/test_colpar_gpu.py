"""Fused column-parallel gather on 2 GPUs: every rank's epilogue writes its
N-shard of C into every rank's full C over peer memory (CUDA IPC); the
gathered matrix must equal the single-GPU GEMM of the unsharded operands
bit for bit (same tiles, same K order).  Skipped with fewer than 2 GPUs."""
import datetime
import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, m, n, k, result_dir):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # A short timeout: a failing rank ends the others' next collective with
    # an error instead of a long hang.
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    from cuda_optimazation_b200 import colpar
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    xa = torch.randn(m, k, generator=gen, device=dev)
    gen.manual_seed(12)
    xb = torch.randn(n, k, generator=gen, device=dev)
    # Every rank quantises the full operands (one global tensor scale each),
    # then keeps its B shard, as a checkpoint loader would.
    a = q.make_nvfp4(xa, layout=q.LAYOUT_MMA_KMAJOR)
    b = q.make_nvfp4(xb, layout=q.LAYOUT_MMA_KMAJOR)
    lo, hi = colpar.shard_range(n, world, rank)
    b_local = colpar.shard_rows(b, lo, hi)
    bufs = colpar.GatherBuffers(m, n, dev)
    bufs.c.fill_(float("nan"))
    torch.cuda.synchronize()
    dist.barrier()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    full = colpar.colpar_gemm_fused(a, b_local, n, bufs, status=status)
    rc, code = q.read_status(status)
    ref = q.block_scaled_gemm(a, b, out_dtype=torch.bfloat16)
    ok = rc == q.OK and torch.equal(full, ref)
    torch.save({"ok": ok, "code": code,
                "mismatch": int((full != ref).sum().item())},
               os.path.join(result_dir, f"r{rank}.pt"))
    dist.barrier()
    bufs.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("m,n,k", [(512, 1024, 512), (300, 1536, 1024)])
def test_fused_gather_two_gpus_matches_single_gpu(tmp_path, m, n, k):
    world = 2
    port = 29731 + (m % 97)
    mp.spawn(_worker, args=(world, port, m, n, k, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        res = torch.load(tmp_path / f"r{r}.pt")
        assert res["ok"], res


def _worker_steps(rank, world, port, m, n, k, result_dir):
    """Three steps with different A; rank 1 reads each result late (after a
    half-second sleep).  The entry barrier of colpar_gemm_fused
    keeps rank 0's next step from overwriting rank 1's buffer before it has
    read the current one."""
    import time
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    from cuda_optimazation_b200 import colpar
    from cuda_optimazation_b200 import qgemm as q
    dev = torch.device("cuda", rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(22)
    b = q.make_nvfp4(torch.randn(n, k, generator=gen, device=dev), layout=q.LAYOUT_MMA_KMAJOR)
    lo, hi = colpar.shard_range(n, world, rank)
    b_local = colpar.shard_rows(b, lo, hi)
    bufs = colpar.GatherBuffers(m, n, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ok, bad = True, []
    for step in range(3):
        gen.manual_seed(100 + step)
        a = q.make_nvfp4(torch.randn(m, k, generator=gen, device=dev), layout=q.LAYOUT_MMA_KMAJOR)
        ref = q.block_scaled_gemm(a, b, out_dtype=torch.bfloat16)
        full = colpar.colpar_gemm_fused(a, b_local, n, bufs, status=status)
        if rank == 1:
            time.sleep(0.5)
        got = full.clone()
        torch.cuda.synchronize()
        if not torch.equal(got, ref):
            ok, bad = False, bad + [step]
    rc, code = q.read_status(status)
    torch.save({"ok": ok and rc == q.OK, "bad_steps": bad, "code": code},
               os.path.join(result_dir, f"s{rank}.pt"))
    dist.barrier()
    bufs.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gather_consecutive_steps_with_slow_reader(tmp_path):
    world = 2
    mp.spawn(_worker_steps, args=(world, 29811, 1024, 2048, 1024, str(tmp_path)), nprocs=world,
             join=True)
    for r in range(world):
        res = torch.load(tmp_path / f"s{r}.pt")
        assert res["ok"], res
