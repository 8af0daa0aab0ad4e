"""Column-parallel partition / broadcast / gather logic on 2 gloo CPU ranks,
checked against the single-process oracle GEMM."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def test_shard_ranges_cover_and_align():
    from cuda_optimazation_b200.colpar import shard_range, shard_sizes
    for n in (256, 1000, 53248, 28672 + 17):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
            for a, b in ranges:
                assert (a % 256 == 0 or a == n) and (b % 256 == 0 or b == n)
            assert sum(shard_sizes(n, world)) == n
    assert shard_range(53248, 8, 3) == (3 * 6656, 4 * 6656)


def _worker(rank, world, port, result_path):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle as om
    from cuda_optimazation_b200 import colpar
    o = om.Oracle()
    m, n, k = 24, 700, 128
    # A: quantised on rank 0 only, broadcast; other ranks start from zeros.
    if rank == 0:
        qa, sa, ta = o.nvfp4_mma(o.normal(m * k, 1).reshape(m, k), 0)
    else:
        qa = np.zeros(m * k // 2, np.uint8)
        sa = np.zeros(o.L.qgo_scale_storage_size(m, k, 16), np.uint8)
        ta = 0.0
    ta_t = torch.tensor([ta], dtype=torch.float32)
    qa_t, sa_t = torch.from_numpy(qa.copy()), torch.from_numpy(sa.copy())
    colpar.broadcast_operand([qa_t, sa_t, ta_t])
    # B: every rank quantises the full seeded B and keeps its shard (as a
    # checkpoint loader would), oracle GEMM stands in for the local GEMM.
    xb = o.normal(n * k, 2).reshape(n, k)
    lo, hi = colpar.shard_range(n, world, rank)
    qb, sb, tb = o.nvfp4_mma(xb, 0)
    bv, bsf = o.nvfp4_decode(qb, sb, n, k)

    def local_gemm(a, b):
        av, asf = o.nvfp4_decode(a[0].numpy(), a[1].numpy(), m, k)
        vb, sfb = b
        d = o.gemm(av, vb, asf, sfb, m, hi - lo, k, 16, threads=1)
        return torch.from_numpy(d * np.float32(np.float32(a[2].item()) * np.float32(tb)))

    b_local = (np.ascontiguousarray(bv.reshape(n, k)[lo:hi]).ravel(),
               np.ascontiguousarray(bsf.reshape(n, k // 16)[lo:hi]).ravel())
    c = colpar.colpar_gemm((qa_t, sa_t, ta_t), b_local, n, local_gemm=local_gemm)
    # The rank-major form of the same gather: shard r in [r, :, :n_r].
    c_local = local_gemm((qa_t, sa_t, ta_t), b_local)
    rm = colpar.gather_columns(c_local, n, rank_major=True)
    assert rm.shape == (world, m, max(colpar.shard_sizes(n, world)))
    for r in range(world):
        a, b = colpar.shard_range(n, world, r)
        assert torch.equal(rm[r, :, : b - a], c[:, a:b])
    if rank == 0:
        np.save(result_path, c.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_colpar_two_gloo_ranks_match_oracle(tmp_path, oracle):
    world, port = 2, 29613
    out = tmp_path / "c.npy"
    mp.spawn(_worker, args=(world, port, str(out)), nprocs=world, join=True)
    got = np.load(out)
    m, n, k = 24, 700, 128
    qa, sa, ta = oracle.nvfp4_mma(oracle.normal(m * k, 1).reshape(m, k), 0)
    qb, sb, tb = oracle.nvfp4_mma(oracle.normal(n * k, 2).reshape(n, k), 0)
    av, asf = oracle.nvfp4_decode(qa, sa, m, k)
    bv, bsf = oracle.nvfp4_decode(qb, sb, n, k)
    ref = oracle.gemm(av, bv, asf, bsf, m, n, k, 16) * np.float32(np.float32(ta) * np.float32(tb))
    assert got.shape == (m, n)
    # The shards run the same O2 per output element: bit equality.
    assert np.array_equal(got, ref)


def test_shard_rows_kmajor_views():
    """Row shards of a K-major NVFP4 operand are contiguous views of the
    values and of whole 128-row scale blocks (checked on CPU tensors)."""
    from cuda_optimazation_b200 import colpar
    from cuda_optimazation_b200.qgemm import LAYOUT_MMA, LAYOUT_MMA_KMAJOR, Nvfp4Result
    rows, k = 768, 512
    sf_blocks = (k // 16 + 3) // 4
    q = torch.arange(rows * k // 2, dtype=torch.int64).to(torch.uint8)
    sf = torch.arange((rows // 128) * sf_blocks * 512, dtype=torch.int64).to(torch.uint8)
    op = Nvfp4Result(q, sf, torch.ones(1), rows, k, LAYOUT_MMA_KMAJOR)
    sh = colpar.shard_rows(op, 256, 512)
    assert sh.rows == 256 and sh.k == k
    assert torch.equal(sh.quantized, q[256 * k // 2: 512 * k // 2])
    assert torch.equal(sh.block_scales, sf[2 * sf_blocks * 512: 4 * sf_blocks * 512])
    with pytest.raises(ValueError):
        colpar.shard_rows(op, 100, 512)
    with pytest.raises(ValueError):
        colpar.shard_rows(Nvfp4Result(q, sf, torch.ones(1), rows, k, LAYOUT_MMA), 0, 256)
