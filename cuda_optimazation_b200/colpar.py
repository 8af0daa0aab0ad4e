"""Column-parallel (N-sharded) block-scaled GEMM over several GPUs of one box.

The reference is single-GPU; BASELINE config 5 asks for the quant GEMM
C = A . B^T at M = 16384, N = 53248, K = 8192 sharded along N over 1/2/4/8
B200s.  The scheme:

* rank r owns B rows ``shard_range(N, world, r)`` and their scale rows
  (weights are sharded once, at load time);
* A (quantised once) is broadcast from rank 0 with NCCL;
* every rank runs its local GEMM with no communication;
* optionally the bf16 output shards are all-gathered over NVLink and laid out
  as the full M x N matrix: either with NCCL after the GEMM
  (``gather_columns``) or fused into the GEMM, whose epilogue stores every
  output tile into every rank's full C over peer memory
  (``GatherBuffers`` + ``colpar_gemm(..., fused=...)``), so the transfer
  overlaps the math.

Shards are multiples of ``align`` rows (256, the CTA-pair tile) so every rank
runs full tiles; the last rank takes the remainder.  ``local_gemm`` is
injectable so the partition / gather logic can be exercised on CPU ranks.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

ALIGN = 256


def shard_range(n: int, world: int, rank: int, align: int = ALIGN) -> tuple[int, int]:
    """[start, stop) of the B rows (output columns) owned by `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    blocks = (n + align - 1) // align
    per = blocks // world
    extra = blocks % world
    b0 = rank * per + min(rank, extra)
    b1 = b0 + per + (1 if rank < extra else 0)
    return min(n, b0 * align), min(n, b1 * align)


def shard_sizes(n: int, world: int, align: int = ALIGN) -> list[int]:
    return [b - a for a, b in (shard_range(n, world, r, align) for r in range(world))]


def broadcast_operand(tensors, src: int = 0, group=None) -> None:
    """Broadcast the tensors of a quantised operand (values, scales, tensor
    scale) from `src` to every rank, in place."""
    for t in tensors:
        dist.broadcast(t, src, group=group)


def gather_columns(c_local: torch.Tensor, n: int, group=None, align: int = ALIGN,
                   rank_major: bool = False) -> torch.Tensor:
    """All-gather the column shards [M, n_r] of every rank.  Returns the full
    [M, N] matrix (rank-major shards padded to the largest, then placed), or
    with ``rank_major`` the gathered [P, M, max n_r] buffer itself (shard r
    in ``[r, :, :n_r]``), which skips the strided placement copy of the
    whole matrix for consumers that index shards (a row-parallel layer)."""
    world = dist.get_world_size(group)
    sizes = shard_sizes(n, world, align)
    m = c_local.shape[0]
    width = max(sizes)
    if c_local.shape[1] != width:
        pad = torch.zeros(m, width, dtype=c_local.dtype, device=c_local.device)
        pad[:, : c_local.shape[1]] = c_local
        c_local = pad
    buf = torch.empty(world, m, width, dtype=c_local.dtype, device=c_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, c_local.contiguous(), group=group)
    else:  # gloo (CPU ranks) has only the list form
        dist.all_gather(list(buf.unbind(0)), c_local.contiguous(), group=group)
    if rank_major:
        return buf
    out = torch.empty(m, n, dtype=c_local.dtype, device=c_local.device)
    for r in range(world):
        a, b = shard_range(n, world, r, align)
        out[:, a:b] = buf[r, :, : b - a]
    return out


def colpar_gemm(a, b_local, n_total: int, local_gemm: Optional[Callable] = None,
                gather: bool = True, group=None, **gemm_kwargs) -> torch.Tensor:
    """One column-parallel GEMM step: local C shard = A . B_local^T, then
    (optionally) the all-gather to the full matrix.  `local_gemm(a, b, **kw)`
    defaults to the tcgen05 ``block_scaled_gemm``."""
    if local_gemm is None:
        from .qgemm import block_scaled_gemm as local_gemm
    c_local = local_gemm(a, b_local, **gemm_kwargs)
    if not gather or dist.get_world_size(group) == 1:
        return c_local
    return gather_columns(c_local, n_total, group=group)


def shard_rows(op, lo: int, hi: int):
    """Rows [lo, hi) of a quantised NVFP4 operand (values, scales, shared
    tensor scale) as views.  Scales must use the K-major chunk layout
    (LAYOUT_MMA_KMAJOR), where a run of whole 128-row blocks is contiguous;
    lo and hi are multiples of 128."""
    from .qgemm import LAYOUT_MMA_KMAJOR, Nvfp4Result
    if op.layout != LAYOUT_MMA_KMAJOR:
        raise ValueError("row shards need the K-major scale layout")
    if lo % 128 or (hi % 128 and hi != op.rows):
        raise ValueError("shard bounds must be 128-row aligned")
    row_bytes = op.k // 2
    chunk_row = ((op.k // 16 + 3) // 4) * 512  # bytes of one 128-row block's scales
    q = op.quantized[lo * row_bytes: hi * row_bytes]
    sf = op.block_scales[(lo // 128) * chunk_row: ((hi + 127) // 128) * chunk_row]
    return Nvfp4Result(q, sf, op.tensor_scale, hi - lo, op.k, op.layout)


class GatherBuffers:
    """Per-rank full bf16 C [m, n_total] plus the peers' buffers mapped into
    this process with CUDA IPC (handles exchanged over the process group).
    ``ptrs`` lists every rank's buffer in rank order (this rank's own
    included) for ``qgemm.gemm_nvfp4_gather``."""

    def __init__(self, m: int, n_total: int, device, group=None):
        from . import qgemm as q
        self.q = q
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > q.MAX_RANKS:
            raise ValueError("at most 8 ranks")
        self.c = torch.empty(m, n_total, dtype=torch.bfloat16, device=device)
        handles = [None] * self.world
        dist.all_gather_object(handles, q.ipc_export(self.c), group=group)
        self.ptrs = []
        self._mapped = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.c.data_ptr())
            else:
                p = q.ipc_import(h)
                self._mapped.append(p)
                self.ptrs.append(p)
        dist.barrier(group=group)

    def close(self):
        for p in self._mapped:
            self.q.ipc_close(p)
        self._mapped = []


def colpar_gemm_fused(a, b_local, n_total: int, bufs: "GatherBuffers", group=None,
                      status=None) -> torch.Tensor:
    """Column-parallel GEMM with the all-gather fused into the epilogue:
    this rank's columns go straight into every rank's ``bufs.c``.  Returns
    this rank's full C once every rank's kernel has finished (device
    synchronise + barrier).

    ``bufs.c`` is shared with the peers, whose kernels write into it, so the
    returned tensor stays valid only until this rank calls again.  The call
    therefore starts with a device synchronise (this rank's readers of the
    previous result, on any stream, are done) and a barrier (so are every
    other rank's) before any kernel writes the next result."""
    torch.cuda.synchronize()
    dist.barrier(group=group)
    lo, _ = shard_range(n_total, dist.get_world_size(group), dist.get_rank(group))
    bufs.q.gemm_nvfp4_gather(a, b_local, bufs.ptrs, lo, n_total, status=status)
    torch.cuda.synchronize()
    dist.barrier(group=group)
    return bufs.c
