"""Column-parallel (N-shard) execution of the 2:4 W4A16 GEMM across GPUs.

The reference has no distributed code; this is the multi-GPU layer of the
B200 build.  Output columns of ``C = A @ W`` are independent, so rank ``r``
of ``g`` owns columns ``[r*N/g, (r+1)*N/g)``: it holds only that slice of the
packed weights, computes its ``(M, N/g)`` block of C with the single-GPU
kernel, and one all-gather assembles C on every rank (the only exchange).

The packed tensors are *sliced*, never re-packed.  All three permutations of
the Sparse-Marlin format act inside 64-column chunks: ``B`` words of chunk
``c`` are columns ``[128c, 128c+128)`` of every ``(K/32, 2N)`` row
(``__init__.py:242-268`` of the reference), the 2:4 metadata reorder stays
inside 64-row groups and the 2x2 swap inside row pairs
(``_semi_structured_conversions.py:21-48``), so the int16 metadata storage
viewed as ``(K/32, N, 2)`` is sliced along its middle axis, and the scale
permutation acts inside 8-column groups.  Shard boundaries must therefore be
multiples of 64 columns (every BASELINE config-3 shard is a multiple of 256).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["column_range", "slice_packed", "gather_columns", "mul_2_4_sharded", "ShardedWeight"]


def column_range(n_out: int, rank: int, world: int) -> Tuple[int, int]:
    """Columns ``[c0, c1)`` owned by ``rank``; shards are equal multiples of 64."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if n_out % (64 * world):
        raise ValueError(f"N={n_out} does not split into {world} shards of whole 64-column chunks")
    w = n_out // world
    return rank * w, (rank + 1) * w


def slice_packed(B: torch.Tensor, meta: torch.Tensor, s: torch.Tensor, c0: int, c1: int):
    """Packed ``(B, meta, s)`` of output columns ``[c0, c1)`` (contiguous copies).

    ``B`` int32 ``(K/32, 2N)``, ``meta`` int16 ``(N, K/16)`` (or int32 3-bit
    metadata of ``N*K*3/128`` words), ``s`` fp16 ``(K/g, N)`` or ``(1, N)``.
    """
    if c0 % 64 or c1 % 64 or not 0 <= c0 < c1:
        raise ValueError("shard columns must be whole 64-column chunks")
    kk = B.size(0)
    n_out = B.size(1) // 2
    if c1 > n_out:
        raise ValueError(f"columns [{c0}, {c1}) exceed N={n_out}")
    B_r = B[:, 2 * c0:2 * c1].contiguous()
    if meta.dtype == torch.int16:
        meta_r = meta.reshape(kk, n_out, 2)[:, c0:c1, :].contiguous().view(c1 - c0, 2 * kk)
    else:
        # 3-bit metadata: each 64-word group of int32 metadata (64 output
        # columns of one 32-K row) is stored as 48 words, in the same order.
        meta_r = meta.reshape(kk, n_out // 64, 48)[:, c0 // 64:c1 // 64, :].contiguous().view(-1)
    s_r = s[:, c0:c1].contiguous()
    return B_r, meta_r, s_r


def gather_columns(C_local: torch.Tensor, group=None, out: Optional[torch.Tensor] = None):
    """All-gather equal column blocks ``(M, N/g)`` into ``(M, N)`` on every rank."""
    world = dist.get_world_size(group)
    m, w = C_local.shape
    C_local = C_local.contiguous()
    if dist.get_backend(group) == "nccl":
        stacked = torch.empty((world, m, w), dtype=C_local.dtype, device=C_local.device)
        dist.all_gather_into_tensor(stacked, C_local, group=group)
    else:
        parts = [torch.empty_like(C_local) for _ in range(world)]
        dist.all_gather(parts, C_local, group=group)
        stacked = torch.stack(parts)
    if out is None:
        out = torch.empty((m, world * w), dtype=C_local.dtype, device=C_local.device)
    # (g, M, N/g) -> (M, g, N/g); a plain copy (the identity at M == 1)
    out.view(m, world, w).copy_(stacked.permute(1, 0, 2))
    return out


class ShardedWeight:
    """This rank's slice of one packed 2:4 layer, ready for :func:`mul_2_4_sharded`."""

    def __init__(self, B, meta, s, rank: int, world: int, meta_bits: int = 4):
        n_out = B.size(1) // 2
        self.n_out = n_out
        self.k_in = B.size(0) * 32
        self.c0, self.c1 = column_range(n_out, rank, world)
        self.B, self.meta, self.s = slice_packed(B, meta, s, self.c0, self.c1)
        self.meta_bits = meta_bits
        self.workspace = torch.zeros((self.c1 - self.c0) // 128 * 16, dtype=torch.int32,
                                     device=B.device)


def mul_2_4_sharded(A: torch.Tensor, shard: ShardedWeight, C: torch.Tensor, group=None,
                    C_local: Optional[torch.Tensor] = None):
    """``C[M, N] = A @ W`` with W column-sharded over ``group``: local GEMM on
    this rank's slice, then an all-gather of the column blocks into ``C``."""
    from . import _mul

    if C_local is None:
        C_local = torch.empty((A.size(0), shard.c1 - shard.c0), dtype=torch.half, device=A.device)
    _mul(A, shard.B, shard.meta, C_local, shard.s, shard.workspace, -1, -1, -1, 16,
         shard.meta_bits)
    return gather_columns(C_local, group=group, out=C)
