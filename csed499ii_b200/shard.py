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

import ctypes
from typing import Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["column_range", "slice_packed", "gather_columns", "mul_2_4_sharded", "ShardedWeight",
           "FusedGather", "mul_2_4_gathered", "check_status"]


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

    @classmethod
    def from_local(cls, B, meta, s, c0: int, c1: int, meta_bits: int = 4):
        """Wrap an already sliced shard (columns ``[c0, c1)`` of the layer)."""
        self = cls.__new__(cls)
        self.B, self.meta, self.s = B, meta, s
        self.k_in = B.size(0) * 32
        self.c0, self.c1 = c0, c1
        self.n_out = None
        self.meta_bits = meta_bits
        self.workspace = torch.zeros((c1 - c0) // 128 * 16, dtype=torch.int32, device=B.device)
        return self

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


class _DevArray:
    """A raw device pointer seen as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr, shape, dtype):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape,
                                         "typestr": dtype, "version": 3, "strides": None}


class FusedGather:
    """Output buffers for the GEMM with the all-gather fused into its epilogue.

    Every rank of ``group`` allocates one device region (CUDA IPC) holding
    three gathered outputs of up to ``max_rows x (world * max_cols)`` fp16
    and, per buffer, an arrival counter and a cumulative target; the regions
    are exported, exchanged with ``all_gather_object`` and mapped into every
    rank.  Calls rotate over the buffers.  All ranks must make the same
    sequence of calls.

    Completion (``pipelined``):

    * ``False``: each call completes on the stream only once this rank's
      buffer holds every rank's block (two buffers in turn suffice: a rank can
      be at most one call ahead).
    * ``True`` (default): no CTA waits for its own peer stores; the next
      call (or :meth:`wait`) releases them once this call's kernel has
      completed, and each call's kernel ends once the PREVIOUS call's
      exchange has completed, so a call's all-gather overlaps the next GEMM.
      A call's output is complete after :meth:`wait` -- call it before
      reading the output, and read it before the next call.  Three buffers
      rotate, because a rank can then be one call further ahead.
    """

    BUFFERS = 3

    def __init__(self, max_rows: int, max_cols: int, group=None, device=None,
                 pipelined: bool = True):
        from . import _ext

        self._lib = _ext.load()
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.max_rows, self.max_cols = max_rows, max_cols
        self.pipelined = pipelined
        nb = self.BUFFERS
        self._c_bytes = (max_rows * self.world * max_cols * 2 + 255) // 256 * 256
        total = nb * self._c_bytes + 256
        base = ctypes.c_void_p()
        self._check(self._lib.sm100_marlin_ipc_alloc(total, self.dev, ctypes.byref(base)))
        self._own = base.value
        self._opened = []
        bases = [self._own]
        if self.world > 1:
            handle = (ctypes.c_char * 64)()
            self._check(self._lib.sm100_marlin_ipc_get_handle(self._own, self.dev, handle))
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for q, h in enumerate(handles):
                if q == self.rank:
                    bases.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                self._check(self._lib.sm100_marlin_ipc_open(h, self.dev, ctypes.byref(peer)))
                self._opened.append(peer.value)
                bases.append(peer.value)
        # region: nb gathered outputs, then per buffer i the arrival counter at
        # +8i and this rank's cumulative target at +128 + 8i (all zero at start)
        tail = nb * self._c_bytes
        self._c = [(ctypes.c_void_p * self.world)(*[b + i * self._c_bytes for b in bases])
                   for i in range(nb)]
        self._flag = [(ctypes.c_void_p * self.world)(*[b + tail + 8 * i for b in bases])
                      for i in range(nb)]
        self._target = [self._own + tail + 128 + 8 * i for i in range(nb)]
        self.next = 0
        self._last = None     # buffer of the last call (pipelined: its completion is pending)
        self._unreleased = None  # buffer of a call whose deferred release is pending

    def _check(self, err):
        from . import _ext

        if err != _ext.OK:
            raise RuntimeError(f"fused all-gather setup failed: {_ext.describe(err)}")

    def _wait_args(self, buf: int):
        """(arrival, target) the launch for ``buf`` waits on before it ends."""
        if not self.pipelined:
            return self._flag[buf][self.rank], self._target[buf]
        if self._last is None:
            return None, None
        return self._flag[self._last][self.rank], self._target[self._last]

    def issue(self, a_ptr, b_ptr, meta_ptr, s_ptr, cols, m, k, workspace_ptr, groupsize,
              stream_ptr, meta_bits):
        """Launch the fused GEMM + all-gather on raw device pointers (the
        operands of :func:`mul_2_4_gathered`) on ``stream_ptr``; returns the
        library status and the buffer written."""
        buf = self.next
        self.next = (self.next + 1) % self.BUFFERS
        wait_arrival, wait_target = self._wait_args(buf)
        release = self._flag[self._unreleased] if self._unreleased is not None else None
        err = self._lib.sm100_marlin_mul_2_4_gather(
            a_ptr, b_ptr, meta_ptr, s_ptr, cols, m, k, workspace_ptr, groupsize, self.dev,
            stream_ptr, meta_bits, self._c[buf], self._flag[buf], self._target[buf], wait_arrival,
            wait_target, release, 1 if self.pipelined else 0, self.world, self.rank)
        if err == 0:
            self._last = buf
            self._unreleased = buf if self.pipelined else None
        return err, buf

    def wait(self, stream_ptr=None) -> None:
        """Make the last call's all-gather complete on the stream (default:
        the current one).  Pipelined mode; a no-op otherwise, where every call
        completes with its own exchange."""
        from . import _ext, _stream_ptr

        if not self.pipelined or self._last is None:
            return
        release = self._flag[self._unreleased] if self._unreleased is not None else None
        err = self._lib.sm100_marlin_gather_wait(
            self._flag[self._last][self.rank], self._target[self._last], release, self.world,
            self.dev, _stream_ptr(self.dev) if stream_ptr is None else stream_ptr)
        if err != _ext.OK:
            raise RuntimeError(f"fused all-gather wait failed: {_ext.describe(err)}")
        self._unreleased = None

    def output(self, buf: int, rows: int, cols: int) -> torch.Tensor:
        """This rank's gathered buffer ``buf`` as an ``(rows, world*cols)`` fp16 tensor."""
        ptr = self._c[buf][self.rank]
        return torch.as_tensor(_DevArray(ptr, (rows, self.world * cols), "<f2"), device=f"cuda:{self.dev}")

    def close(self):
        """Unmap the peers' regions and free this rank's (after a device sync)."""
        torch.cuda.synchronize(self.dev)
        for ptr in self._opened:
            self._lib.sm100_marlin_ipc_close(ptr, self.dev)
        self._opened = []
        if self._own:
            self._lib.sm100_marlin_ipc_free(self._own, self.dev)
            self._own = 0


GATHER_WAIT_TIMEOUT = 8  # SM100_MARLIN_STATUS_GATHER_WAIT_TIMEOUT


def check_status(dev: int) -> None:
    """Raise if a kernel on ``dev`` gave up a bounded wait since the last check.

    Synchronises the device (reads and clears the library's status word).  A
    fused all-gather whose peers did not all arrive in time sets
    ``GATHER_WAIT_TIMEOUT``: its output then lacks some ranks' blocks.
    """
    from . import _ext

    status = _ext.device_status(dev)
    if status & GATHER_WAIT_TIMEOUT:
        raise RuntimeError(f"fused all-gather timed out waiting for other ranks (status {status})")
    if status:
        raise RuntimeError(f"a GEMM kernel gave up a bounded wait (status {status})")


def mul_2_4_gathered(A: torch.Tensor, shard: ShardedWeight, gather: FusedGather,
                     check: bool = False):
    """``A @ W`` for the column-sharded W with the all-gather fused into the
    GEMM: returns this rank's ``(M, world * N/world)`` fp16 result (a view of
    the fused buffer).

    The call is asynchronous.  With a pipelined ``gather`` (the default) the
    result is complete after ``gather.wait()`` and must be read before the
    next call on ``gather``; otherwise it is complete when the call completes
    on the stream and stays valid until the call after next.  A rank whose
    peers do not arrive within the kernel's wait limit gets an incomplete
    result and a device status bit; ``check=True`` waits (pipelined),
    synchronises and raises in that case (otherwise call
    :func:`check_status` at a synchronisation point of your own)."""
    from . import _ext, _groupsize, _stream_ptr

    m, k = A.shape
    cols = shard.c1 - shard.c0
    if m > 64 or m > gather.max_rows or cols > gather.max_cols:
        raise ValueError("fused all-gather: at most 64 (and max_rows) rows, max_cols columns")
    if not (A.is_cuda and A.dtype == torch.half and A.is_contiguous()):
        raise RuntimeError("A must be a contiguous CUDA half tensor")
    dev = A.get_device()
    if dev != gather.dev:
        raise ValueError("A must be on the FusedGather's device")
    err, buf = gather.issue(A.data_ptr(), shard.B.data_ptr(), shard.meta.data_ptr(),
                            shard.s.data_ptr(), cols, m, k, shard.workspace.data_ptr(),
                            _groupsize(k, shard.s), _stream_ptr(dev), shard.meta_bits)
    if err != _ext.OK:
        raise RuntimeError(f"fused sharded GEMM failed: {_ext.describe(err)}")
    if check:
        gather.wait()
        check_status(dev)
    return gather.output(buf, m, cols)
