"""Metadata-cost diagnostics: the GEMM with parts of the metadata path removed.

Mirrors the reference's ``metadata_diagnostics`` extension
(``kernel_experiments/sparse_marlin/kernel_profile/setup.py:14-38``), whose
functions take the operands of ``mul_2_4`` and run a copy of the kernel with
the metadata path cut:

* :func:`no_gmem` -- no metadata copy from global memory; the kernel's
  shared-memory metadata is the constant 0xEEEE from its start;
* :func:`no_reg`  -- the metadata is copied as usual, but the constant is used
  in place of the shared-memory (decode kernel) or tensor-memory-bound
  (prefill kernel) load;
* :func:`no_all`  -- both.

Results are only meaningful when every metadata nibble is 0xE (int16 -4370,
the reference's ``get_problem_24`` metadata); then they equal ``mul_2_4`` bit
for bit (``kernel_profile/run.py:62-70``) as long as ``mul_2_4`` runs the same
kernel: the diagnostics are instances of the warp-level decode kernel and the
CTA-pair kernel, so for 17-64 rows, which ``mul_2_4`` sends to the
tensor-memory decode kernel by default, compare against a call made after
``sm100_marlin_set_decode_kernel(DECODE_STREAM_K)``.  Group-128 scales only.
"""
from __future__ import annotations

import torch

from . import _ext, _groupsize, _stream_ptr

__all__ = ["no_gmem", "no_reg", "no_all", "VARIANTS", "UNIFORM_META"]

VARIANTS = {"no_gmem": 1, "no_reg": 2, "no_all": 3}
UNIFORM_META = -4370  # int16 0xEEEE: every group of four keeps positions 2 and 3


def _run(variant: int, a, b, meta, c, s, workspace):
    lib = _ext.load()
    for name, t, dt in (("a", a, torch.half), ("b", b, torch.int32), ("meta", meta, torch.int16),
                        ("c", c, torch.half), ("s", s, torch.half), ("workspace", workspace, torch.int32)):
        if not t.is_cuda or t.dtype != dt or not t.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous CUDA {dt} tensor")
    k, n, batch = a.size(1), c.size(1), a.size(0)
    dev = a.get_device()
    group = _groupsize(k, s)
    if group == -1:
        raise RuntimeError("metadata diagnostics need group-128 scales")
    err = lib.sm100_marlin_mul_2_4_meta_diag(a.data_ptr(), b.data_ptr(), meta.data_ptr(),
                                             c.data_ptr(), s.data_ptr(), n, batch, k,
                                             workspace.data_ptr(), group, dev, _stream_ptr(dev),
                                             variant)
    if err != _ext.OK:
        raise RuntimeError(f"diagnostic kernel error {err}: {_ext.describe(err)}")


def no_gmem(a, b, meta, c, s, workspace):
    _run(1, a, b, meta, c, s, workspace)


def no_reg(a, b, meta, c, s, workspace):
    _run(2, a, b, meta, c, s, workspace)


def no_all(a, b, meta, c, s, workspace):
    _run(3, a, b, meta, c, s, workspace)
