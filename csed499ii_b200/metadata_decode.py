"""3-bit 2:4 metadata: codec and GEMM.

Mirrors the reference extension module ``metadata_decode``
(hyeonu453/CSED499II ``kernel_experiments/sparse_marlin/metadata_decode``):

* :func:`pack` / :func:`unpack` -- ``codec.cu:30-41`` (same checks and
  messages);
* :func:`fetch` / :func:`matmul` -- the two generated 3-bit GEMM variants
  (``setup.py:77-85``).  The reference's variants differ only in *where*
  the metadata decode sits inside its kernel; this library has one kernel
  whose consumer warps decode right after the shared-memory load, so both
  names run it.
"""
from __future__ import annotations

import torch

from . import _ext
from . import _mul, _stream_ptr

__all__ = ["pack", "unpack", "fetch", "matmul", "decode_words"]


def pack(x: torch.Tensor) -> torch.Tensor:
    """4-bit 2:4 metadata (int16, numel % 128 == 0) -> 3-bit metadata (int32)."""
    if not (x.is_cuda and x.is_contiguous() and x.dtype == torch.int16 and x.numel() % 128 == 0):
        raise RuntimeError("expected CUDA contiguous int16 metadata, multiple of 256 bytes")
    dev = x.get_device()
    y = torch.empty(x.numel() * 3 // 8, dtype=torch.int32, device=x.device)
    errors = torch.zeros(1, dtype=torch.int32, device=x.device)
    err = _ext.load().sm100_marlin_meta3_pack(x.data_ptr(), y.data_ptr(), x.numel(),
                                               errors.data_ptr(), _stream_ptr(dev))
    if err != _ext.OK:
        raise RuntimeError(f"meta3 pack failed: {_ext.describe(err)}")
    if int(errors.item()) != 0:
        raise RuntimeError("metadata contains unsupported 2:4 nibbles")
    return y


def unpack(x: torch.Tensor) -> torch.Tensor:
    """3-bit metadata (int32, numel % 48 == 0) -> 4-bit metadata (int16, flat)."""
    if not (x.is_cuda and x.is_contiguous() and x.dtype == torch.int32 and x.numel() % 48 == 0):
        raise RuntimeError("expected compressed metadata")
    dev = x.get_device()
    y = torch.empty(x.numel() * 8 // 3, dtype=torch.int16, device=x.device)
    err = _ext.load().sm100_marlin_meta3_unpack(x.data_ptr(), y.data_ptr(), x.numel(),
                                                 _stream_ptr(dev))
    if err != _ext.OK:
        raise RuntimeError(f"meta3 unpack failed: {_ext.describe(err)}")
    return y


def _check_meta3(a, b, meta, c, s, w):
    if not (a.is_cuda and a.dtype == torch.float16 and a.is_contiguous()):
        raise RuntimeError("a must be contiguous CUDA half")
    k, n = a.size(1), c.size(1)
    if not (n % 256 == 0 and k % 128 == 0 and meta.dtype == torch.int32 and meta.is_contiguous()
            and meta.numel() == n * k * 3 // 128):
        raise RuntimeError("unsupported compressed metadata shape")


def fetch(a, b, meta, c, s, w) -> None:
    """3-bit-metadata GEMM ``c = a . dequant(b, meta, s)`` (in place)."""
    _check_meta3(a, b, meta, c, s, w)
    _mul(a, b, meta, c, s, w, -1, -1, -1, 16, 3)


def matmul(a, b, meta, c, s, w) -> None:
    """Same operation as :func:`fetch` (see module docstring)."""
    _check_meta3(a, b, meta, c, s, w)
    _mul(a, b, meta, c, s, w, -1, -1, -1, 16, 3)


def decode_words(x: torch.Tensor):
    """Device decoders on raw words: returns (high-table, low-table) decodes
    of bits [0, 24) of every int32 of ``x`` (known-answer testing)."""
    if not (x.is_cuda and x.is_contiguous() and x.dtype == torch.int32):
        raise RuntimeError("expected a contiguous CUDA int32 tensor")
    dev = x.get_device()
    hi = torch.empty_like(x)
    lo = torch.empty_like(x)
    err = _ext.load().sm100_marlin_meta3_decode_words(x.data_ptr(), hi.data_ptr(), lo.data_ptr(),
                                                       x.numel(), _stream_ptr(dev))
    if err != _ext.OK:
        raise RuntimeError(f"meta3 decode failed: {_ext.describe(err)}")
    return hi, lo
