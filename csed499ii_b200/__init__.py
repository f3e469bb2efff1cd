"""B200 (sm_100a) drop-in for the Sparse-Marlin 2:4 sparse W4A16 operator.

Python surface mirrors the reference's ``marlin`` package
(hyeonu453/CSED499II ``kernel_experiments/sparse_marlin/src/marlin``):

* :func:`mul_2_4` -- same positional arguments, tensor contract and error
  messages as ``marlin.mul_2_4`` / ``marlin_cuda.mul_2_4``
  (``__init__.py:45-58``, ``marlin_cuda.cpp:66-94``);
* :mod:`csed499ii_b200.metadata_decode` -- the 3-bit metadata codec and the
  3-bit GEMM (``metadata_decode`` extension: ``pack``, ``unpack``, ``fetch``,
  ``matmul``);
* :class:`Layer_2_4` / :func:`replace_linear` -- the torch module surface
  (``__init__.py:274-415``), packing on the GPU;
* :mod:`csed499ii_b200.shard` -- column-parallel execution across GPUs.

All compute runs in the in-tree CUDA library through its C ABI
(``include/sm100_marlin.h``); nothing here computes on the CPU.
"""
from __future__ import annotations

import torch

from . import _ext

__all__ = ["mul_2_4", "mul_2_4_epilogue", "ACTIVATIONS", "scratch_bytes", "device_status",
           "Layer_2_4", "replace_linear"]

# fused-epilogue activations (SM100_MARLIN_ACT_* of the C header)
ACTIVATIONS = {"none": 0, "relu": 1, "silu": 2, "gelu_tanh": 3}


def _stream_ptr(dev: int) -> int:
    return torch._C._cuda_getCurrentRawStream(dev)


def _check_cuda(name: str, t: torch.Tensor, dtype: torch.dtype, dev: int) -> None:
    if not t.is_cuda or t.get_device() != dev:
        raise RuntimeError(f"{name} must be a CUDA tensor on device {dev}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must have dtype {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _groupsize(prob_k: int, s: torch.Tensor) -> int:
    """Compressed group size as derived by ``marlin_cuda.cpp:74-77``."""
    groupsize = -1 if s.size(0) == 1 else prob_k // 2 // s.size(0)
    if groupsize != -1 and groupsize * s.size(0) != prob_k // 2:
        raise RuntimeError(f"k={prob_k} not compatible with {s.size(0)} groups.")
    return groupsize


def _raise_for(err: int, prob_m, prob_n, prob_k, thread_k, thread_m, groupsize) -> None:
    if err == _ext.OK:
        return
    if err == _ext.ERR_PROB_SHAPE:
        raise RuntimeError(
            f"Problem (m={prob_m}, n={prob_n}, k={prob_k}) not compatible with "
            f"thread_k={thread_k}, thread_m={thread_m}."
        )
    if err == _ext.ERR_KERN_SHAPE:
        raise RuntimeError(
            f"No kernel implementation for thread_k={thread_k}, thread_m={thread_m}, "
            f"groupsize={groupsize}."
        )
    raise RuntimeError(f"sm100_marlin error {err}: {_ext.describe(err)}")


_HALF, _INT32, _INT16 = torch.half, torch.int32, torch.int16


def _mul(A, B, meta, C, s, workspace, thread_k, thread_m, sms, max_par, meta_bits, bias=None,
         act=0):
    lib = _ext._lib or _ext.load()
    prob_n, prob_k = A.shape  # batch rows, input features
    prob_m = C.shape[1]       # output features
    groupsize = _groupsize(prob_k, s)
    if workspace.numel() < prob_m // 128 * max_par:
        raise RuntimeError(f"workspace must be of size at least {prob_m // 128 * max_par}.")
    dev = A.get_device()
    if dev < 0:
        raise RuntimeError("A must be a CUDA tensor")
    meta_dtype = _INT16 if meta_bits == 4 else _INT32
    # one combined test on the hot path; the per-tensor checks (with their
    # messages) only run when it fails
    if not (A.dtype is _HALF and C.dtype is _HALF and s.dtype is _HALF and B.dtype is _INT32
            and meta.dtype is meta_dtype and workspace.dtype is _INT32
            and B.get_device() == dev and meta.get_device() == dev and C.get_device() == dev
            and s.get_device() == dev and workspace.get_device() == dev
            and A.is_contiguous() and B.is_contiguous() and meta.is_contiguous()
            and C.is_contiguous() and s.is_contiguous() and workspace.is_contiguous()):
        _check_cuda("A", A, _HALF, dev)
        _check_cuda("B", B, _INT32, dev)
        _check_cuda("meta", meta, meta_dtype, dev)
        _check_cuda("C", C, _HALF, dev)
        _check_cuda("s", s, _HALF, dev)
        _check_cuda("workspace", workspace, _INT32, dev)
    fc = _ext._fast if _ext._fast_tried else _ext.fast()
    if bias is not None:
        _check_cuda("bias", bias, _HALF, dev)
        if bias.numel() != prob_m:
            raise RuntimeError(f"bias must have {prob_m} elements (one per output column)")
    if fc is not None:
        err = fc.mul(A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), prob_m,
                     prob_n, prob_k, workspace.data_ptr(), groupsize, dev, _stream_ptr(dev), thread_k,
                     thread_m, sms, max_par, meta_bits, bias.data_ptr() if bias is not None else 0,
                     act)
    elif bias is None and act == 0:
        fn = lib.sm100_marlin_mul_2_4 if meta_bits == 4 else lib.sm100_marlin_mul_2_4_meta3
        err = fn(A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), prob_m,
                 prob_n, prob_k, workspace.data_ptr(), groupsize, dev, _stream_ptr(dev), thread_k,
                 thread_m, sms, max_par)
    else:
        err = lib.sm100_marlin_mul_2_4_epilogue(
            A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), prob_m,
            prob_n, prob_k, workspace.data_ptr(), groupsize, dev, _stream_ptr(dev), thread_k,
            thread_m, sms, max_par, meta_bits, bias.data_ptr() if bias is not None else None, act)
    if err:
        _raise_for(err, prob_m, prob_n, prob_k, thread_k, thread_m, groupsize)


def mul_2_4(A, B, meta, C, s, workspace, thread_k=-1, thread_m=-1, sms=-1, max_par=16):
    """FP16 x (INT4 + 2:4 sparsity) multiply into ``C`` (in place).

    @A: ``torch.half`` activations ``(n, k)`` row-major (n = batch rows)
    @B: ``torch.int`` packed weights ``(k/32, 2m)`` in Sparse-Marlin format
    @meta: ``torch.int16`` 2:4 metadata ``(m, k/16)``
    @C: ``torch.half`` output ``(n, m)`` row-major, written in place
    @s: ``torch.half`` scales ``(k/128, m)`` or ``(1, m)``
    @workspace: ``torch.int`` with at least ``m / 128 * max_par`` zero entries
    @thread_k, @thread_m: -1 or a reference tile shape (shape checks only)
    @sms: persistent CTAs (-1 = all SMs)
    @max_par: as in the reference; only sizes the workspace requirement
    """
    _mul(A, B, meta, C, s, workspace, thread_k, thread_m, sms, max_par, 4)


def mul_2_4_epilogue(A, B, meta, C, s, workspace, bias=None, activation="none", thread_k=-1,
                     thread_m=-1, sms=-1, max_par=16, meta_bits=4):
    """``mul_2_4`` with a fused epilogue: ``C = act(A @ W + bias)``.

    Not in the reference (its ``Layer_2_4`` is "without bias" and callers
    apply bias and activation as separate ops); computed in fp32 and rounded
    once to fp16 in the GEMM's store.
    @bias: ``torch.half`` ``(m,)`` per output column, or None
    @activation: one of ``ACTIVATIONS`` ("none", "relu", "silu", "gelu_tanh")
    @meta_bits: 4 (int16 metadata) or 3 (``metadata_decode.pack`` output)
    Other arguments as ``mul_2_4``.
    """
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}")
    if meta_bits not in (3, 4):
        raise ValueError("meta_bits must be 3 or 4")
    _mul(A, B, meta, C, s, workspace, thread_k, thread_m, sms, max_par, meta_bits, bias,
         ACTIVATIONS[activation])


def scratch_bytes(prob_m: int, prob_n: int, prob_k: int, dev: int = 0, sms: int = -1) -> int:
    """Split-K scratch bytes the library keeps per (device, stream) for a call."""
    return int(_ext.load().sm100_marlin_scratch_bytes(prob_m, prob_n, prob_k, dev, sms))


def device_status(dev: int = 0) -> int:
    """Read and clear the device status word (nonzero = a bounded wait gave up)."""
    return _ext.device_status(dev)


from .layer import Layer_2_4, replace_linear  # noqa: E402  (needs mul_2_4 above)
