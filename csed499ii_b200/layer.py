"""``Layer_2_4`` / ``replace_linear``: the torch module surface of the 2:4 path.

Mirrors ``Layer_2_4`` and ``replace_linear`` of the reference package
(hyeonu453/CSED499II ``kernel_experiments/sparse_marlin/src/marlin/__init__.py:274-415``):
same constructor arguments and checks, the same buffers (``B``, ``meta``,
``s``; ``workspace`` non-persistent) so ``state_dict`` files carry the same
tensors, ``forward`` through :func:`csed499ii_b200.mul_2_4`, and ``pack``
producing bit-identical operands -- on the GPU (``sm100_marlin_pack_2_4``)
instead of the reference's CPU loop.

Differences a caller may notice:

* the reference allocates ``B`` as ``(K/16, 2N)`` and ``s`` as
  ``(K/groupsize, N)`` in ``__init__`` but ``pack`` produces ``(K/32, 2N)``
  (its own tests replace the buffers before packing); here the buffers have
  the packed shapes from the start;
* ``pack`` keeps ``k``/``groupsize`` in uncompressed units (the reference
  halves them in place);
* only ``trans=True`` is accepted: ``trans=False`` selects the dense Marlin
  permutation, a layout the 2:4 kernel does not read.

Extension (off by default, so the defaults match the reference): ``bias=True``
adds a ``bias`` buffer (fp16, one per output feature, filled by ``pack`` from
``linear.bias``) and ``activation`` names an activation; both are fused into
the GEMM's store (:func:`csed499ii_b200.mul_2_4_epilogue`).
``replace_linear(..., keep_bias=True)`` keeps each ``nn.Linear``'s bias.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ACTIVATIONS, _ext, mul_2_4, mul_2_4_epilogue

__all__ = ["Layer_2_4", "replace_linear"]


class Layer_2_4(nn.Module):
    """2:4-sparse INT4 (symmetric, grouped) linear layer; without bias unless
    ``bias=True`` (an extension: bias and ``activation`` fused into the store)."""

    def __init__(self, infeatures, outfeatures, groupsize=-1, bias=False, activation="none"):
        super().__init__()
        if activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}")
        if groupsize not in [-1, 128]:
            raise ValueError("Only groupsize -1 and 128 are supported.")
        if infeatures % 128 != 0 or outfeatures % 256 != 0:
            raise ValueError("`infeatures` must be divisible by 64 and `outfeatures` by 256.")
        if groupsize == -1:
            groupsize = infeatures
        if infeatures % groupsize != 0:
            raise ValueError("`infeatures` must be divisible by `groupsize`.")
        self.k = infeatures
        self.n = outfeatures
        self.groupsize = groupsize
        self.register_buffer("B", torch.empty((self.k // 32, self.n * 2), dtype=torch.int))
        self.register_buffer("meta", torch.empty((self.n, self.k // 16), dtype=torch.int16))
        self.register_buffer("s", torch.empty((self.k // groupsize, self.n), dtype=torch.half))
        self.register_buffer("workspace", torch.zeros(self.n // 128 * 16, dtype=torch.int32),
                             persistent=False)
        self.activation = activation
        if bias:
            self.register_buffer("bias", torch.zeros(self.n, dtype=torch.half))
        else:
            self.bias = None

    def forward(self, A):
        C = torch.empty(A.shape[:-1] + (self.s.shape[1],), dtype=A.dtype, device=A.device)
        if self.workspace.device != A.device:
            self.workspace = self.workspace.to(A.device)
        A2, C2 = A.view((-1, A.shape[-1])), C.view((-1, C.shape[-1]))
        if self.bias is None and self.activation == "none":
            mul_2_4(A2, self.B, self.meta, C2, self.s, self.workspace)
        else:
            mul_2_4_epilogue(A2, self.B, self.meta, C2, self.s, self.workspace, bias=self.bias,
                             activation=self.activation)
        return C

    def pack(self, linear, scales, trans=True):
        """Pack a fake-quantised layer into the 2:4 representation (on the GPU).

        @linear: module whose ``weight.data`` is the fp16 weight as (infeatures,
                 outfeatures), as the reference's tests pass it with trans=True
        @scales: fp16 quantisation scales, ``(infeatures/groupsize, outfeatures)``
                 (or ``(1, outfeatures)`` for one scale per column)
        """
        if not trans:
            raise NotImplementedError(
                "only trans=True is supported: trans=False selects the dense Marlin permutation, "
                "which the 2:4 kernel does not read")
        w = linear.weight.data
        if w.dtype != torch.half:
            raise ValueError("Only `torch.half` weights are supported.")
        if tuple(w.shape) != (self.k, self.n):
            raise ValueError(f"weight must be ({self.k}, {self.n}) (in, out) for trans=True")
        dev = self.B.device if self.B.is_cuda else (w.device if w.is_cuda else torch.device("cuda"))
        g = -1 if self.groupsize == self.k else self.groupsize
        w = w.to(dev).contiguous()
        s = scales.to(device=dev, dtype=torch.half).reshape(-1, self.n).contiguous()
        if s.size(0) != self.k // self.groupsize:
            raise ValueError(f"scales must have {self.k // self.groupsize} rows")
        B = torch.empty((self.k // 32, 2 * self.n), dtype=torch.int32, device=dev)
        meta = torch.empty((self.n, self.k // 16), dtype=torch.int16, device=dev)
        s_out = torch.empty_like(s)
        di = dev.index if dev.index is not None else torch.cuda.current_device()
        err = _ext.load().sm100_marlin_pack_2_4(
            w.data_ptr(), s.data_ptr(), self.k, self.n, g, B.data_ptr(), meta.data_ptr(),
            s_out.data_ptr(), di, torch.cuda.current_stream(di).cuda_stream)
        if err != _ext.OK:
            raise RuntimeError(f"pack failed: {_ext.describe(err)}")
        self.B = B.to(self.B.device)
        self.meta = meta.to(self.meta.device)
        self.s = s_out.to(self.s.device)
        if self.bias is not None and getattr(linear, "bias", None) is not None:
            b = linear.bias.data.reshape(-1)
            if b.numel() != self.n:
                raise ValueError(f"bias must have {self.n} elements")
            self.bias = b.to(device=self.bias.device, dtype=torch.half).contiguous()


def replace_linear(module, name_filter=lambda n: True, groupsize=-1, name="", keep_bias=False):
    """Recursively replace every ``torch.nn.Linear`` by an empty ``Layer_2_4``.

    Same traversal as the reference (``__init__.py:391-415``): attributes of
    ``module`` that are ``nn.Linear`` and pass ``name_filter`` (dotted name)
    are replaced, then children are visited.  ``keep_bias=True`` (not in the
    reference, which drops biases) gives layers with a bias buffer where the
    ``nn.Linear`` has one.
    """
    if isinstance(module, Layer_2_4):
        return
    for attr in dir(module):
        tmp = getattr(module, attr)
        name1 = name + "." + attr if name != "" else attr
        if isinstance(tmp, nn.Linear) and name_filter(name1):
            setattr(module, attr, Layer_2_4(tmp.in_features, tmp.out_features, groupsize=groupsize,
                                            bias=keep_bias and tmp.bias is not None))
    for name1, child in module.named_children():
        replace_linear(child, name_filter, groupsize=groupsize,
                       name=name + "." + name1 if name != "" else name1, keep_bias=keep_bias)
