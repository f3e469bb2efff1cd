"""Generate the golden packer / GEMM fixtures from the reference's own code.

Run once in a container where the reference checkout is importable::

    python tests/golden/make_golden.py /path/to/CSED499II

It imports the reference's Python packers
(``kernel_experiments/sparse_marlin/src/marlin/__init__.py`` and
``_semi_structured_conversions.py``) on the CPU -- stubbing only the CUDA
extension module and the ``.cuda()`` / ``device=`` placements that the
reference hard-codes -- and replays the data flow of
``kernel_experiments/sparse_marlin/src/test_2_4.py:22-70`` (gen_quant4_NT) to
produce, per case:

* ``w``         fp16 (K, N)  the random weight before quantisation
* ``s_raw``     fp16 (K/g, N) per-group scales (absmax * 2/15)
* ``B``         int32 (K/32, 2N) packed by ``Layer_2_4.pack(trans=True)``
* ``meta``      int16 (N, K/16) reordered 2:4 metadata
* ``s``         fp16 scales in the kernel's permuted layout
* ``A``         fp16 (16, K) activations
* ``C_ref``     fp32 (16, K) x (K, N): ``A.float() @ uncompress.float()``

The fixtures are small ``.npz`` files committed next to this script; the
tests never import the reference.
"""
import os
import sys
import types

import numpy as np

CASES = [
    # (N out-features, K in-features, groupsize, seed)
    (256, 256, -1, 0),
    (256, 512, 128, 1),
    (512, 256, 128, 2),
    (768, 192, -1, 3),
    (256, 1024, -1, 4),
    (256, 1024, 128, 5),
]
M_ROWS = 16


def _import_reference(root):
    import torch

    sys.modules["marlin_cuda"] = types.ModuleType("marlin_cuda")
    torch.Tensor.cuda = lambda self, *a, **k: self
    zeros = torch.zeros

    def zeros_cpu(*a, **k):
        k.pop("device", None)
        return zeros(*a, **k)

    torch.zeros = zeros_cpu
    sys.path.insert(0, os.path.join(root, "kernel_experiments/sparse_marlin/src"))
    import marlin
    from marlin._semi_structured_conversions import mask_creator

    return torch, marlin, mask_creator


def reference_case(torch, marlin, mask_creator, N, K, groupsize, seed):
    """gen_quant4_NT(m=N, k=K, groupsize) on the CPU (test_2_4.py:22-70)."""
    import torch.nn as nn

    torch.manual_seed(seed)
    maxq = 15
    w = torch.randn((N, K), dtype=torch.half)
    w_kn = w.t().contiguous().clone()
    w = w.t()
    if groupsize != -1:
        w = w.reshape((-1, groupsize, N)).permute(1, 0, 2).reshape((groupsize, -1))
    s = torch.max(torch.abs(w), 0, keepdim=True)[0]
    s *= 2 / maxq
    q = torch.round(w / s).int()
    q += (maxq + 1) // 2
    q = torch.clamp(q, 0, maxq)
    ref = (q - (maxq + 1) // 2).half() * s
    if groupsize != -1:
        def reshape(t):
            return t.reshape((groupsize, -1, N)).permute(1, 0, 2).reshape((K, N)).contiguous()

        ref = reshape(ref)
        q = reshape(q)
    mask = mask_creator(q.T).bool()
    uncompress = (mask * ref.T).T
    s = s.reshape((-1, N)).contiguous()
    linear = nn.Linear(K, N)
    linear.weight.data = ref
    layer = marlin.Layer_2_4(256, 256, groupsize=groupsize)
    g = K if groupsize == -1 else groupsize
    layer.k, layer.n, layer.groupsize = K, N, g
    layer.B = torch.empty((K // 2 // 16, N * 16 // 8), dtype=torch.int)
    layer.meta = torch.empty((N, K // 16), dtype=torch.int16)
    layer.s = torch.empty((K // 2 // (g // 2), N), dtype=torch.half)
    layer.pack(linear, s, True)
    A = torch.randn((M_ROWS, K), dtype=torch.half)
    C_ref = A.float() @ uncompress.float()
    return dict(
        w=w_kn.numpy(), s_raw=s.numpy(), B=layer.B.numpy(), meta=layer.meta.numpy(),
        s=layer.s.numpy(), A=A.numpy(), C_ref=C_ref.numpy(),
        N=np.int64(N), K=np.int64(K), groupsize=np.int64(groupsize), seed=np.int64(seed),
    )


def main(root):
    torch, marlin, mask_creator = _import_reference(root)
    here = os.path.dirname(os.path.abspath(__file__))
    for N, K, g, seed in CASES:
        case = reference_case(torch, marlin, mask_creator, N, K, g, seed)
        name = f"pack_n{N}_k{K}_g{g}.npz"
        np.savez_compressed(os.path.join(here, name), **case)
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CSED499II_ROOT", ""))
