"""The reference's own GEMM kernel, built for sm_100a, as a second checker and speed bar.

``oracle/_ref/libref_marlin24.so`` is the reference launcher and kernel
(``kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu``)
compiled from its source by ``oracle/build_ref.py``.  These tests

* pin the oracle's reading of the packed format to the reference kernel's:
  the reference kernel's output must match ``A @ dequant_2_4(B, meta, s)``
  at batch sizes where the reference is known to be correct (<= 16 rows,
  ``SMOKE_K4096.md`` of the reference);
* check this library's output against the reference kernel's on the same
  inputs;
* time both kernels on the Llama-2-7B decode shapes on the same GPU, with the
  same eager launches and weights rotated through more than the L2 size.

They skip when the reference build is absent (it needs the reference source
tree at build time).
"""
import ctypes
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT, golden_cases
from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_marlin24.so")
LLAMA7B = [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]  # (K, N)


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference kernel not built (oracle/build_ref.py needs the reference tree)")
    lib = ctypes.CDLL(REF_LIB)
    fn = lib.ref_marlin_cuda_2_4
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int,
                                                                 ctypes.c_int, ctypes.c_void_p] + \
        [ctypes.c_int] * 4
    torch.backends.cuda.matmul.allow_tf32 = False
    return fn


def _args(A, B, meta, C, s, ws, N, K, groupsize, stream, tk=-1, tm=-1, sms=-1):
    gs = -1 if groupsize == -1 else groupsize // 2
    return (A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), N,
            A.shape[0], K, ws.data_ptr(), gs, 0, stream, tk, tm, sms, 16)


def _both(ref, A_np, B_np, meta_np, s_np, N, K, groupsize):
    from csed499ii_b200 import _ext

    lib = _ext.load()
    A, B = torch.from_numpy(A_np).to(DEV), torch.from_numpy(B_np).to(DEV)
    meta, s = torch.from_numpy(meta_np).to(DEV), torch.from_numpy(s_np).to(DEV)
    stream = torch.cuda.current_stream(0).cuda_stream
    out = []
    for fn in (ref, lib.sm100_marlin_mul_2_4):
        C = torch.zeros((A.shape[0], N), dtype=torch.half, device=DEV)
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
        assert fn(*_args(A, B, meta, C, s, ws, N, K, groupsize, stream)) == 0
        torch.cuda.synchronize()
        assert int(ws.abs().sum().item()) == 0
        out.append(C)
    return A, out[0], out[1]


def _check(C, C_ref):
    rel_mae, rel_fro, _ = errors(C, C_ref)
    assert torch.isfinite(C).all()
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)


@pytest.mark.parametrize("M", [1, 16])
@pytest.mark.parametrize("name", [n for n in golden_cases() if "k192" not in n])
def test_reference_kernel_agrees_with_oracle_on_golden(ref, name, M):
    # C_ref = A @ uncompress, written by the reference's own packing flow
    z = np.load(os.path.join(GOLDEN, name))
    N, K, g = int(z["N"]), int(z["K"]), int(z["groupsize"])
    A_np = np.ascontiguousarray(z["A"][:M])
    A, C_ref_kernel, C_ours = _both(ref, A_np, z["B"], z["meta"], z["s"], N, K, g)
    oracle = torch.from_numpy(z["C_ref"][:M]).to(DEV)
    _check(C_ours, oracle)
    _check(C_ref_kernel, oracle)
    _check(C_ours, C_ref_kernel.float())


@pytest.mark.parametrize("K,N", LLAMA7B)
def test_reference_kernel_agrees_with_oracle_on_llama_shapes(ref, K, N):
    W, B, s, meta = random_packed_problem(N, K, 128, seed=K + N)
    A_np = activations(16, K, seed=5)
    A, C_ref_kernel, C_ours = _both(ref, A_np, B, meta, s, N, K, 128)
    oracle = A.float() @ torch.from_numpy(W).to(DEV).float()
    _check(C_ours, oracle)
    _check(C_ref_kernel, oracle)


def test_speed_against_reference_kernel(ref):
    """Both kernels, eager launches on one stream, weights rotated past L2."""
    from csed499ii_b200 import _ext

    lib = _ext.load()
    M, reps = 16, 40
    gen = torch.Generator(device=DEV)
    gen.manual_seed(7)
    stream = torch.cuda.current_stream(0).cuda_stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    result = {}
    for K, N in LLAMA7B:
        per_copy = K * N // 4 + K * N // 8 + 2 * N * K // 128
        copies = max(2, -(-4 * 126 * 2**20 // per_copy))
        B = torch.randint(-2**31, 2**31 - 1, (copies, K // 32, 2 * N), dtype=torch.int32,
                          device=DEV, generator=gen)
        meta = torch.full((copies, N, K // 16), 0x4E4E, dtype=torch.int16, device=DEV)
        s = (torch.rand((copies, K // 128, N), device=DEV, generator=gen) * 0.003).half()
        A = torch.randn((M, K), dtype=torch.half, device=DEV, generator=gen)
        C = torch.empty((M, N), dtype=torch.half, device=DEV)
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
        row = {}
        for name, fn in (("reference_us", ref), ("ours_us", lib.sm100_marlin_mul_2_4)):
            def call(i):
                c = i % copies
                rc = fn(*_args(A, B[c], meta[c], C, s[c], ws, N, K, 128, stream))
                assert rc == 0
            for i in range(5):
                call(i)
            torch.cuda.synchronize()
            ev0.record()
            for i in range(reps):
                call(i)
            ev1.record()
            torch.cuda.synchronize()
            row[name] = round(ev0.elapsed_time(ev1) * 1e3 / reps, 2)
        byts = per_copy + 2 * M * K + 2 * M * N
        row["reference_GB/s"] = round(byts / row["reference_us"] / 1e3, 1)
        row["ours_GB/s"] = round(byts / row["ours_us"] / 1e3, 1)
        row["speedup"] = round(row["reference_us"] / row["ours_us"], 2)
        result[f"{K}x{N}"] = row
        del B, meta, s
    print("\nREFERENCE_KERNEL_TIMING " + json.dumps(result))
    for row in result.values():
        assert row["ours_us"] < row["reference_us"]
