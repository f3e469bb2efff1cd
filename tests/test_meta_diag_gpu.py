"""Metadata-cost diagnostics (BASELINE config 4's ablation).

The reference builds copies of its kernel with the metadata path cut --
``no_gmem`` (no global-memory copy, constant metadata in shared memory),
``no_reg`` (constant register instead of the shared-memory load) and
``no_all`` -- and requires each to equal the baseline bit for bit on inputs
whose metadata is the uniform pattern 0xEEEE
(``kernel_experiments/sparse_marlin/kernel_profile/run.py:44-70``: random
packed INT4 weights, scales 0.01, metadata -4370).  The same check here, on
the decode kernel (1-16 rows and the 32-row tile), the CTA-pair route for
33-64 rows and the CTA-pair prefill kernel.  The diagnostics are instances
of those kernels, so the baseline call pins them
(``sm100_marlin_set_decode_kernel(DECODE_STREAM_K)``; by default 17-64 rows
run on the tensor-memory decode kernel, whose sums come in another order).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _uniform_problem(M, N, K, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    A = torch.randn((M, K), dtype=torch.half, device=DEV, generator=g)
    B = torch.randint(-(2**31), 2**31 - 1, (K // 32, 2 * N), dtype=torch.int32, device=DEV, generator=g)
    s = torch.full((K // 128, N), 0.01, dtype=torch.half, device=DEV)
    meta = torch.full((N, K // 16), -4370, dtype=torch.int16, device=DEV)
    return A, B, meta, s


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 4096, 4096), (32, 4096, 4096),
                                   (1, 1024, 1024), (48, 4096, 4096), (64, 12288, 4096),
                                   (512, 4096, 4096), (200, 2048, 1024)])
def test_diagnostics_equal_baseline_on_uniform_metadata(M, N, K):
    import csed499ii_b200 as m
    from csed499ii_b200 import _ext
    from csed499ii_b200 import metadata_diagnostics as diag

    A, B, meta, s = _uniform_problem(M, N, K, seed=M + N)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    C0 = torch.empty((M, N), dtype=torch.half, device=DEV)
    lib = _ext.load()
    assert lib.sm100_marlin_set_decode_kernel(_ext.DECODE_STREAM_K) == 0
    try:
        m.mul_2_4(A, B, meta, C0, s, ws)
        torch.cuda.synchronize()
    finally:
        lib.sm100_marlin_set_decode_kernel(_ext.DECODE_AUTO)
    assert torch.isfinite(C0).all()
    for name in ("no_gmem", "no_reg", "no_all"):
        C = torch.full((M, N), float("nan"), dtype=torch.half, device=DEV)
        getattr(diag, name)(A, B, meta, C, s, ws)
        torch.cuda.synchronize()
        assert torch.equal(C, C0), name
    assert int(ws.abs().sum().item()) == 0
    assert m.device_status(0) == 0


def test_diagnostics_argument_checks():
    from csed499ii_b200 import _ext

    lib = _ext.load()
    A, B, meta, s = _uniform_problem(16, 1024, 1024, seed=3)
    C = torch.empty((16, 1024), dtype=torch.half, device=DEV)
    ws = torch.zeros(1024 // 128 * 16, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(0).cuda_stream
    args = (A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), 1024, 16, 1024,
            ws.data_ptr())
    assert lib.sm100_marlin_mul_2_4_meta_diag(*args, 64, 0, stream, 0) == _ext.ERR_ARGUMENT
    assert lib.sm100_marlin_mul_2_4_meta_diag(*args, 64, 0, stream, 4) == _ext.ERR_ARGUMENT
    assert lib.sm100_marlin_mul_2_4_meta_diag(*args, -1, 0, stream, 1) == _ext.ERR_ARGUMENT
