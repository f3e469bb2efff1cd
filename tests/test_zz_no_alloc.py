"""The allocation-free GEMM entry point (sm100_marlin_mul_2_4_noalloc).

Some callers cannot allocate device memory when they call the GEMM: code
inside CUDA graph capture, serving runtimes and plugins whose host framework
owns every device allocation, real-time loops that forbid allocation after
start-up.  For them the library keeps its split-K scratch (the fp32 partial
sums that CTAs sharing an output tile hand to each other) in a fixed static
device buffer.  This test calls that entry point through the C ABI on layer
shapes whose plan splits K across CTAs -- so the partials really go through
the static buffer -- two different shapes back to back and each twice in a
row, and checks every result against the regular entry point's with the
tolerances of the other GEMM tests, and that free device memory does not
change.  The file sorts last so that a run that stops at the first failure
has already run every other test.
"""
import pytest
import torch

from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

# Llama-2-7B gate+up and Llama-2-70B qkv projections: at 1 and 16 batch rows
# the plan splits K across CTAs through the scratch (stream-K: more column
# tiles than CTAs, and too many for a cluster per tile).
SPLIT_K_CASES = [(22016, 4096, 1), (10240, 8192, 16), (22016, 4096, 16), (10240, 8192, 1)]


def _call(fn, A, B, meta, C, s, ws, N, M, K):
    stream = torch.cuda.current_stream(0).cuda_stream
    return fn(A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), N, M, K,
              ws.data_ptr(), 64, 0, stream, -1, -1, -1, 16)


def test_noalloc_matches_regular_entry_point_on_two_calls():
    from csed499ii_b200 import _ext

    lib = _ext.load()
    cases = []
    for (N, K, M) in SPLIT_K_CASES:
        assert lib.sm100_marlin_scratch_bytes(N, M, K, 0, -1) > 0, "case must split K"
        W, B_np, s_np, meta_np = random_packed_problem(N, K, 128, seed=31)
        A = torch.from_numpy(activations(M, K, seed=32)).to(DEV)
        B = torch.from_numpy(B_np).to(DEV)
        meta = torch.from_numpy(meta_np).to(DEV)
        s = torch.from_numpy(s_np).to(DEV)
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
        C_ref = torch.zeros((M, N), dtype=torch.half, device=DEV)
        assert _call(lib.sm100_marlin_mul_2_4, A, B, meta, C_ref, s, ws, N, M, K) == 0
        cases.append((N, K, M, W, A, B, meta, s, ws, C_ref))
    torch.cuda.synchronize()

    # everything the calls below touch exists already: no allocation may
    # happen from here on (the checks, which allocate torch temporaries, run
    # after the second measurement)
    outs = [[torch.full((M, N), float("nan"), dtype=torch.half, device=DEV)
             for (N, K, M, *_) in cases] for _ in range(2)]
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(0)
    for call in range(2):
        for (N, K, M, W, A, B, meta, s, ws, C_ref), C in zip(cases, outs[call]):
            rc = _call(lib.sm100_marlin_mul_2_4_noalloc, A, B, meta, C, s, ws, N, M, K)
            assert rc == 0, _ext.describe(rc)
            torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(0)
    assert free_after == free_before, "the allocation-free entry point allocated device memory"
    for call in range(2):
        for (N, K, M, W, A, B, meta, s, ws, C_ref), C in zip(cases, outs[call]):
            assert torch.isfinite(C).all(), (call, N, K, M)
            rel_mae, rel_fro, _ = errors(C, C_ref)
            assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (call, N, K, M, rel_mae, rel_fro)
            assert int(ws.abs().sum().item()) == 0, "workspace must be left zero"
    assert all(torch.equal(a, b) for a, b in zip(*outs)), "the two calls must agree bit for bit"

    # the result also matches the oracle weight
    for (N, K, M, W, A, *_), C in zip(cases, outs[1]):
        oracle = A.float() @ torch.from_numpy(W).to(DEV).float()
        rel_mae, rel_fro, _ = errors(C, oracle)
        assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (N, K, M, rel_mae, rel_fro)
    assert _ext.device_status(0) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    from csed499ii_b200 import _ext

    lib = _ext.load()
    # 64 batch rows on a very wide layer (Llama-2-70B gate+up) need more than
    # the static 8 MiB of scratch
    N, K, M = 57344, 1024, 64
    A = torch.zeros((M, K), dtype=torch.half, device=DEV)
    C = torch.zeros((M, N), dtype=torch.half, device=DEV)
    B = torch.zeros((K // 32, 2 * N), dtype=torch.int32, device=DEV)
    meta = torch.zeros((N, K // 16), dtype=torch.int16, device=DEV)
    s = torch.zeros((K // 128, N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    needed = lib.sm100_marlin_scratch_bytes(N, M, K, 0, -1)
    if needed <= (8 << 20):
        pytest.skip("this device needs no more than the static scratch for the case")
    rc = _call(lib.sm100_marlin_mul_2_4_noalloc, A, B, meta, C, s, ws, N, M, K)
    assert rc == 6
    assert b"static buffer" in lib.sm100_marlin_last_cuda_error()
