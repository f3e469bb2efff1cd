"""GPU parity of the sm_100a 2:4 W4A16 GEMM against the CPU oracle.

Cases follow the reference's own test matrix
(``kernel_experiments/sparse_marlin/src/test_2_4.py:91-135``), extended to
batch sizes where the reference kernel itself fails (48..256) and checked for
run-to-run determinism.
"""
import os

import numpy as np
import pytest
import torch

import marlin24_oracle as O
from conftest import GOLDEN, golden_cases
from problems import (REL_FRO_TOL, REL_MAE_TOL, activations, chunk_columns, errors,
                      oracle_columns, packed_problem_gpu, quantized_problem, random_packed_problem,
                      sample_chunks)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _setup():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    import csed499ii_b200 as m

    assert m.device_status(0) == 0


def run(A, B, meta, s, N, thread_k=-1, thread_m=-1, sms=-1, max_par=16):
    import csed499ii_b200 as m

    A_d = torch.from_numpy(A).to(DEV)
    C = torch.zeros((A.shape[0], N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * max_par, dtype=torch.int32, device=DEV)
    m.mul_2_4(A_d, torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV), C,
              torch.from_numpy(s).to(DEV), ws, thread_k, thread_m, sms, max_par)
    torch.cuda.synchronize()
    assert int(ws.abs().sum().item()) == 0, "workspace must be left zero"
    return C


def oracle_c(A, W):
    return torch.from_numpy(A).to(DEV).float() @ torch.from_numpy(W).to(DEV).float()


def check(C, C_ref):
    rel_mae, rel_fro, _ = errors(C, C_ref)
    assert torch.isfinite(C).all()
    assert rel_mae < REL_MAE_TOL, rel_mae
    assert rel_fro <= REL_FRO_TOL, rel_fro


@pytest.mark.parametrize("name", golden_cases())
def test_golden_fixtures(name):
    z = np.load(os.path.join(GOLDEN, name))
    N, K = int(z["N"]), int(z["K"])
    # K not a multiple of 128 needs the reference's 64x256 tile (test_2_4.py:108-111)
    tk, tm = (64, 256) if K % 128 else (-1, -1)
    for rows in (1, 5, 16):
        A = np.ascontiguousarray(z["A"][:rows])
        C = run(A, z["B"], z["meta"], z["s"], N, tk, tm)
        check(C, torch.from_numpy(z["C_ref"][:rows]).to(DEV))


def test_correctness():
    # test_2_4.py:91-93
    for (N, M, K, tk, tm, g) in [(256, 16, 256, 128, 128, -1), (21504, 16, 4096, 64, 256, 128)]:
        W, B, s, meta = quantized_problem(N, K, g, seed=0)
        A = activations(M, K)
        check(run(A, B, meta, s, N, tk, tm), oracle_c(A, W))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7, 8, 9, 12, 16, 24, 32, 48, 64, 65, 96, 128, 192, 256])
@pytest.mark.parametrize("g", [-1, 128])
def test_batch_sweep(M, g):
    # test_2_4.py:95-101 (tiles) plus the batches where the reference fails
    N, K = 512, 1024
    W, B, s, meta = quantized_problem(N, K, g, seed=2)
    A = activations(M, K, seed=M)
    check(run(A, B, meta, s, N), oracle_c(A, W))


@pytest.mark.parametrize("tk,tm", [(64, 256), (128, 128)])
@pytest.mark.parametrize("M", [1, 8, 16])
def test_explicit_tiles(tk, tm, M):
    N, K = 512, 1024
    W, B, s, meta = quantized_problem(N, K, -1, seed=3)
    A = activations(M, K)
    check(run(A, B, meta, s, N, tk, tm), oracle_c(A, W))


@pytest.mark.parametrize("K", [704, 768, 832])
def test_k_stages_divisibility(K):
    # test_2_4.py:103-106
    W, B, s, meta = quantized_problem(512, K, -1, seed=4)
    A = activations(16, K)
    check(run(A, B, meta, s, 512, 64, 256), oracle_c(A, W))


@pytest.mark.parametrize("K", [64, 128, 192])
def test_very_few_stages(K):
    # test_2_4.py:108-111
    W, B, s, meta = quantized_problem(768, K, -1, seed=5)
    A = activations(16, K)
    check(run(A, B, meta, s, 768, 64, 256), oracle_c(A, W))


@pytest.mark.parametrize("N,K", [(256, 512), (256, 1024), (256 * 128, 1024)])
@pytest.mark.parametrize("tk,tm", [(128, 128), (64, 256)])
def test_groups(N, K, tk, tm):
    # test_2_4.py:129-135
    W, B, s, meta = quantized_problem(N, K, 128, seed=6)
    A = activations(16, K)
    check(run(A, B, meta, s, N, tk, tm), oracle_c(A, W))


@pytest.mark.parametrize("N", [128, 384, 640])
def test_column_tile_widths(N):
    # N % 256 != 0 exercises the 128- and 64-column tile variants
    K = 512
    W, B, s, meta = quantized_problem(N, K, 128, seed=7)
    A = activations(16, K)
    check(run(A, B, meta, s, N), oracle_c(A, W))


@pytest.mark.parametrize("sms", [1, 3, 20, 77, 148, 300])
def test_grid_sizes(sms):
    W, B, s, meta = quantized_problem(1024, 2048, 128, seed=8)
    A = activations(16, 2048)
    check(run(A, B, meta, s, 1024, sms=sms), oracle_c(A, W))


@pytest.mark.parametrize("M", [16, 48, 64, 128])
def test_deterministic_repeats(M):
    # The reference kernel is nondeterministic at M >= 48
    # (kernel_profile/SMOKE_K4096.md:7-23); this one must not be.
    N, K = 4096, 4096
    W, B, s, meta = random_packed_problem(N, K, 128, seed=9)
    A = activations(M, K)
    outs = [run(A, B, meta, s, N) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    check(outs[0], oracle_c(A, W))


LLAMA7B = [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]


# every Llama-2-7B decode layer shape at every batch of the
# config (M = 1 ... 128 covers the decode kernel at 1-4 row blocks, the
# CTA-pair route for 33-64 rows and the prefill kernel above 64), each
# against the oracle and bit-identical over three runs.
@pytest.mark.parametrize("K,N", LLAMA7B)
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 32, 64, 128])
def test_llama7b_shapes(K, N, M):
    W, B, s, meta = random_packed_problem(N, K, 128, seed=10)
    A = activations(M, K)
    outs = [run(A, B, meta, s, N) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    check(outs[0], oracle_c(A, W))


LLAMA70B = [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]


def _check_sampled(C, A, B, meta, s, K, N, seed):
    """C against the oracle on a sample of 64-column chunks (first, last and
    random ones) and finite everywhere."""
    assert torch.isfinite(C).all()
    chunks = sample_chunks(N, 8, seed)
    W = torch.from_numpy(oracle_columns(B, meta, s, K, chunks)).to(DEV).float()
    cols = torch.from_numpy(chunk_columns(chunks)).to(DEV)
    check(C[:, cols], A.float() @ W)


def _run_dev(A, B, meta, s, N, sms=-1):
    import csed499ii_b200 as m

    C = torch.zeros((A.shape[0], N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    m.mul_2_4(A, B, meta, C, s, ws, -1, -1, sms, 16)
    torch.cuda.synchronize()
    assert int(ws.abs().sum().item()) == 0, "workspace must be left zero"
    return C


# BASELINE config 3 on one GPU: the Llama-2-70B layer shapes (W ~ N(0, 0.01)
# scale magnitudes) at M = 1, 16, 128.  Whole-matrix numpy dequantisation of
# these layers is too large for a test, so the oracle checks a sample of
# column chunks; the whole output is checked for determinism.
@pytest.mark.parametrize("K,N", LLAMA70B)
@pytest.mark.parametrize("M", [1, 16, 128])
def test_llama70b_shapes(K, N, M):
    B, meta, s = packed_problem_gpu(N, K, seed=K + N, sigma=0.01)
    A = torch.from_numpy(activations(M, K, seed=M)).to(DEV)
    outs = [_run_dev(A, B, meta, s, N) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    _check_sampled(outs[0], A, B, meta, s, K, N, seed=M)


# BASELINE config 3 column-sharded g = 2 / 4 / 8 ways, the shards run one
# after another on one GPU (tests/test_shard_gpu.py covers the exchange):
# each shard's block must match the unsharded GEMM (both are checked against
# the oracle on sampled chunks).
@pytest.mark.parametrize("K,N", LLAMA70B)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_llama70b_sharded_on_one_gpu(K, N, world):
    from csed499ii_b200 import shard

    B, meta, s = packed_problem_gpu(N, K, seed=K + N, sigma=0.01)
    for M in (1, 16, 128):
        A = torch.from_numpy(activations(M, K, seed=M)).to(DEV)
        full = _run_dev(A, B, meta, s, N)
        C = torch.empty((M, N), dtype=torch.half, device=DEV)
        for r in range(world):
            w = shard.ShardedWeight(B, meta, s, r, world)
            C[:, w.c0:w.c1] = _run_dev(A, w.B, w.meta, w.s, w.c1 - w.c0)
        torch.cuda.synchronize()
        rel_mae, rel_fro, _ = errors(C, full)
        assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (M, rel_mae, rel_fro)
        _check_sampled(C, A, B, meta, s, K, N, seed=world + M)


def test_reference_error_messages():
    import csed499ii_b200 as m

    A = torch.zeros((32, 256), dtype=torch.half, device=DEV)
    C = torch.zeros((32, 384), dtype=torch.half, device=DEV)
    B = torch.zeros((8, 768), dtype=torch.int32, device=DEV)
    meta = torch.zeros((384, 16), dtype=torch.int16, device=DEV)
    s = torch.zeros((1, 384), dtype=torch.half, device=DEV)
    ws = torch.zeros(48, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match=r"Problem \(m=384, n=32, k=256\) not compatible"):
        m.mul_2_4(A, B, meta, C, s, ws)
    with pytest.raises(RuntimeError, match="No kernel implementation for thread_k=128"):
        m.mul_2_4(A, B, meta, C[:, :256].contiguous(), s[:, :256].contiguous(), ws, 128, 128)


# Batches above 64 rows run on the tensor-memory (tcgen05) kernel in one
# launch: BASELINE config-4 shapes at the small end of its batch range,
# ragged batch tiles, both scale modes, and K not a multiple of 128.
@pytest.mark.parametrize("K,N,M", [(4096, 4096, 512), (4096, 11008, 512), (4096, 4096, 2048),
                                   (1024, 512, 300), (2048, 768, 1000), (4096, 4096, 257)])
def test_prefill_shapes(K, N, M):
    W, B, s, meta = random_packed_problem(N, K, 128, seed=K + M)
    A = activations(M, K, seed=M)
    check(run(A, B, meta, s, N), oracle_c(A, W))


# BASELINE config 4 headline shapes: M = 2048 and 8192 at K = N = 8192, and
# M = 8192 at (4096, 4096) and (4096, 11008), against the whole-matrix oracle.
@pytest.mark.parametrize("K,N,M", [(8192, 8192, 2048), (8192, 8192, 8192), (4096, 4096, 8192),
                                   (4096, 11008, 8192)])
def test_prefill_headline_shapes(K, N, M):
    W, B, s, meta = random_packed_problem(N, K, 128, seed=K + N)
    A = activations(M, K, seed=M)
    check(run(A, B, meta, s, N), oracle_c(A, W))


@pytest.mark.parametrize("K", [512, 704])
def test_prefill_per_column_scales(K):
    W, B, s, meta = quantized_problem(512, K, -1, seed=9)
    A = activations(160, K, seed=10)
    check(run(A, B, meta, s, 512, 64, 256), oracle_c(A, W))


# 256-row tiles on CTA pairs (tcgen05.mma.sp.cta_group::2, N % 256 == 0): a
# small `sms` makes the launcher choose the 256-row tile; ragged batches put
# the odd CTA's rows partly or wholly past M; both scale modes.
@pytest.mark.parametrize("K,N,M,g", [(512, 1024, 300, 128), (1024, 2048, 129, 128),
                                     (1024, 1536, 257, -1), (2048, 512, 640, 128),
                                     (4096, 4096, 1000, 128)])
def test_prefill_pair(K, N, M, g):
    if g == -1:
        W, B, s, meta = quantized_problem(N, K, -1, seed=K + N)
    else:
        W, B, s, meta = random_packed_problem(N, K, 128, seed=K + N + M)
    A = activations(M, K, seed=M + 1)
    check(run(A, B, meta, s, N, sms=8), oracle_c(A, W))


def test_prefill_pair_deterministic():
    W, B, s, meta = random_packed_problem(2048, 1024, 128, seed=14)
    A = activations(384, 1024, seed=15)
    C0 = run(A, B, meta, s, 2048, sms=8)
    for _ in range(3):
        assert torch.equal(run(A, B, meta, s, 2048, sms=8), C0)


def test_prefill_deterministic():
    W, B, s, meta = random_packed_problem(1024, 2048, 128, seed=12)
    A = activations(384, 2048, seed=13)
    C0 = run(A, B, meta, s, 1024)
    for _ in range(3):
        assert torch.equal(run(A, B, meta, s, 1024), C0)
