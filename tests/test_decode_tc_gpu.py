"""The tensor-memory decode kernel (batches of up to 64 rows) against the oracle.

``mul_2_4`` routes batches of 17-64 rows (33-64 with 3-bit metadata) with N a
multiple of 128 and K a multiple of 256 to the tcgen05 kernel of
``marlin24_decode_tc.cuh``: clusters of 1, 2 or 4 CTAs split K and reduce
through distributed shared memory.  These tests pin that kernel for every
batch of 1-64 rows with ``sm100_marlin_set_decode_kernel(DECODE_TMEM)``.  The
planner's choice is steered with ``sms``: few SMs give clusters several
128-feature blocks each (two alternating accumulators and exchange buffers),
many SMs give clusters of four on one block.  Every case is checked against
the oracle, rerun for bit-identical output, and compared with the stream-K
kernel (``sm100_marlin_mul_2_4_ex``, which takes the caller's split-K scratch
and so keeps the warp-level kernel), which is checked against the oracle as
well.
"""
import pytest
import torch

from csed499ii_b200 import metadata_decode as md
from problems import (REL_FRO_TOL, REL_MAE_TOL, activations, errors, quantized_problem,
                      random_packed_problem)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture
def tmem_kernel():
    from csed499ii_b200 import _ext

    lib = _ext.load()
    assert lib.sm100_marlin_set_decode_kernel(_ext.DECODE_TMEM) == 0
    yield lib
    assert lib.sm100_marlin_set_decode_kernel(_ext.DECODE_AUTO) == 0


def _run(lib, A, B, meta, s, N, M, K, g, sms, meta_bits, entry="tc"):
    C = torch.full((M, N), float("nan"), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(0).cuda_stream
    args = (A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), N, M, K,
            ws.data_ptr(), g, 0, stream, -1, -1, sms, 16)
    if entry == "tc":
        fn = lib.sm100_marlin_mul_2_4 if meta_bits == 4 else lib.sm100_marlin_mul_2_4_meta3
        rc = fn(*args)
    else:
        scratch = torch.empty(max(lib.sm100_marlin_scratch_bytes(N, M, K, 0, sms), 16),
                              dtype=torch.uint8, device=DEV)
        rc = lib.sm100_marlin_mul_2_4_ex(*args, meta_bits, scratch.data_ptr(), scratch.numel())
    torch.cuda.synchronize()
    assert rc == 0
    assert int(ws.abs().sum().item()) == 0, "workspace must be left zero"
    return C


CASES = [
    # (N, K, M, groupsize, sms)
    (4096, 4096, 16, 128, -1),     # clusters of 4, one block each
    (12288, 4096, 1, 128, -1),     # clusters of 4, three blocks each
    (22016, 4096, 16, 128, -1),    # many blocks per cluster
    (4096, 11008, 7, 128, -1),     # uneven K split across the cluster
    (4096, 4096, 64, 128, -1),
    (4096, 4096, 33, 128, -1),
    (2048, 2048, 48, 128, 8),      # few SMs: several blocks per cluster
    (1024, 1024, 20, 128, 2),      # two SMs
    (1024, 512, 5, 128, 1),        # one CTA, all blocks
    (128, 128, 1, 128, -1),        # one block, one K step
    (384, 256, 9, 128, 3),
    (640, 1024, 16, -1, -1),       # one scale per column
    (1024, 1024, 64, -1, 8),
]


@pytest.mark.parametrize("N,K,M,g,sms", CASES)
@pytest.mark.parametrize("meta_bits", [4, 3])
def test_decode_tc_against_oracle_and_stream_k(N, K, M, g, sms, meta_bits, tmem_kernel):
    from csed499ii_b200 import _ext

    lib = tmem_kernel
    if g == -1:
        W, B, s, meta = quantized_problem(N, K, -1, seed=N + K)
    else:
        W, B, s, meta = random_packed_problem(N, K, 128, seed=N + K + 1)
    A = torch.from_numpy(activations(M, K, seed=M + 3)).to(DEV)
    Bd, sd = torch.from_numpy(B).to(DEV), torch.from_numpy(s).to(DEV)
    md_ = torch.from_numpy(meta).to(DEV)
    mm = md_ if meta_bits == 4 else md.pack(md_)
    gs = 64 if g != -1 else -1
    ref = A.float() @ torch.from_numpy(W).to(DEV).float()
    C = _run(lib, A, Bd, mm, sd, N, M, K, gs, sms, meta_bits)
    assert torch.isfinite(C).all()
    rel_mae, rel_fro, _ = errors(C, ref)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)
    assert torch.equal(_run(lib, A, Bd, mm, sd, N, M, K, gs, sms, meta_bits), C)
    C_sk = _run(lib, A, Bd, mm, sd, N, M, K, gs, sms, meta_bits, entry="stream_k")
    rel_mae, rel_fro, _ = errors(C_sk, ref)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, ("stream-K", rel_mae, rel_fro)
    # the two kernels sum in different orders; both are within fp32 rounding
    rel_mae, rel_fro, _ = errors(C, C_sk.float())
    assert rel_mae < 1e-3 and rel_fro < 1e-3, (rel_mae, rel_fro)
    assert _ext.device_status(0) == 0


def test_decode_tc_pdl_chain(tmem_kernel):
    """Back-to-back dependent calls (each GEMM's input is the previous one's
    output) with programmatic dependent launch, captured in a CUDA graph:
    every result must equal the same chain run with launch overlap off."""
    import csed499ii_b200 as m
    from csed499ii_b200 import _ext

    lib = tmem_kernel
    N = K = 1024
    layers = []
    for i in range(6):
        W, B, s, meta = random_packed_problem(N, K, 128, seed=50 + i)
        # scales x3.5 keep the chain's activations near unit size
        layers.append((torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV),
                       torch.from_numpy(s).to(DEV) * 3.5))
    x0 = torch.from_numpy(activations(16, K, seed=7)).to(DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    outs = [torch.empty((16, N), dtype=torch.half, device=DEV) for _ in layers]

    def chain():
        x = x0
        for (B, meta, s), out in zip(layers, outs):
            m.mul_2_4(x, B, meta, out, s, ws)
            x = out

    results = []
    for overlap in (0, 1):
        lib.sm100_marlin_set_overlap(overlap)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            chain()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                chain()
            for o in outs:
                o.fill_(float("nan"))
            g.replay()
        torch.cuda.synchronize()
        results.append([o.clone() for o in outs])
        del g
    lib.sm100_marlin_set_overlap(1)
    for a, b in zip(*results):
        assert torch.isfinite(a).all() and torch.equal(a, b)
    assert _ext.device_status(0) == 0


def test_decode_kernel_selection_routes_and_agrees():
    """Default routing against both pinned kernels at the rows where the
    choice flips (16/17 rows with 4-bit metadata, 32/33 with 3-bit): auto
    must equal the pinned kernel its rule names, bit for bit."""
    from csed499ii_b200 import _ext

    lib = _ext.load()
    N, K = 1024, 2048
    W, B, s, meta = random_packed_problem(N, K, 128, seed=11)
    Bd, sd, md_ = (torch.from_numpy(x).to(DEV) for x in (B, s, meta))
    assert lib.sm100_marlin_set_decode_kernel(3) == _ext.ERR_ARGUMENT
    try:
        for meta_bits, rows in ((4, 16), (4, 17), (3, 32), (3, 33)):
            mm = md_ if meta_bits == 4 else md.pack(md_)
            A = torch.from_numpy(activations(rows, K, seed=rows)).to(DEV)
            out = {}
            for which in (_ext.DECODE_AUTO, _ext.DECODE_STREAM_K, _ext.DECODE_TMEM):
                assert lib.sm100_marlin_set_decode_kernel(which) == 0
                out[which] = _run(lib, A, Bd, mm, sd, N, rows, K, 64, -1, meta_bits)
            tmem_rule = rows > (32 if meta_bits == 3 else 16)
            expect = _ext.DECODE_TMEM if tmem_rule else _ext.DECODE_STREAM_K
            assert torch.equal(out[_ext.DECODE_AUTO], out[expect]), (meta_bits, rows)
            rel_mae, rel_fro, _ = errors(out[_ext.DECODE_TMEM], out[_ext.DECODE_STREAM_K].float())
            assert rel_mae < 1e-3 and rel_fro < 1e-3, (meta_bits, rows, rel_mae, rel_fro)
    finally:
        lib.sm100_marlin_set_decode_kernel(_ext.DECODE_AUTO)
    assert _ext.device_status(0) == 0
