"""Cluster split-K of the warp-level decode kernel (batches of up to 16 rows).

When the column tiles times 2 or 3 fill the SMs, ``mul_2_4`` launches one
thread-block cluster per tile: the tile's CTAs split K, and the non-zero
ranks store their fp32 partials into the finisher's shared memory with
``st.async`` instead of going through the split-K scratch and the
workspace counters.  These cases take that plan on 148 SMs (clusters of 2
with 64- and 128-column tiles on Llama shapes, clusters of 3 with 64-column
tiles); each is checked against the oracle, for bit-identical reruns, for
an untouched workspace, and for needing no scratch.
"""
import pytest
import torch

from csed499ii_b200 import metadata_decode as md
from problems import (REL_FRO_TOL, REL_MAE_TOL, activations, errors, quantized_problem,
                      random_packed_problem)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

CASES = [
    # (N, K): cluster size and tile width the plan picks on 148 SMs
    (4096, 4096),    # 2, 64 columns
    (4096, 11008),   # 2, 64 columns, 8-row units
    (8192, 8192),    # 2, 128 columns
    (3072, 4096),    # 3, 64 columns
]


@pytest.mark.parametrize("N,K", CASES)
@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("meta_bits", [4, 3])
def test_cluster_split_against_oracle(N, K, M, meta_bits):
    from csed499ii_b200 import _ext

    lib = _ext.load()
    assert lib.sm100_marlin_scratch_bytes(N, M, K, 0, -1) == 0, "plan must be cluster split-K"
    W, B, s, meta = random_packed_problem(N, K, 128, seed=N + K + M)
    A = torch.from_numpy(activations(M, K, seed=M)).to(DEV)
    Bd, sd, md_ = (torch.from_numpy(x).to(DEV) for x in (B, s, meta))
    mm = md_ if meta_bits == 4 else md.pack(md_)
    fn = lib.sm100_marlin_mul_2_4 if meta_bits == 4 else lib.sm100_marlin_mul_2_4_meta3
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(0).cuda_stream
    outs = []
    for _ in range(2):
        C = torch.full((M, N), float("nan"), dtype=torch.half, device=DEV)
        rc = fn(A.data_ptr(), Bd.data_ptr(), mm.data_ptr(), C.data_ptr(), sd.data_ptr(), N, M, K,
                ws.data_ptr(), 64, 0, stream, -1, -1, -1, 16)
        assert rc == 0, _ext.describe(rc)
        outs.append(C)
    torch.cuda.synchronize()
    ref = A.float() @ torch.from_numpy(W).to(DEV).float()
    rel_mae, rel_fro, _ = errors(outs[0], ref)
    assert torch.isfinite(outs[0]).all()
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)
    assert torch.equal(outs[0], outs[1]), "cluster split-K must be deterministic"
    assert int(ws.abs().sum().item()) == 0, "the workspace counters are not used"
    assert _ext.device_status(0) == 0


def test_cluster_split_per_column_scales_and_epilogue():
    """One scale per column (applied by the finisher) and the fused bias +
    SiLU epilogue on a cluster plan."""
    import csed499ii_b200 as m

    N, K, M = 4096, 4096, 16
    W, B, s, meta = quantized_problem(N, K, -1, seed=77)
    A = torch.from_numpy(activations(M, K, seed=78)).to(DEV)
    Bd, sd, md_ = (torch.from_numpy(x).to(DEV) for x in (B, s, meta))
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    bias = torch.randn(N, dtype=torch.half, device=DEV, generator=torch.Generator(DEV).manual_seed(5))
    C = torch.empty((M, N), dtype=torch.half, device=DEV)
    m.mul_2_4(A, Bd, md_, C, sd, ws)
    C_epi = torch.empty((M, N), dtype=torch.half, device=DEV)
    m.mul_2_4_epilogue(A, Bd, md_, C_epi, sd, ws, bias=bias, activation="silu")
    torch.cuda.synchronize()
    ref = A.float() @ torch.from_numpy(W).to(DEV).float()
    rel_mae, rel_fro, _ = errors(C, ref)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)
    ref_epi = torch.nn.functional.silu(ref + bias.float())
    rel_mae, rel_fro, _ = errors(C_epi, ref_epi)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)
    assert m.device_status(0) == 0
