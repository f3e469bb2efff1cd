"""A bounded wait that runs out, without faulting or hanging the GPU.

Every wait in the library's kernels gives up after a fixed limit (0.5 s of
%globaltimer), records a bit in the device status word and lets the kernel
return.  Here one process issues the fused all-gather GEMM declaring a world
of two ranks whose second rank never exists: rank 0 stores its block into
both "ranks'" buffers (two buffers of this GPU) and counts it on both arrival
counters, then waits on its own counter for the second rank's block, which
never comes.  The wait must expire with SM100_MARLIN_STATUS_GATHER_WAIT_TIMEOUT,
the host check must raise, the buffer's cumulative arrival target must still
move by this call's blocks, and the GPU must go on computing correct results.
"""
import ctypes

import pytest
import torch

from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_gather_wait_expires_and_gpu_keeps_working():
    import csed499ii_b200 as m
    from csed499ii_b200 import _ext, shard

    lib = _ext.load()
    assert m.device_status(0) == 0
    N, K, M = 4096, 4096, 16
    W, B_np, s_np, meta_np = random_packed_problem(N, K, 128, seed=41)
    A = torch.from_numpy(activations(M, K, seed=42)).to(DEV)
    B = torch.from_numpy(B_np).to(DEV)
    meta = torch.from_numpy(meta_np).to(DEV)
    s = torch.from_numpy(s_np).to(DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    world = 2
    bufs = [torch.zeros((M, world * N), dtype=torch.half, device=DEV) for _ in range(world)]
    flags = torch.zeros(world, dtype=torch.int64, device=DEV)
    target = torch.zeros(1, dtype=torch.int64, device=DEV)
    c_ptrs = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    f_ptrs = (ctypes.c_void_p * world)(*[flags.data_ptr() + 8 * q for q in range(world)])
    stream = torch.cuda.current_stream(0).cuda_stream
    # per-call completion: the launch waits on its own buffer's counter
    rc = lib.sm100_marlin_mul_2_4_gather(A.data_ptr(), B.data_ptr(), meta.data_ptr(), s.data_ptr(),
                                         N, M, K, ws.data_ptr(), 64, 0, stream, 4, c_ptrs, f_ptrs,
                                         target.data_ptr(), flags.data_ptr(), target.data_ptr(),
                                         None, 0, world, 0)
    assert rc == 0, _ext.describe(rc)
    with pytest.raises(RuntimeError, match="fused all-gather timed out"):
        shard.check_status(0)  # synchronises: the kernel returned after its wait expired
    # rank 0's blocks arrived on both counters; the target moved by the
    # call's blocks (both ranks') although only half of them came
    own = int(flags[0].item())
    assert own > 0 and int(flags[1].item()) == own
    assert int(target.item()) == world * own
    # this rank's block of its own buffer is complete and correct
    oracle = A.float() @ torch.from_numpy(W).to(DEV).float()
    rel_mae, rel_fro, _ = errors(bufs[0][:, :N], oracle)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL
    # the status word was cleared by the check, and the GPU keeps computing
    C = torch.zeros((M, N), dtype=torch.half, device=DEV)
    m.mul_2_4(A, B, meta, C, s, ws)
    torch.cuda.synchronize()
    rel_mae, rel_fro, _ = errors(C, oracle)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL
    assert m.device_status(0) == 0


def test_pipelined_gather_wait_expires():
    """The pipelined completion point (sm100_marlin_gather_wait) on a buffer
    whose second rank never stores: the one-thread wait kernel must expire
    with the gather status bit, and the device keeps working."""
    from csed499ii_b200 import _ext, shard

    lib = _ext.load()
    flags = torch.zeros(2, dtype=torch.int64, device=DEV)
    target = torch.full((1,), 5, dtype=torch.int64, device=DEV)
    flags[0] = 3  # three of five blocks arrived
    stream = torch.cuda.current_stream(0).cuda_stream
    assert lib.sm100_marlin_gather_wait(flags.data_ptr(), target.data_ptr(), None, 0, 0, stream) == 0
    with pytest.raises(RuntimeError, match="fused all-gather timed out"):
        shard.check_status(0)
    flags[0] = 4  # four arrived; the release adds this rank's fifth before the wait
    rel = (ctypes.c_void_p * 2)(flags.data_ptr(), flags.data_ptr() + 8)
    assert lib.sm100_marlin_gather_wait(flags.data_ptr(), target.data_ptr(), rel, 2, 0, stream) == 0
    torch.cuda.synchronize()
    assert _ext.device_status(0) == 0
    assert int(flags[0].item()) == 5 and int(flags[1].item()) == 1
    assert lib.sm100_marlin_gather_wait(None, target.data_ptr(), None, 0, 0, stream) == _ext.ERR_ARGUMENT
