"""Column-parallel sharded GEMM on the GPU.

* One GPU: each rank's slice is multiplied by the sm_100a kernel in turn and
  placed in its column block; the assembled C must match the oracle.
* Two GPUs (skipped with fewer): two NCCL ranks run ``mul_2_4_sharded`` (local
  GEMM + all-gather of C) and both must hold the oracle's C.
* The all-gather fused into the GEMM (``mul_2_4_gathered``), with per-call and
  with pipelined completion (``FusedGather.wait()`` before reading), on one
  rank and on two GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from csed499ii_b200 import shard
from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("N,K,M,world", [(4096, 4096, 16, 2), (4096, 4096, 1, 8), (8192, 1024, 16, 4),
                                         (1536, 2048, 33, 3)])
def test_shards_on_one_gpu(N, K, M, world):
    import csed499ii_b200 as m

    W, B, s, meta = random_packed_problem(N, K, 128, seed=N + world)
    A = torch.from_numpy(activations(M, K, seed=2)).to(DEV)
    Bd, md, sd = torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV), torch.from_numpy(s).to(DEV)
    C = torch.empty((M, N), dtype=torch.half, device=DEV)
    for r in range(world):
        w = shard.ShardedWeight(Bd, md, sd, r, world)
        C_r = torch.empty((M, w.c1 - w.c0), dtype=torch.half, device=DEV)
        m.mul_2_4(A, w.B, w.meta, C_r, w.s, w.workspace)
        C[:, w.c0:w.c1] = C_r
    torch.cuda.synchronize()
    rel_mae, rel_fro, _ = errors(C, A.float() @ torch.from_numpy(W).to(DEV).float())
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        N, K, M = 4096, 4096, 16
        W, B, s, meta = random_packed_problem(N, K, 128, seed=77)
        dev = torch.device("cuda", rank)
        sw = shard.ShardedWeight(torch.from_numpy(B).to(dev), torch.from_numpy(meta).to(dev),
                                 torch.from_numpy(s).to(dev), rank, world)
        A = torch.from_numpy(activations(M, K, seed=9)).to(dev)
        C = torch.empty((M, N), dtype=torch.half, device=dev)
        shard.mul_2_4_sharded(A, sw, C)
        torch.cuda.synchronize(dev)
        rel_mae, rel_fro, _ = errors(C, A.float() @ torch.from_numpy(W).to(dev).float())
        q.put((rank, rel_mae, rel_fro))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_nccl_all_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    for _ in range(world):
        rank, rel_mae, rel_fro = q.get(timeout=5)
        assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rank, rel_mae, rel_fro)


@pytest.mark.parametrize("pipelined", [True, False])
def test_fused_gather_one_rank(pipelined):
    """The fused path with a single rank (its own buffer is the only peer):
    rotating buffers, changing shapes, the device-side arrival accounting."""
    import csed499ii_b200 as m

    gather = shard.FusedGather(64, 4096, device=DEV, pipelined=pipelined)
    try:
        cases = [(4096, 4096, 16), (4096, 2048, 1), (1024, 4096, 64), (4096, 4096, 16),
                 (2048, 1024, 5)]
        for i, (N, K, M) in enumerate(cases):
            W, B, s, meta = random_packed_problem(N, K, 128, seed=100 + i)
            sw = shard.ShardedWeight(torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV),
                                     torch.from_numpy(s).to(DEV), 0, 1)
            A = torch.from_numpy(activations(M, K, seed=i)).to(DEV)
            C = shard.mul_2_4_gathered(A, sw, gather)
            gather.wait()
            torch.cuda.synchronize()
            assert C.shape == (M, N)
            rel_mae, rel_fro, _ = errors(C, A.float() @ torch.from_numpy(W).to(DEV).float())
            assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (i, rel_mae, rel_fro)
        assert m.device_status(0) == 0
    finally:
        gather.close()


def test_fused_gather_pipelined_sequence():
    """Pipelined completion over a sequence with no waits in between (each
    launch waits on its predecessor's exchange): the last result, after one
    wait, is complete; nothing timed out."""
    import csed499ii_b200 as m

    gather = shard.FusedGather(16, 4096, device=DEV)
    try:
        N, K, M = 4096, 4096, 16
        outs = []
        for i in range(7):
            W, B, s, meta = random_packed_problem(N, K, 128, seed=300 + i)
            sw = shard.ShardedWeight(torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV),
                                     torch.from_numpy(s).to(DEV), 0, 1)
            A = torch.from_numpy(activations(M, K, seed=40 + i)).to(DEV)
            outs.append((shard.mul_2_4_gathered(A, sw, gather), A, W))
        gather.wait()
        torch.cuda.synchronize()
        C, A, W = outs[-1]
        rel_mae, rel_fro, _ = errors(C, A.float() @ torch.from_numpy(W).to(DEV).float())
        assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)
        assert m.device_status(0) == 0
    finally:
        gather.close()


def _fused_worker(rank, world, port, q, pipelined):
    import datetime

    import torch.distributed as dist

    import csed499ii_b200 as m

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    dev = torch.device("cuda", rank)
    gather = shard.FusedGather(16, 12288 // world, device=dev, pipelined=pipelined)
    try:
        shapes = [(4096, 4096), (11008, 4096), (4096, 4096), (12288, 4096), (4096, 11008)]
        for i, (N, K) in enumerate(shapes):
            W, B, s, meta = random_packed_problem(N, K, 128, seed=200 + i)
            sw = shard.ShardedWeight(torch.from_numpy(B).to(dev), torch.from_numpy(meta).to(dev),
                                     torch.from_numpy(s).to(dev), rank, world)
            A = torch.from_numpy(activations(16, K, seed=30 + i)).to(dev)
            C = shard.mul_2_4_gathered(A, sw, gather)
            gather.wait()
            torch.cuda.synchronize(dev)
            rel_mae, rel_fro, _ = errors(C, A.float() @ torch.from_numpy(W).to(dev).float())
            q.put((rank, i, rel_mae, rel_fro))
        q.put((rank, -1, float(m.device_status(rank)), 0.0))
        dist.barrier()
    finally:
        gather.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("pipelined", [True, False])
def test_fused_gather_two_ranks(pipelined):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, q, pipelined))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    got = [q.get(timeout=5) for _ in range(world * 6)]
    for rank, i, a, b in got:
        if i < 0:
            assert a == 0.0, f"rank {rank} device status {a}"
        else:
            assert a < REL_MAE_TOL and b <= REL_FRO_TOL, (rank, i, a, b)
