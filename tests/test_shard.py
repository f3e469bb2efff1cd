"""Column-parallel sharding of packed 2:4 weights (CPU; gloo for the exchange).

The multi-GPU layer has no reference counterpart; its oracle is the
single-device result.  Slicing the packed tensors must equal packing the
sliced weight (checked through the pinned dequantisation oracle, bit-exact),
and the all-gather of per-rank column blocks must reassemble the full
product.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import marlin24_oracle as O
from csed499ii_b200 import shard
from problems import quantized_problem, random_packed_problem


def test_column_range():
    assert shard.column_range(4096, 0, 2) == (0, 2048)
    assert shard.column_range(4096, 1, 2) == (2048, 4096)
    assert shard.column_range(57344, 7, 8) == (50176, 57344)
    with pytest.raises(ValueError):
        shard.column_range(4096 + 64, 0, 2)  # 4160 / 2 = 2080 is not whole chunks
    with pytest.raises(ValueError):
        shard.column_range(4096, 2, 2)


@pytest.mark.parametrize("N,K,g,world", [(512, 256, 128, 2), (1024, 512, -1, 4), (768, 384, 128, 3),
                                         (2048, 256, 128, 8)])
def test_slice_equals_dequantised_column_block(N, K, g, world):
    W, B, s, meta = quantized_problem(N, K, g, seed=11)
    full = O.dequant_2_4(B, meta, s, K, N, g)
    Bt, mt, st = torch.from_numpy(B), torch.from_numpy(meta), torch.from_numpy(s)
    for r in range(world):
        c0, c1 = shard.column_range(N, r, world)
        B_r, m_r, s_r = shard.slice_packed(Bt, mt, st, c0, c1)
        assert B_r.shape == (K // 32, 2 * (c1 - c0)) and m_r.shape == (c1 - c0, K // 16)
        part = O.dequant_2_4(B_r.numpy(), m_r.numpy(), s_r.numpy(), K, c1 - c0, g)
        np.testing.assert_array_equal(part.view(np.uint16), full[:, c0:c1].view(np.uint16))


def test_slice_equals_packing_the_slice():
    # pack the whole weight, and pack its column block separately, with the
    # same scales and mask: the packed bytes must be identical
    rng = np.random.default_rng(5)
    K, N, g = 256, 512, 128
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    s = O.group_scales(w, g)
    B, meta, s_p = O.pack_2_4(w, s, g)
    c0, c1 = 128, 384
    B2, meta2, s_p2 = O.pack_2_4(np.ascontiguousarray(w[:, c0:c1]), np.ascontiguousarray(s[:, c0:c1]), g)
    B_r, m_r, s_r = shard.slice_packed(torch.from_numpy(B), torch.from_numpy(meta),
                                       torch.from_numpy(s_p), c0, c1)
    np.testing.assert_array_equal(B_r.numpy(), B2)
    np.testing.assert_array_equal(m_r.numpy(), meta2)
    np.testing.assert_array_equal(s_r.numpy().view(np.uint16), s_p2.view(np.uint16))


def test_oracle_columns_equals_whole_matrix_oracle():
    # the column-sampled oracle of the large-layer GPU tests (problems.py)
    # dequantises exactly the chosen columns of the whole-matrix oracle
    from problems import chunk_columns, oracle_columns, sample_chunks

    N, K = 1024, 512
    W, B, s, meta = random_packed_problem(N, K, 128, seed=21)
    chunks = sample_chunks(N, 5, seed=3)
    assert chunks[0] == 0 and chunks[-1] == N // 64 - 1
    part = oracle_columns(B, meta, s, K, chunks)
    np.testing.assert_array_equal(part.view(np.uint16), W[:, chunk_columns(chunks)].view(np.uint16))


def test_slice_of_3bit_metadata():
    N, K = 1024, 512
    _, B, s, meta = random_packed_problem(N, K, 128, seed=4)
    m3 = torch.from_numpy(O.meta3_pack(meta)[0])
    for c0, c1 in [(0, 256), (256, 768), (960, 1024)]:
        _, m_r, _ = shard.slice_packed(torch.from_numpy(B), m3, torch.from_numpy(s), c0, c1)
        _, m16_r, _ = shard.slice_packed(torch.from_numpy(B), torch.from_numpy(meta),
                                         torch.from_numpy(s), c0, c1)
        np.testing.assert_array_equal(m_r.numpy(), O.meta3_pack(m16_r.numpy())[0])


def test_slice_rejects_partial_chunks():
    _, B, s, meta = random_packed_problem(256, 128, 128, seed=1)
    with pytest.raises(ValueError):
        shard.slice_packed(torch.from_numpy(B), torch.from_numpy(meta), torch.from_numpy(s), 32, 128)


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _gather_worker(rank, world, port, N, K, M, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, B, s, meta = random_packed_problem(N, K, 128, seed=21)
        A = np.random.default_rng(3).standard_normal((M, K)).astype(np.float32)
        c0, c1 = shard.column_range(N, rank, world)
        B_r, m_r, s_r = shard.slice_packed(torch.from_numpy(B), torch.from_numpy(meta),
                                           torch.from_numpy(s), c0, c1)
        W_r = O.dequant_2_4(B_r.numpy(), m_r.numpy(), s_r.numpy(), K, c1 - c0, 128)
        C_r = torch.from_numpy(A @ W_r.astype(np.float32))
        C = shard.gather_columns(C_r)
        ref = A @ W.astype(np.float32)
        q.put((rank, float(np.abs(C.numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_columns_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, 512, 256, 5, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(err == 0.0 for err in res.values()), res
