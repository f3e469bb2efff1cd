"""Seeded problem generation and error metrics shared by the GPU tests.

Two generators, both built on the CPU oracle:

* :func:`quantized_problem` -- the reference's data flow (``gen_quant4_NT``,
  ``test_2_4.py:22-70``): random fp16 W, absmax*2/15 scales, codes, 2:4 mask
  on codes, Sparse-Marlin packing.
* :func:`random_packed_problem` -- random operator inputs in the packed
  format (random INT4 codes, random legal 2:4 metadata nibbles, random
  positive scales); used for full-size shapes where packing from dense would
  dominate the test time.  Either way the oracle weight is
  ``dequant_2_4(B, meta, s)``.
* :func:`packed_problem_gpu` + :func:`oracle_columns` -- the same kind of
  inputs made on the GPU for layers too large for a whole-matrix numpy
  oracle (Llama-2-70B); the oracle then dequantises a sample of 64-column
  chunks, sliced from the packed tensors the way column shards are (every
  permutation of the format stays inside a 64-column chunk; pinned bit-exact
  by ``tests/test_shard.py``).
"""
from __future__ import annotations

import functools

import numpy as np

import marlin24_oracle as O

LEGAL_NIBBLES = np.array([0x4, 0x8, 0x9, 0xC, 0xD, 0xE], dtype=np.uint16)


@functools.lru_cache(maxsize=16)
def quantized_problem(N: int, K: int, groupsize: int, seed: int = 0, sigma: float = 1.0):
    rng = np.random.default_rng(seed)
    unc, B, s, meta = O.gen_quant4_nt(N, K, groupsize, rng, sigma)
    return unc, B, s, meta


@functools.lru_cache(maxsize=16)
def random_packed_problem(N: int, K: int, groupsize: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    B = rng.integers(0, 2**32, size=(K // 32, 2 * N), dtype=np.uint64).astype(np.uint32).view(np.int32)
    nib = rng.choice(LEGAL_NIBBLES, size=(N * K // 16, 4))
    meta = (nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)).astype(np.uint16)
    meta = meta.view(np.int16).reshape(N, K // 16)
    rows = 1 if groupsize == -1 else K // groupsize
    s = (rng.uniform(0.5, 1.5, size=(rows, N)) * 0.02 * 2 / 15).astype(np.float16)
    W = O.dequant_2_4(B, meta, s, K, N, groupsize)
    return W, B, s, meta


def activations(M: int, K: int, seed: int = 1):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K)).astype(np.float16)


def errors(C, C_ref):
    """(relative MAE, relative Frobenius, max abs) of C against C_ref (fp32)."""
    import torch

    C = C.float()
    C_ref = C_ref.float()
    d = (C - C_ref).abs()
    rel_mae = (d.mean() / C_ref.abs().mean()).item()
    rel_fro = (torch.linalg.norm(C - C_ref) / torch.linalg.norm(C_ref)).item()
    return rel_mae, rel_fro, d.max().item()


# Tolerances: relative MAE from the reference's tests (test_2_4.py:87-89),
# relative Frobenius error from the north-star statement.
REL_MAE_TOL = 0.002
REL_FRO_TOL = 1e-2


def packed_problem_gpu(N: int, K: int, seed: int, sigma: float = 0.02, device: str = "cuda:0"):
    """Random packed operator inputs made on the GPU: INT4 codes, legal 2:4
    metadata nibbles, group-128 scales of the size absmax*2/15 gives for
    weights ~N(0, sigma) (about 4.5 sigma * 2/15, +-50 %)."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    legal = torch.tensor([int(v) for v in LEGAL_NIBBLES], dtype=torch.int32, device=device)
    B = torch.randint(-(2**31), 2**31 - 1, (K // 32, 2 * N), dtype=torch.int32, device=device,
                      generator=gen)
    idx = torch.randint(0, 6, (N * K // 16, 4), device=device, generator=gen)
    nib = legal[idx]
    meta = (nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)).to(torch.int16)
    meta = meta.view(N, K // 16).contiguous()
    del idx, nib
    s = ((torch.rand((K // 128, N), device=device, generator=gen) + 0.5) * (4.5 * sigma * 2 / 15)).half()
    return B, meta, s.contiguous()


def sample_chunks(N: int, count: int = 8, seed: int = 0):
    """Indices of `count` 64-column chunks: the first, the last and random ones."""
    n = N // 64
    rng = np.random.default_rng(seed)
    inner = rng.permutation(np.arange(1, n - 1))[:max(0, count - 2)] if n > 2 else []
    return sorted({0, n - 1} | set(int(c) for c in inner))


def oracle_columns(B, meta, s, K: int, chunks):
    """Oracle weight (K, 64*len(chunks)) of the given 64-column chunks, from
    the packed tensors (torch or numpy) sliced per chunk."""
    def host(t):
        return t.cpu().numpy() if hasattr(t, "cpu") else np.asarray(t)

    B, meta, s = host(B), host(meta), host(s)
    kk = B.shape[0]
    n_out = B.shape[1] // 2
    parts = []
    for c in chunks:
        c0, c1 = 64 * c, 64 * c + 64
        B_r = np.ascontiguousarray(B[:, 2 * c0:2 * c1])
        meta_r = np.ascontiguousarray(meta.reshape(kk, n_out, 2)[:, c0:c1, :]).reshape(c1 - c0, 2 * kk)
        s_r = np.ascontiguousarray(s[:, c0:c1])
        parts.append(O.dequant_2_4(B_r, meta_r, s_r, K, c1 - c0, 128))
    return np.concatenate(parts, axis=1)


def chunk_columns(chunks):
    return np.concatenate([np.arange(64 * c, 64 * c + 64) for c in chunks])
