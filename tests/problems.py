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
