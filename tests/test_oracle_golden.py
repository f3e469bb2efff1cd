"""Pin the CPU oracle against the reference's own packers (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference's ``Layer_2_4.pack`` / ``gen_quant4_NT`` flow
(``kernel_experiments/sparse_marlin/src/test_2_4.py:22-70``).
"""
import os

import numpy as np
import pytest

import marlin24_oracle as O
from conftest import GOLDEN, golden_cases

CASES = golden_cases()


def load(name):
    z = np.load(os.path.join(GOLDEN, name))
    return {k: z[k] for k in z.files}


def test_fixtures_present():
    assert len(CASES) >= 5


@pytest.mark.parametrize("name", CASES)
def test_scales_bit_exact(name):
    c = load(name)
    s = O.group_scales(c["w"], int(c["groupsize"]))
    assert np.array_equal(s.view(np.uint16), c["s_raw"].view(np.uint16))


@pytest.mark.parametrize("name", CASES)
def test_pack_bit_exact(name):
    c = load(name)
    g = int(c["groupsize"])
    codes = O.quantize_codes(c["w"], c["s_raw"], g)
    ref = O.dequant_codes(codes, c["s_raw"], g)
    B, meta, s = O.pack_2_4(ref, c["s_raw"], g)
    assert B.dtype == np.int32 and B.shape == c["B"].shape
    assert np.array_equal(B, c["B"])
    assert meta.dtype == np.int16 and np.array_equal(meta, c["meta"])
    assert np.array_equal(s.view(np.uint16), c["s"].view(np.uint16))


@pytest.mark.parametrize("name", CASES)
def test_unpack_inverts_reference_pack(name):
    c = load(name)
    K, N, g = int(c["K"]), int(c["N"]), int(c["groupsize"])
    codes = O.unpack_2_4(c["B"], c["meta"], K, N)
    # exactly two kept entries in every group of 4 along K
    kept = (codes >= 0).reshape(K // 4, 4, N).sum(axis=1)
    assert np.all(kept == 2)
    B, meta = O.pack_values(np.ascontiguousarray(
        O.compress_2_4(np.where(codes < 0, 0, codes).T)[0].T)), None
    assert np.array_equal(B, c["B"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_gemm_matches_reference_oracle(name):
    c = load(name)
    g = int(c["groupsize"])
    C = O.gemm_oracle(c["A"], c["B"], c["meta"], c["s"], g)
    ref = c["C_ref"]
    # same products, different fp32 summation order
    assert np.allclose(C, ref, rtol=1e-5, atol=1e-4 * np.abs(ref).max())


def test_stable_mask_tie_breaking():
    x = np.array([[3, 3, 3, 3, 1, 5, 5, 1, 7, 0, 7, 0, 2, 2, 9, 2]], dtype=np.int32)
    m = O.mask_2_4(x)
    # ties: the lower indices are dropped first
    assert m.astype(int).tolist() == [[0, 0, 1, 1, 0, 1, 1, 0, 1, 0, 1, 0, 0, 0, 1, 1]]
