"""CPU known-answer tests of the 3-bit metadata codec restatement.

Truth tables come from the reference's own exhaustive checks:
``decoder_dependency/pair.cu:11`` (high map), ``decoder_dependency/
experiment.cu:12`` (low map), ``3bit_encoding/experiment.cu:83`` (earlier
code), encoder tables from ``metadata_decode/codec.cu:11-13``.
"""
import numpy as np
import pytest

import marlin24_oracle as O

LEGAL = [0x4, 0x8, 0x9, 0xC, 0xD, 0xE]


def test_truth_tables_match_reference_tests():
    assert [int(v) for v in O.DEC_HIGH] == [14, 13, 8, 13, 3, 4, 9, 12]
    assert [int(v) for v in O.DEC_LOW] == [12, 13, 14, 10, 8, 9, 4, 0]
    assert [int(v) for v in O.DEC_3BIT_ENCODING] == [4, 4, 9, 8, 14, 14, 13, 12]


def test_encoders_invert_decoders_on_legal_nibbles():
    for nib in LEGAL:
        assert O.DEC_HIGH[O.ENC_HIGH[nib]] == nib
        assert O.DEC_LOW[O.ENC_LOW[nib]] == nib
    for nib in range(16):
        if nib not in LEGAL:
            assert O.ENC_HIGH[nib] == -1 and O.ENC_LOW[nib] == -1


def test_decode24_exhaustive_ignores_top_byte():
    x = np.arange(1 << 24, dtype=np.uint32)
    garbage = ((x * np.uint32(1664525) + np.uint32(1013904223)) & np.uint32(0xFF)) << np.uint32(24)
    for table in (O.DEC_HIGH, O.DEC_LOW):
        a = O.decode24(x, table)
        b = O.decode24(x | garbage, table)
        assert np.array_equal(a, b)
    # spot values: all codes = c -> nibble table[c] everywhere
    for c in range(8):
        word = np.uint32(int("".join(f"{c:03b}" for _ in range(8)), 2))
        assert int(O.decode24(np.array([word]), O.DEC_LOW)[0]) == int(O.DEC_LOW[c]) * 0x11111111


def random_legal_meta(rng, n_int16):
    nib = rng.choice(np.array(LEGAL, dtype=np.uint16), size=(n_int16, 4))
    v = nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)
    return v.astype(np.uint16).view(np.int16)


@pytest.mark.parametrize("blocks", [1, 3, 64])
def test_meta3_roundtrip(blocks):
    rng = np.random.default_rng(20261019)
    meta = random_legal_meta(rng, 128 * blocks)
    packed, errors = O.meta3_pack(meta)
    assert errors == 0
    assert packed.dtype == np.int32 and packed.size == meta.size * 3 // 8
    assert np.array_equal(O.meta3_unpack(packed), meta)


def test_meta3_plane_layout():
    # word p of a block -> first of lane pair p; check X/Y/Z planes by hand
    w = np.zeros(64, dtype=np.uint32)
    w[:] = 0xEEEEEEEE  # high code 0, low code 2
    w[5] = 0xDDDDDDDD  # high code 1 at lane pair 5 (first word)
    packed, errors = O.meta3_pack(w.view(np.int16))
    assert errors == 0
    p = packed.view(np.uint32)
    low_e = 0o22222222  # eight low codes of 2
    assert p[5] == (0o11111111 | ((low_e & 0xFF) << 24))
    assert p[0] == ((low_e & 0xFF) << 24)
    assert p[16] == ((low_e >> 8) | ((0 & 0xFFFF) << 16))


def test_meta3_rejects_illegal_nibbles():
    meta = np.full(128, 0x4444, dtype=np.uint16).view(np.int16).copy()
    meta.view(np.uint16)[7] = 0x4F44  # one illegal nibble (F)
    _, errors = O.meta3_pack(meta)
    assert errors == 1


def test_meta3_of_reference_metadata():
    import os
    from conftest import GOLDEN, golden_cases

    for name in golden_cases():
        z = np.load(os.path.join(GOLDEN, name))
        meta = z["meta"].reshape(-1)
        packed, errors = O.meta3_pack(meta)
        assert errors == 0
        assert np.array_equal(O.meta3_unpack(packed), meta)
