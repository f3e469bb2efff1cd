"""The C-ABI library builds, loads and exports what include/sm100_marlin.h declares.

Only argument-validation paths that return before touching CUDA are called
here (no GPU in the CPU suite).
"""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sm100_marlin.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sm100_marlin_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from csed499ii_b200 import build, _ext

    build.build()
    return _ext.load()


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("sm100_marlin_mul_2_4", "sm100_marlin_mul_2_4_meta3", "sm100_marlin_meta3_pack",
              "sm100_marlin_meta3_unpack", "sm100_marlin_error_string"):
        assert n in names


def test_every_declared_symbol_is_exported(lib):
    from csed499ii_b200 import _ext

    names = declared_functions()
    for n in names:
        assert hasattr(lib, n), n
    # the ctypes signature table covers exactly the header
    assert sorted(_ext.SIGNATURES) == names


def test_library_has_no_torch_dependency():
    from csed499ii_b200 import build

    with open(build.LIB_PATH, "rb") as f:
        blob = f.read()
    assert b"libtorch" not in blob and b"libc10" not in blob


def _mul(lib, **kw):
    args = dict(A=None, B=None, meta=None, C=None, s=None, prob_m=256, prob_n=16, prob_k=256,
                workspace=None, groupsize=-1, dev=0, stream=None, thread_k=-1, thread_m=-1,
                sms=-1, max_par=16)
    args.update(kw)
    return lib.sm100_marlin_mul_2_4(*args.values())


def test_reference_shape_rules(lib):
    # marlin_cuda_kernel_nm.cu:779-781: N % thread_m, K % thread_k -> ERR_PROB_SHAPE
    assert _mul(lib, prob_m=200) == 1
    assert _mul(lib, prob_k=200) == 1
    assert _mul(lib, prob_m=384, prob_n=32) == 1          # auto tile 64x256 at n > 16
    # no instance for explicit (128,128) with more than 16 rows (nm.cu:813-823)
    assert _mul(lib, prob_n=32, thread_k=128, thread_m=128) == 2
    assert _mul(lib, thread_k=256, thread_m=128) == 2
    assert _mul(lib, groupsize=32) == 2
    # zero-sized problems are a no-op (nm.cu:782-783)
    assert _mul(lib, prob_n=0) == 0


def test_meta3_argument_checks(lib):
    assert lib.sm100_marlin_meta3_pack(None, None, 100, None, None) == 5
    assert lib.sm100_marlin_meta3_pack(None, None, 0, None, None) == 0
    assert lib.sm100_marlin_meta3_unpack(None, None, 47, None) == 5


def test_error_strings(lib):
    for code in range(7):
        assert lib.sm100_marlin_error_string(code)
    assert b"unknown" in lib.sm100_marlin_error_string(99)


def test_python_mirror_raises_reference_messages():
    import torch
    import csed499ii_b200 as m

    A = torch.zeros(16, 256, dtype=torch.half)
    C = torch.zeros(16, 256, dtype=torch.half)
    s = torch.zeros(3, 256, dtype=torch.half)
    ws = torch.zeros(32, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="k=256 not compatible with 3 groups."):
        m.mul_2_4(A, None, None, C, s, ws)
    s1 = torch.zeros(1, 256, dtype=torch.half)
    with pytest.raises(RuntimeError, match="workspace must be of size at least 32."):
        m.mul_2_4(A, None, None, C, s1, torch.zeros(31, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        m.mul_2_4(A, None, None, C, s1, ws)
