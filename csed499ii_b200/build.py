"""Build recipe for the in-tree CUDA library (sm_100a only).

``python -m csed499ii_b200.build`` compiles ``csrc/sm100_marlin.cu`` with
nvcc into ``csed499ii_b200/_lib/libsm100_marlin.so``.  The library is a plain
C-ABI shared object (no torch, no Python symbols); ``csed499ii_b200._ext``
loads it with ctypes.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sysconfig
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libsm100_marlin.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    "-shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".h"))] + [
        os.path.join(ROOT, "include", "sm100_marlin.h")
    ]


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False,
          out: str = LIB_PATH, defines=()) -> str:
    """Compile the library if any source is newer than it; return its path.

    ``defines`` (e.g. ``["SM100_MARLIN_TRACE=1"]``) build a variant into
    ``out``; the default build has none.
    """
    if not force and not ptxas_info and not defines and out == LIB_PATH and up_to_date():
        return LIB_PATH
    os.makedirs(os.path.dirname(out), exist_ok=True)
    tmp = out + ".tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS] + [f"-D{d}" for d in defines]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-cudart", "static", "-o", tmp, os.path.join(CSRC, "sm100_marlin.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose or ptxas_info:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, out)
    return out


FAST_NAME = "_fastcall" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so")
FAST_PATH = os.path.join(HERE, FAST_NAME)


def build_fastcall(force: bool = False) -> str:
    """Compile the CPython binding (csrc/pybind_fast.c) next to the package;
    it links the C-ABI library from _lib/ (rpath $ORIGIN/_lib)."""
    src = os.path.join(CSRC, "pybind_fast.c")
    hdr = os.path.join(ROOT, "include", "sm100_marlin.h")
    if (not force and os.path.exists(FAST_PATH)
            and os.path.getmtime(FAST_PATH) >= max(os.path.getmtime(src), os.path.getmtime(hdr),
                                                   os.path.getmtime(LIB_PATH))):
        return FAST_PATH
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the CPython binding")
    tmp = FAST_PATH + ".tmp"
    cmd = [cc, "-O2", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], src, "-o", tmp,
           "-L", LIB_DIR, "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN/_lib"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("building the CPython binding failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, FAST_PATH)
    return FAST_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    build_fastcall(force="--force" in sys.argv)
