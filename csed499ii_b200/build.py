"""Build recipe for the in-tree CUDA library (sm_100a only).

``python -m csed499ii_b200.build`` compiles every ``csrc/*.cu`` translation
unit with nvcc (in parallel, objects under ``csed499ii_b200/_build/``) and
links them into ``csed499ii_b200/_lib/libsm100_marlin.so``: the host launcher
and C ABI (``sm100_marlin.cu``) and the kernel instances (``k_*.cu``).  The
library is a plain C-ABI shared object (no torch, no Python symbols);
``csed499ii_b200._ext`` loads it with ctypes.
"""
from __future__ import annotations

import concurrent.futures
import hashlib
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
]
BUILD_DIR = os.path.join(HERE, "_build")


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def _units():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith(".cu")]


def _headers():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cuh", ".h"))] + [
        os.path.join(ROOT, "include", "sm100_marlin.h")
    ]


def _sources():
    return _units() + _headers()


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


def _compile(unit: str, obj: str, defines, ptxas_info: bool):
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS] + [f"-D{d}" for d in defines]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-c", "-o", obj + ".tmp", unit]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(unit)}:\n" + res.stdout + res.stderr)
    os.replace(obj + ".tmp", obj)
    return " ".join(cmd), res.stdout + res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False,
          out: str = LIB_PATH, defines=()) -> str:
    """Compile the library if any source is newer than it; return its path.

    Each translation unit is recompiled when it or any header is newer than
    its object.  ``defines`` (e.g. ``["SM100_MARLIN_TRACE=1"]``) build a
    variant into ``out`` (objects in their own directory); the default build
    has none.
    """
    if not force and not ptxas_info and not defines and out == LIB_PATH and up_to_date():
        return LIB_PATH
    tag = hashlib.sha1(" ".join(sorted(defines)).encode()).hexdigest()[:8] if defines else "default"
    bdir = os.path.join(BUILD_DIR, tag)
    os.makedirs(bdir, exist_ok=True)
    os.makedirs(os.path.dirname(out), exist_ok=True)
    newest_header = max(os.path.getmtime(h) for h in _headers())
    jobs = []
    objs = []
    for unit in _units():
        obj = os.path.join(bdir, os.path.basename(unit)[:-3] + ".o")
        objs.append(obj)
        stale = (force or ptxas_info or not os.path.exists(obj)
                 or os.path.getmtime(obj) < max(os.path.getmtime(unit), newest_header))
        if stale:
            jobs.append((unit, obj))
    workers = max(1, min(len(jobs), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        futs = [pool.submit(_compile, u, o, defines, ptxas_info) for u, o in jobs]
        for f in futs:
            cmd, log = f.result()
            if verbose:
                print(cmd, flush=True)
            if verbose or ptxas_info:
                sys.stdout.write(log)
    tmp = out + ".tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("linking the library failed:\n" + res.stdout + res.stderr)
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
