"""Build the reference's own CUDA code for sm_100a into ``oracle/_ref/``.

Test infrastructure only (the product never loads these):

* ``libref_marlin24.so`` -- the reference launcher and kernel
  (``kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu``
  with its ``common/*.h``) behind the C function ``ref_marlin_cuda_2_4``
  (``ref_marlin24_wrap.cu``).  Used by the GPU tests to check the reference
  kernel against the oracle at batch sizes where it is known to be correct
  (M <= 16) and to time it beside this library on the same B200.
* ``ref_codec*.so`` -- the reference 3-bit metadata codec
  (``kernel_experiments/sparse_marlin/metadata_decode/codec.cu`` +
  ``decoder_dependency/pair.cuh``) as a torch extension (``ref_codec_bind.cpp``).

Sources are compiled where they lie in the reference checkout (path from
``CSED499II_ROOT`` or the first argument); nothing is copied.  Outputs go to
``oracle/_ref/`` only (git-ignored, shipped to the GPU box with the tree).
Without the checkout this script does nothing.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def ref_root():
    cands = [a for a in sys.argv[1:] if not a.startswith("-")] + [os.environ.get("CSED499II_ROOT", ""),
                                                                 "/root/reference"]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "kernel_experiments", "sparse_marlin")):
            return c
    return None


def build_kernel(root):
    src = os.path.join(root, "kernel_experiments/sparse_marlin/src/marlin/marlin_cuda_kernel_nm.cu")
    out = os.path.join(OUT, "libref_marlin24.so")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, *ARCH, "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
           "-shared", "-cudart", "static", f'-DREF_NM_CU="{src}"', "-o", out,
           os.path.join(HERE, "ref_marlin24_wrap.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        print("reference kernel build failed:\n" + r.stderr[-4000:])
        return False
    print("built", out)
    return True


def build_codec(root):
    from torch.utils.cpp_extension import load

    codec = os.path.join(root, "kernel_experiments/sparse_marlin/metadata_decode/codec.cu")
    inc = os.path.join(root, "kernel_experiments/sparse_marlin/decoder_dependency")
    bdir = os.path.join(OUT, "build_codec")
    os.makedirs(bdir, exist_ok=True)
    try:
        load(name="ref_codec", sources=[os.path.join(HERE, "ref_codec_bind.cpp"), codec],
             extra_include_paths=[inc], extra_cuda_cflags=[*ARCH, "-O3", "-std=c++17"],
             build_directory=bdir, verbose=False, is_python_module=True)
    except Exception as e:  # the import after building may fail without a GPU; the .so is what matters
        if not any(f.endswith(".so") for f in os.listdir(bdir)):
            print("reference codec build failed:", e)
            return False
    for f in os.listdir(bdir):
        if f.endswith(".so"):
            shutil.copy(os.path.join(bdir, f), os.path.join(OUT, f))
            print("built", os.path.join(OUT, f))
    return True


def main():
    root = ref_root()
    if root is None:
        print("reference checkout not found; oracle/_ref not built")
        return 0
    os.makedirs(OUT, exist_ok=True)
    ok = build_kernel(root)
    ok = build_codec(root) and ok
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
