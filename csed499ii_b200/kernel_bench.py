"""The reference's kernel benchmark harness, driving this library.

Mirrors the Sparse-Marlin parts of hyeonu453/CSED499II ``kernel_bench/bench.py``
so that its sweeps and their output lines can be reproduced on B200:

* ``python -m csed499ii_b200.kernel_bench compare sparse [--models ...]
  [--batchsizes ...]`` -- cuSPARSELt fp16 2:4 against the 2:4 INT4 kernel on
  each model's four layer shapes, one summary line per batch size
  (``benchmark_sparse_kernels`` + ``run_sweep``, ``bench.py:293-314,379-392``);
* ``python -m csed499ii_b200.kernel_bench single sparse-marlin -m M -n N -k K``
  -- one kernel, one shape (``benchmark_kernel``, ``bench.py:443-455``), as
  the target of an ``ncu --profile-from-start off`` capture;
* :func:`benchmark_sparse_marlin` returns ``{"s", "TFLOP/s", "GB/s"}`` with
  the reference's byte count (``bench.py:159-173``).

Inputs are the reference's synthetic timing problem (``get_problem_24``,
``bench.py:108-124``): random packed codes, uniform metadata 0xEEEE, zero
scales; only the kernel's time is measured.  The other kernels of the
reference harness (dense Marlin, EXL2, MACKO, cuSPARSE SpMV) are not part of
this library.
"""
from __future__ import annotations

import argparse
import time

import torch

import csed499ii_b200 as marlin

# bench.py:283-290 (the reference's model table)
MODELS = {
    "Llama7B": [(4096, 3 * 4096), (4096, 4096), (4096, 2 * 10752), (10752, 4096)],
    "Llama13B": [(5120, 3 * 5120), (5120, 5120), (5120, 2 * 13568), (13568, 5120)],
    "Llama33B": [(6656, 3 * 6656), (6656, 6656), (6656, 2 * 17664), (17664, 6656)],
}
DEFAULT_BATCHES = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048]


def _dev():
    return torch.device("cuda:0")


def benchmark(f, warmup=1, iter=10, profile=False, cooldown=1.0):
    """Average CUDA-event seconds per call (bench.py:17-45); ``profile`` opens
    a cudaProfilerStart/Stop range around the timed calls."""
    if warmup < 0 or iter <= 0:
        raise ValueError("warmup must be nonnegative and iter must be positive")
    for _ in range(warmup):
        f()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if profile:
        torch.cuda.profiler.start()
    try:
        start.record()
        for _ in range(iter):
            f()
        end.record()
        torch.cuda.synchronize()
    finally:
        if profile:
            torch.cuda.profiler.stop()
    res = start.elapsed_time(end) / iter / 1000
    if cooldown:
        time.sleep(cooldown)
    return res


def get_problem_24(m, n, k, groupsize=-1):
    """(B, B_ref, s, meta) of the reference's synthetic 2:4 timing problem."""
    dev = _dev()
    B = torch.randint(low=-(2**31), high=2**31 - 1, size=(k * n // 8 // 2,), dtype=torch.int32,
                      device=dev)
    B_ref = torch.randn((k, n), dtype=torch.half, device=dev)
    meta = torch.full((n * k // 16,), -4370, dtype=torch.int16, device=dev)
    rows = 1 if groupsize == -1 else (k // 2) // (groupsize // 2)
    s = torch.zeros((rows, n), dtype=torch.half, device=dev)
    torch.cuda.synchronize()
    return B.view(k // 32, 2 * n), B_ref, s, meta.view(n, k // 16)


def benchmark_sparse_marlin(A, B, meta, C, s, warmup=1, iter=10, profile=False, cooldown=1.0):
    workspace = torch.zeros(C.shape[1] // 128 * 16, device=A.device, dtype=torch.int32)
    sms = torch.cuda.get_device_properties(A.device).multi_processor_count

    def f():
        marlin.mul_2_4(A, B, meta, C, s, workspace, -1, -1, sms)

    res = benchmark(f, warmup, iter, profile=profile, cooldown=cooldown)
    return {
        "s": res,
        "TFLOP/s": 2 * A.numel() * C.shape[1] / res / 10**12,
        "GB/s": (2 * A.numel() + 4 * B.numel() + 2 * meta.numel() + 2 * C.numel() + 2 * s.numel())
        / res / 10**9,
    }


def benchmark_cusparselt(A, B, warmup=1, iter=10, profile=False, cooldown=1.0):
    """fp16 x fp16 2:4 GEMM through cuSPARSELt (bench.py:249-277); B is the
    dense (k, n) weight with two nonzeros in every four along k."""
    m = A.shape[0]
    padded_m = max(8, m)
    k, n = B.shape
    B_t = B.t().contiguous()
    B_compressed = torch._cslt_compress(B_t)
    if m < 8:
        A_padded = torch.zeros((padded_m, k), dtype=A.dtype, device=A.device)
        A_padded[:m].copy_(A)
    else:
        A_padded = A.contiguous()
    V = A_padded.t()

    def f():
        torch._cslt_sparse_mm(B_compressed, V)

    res = benchmark(f, warmup, iter, profile=profile, cooldown=cooldown)
    return {
        "s": res,
        "TFLOP/s": 2 * A.numel() * n / res / 10**12,
        "GB/s": (2 * A_padded.numel() + B_compressed.numel() * B_compressed.element_size()
                 + 2 * padded_m * n) / res / 10**9,
        "padded_m": padded_m,
    }


def format_line(name, batch, total):
    return ("[%s] batch=%04d: s=%.5f, TFLOP/s=%07.3f, GB/s=%08.3f, speedup=%.2f"
            % (name, batch, total["s"], total["TFLOP/s"], total["GB/s"], total["speedup"]))


def run_sweep(models, batchsizes, run_case, out=print):
    """Time-weighted totals over a model's layers per batch (bench.py:293-314)."""
    for model, layers in models.items():
        out(model)
        for batch in batchsizes:
            totals = {}
            for k, n in layers:
                results = run_case(batch, n, k)
                baseline = next(iter(results.values()))["s"]
                for name, res in results.items():
                    total = totals.setdefault(name, {"s": 0, "TFLOP/s": 0, "GB/s": 0, "speedup": 0})
                    total["s"] += res["s"]
                    total["TFLOP/s"] += res["TFLOP/s"] * res["s"]
                    total["GB/s"] += res["GB/s"] * res["s"]
                    total["speedup"] += baseline
            for name, total in totals.items():
                for key in ("TFLOP/s", "GB/s", "speedup"):
                    total[key] /= total["s"]
                out(format_line(name, batch, total))
        out("")


def benchmark_sparse_kernels(models, batchsizes, warmup=1, iter=10, profile=False, out=print,
                             cooldown=1.0):
    """cuSPARSELt vs the 2:4 INT4 kernel; speedup relative to cuSPARSELt."""
    dev = _dev()

    def run_case(m, n, k):
        A = torch.randn((m, k), dtype=torch.half, device=dev)
        C = torch.zeros((m, n), dtype=torch.half, device=dev)
        B_ref = torch.rand((k // 4, 4, n), dtype=torch.half, device=dev) + 0.5
        B_ref[:, :2] = 0
        results = {"cuSPARSELt": benchmark_cusparselt(A, B_ref.view(k, n), warmup, iter, profile,
                                                      cooldown)}
        del B_ref
        B, B_ref, s, meta = get_problem_24(m, n, k, groupsize=128)
        results["2:4"] = benchmark_sparse_marlin(A, B, meta, C, s, warmup, iter, profile, cooldown)
        return results

    out("groupsize=128\n")
    run_sweep(models, batchsizes, run_case, out=out)


def benchmark_kernel(kernel, m, n, k, groupsize=128, warmup=1, iter=10):
    dev = _dev()
    A = torch.randn((m, k), dtype=torch.half, device=dev)
    C = torch.zeros((m, n), dtype=torch.half, device=dev)
    if kernel == "sparse-marlin":
        B, B_ref, s, meta = get_problem_24(m, n, k, groupsize)
        return benchmark_sparse_marlin(A, B, meta, C, s, warmup, iter, profile=True)
    if kernel == "cusparselt":
        B_t = torch.zeros((n, k // 4, 4), dtype=torch.half, device=dev)
        idx = torch.rand((n, k // 4, 4), device=dev).argsort(dim=-1)[..., :2]
        vals = torch.rand((n, k // 4, 2), dtype=torch.half, device=dev) + 0.5
        B_t.scatter_(-1, idx, vals)
        return benchmark_cusparselt(A, B_t.view(n, k).t().contiguous(), warmup, iter, profile=True)
    if kernel == "cublas":
        B = torch.randn((k, n), dtype=torch.half, device=dev)
        return benchmark(lambda: torch.mm(A, B, out=C), warmup, iter, profile=True)
    raise ValueError(f"Unsupported Kernel: {kernel}")


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description="Kernel performance benchmarks (B200)")
    sub = parser.add_subparsers(dest="mode", required=True)
    compare = sub.add_parser("compare", help="Compare kernels across model layers")
    compare.add_argument("comparison", choices=["sparse"])
    compare.add_argument("--models", nargs="+", choices=list(MODELS), default=list(MODELS))
    compare.add_argument("--batchsizes", type=int, nargs="+", default=DEFAULT_BATCHES)
    compare.add_argument("--warmup", type=int, default=1)
    compare.add_argument("--iter", type=int, default=10)
    compare.add_argument("--profile", action="store_true",
                         help="Enable profiler ranges; run ncu with --profile-from-start off")
    single = sub.add_parser("single", help="Profile one kernel with ncu --profile-from-start off")
    single.add_argument("kernel", choices=["sparse-marlin", "cusparselt", "cublas"])
    single.add_argument("-m", type=int, required=True)
    single.add_argument("-n", type=int, required=True)
    single.add_argument("-k", type=int, required=True)
    single.add_argument("--groupsize", type=int, default=128)
    single.add_argument("--warmup", type=int, default=1)
    single.add_argument("--iter", type=int, default=10)
    args = parser.parse_args(argv)
    if args.warmup < 0 or args.iter <= 0:
        parser.error("--warmup must be nonnegative and --iter must be positive")
    if args.mode == "single" and min(args.m, args.n, args.k) <= 0:
        parser.error("-m, -n and -k must be positive")
    if args.mode == "compare" and any(b <= 0 for b in args.batchsizes):
        parser.error("--batchsizes must be positive")
    return args


def main(argv=None):
    args = parse_args(argv)
    if args.mode == "single":
        print(benchmark_kernel(args.kernel, args.m, args.n, args.k, groupsize=args.groupsize,
                               warmup=args.warmup, iter=args.iter))
        return
    models = {name: MODELS[name] for name in args.models}
    benchmark_sparse_kernels(models, args.batchsizes, warmup=args.warmup, iter=args.iter,
                             profile=args.profile)


if __name__ == "__main__":
    main()
