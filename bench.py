"""Benchmark of the sm_100a 2:4 sparse W4A16 GEMM (driver contract).

Workload (Llama-2-7B decode): one *step* is one decode
step of all 32 transformer layers' four projection GEMMs --
(K, N) in {(4096, 12288) qkv, (4096, 4096) o, (4096, 22016) gate+up,
(11008, 4096) down} -- at M = 16 batch rows, 2:4 INT4 weights with group-128
fp16 scales and 4-bit 2:4 metadata (``--meta-bits 3`` for the 3-bit variant).
Every layer has its own weights (2.4 GB per GPU, far above the 126 MB L2), so
each step streams its weights from HBM.  The 128 launches of a step are
captured in a CUDA graph and replayed.

Lines printed (rank 0, one JSON line):
* ``value``  -- algorithmic bytes (bench.py:170 of the reference: A + B + meta
  + s + C) of all ranks / max-over-ranks device time, GB/s, inputs resident.
* ``e2e``    -- same metric through the public Python operator
  (``csed499ii_b200.mul_2_4``), eager launches, with the step's activations
  copied from pinned host memory and the last layer's outputs copied back
  inside the timed region.
* ``roofline`` -- GEMM kernel achieved GB/s vs the measured HBM copy peak.
* ``cpu_baseline`` -- the CPU oracle (numpy dequantise-then-matmul, the
  reference's torch fp32 oracle path) on a bounded sample, plus the variant
  that decompresses the packed weights on every call.
* ``detail`` -- per-shape kernel times of the step and a small prefill
  sample (config 4 shapes, TFLOP/s against the derived 2:4 peak).

``--impl reference`` times the reference's CPU path (the oracle port) alone.
``--workload prefill`` runs the config-4 sweep (with the cuSPARSELt bar);
``--workload ablation`` runs the metadata-cost ablation (the reference's
``kernel_profile/run.py bench`` protocol).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS = 32
SHAPES = [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]  # (K, N)
# one Llama-2-70B layer set (qkv, o, gate+up, down)
SHAPES_70B = [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]
GROUP = 128
# (batch rows, metadata bits) -> mean DRAM bytes per GEMM launch over SHAPES,
# `dram__bytes_read.sum + dram__bytes_write.sum` from one ncu capture of the
# same kernel and shapes, made separately (ncu cannot run inside this
# timing); reported as a constant with its source, not measured in the run.
MEASURED_TRAFFIC = {(16, 4): 20.002e6}


def algo_bytes(M, K, N, meta_bits):
    meta = K * N // 8 if meta_bits == 4 else 3 * K * N // 32
    return K * N // 4 + meta + 2 * N * K // GROUP + 2 * M * K + 2 * M * N


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------
# clocks sampled during the timed region (NVML)
# ----------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [k for k, v in self.REASONS.items() if self.reasons & v and k != "gpu_idle"]
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ----------------------------------------------------------------------------
# synthetic weights (random packed operator inputs; timing is data-independent)
# ----------------------------------------------------------------------------
def make_layer(torch, K, N, dev, gen, meta_bits):
    legal = torch.tensor([0x4, 0x8, 0x9, 0xC, 0xD, 0xE], dtype=torch.int32, device=dev)
    B = torch.randint(-(2**31), 2**31 - 1, (K // 32, 2 * N), dtype=torch.int32, device=dev, generator=gen)
    idx = torch.randint(0, 6, (N * K // 16, 4), device=dev, generator=gen)
    nib = legal[idx]
    meta = (nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)).to(torch.int16)
    meta = meta.view(N, K // 16).contiguous()
    s = (torch.rand((K // GROUP, N), device=dev, generator=gen) * 0.02 + 0.01).half() * (2 / 15)
    if meta_bits == 3:
        from csed499ii_b200 import metadata_decode as md

        meta = md.pack(meta)
    return B, meta, s.contiguous()


def bench_ours(args, torch, dist, rank, world, dev):
    import csed499ii_b200 as m
    from csed499ii_b200 import metadata_decode as md
    from csed499ii_b200 import shard

    lib = m._ext.load()
    M = args.m
    shapes = args.shapes
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    layers = [[make_layer(torch, K, N, dev, gen, args.meta_bits) for (K, N) in shapes]
              for _ in range(args.layers)]
    A = {K: torch.randn((M, K), dtype=torch.half, device=dev, generator=gen)
         for K in sorted({K for K, _ in shapes})}
    C = {N: torch.empty((M, N), dtype=torch.half, device=dev) for (_, N) in shapes}
    # N > 1: column-parallel layers of width world * N; this rank holds one
    # N-wide shard and every GEMM is followed by the all-gather of C
    Cg = {N: torch.empty((M, world * N), dtype=torch.half, device=dev) for (_, N) in shapes}

    def gather(N):
        if world > 1:
            shard.gather_columns(C[N], out=Cg[N])
    ws = torch.zeros(max(N for _, N in shapes) // 128 * 16, dtype=torch.int32, device=dev)
    devi = dev.index
    fn = lib.sm100_marlin_mul_2_4 if args.meta_bits == 4 else lib.sm100_marlin_mul_2_4_meta3
    stream = torch.cuda.Stream(device=dev)
    # N > 1, default: the all-gather fused into the GEMM epilogue (peer stores
    # over NVLink into buffers shared by CUDA IPC), pipelined: each GEMM's
    # kernel ends once the previous call's exchange has completed, and every
    # step ends with a wait for its last exchange (so each step's all-gathers
    # are complete inside the timed region); --gather nccl: separate NCCL
    # all-gather after each GEMM
    fused = world > 1 and args.gather in ("fused", "fused-sync")
    fg = (shard.FusedGather(M, max(N for _, N in shapes), device=dev,
                            pipelined=args.gather == "fused") if fused else None)
    shards = [[shard.ShardedWeight.from_local(B, meta, s, rank * N, (rank + 1) * N, args.meta_bits)
               for (K, N), (B, meta, s) in zip(shapes, lay)] for lay in layers] if fused else None

    def step_raw(s_ptr):
        for li, lay in enumerate(layers):
            for si, ((K, N), (B, meta, s)) in enumerate(zip(shapes, lay)):
                if fused:
                    rc, _ = fg.issue(A[K].data_ptr(), B.data_ptr(), meta.data_ptr(), s.data_ptr(),
                                     N, M, K, shards[li][si].workspace.data_ptr(), GROUP // 2,
                                     s_ptr, args.meta_bits)
                else:
                    rc = fn(A[K].data_ptr(), B.data_ptr(), meta.data_ptr(), C[N].data_ptr(),
                            s.data_ptr(), N, M, K, ws.data_ptr(), GROUP // 2, devi, s_ptr, -1, -1,
                            -1, 16)
                if rc != 0:
                    raise RuntimeError(f"mul_2_4 failed: {m._ext.describe(rc)}")
                if not fused:
                    gather(N)
        if fused:
            fg.wait(s_ptr)

    bytes_step = args.layers * sum(algo_bytes(M, K, N, args.meta_bits) for (K, N) in shapes)
    launches_step = args.layers * len(shapes) * ((M + 63) // 64)

    # warm-up eagerly (sizes the split-K scratch before capture), then capture
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step_raw(stream.cuda_stream)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_raw(torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(devi) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / args.steps
    value = bytes_step * world * args.steps / (ms * 1e-3) / 1e9
    per_launch_us = ms * 1e3 / (args.steps * launches_step)
    status = m.device_status(devi)
    if status != 0:
        raise RuntimeError(f"device status {status}: a bounded wait timed out")

    # ---- per-shape kernel times (for the detail block), inputs resident
    detail = {}
    for (K, N), idx in zip(shapes, range(len(shapes))):
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            sp = torch.cuda.current_stream(dev).cuda_stream
            for li, lay in enumerate(layers):
                B, meta, s = lay[idx]
                if fused:
                    fg.issue(A[K].data_ptr(), B.data_ptr(), meta.data_ptr(), s.data_ptr(), N, M, K,
                             shards[li][idx].workspace.data_ptr(), GROUP // 2, sp, args.meta_bits)
                else:
                    fn(A[K].data_ptr(), B.data_ptr(), meta.data_ptr(), C[N].data_ptr(),
                       s.data_ptr(), N, M, K, ws.data_ptr(), GROUP // 2, devi, sp, -1, -1, -1, 16)
                    gather(N)
            if fused:
                fg.wait(sp)
        for _ in range(3):
            g2.replay()
        torch.cuda.synchronize(dev)
        reps = max(3, min(50, args.steps))
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                g2.replay()
            ev1.record(stream)
        torch.cuda.synchronize(dev)
        us = ev0.elapsed_time(ev1) * 1e3 / (reps * args.layers)
        b = algo_bytes(M, K, N, args.meta_bits)
        detail[f"{K}x{N}"] = {"us": round(us, 3), "GB/s": round(b / us / 1e3, 1),
                              "TFLOP/s": round(2 * M * K * N / us / 1e6, 2)}
        del g2

    # ---- end to end through the public operator, host buffers
    A_h = {K: A[K].cpu().pin_memory() for K in A}
    C_h = {N: torch.empty((M, world * N), dtype=torch.half).pin_memory() for N in C}
    C_out = dict(Cg) if world > 1 else C
    A_d = {K: torch.empty_like(A[K]) for K in A}
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        for K in A_h:
            A_d[K].copy_(A_h[K], non_blocking=True)
        for li, lay in enumerate(layers):
            for si, ((K, N), (B, meta, s)) in enumerate(zip(shapes, lay)):
                if fused:
                    C_out[N] = shard.mul_2_4_gathered(A_d[K], shards[li][si], fg)
                    continue
                if args.meta_bits == 4:
                    m.mul_2_4(A_d[K], B, meta, C[N], s, ws)
                else:
                    md.matmul(A_d[K], B, meta, C[N], s, ws)
                gather(N)
        if fused:
            fg.wait()
        for N in C_h:
            C_h[N].copy_(C_out[N], non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        ev0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        ev1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = bytes_step * world * e2e_steps / (e2e_ms * 1e-3) / 1e9
    h2d = sum(t.numel() * 2 for t in A_h.values())
    d2h = sum(t.numel() * 2 for t in C_h.values())

    # the graphs hold launches that reference the fused-gather buffers
    del graph
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    if fg is not None:
        fg.close()

    peak, peak_kind = load_peaks()
    # DRAM bytes (read + write) per launch from a separate ncu capture of the
    # same kernel and shapes, averaged over the four shapes like `achieved`;
    # only known for the default case.
    traffic = MEASURED_TRAFFIC.get((M, args.meta_bits)) if shapes == SHAPES else None
    achieved = bytes_step / args.layers / len(shapes) / (per_launch_us * 1e-6) / 1e9 if M <= 64 else None
    return dict(
        value=value, ms_step=ms_step, per_launch_us=per_launch_us, bytes_step=bytes_step,
        launches=launches_step * args.steps, clocks=clk.summary(), detail=detail,
        e2e=dict(value=round(e2e_value, 2), unit="GB/s", h2d_bytes_per_step=h2d,
                 d2h_bytes_per_step=d2h, steps=e2e_steps,
                 ms_per_step=round(e2e_ms / e2e_steps, 4)),
        roofline=dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s",
                      frac=round(achieved / peak, 4), traffic=traffic,
                      traffic_source=("constant: ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                      "per launch from a separate capture of this kernel on these "
                                      "shapes, not measured in this run") if traffic else None,
                      peak_source=f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"),
    )


# ----------------------------------------------------------------------------
# CPU oracle (the reference's dequantise-then-matmul path)
# ----------------------------------------------------------------------------
def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        return max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        return os.cpu_count() or 1


def _random_packed(rng, K, N):
    B = rng.integers(0, 2**32, size=(K // 32, 2 * N), dtype=np.uint64).astype(np.uint32).view(np.int32)
    nib = rng.choice(np.array([0x4, 0x8, 0x9, 0xC, 0xD, 0xE], dtype=np.uint16), size=(N * K // 16, 4))
    meta = (nib[:, 0] | (nib[:, 1] << 4) | (nib[:, 2] << 8) | (nib[:, 3] << 12)).astype(np.uint16)
    meta = meta.view(np.int16).reshape(N, K // 16)
    s = (rng.uniform(0.01, 0.03, size=(K // GROUP, N)) * 2 / 15).astype(np.float16)
    return B, meta, s


def cpu_reference(M, meta_bits, reps, budget_s=25.0):
    """The reference's CPU path on one Llama-2-7B layer (its four GEMMs):
    ``A.float() @ W.float()`` with W the oracle's dequantised 2:4 weight,
    dequantised once (``metadata_decode/smoke.py:26``).  One *step* of this
    arm is that one layer; ``seconds_per_step`` is its measured median."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import marlin24_oracle as O

    rng = np.random.default_rng(0)
    Ws, As = [], {}
    for (K, N) in SHAPES:
        B, meta, s = _random_packed(rng, K, N)
        Ws.append(O.dequant_2_4(B, meta, s, K, N, GROUP).astype(np.float32))
        As.setdefault(K, rng.standard_normal((M, K)).astype(np.float16).astype(np.float32))
    bytes_layer = sum(algo_bytes(M, K, N, meta_bits) for (K, N) in SHAPES)
    times = []
    t_start = time.perf_counter()
    for r in range(reps):
        t0 = time.perf_counter()
        for (K, N), W in zip(SHAPES, Ws):
            _ = As[K] @ W
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    return dict(value=round(bytes_layer / t / 1e9, 3), unit="GB/s", cores=_cpu_threads(), kind="port",
                cpu_model=cpu_model(), os_cpu_count=os.cpu_count(),
                sample=(f"step = one Llama-2-7B layer (its 4 GEMMs, M={M}) of the 32-layer decode "
                        f"step; numpy fp32 A @ dequant(W), W dequantised once by the oracle "
                        f"(the reference's torch fp32 path); median of {len(times)} steps"),
                seconds_per_step=t, steps_run=len(times))


def cpu_reference_decompress(M, reps=3, budget_s=15.0):
    """The variant that decompresses on every call: the packed (B, meta, s)
    are expanded to the dense weight (the reference's
    ``sparse_semi_structured_to_dense_cutlass`` + scale multiply,
    ``_semi_structured_conversions.py:186-283``, restated by the oracle) and
    multiplied, per call, on the (4096, 4096) layer."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import marlin24_oracle as O

    K = N = 4096
    rng = np.random.default_rng(1)
    B, meta, s = _random_packed(rng, K, N)
    A = rng.standard_normal((M, K)).astype(np.float16).astype(np.float32)
    times = []
    t_start = time.perf_counter()
    for _ in range(reps):
        t0 = time.perf_counter()
        W = O.dequant_2_4(B, meta, s, K, N, GROUP).astype(np.float32)
        _ = A @ W
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    return dict(value=round(algo_bytes(M, K, N, 4) / t / 1e9, 4), unit="GB/s", cores=_cpu_threads(),
                kind="port", sample=(f"one (K, N) = (4096, 4096) GEMM at M={M} with the packed weight "
                                     f"decompressed on every call; median of {len(times)} calls"),
                us_per_call=round(t * 1e6, 1))


PREFILL_SHAPES = [(4096, 4096), (8192, 8192), (4096, 11008)]  # (K, N)
PREFILL_M = [512, 2048, 8192]


def bench_prefill(args, torch, dev):
    """Compute-bound regime: dense-equivalent TFLOP/s of single GEMMs."""
    import csed499ii_b200 as m

    lib = m._ext.load()
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321)
    devi = dev.index
    detail, flops_total, sec_total = {}, 0.0, 0.0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.Stream(device=dev)
    fn = lib.sm100_marlin_mul_2_4 if args.meta_bits == 4 else lib.sm100_marlin_mul_2_4_meta3
    for (K, N) in PREFILL_SHAPES:
        B, meta, s = make_layer(torch, K, N, dev, gen, args.meta_bits)
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=dev)
        for M in PREFILL_M:
            A = torch.randn((M, K), dtype=torch.half, device=dev, generator=gen)
            C = torch.empty((M, N), dtype=torch.half, device=dev)

            def call():
                rc = fn(A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(), s.data_ptr(), N, M,
                        K, ws.data_ptr(), GROUP // 2, devi, stream.cuda_stream, -1, -1, -1, 16)
                if rc != 0:
                    raise RuntimeError(f"mul_2_4 failed: {m._ext.describe(rc)}")
            for _ in range(args.warmup):
                call()
            torch.cuda.synchronize(dev)
            reps = max(3, min(args.steps, 20))
            with torch.cuda.stream(stream):
                ev0.record(stream)
                for _ in range(reps):
                    call()
                ev1.record(stream)
            torch.cuda.synchronize(dev)
            t = ev0.elapsed_time(ev1) * 1e-3 / reps
            fl = 2.0 * M * N * K
            detail[f"M{M}_K{K}_N{N}"] = {"us": round(t * 1e6, 1), "TFLOP/s": round(fl / t / 1e12, 1)}
            flops_total += fl
            sec_total += t
    return flops_total / sec_total / 1e12, detail


def dense_peak():
    """(dense bf16 TFLOP/s, label): the derived 2:4 peak is twice it."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "derived: 2 x measured dense bf16 (MEASURED_PEAKS.json)"
    except Exception:
        return 1590.0, "derived: 2 x fallback dense"


PREFILL_SAMPLE = [(2048, 4096, 4096), (8192, 4096, 4096), (2048, 8192, 8192), (8192, 8192, 8192)]


def prefill_sample(torch, dev, reps=10):
    """Config-4 sample carried in the decode line's `detail`: single GEMMs at
    M = 2048 / 8192 and K = N = 4096 / 8192, inputs resident, CUDA events on
    the launching stream; TFLOP/s dense-equivalent against the derived 2:4
    peak."""
    import csed499ii_b200 as m

    lib = m._ext.load()
    gen = torch.Generator(device=dev)
    gen.manual_seed(4323)
    stream = torch.cuda.Stream(device=dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dense, kind = dense_peak()
    out, layers = {}, {}
    for (M, K, N) in PREFILL_SAMPLE:
        if (K, N) not in layers:
            layers[(K, N)] = make_layer(torch, K, N, dev, gen, 4)
        B, meta, s = layers[(K, N)]
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=dev)
        A = torch.randn((M, K), dtype=torch.half, device=dev, generator=gen)
        C = torch.empty((M, N), dtype=torch.half, device=dev)

        def call():
            rc = lib.sm100_marlin_mul_2_4(A.data_ptr(), B.data_ptr(), meta.data_ptr(), C.data_ptr(),
                                          s.data_ptr(), N, M, K, ws.data_ptr(), GROUP // 2, dev.index,
                                          stream.cuda_stream, -1, -1, -1, 16)
            if rc != 0:
                raise RuntimeError(f"mul_2_4 failed: {m._ext.describe(rc)}")
        for _ in range(3):
            call()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                call()
            ev1.record(stream)
        torch.cuda.synchronize(dev)
        t = ev0.elapsed_time(ev1) * 1e-3 / reps
        tf = 2.0 * M * N * K / t / 1e12
        out[f"M{M}_K{K}_N{N}"] = {"us": round(t * 1e6, 1), "TFLOP/s": round(tf, 1),
                                  "frac_of_2to4_peak": round(tf / (2 * dense), 4)}
    out["peak"] = {"value": 2 * dense, "unit": "TFLOP/s", "source": kind}
    return out


ABLATION_SHAPES = [(1, 4096, 4096), (16, 4096, 4096), (32, 4096, 4096), (1, 1024, 1024),
                   (64, 4096, 4096), (2048, 4096, 4096)]


def bench_ablation(args, torch, dev, samples=9, graph_calls=100, replays=5):
    """Metadata-cost ablation, the reference's `kernel_profile/run.py bench`
    protocol: uniform inputs (random packed codes, scales 0.01, metadata
    0xEEEE), every variant checked bit-exact against the baseline first, then
    `graph_calls` calls captured in one CUDA graph per variant, `samples`
    measurements of `replays` replays each in a shuffled order (seeded), and
    the median per-call microseconds.  The diagnostics are instances of the
    warp-level decode kernel and the CTA-pair kernel, so the baseline is
    pinned to those (`sm100_marlin_set_decode_kernel(DECODE_STREAM_K)`)."""
    from csed499ii_b200 import _ext

    lib = _ext.load()
    lib.sm100_marlin_set_decode_kernel(_ext.DECODE_STREAM_K)
    try:
        return _bench_ablation_pinned(torch, dev, samples, graph_calls, replays)
    finally:
        lib.sm100_marlin_set_decode_kernel(_ext.DECODE_AUTO)


def _bench_ablation_pinned(torch, dev, samples, graph_calls, replays):
    import random

    import csed499ii_b200 as m
    from csed499ii_b200 import metadata_diagnostics as diag

    gen = torch.Generator(device=dev)
    gen.manual_seed(20261019)
    rows = {}
    for (M, N, K) in ABLATION_SHAPES:
        a = torch.randn((M, K), dtype=torch.half, device=dev, generator=gen)
        b = torch.randint(-(2**31), 2**31 - 1, (K // 32, 2 * N), dtype=torch.int32, device=dev,
                          generator=gen)
        s = torch.full((K // 128, N), 0.01, dtype=torch.half, device=dev)
        meta = torch.full((N, K // 16), -4370, dtype=torch.int16, device=dev)
        c = torch.empty((M, N), dtype=torch.half, device=dev)
        ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=dev)
        fns = {"baseline": m.mul_2_4, "no_gmem": diag.no_gmem, "no_reg": diag.no_reg,
               "no_all": diag.no_all}
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            fns["baseline"](a, b, meta, c, s, ws)
            torch.cuda.synchronize(dev)
            ref = c.clone()
            for name, f in fns.items():
                c.fill_(float("nan"))
                f(a, b, meta, c, s, ws)
                torch.cuda.synchronize(dev)
                if not torch.equal(c, ref):
                    raise RuntimeError(f"ablation {name} differs from the baseline at {(M, N, K)}")
        graphs = {}
        for name, f in fns.items():
            with torch.cuda.stream(stream):
                for _ in range(3):
                    f(a, b, meta, c, s, ws)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(graph_calls):
                    f(a, b, meta, c, s, ws)
            graphs[name] = g
        jobs = [(name, i) for name in fns for i in range(samples)]
        random.Random(20261019).shuffle(jobs)
        per = {name: [] for name in fns}
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for name, _ in jobs:
            with torch.cuda.stream(stream):
                graphs[name].replay()
                ev0.record(stream)
                for _ in range(replays):
                    graphs[name].replay()
                ev1.record(stream)
            ev1.synchronize()
            per[name].append(ev0.elapsed_time(ev1) * 1000 / (graph_calls * replays))
        med = {name: round(statistics.median(v), 3) for name, v in per.items()}
        base = med["baseline"]
        rows[f"M{M}_N{N}_K{K}"] = {"us": med, "saved_vs_baseline": {
            name: round(1 - med[name] / base, 4) for name in fns if name != "baseline"}}
        del graphs
    if m.device_status(dev.index) != 0:
        raise RuntimeError("a bounded wait timed out during the ablation")
    return rows


def bench_cusparselt(args, torch, dev):
    """Library bar for the prefill sweep, as the reference's own comparator
    (kernel_bench/bench.py:249-277): an fp16 2:4 GEMM through cuSPARSELt
    (torch._cslt_compress / torch._cslt_sparse_mm) on the same shapes, fp16
    weights (4x the bytes of the INT4 ones), timed the same way."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(4322)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.Stream(device=dev)
    detail, flops_total, sec_total = {}, 0.0, 0.0
    for (K, N) in PREFILL_SHAPES:
        W = torch.randn((N, K), dtype=torch.half, device=dev, generator=gen)
        keep = W.abs().view(N, K // 4, 4).topk(2, dim=-1).indices
        mask = torch.zeros((N, K // 4, 4), dtype=torch.bool, device=dev).scatter_(-1, keep, True)
        Wc = torch._cslt_compress((W.view(N, K // 4, 4) * mask).view(N, K))
        del W, mask, keep
        for M in PREFILL_M:
            A = torch.randn((M, K), dtype=torch.half, device=dev, generator=gen)
            At = A.t()
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    torch._cslt_sparse_mm(Wc, At)
                torch.cuda.synchronize(dev)
                reps = max(3, min(args.steps, 20))
                ev0.record(stream)
                for _ in range(reps):
                    torch._cslt_sparse_mm(Wc, At)
                ev1.record(stream)
            torch.cuda.synchronize(dev)
            t = ev0.elapsed_time(ev1) * 1e-3 / reps
            fl = 2.0 * M * N * K
            detail[f"M{M}_K{K}_N{N}"] = {"us": round(t * 1e6, 1), "TFLOP/s": round(fl / t / 1e12, 1)}
            flops_total += fl
            sec_total += t
        del Wc
    return flops_total / sec_total / 1e12, detail


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--meta-bits", type=int, choices=[3, 4], default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", choices=["fused", "fused-sync", "nccl"], default="fused",
                    help="N > 1: all-gather of C fused into the GEMM epilogue (NVLink peer "
                         "stores) with pipelined completion (each step ends with a wait for "
                         "its last exchange), the same with per-call completion, or a "
                         "separate NCCL all-gather")
    ap.add_argument("--workload", choices=["decode", "llama70b", "prefill", "ablation"],
                    default="decode",
                    help="decode: Llama-2-7B decode step (config 1, the headline; N > 1: weak "
                         "scaling); llama70b: Llama-2-70B layer set (config 3), N-sharded across "
                         "the ranks (strong scaling); prefill: compute-bound sweep (config 4); "
                         "ablation: metadata-cost diagnostics (config 4's ablation)")
    ap.add_argument("--no-prefill-sample", action="store_true",
                    help="decode: skip the config-4 prefill sample in `detail`")
    ap.add_argument("--no-comparator", action="store_true",
                    help="prefill: skip the cuSPARSELt fp16 2:4 comparator")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers per step (32 = Llama-2-7B; fewer only for profiling)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    strong = args.workload == "llama70b"
    if strong:
        if any(N % (128 * world) for _, N in SHAPES_70B):
            raise SystemExit(f"llama70b: the layer widths do not split into {world} shards")
        args.shapes = [(K, N // world) for (K, N) in SHAPES_70B]
        if args.layers == LAYERS:
            args.layers = 8  # 2.7 GB of weights per step on one GPU
        args.no_cpu_baseline = True
        args.no_prefill_sample = True
    else:
        args.shapes = SHAPES
    config = {"workload": f"Llama-2-7B decode step: {args.layers} layers x 4 GEMMs "
                          f"(K,N) in {SHAPES}, M={args.m}, 2:4 INT4 g128, {args.meta_bits}-bit meta",
              "model_shapes": "Llama-2-7B", "batch_rows": args.m, "groupsize": GROUP,
              "meta_bits": args.meta_bits, "layers": args.layers,
              "l2": f"inputs larger than L2: {args.layers} distinct layers' weights "
                    f"({args.layers * 75.4 / 1024:.2f} GB) per step",
              "parallelism": ("single GPU" if args.gpus == 1 else
                              f"tp{args.gpus} column-parallel: each rank holds an N-wide shard of "
                              f"{args.gpus}N-wide layers (weak scaling), all-gather of C after "
                              f"every GEMM ({'fused into the GEMM epilogue over NVLink' if args.gather == 'fused' else 'NCCL'})")}
    metric = f"2:4 W4A16 GEMM HBM GB/s (Llama-2-7B decode layer set, M={args.m})"
    if strong:
        layer_gb = sum(algo_bytes(args.m, K, N, args.meta_bits) for (K, N) in SHAPES_70B) / 1e9
        config = {"workload": f"Llama-2-70B layer set: {args.layers} layers x 4 GEMMs (K,N) in "
                              f"{SHAPES_70B}, M={args.m}, 2:4 INT4 g128, {args.meta_bits}-bit meta, "
                              f"every layer's columns split over {world} ranks",
                  "model_shapes": "Llama-2-70B", "batch_rows": args.m, "groupsize": GROUP,
                  "meta_bits": args.meta_bits, "layers": args.layers,
                  "l2": f"inputs larger than L2: {args.layers * layer_gb / world:.2f} GB of "
                        f"weights per rank per step",
                  "parallelism": ("single GPU" if world == 1 else
                                  f"tp{world} column-parallel (strong scaling): each rank holds "
                                  f"1/{world} of every layer's columns, all-gather of C after every "
                                  f"GEMM ({args.gather})")}
        metric = f"2:4 W4A16 GEMM HBM GB/s (Llama-2-70B layer set, M={args.m}, column-sharded)"

    if args.impl == "reference":
        if rank != 0:
            return
        if strong:
            print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm times the "
                              "Llama-2-7B decode workload only"}), flush=True)
            return
        ref = cpu_reference(args.m, args.meta_bits, reps=max(args.steps, 1))
        keys = ("value", "unit", "cores", "kind", "sample", "cpu_model", "os_cpu_count")
        line = dict(metric=metric, value=ref["value"], unit="GB/s", n_gpus=args.gpus,
                    steps=ref["steps_run"], warmup=args.warmup,
                    ms_per_step=round(ref["seconds_per_step"] * 1e3, 3),
                    higher_is_better=True, scaling="weak", vs_baseline=None, dtype="f32",
                    data="synthetic", config=config, impl="reference",
                    cpu_baseline={k: ref[k] for k in keys},
                    e2e={"value": ref["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)

    if args.workload == "prefill":
        value, detail = bench_prefill(args, torch, dev)
        dense, kind = dense_peak()
        line = dict(metric="2:4 W4A16 GEMM dense-equivalent TFLOP/s (prefill sweep, config 4)"
                    + ("" if args.meta_bits == 4 else ", 3-bit metadata"),
                    value=round(value, 1), unit="TFLOP/s", n_gpus=1, steps=args.steps,
                    warmup=args.warmup, higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype="f16", data="synthetic (random packed INT4 codes, legal 2:4 metadata)",
                    config={"workload": f"M in {PREFILL_M} x (K,N) in {PREFILL_SHAPES}, g128",
                            "meta_bits": args.meta_bits},
                    roofline={"bound": "tensor", "achieved": round(value, 1), "peak": 2 * dense,
                              "unit": "TFLOP/s", "frac": round(value / (2 * dense), 4),
                              "peak_source": kind},
                    detail=detail)
        if not args.no_comparator:
            try:
                cv, cdetail = bench_cusparselt(args, torch, dev)
                line["comparator"] = {
                    "library": "cuSPARSELt fp16 x fp16 2:4 (torch._cslt_sparse_mm), fp16 weights",
                    "value": round(cv, 1), "unit": "TFLOP/s", "ours_over_library": round(value / cv, 3),
                    "detail": cdetail}
            except Exception as e:  # comparator only; never fails the bench line
                line["comparator"] = {"library": "cuSPARSELt", "unavailable": str(e)[:200]}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    if args.workload == "ablation":
        rows = bench_ablation(args, torch, dev)
        if rank == 0:
            print(json.dumps(dict(
                metric="metadata-cost ablation: per-call us, uniform 0xEEEE metadata (config 4)",
                unit="us", higher_is_better=False, n_gpus=1, dtype="f16",
                data="synthetic uniform (random packed INT4 codes, scales 0.01, metadata 0xEEEE)",
                config={"workload": "kernel_profile/run.py bench protocol: 100 calls per CUDA graph, "
                                    "9 shuffled samples of 5 replays, median",
                        "shapes": [f"M{M}_N{N}_K{K}" for (M, N, K) in ABLATION_SHAPES]},
                detail=rows)), flush=True)
        return
    res = bench_ours(args, torch, dist, rank, world, dev)
    if rank == 0 and world == 1 and args.workload == "decode" and not args.no_prefill_sample:
        res["detail"]["prefill_sample"] = prefill_sample(torch, dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = cpu_reference(args.m, args.meta_bits, reps=10)
        cpu = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model",
                                   "os_cpu_count")}
        cpu["per_call_decompression"] = cpu_reference_decompress(args.m)
    if rank == 0:
        line = dict(metric=metric, value=round(res["value"], 2), unit="GB/s", n_gpus=world,
                    steps=args.steps, warmup=args.warmup, ms_per_step=round(res["ms_step"], 5),
                    higher_is_better=True, scaling="strong" if strong else "weak",
                    vs_baseline=None, dtype="f16",
                    data="synthetic (random packed INT4 codes, random legal 2:4 metadata, "
                         "random fp16 group scales; seeded)",
                    config=config, e2e=res["e2e"], roofline=res["roofline"],
                    cpu_baseline=cpu, clocks=res["clocks"], gpu_launches=res["launches"],
                    per_launch_us=round(res["per_launch_us"], 3), detail=res["detail"])
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
