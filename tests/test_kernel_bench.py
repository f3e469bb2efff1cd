"""The reference harness surface (csed499ii_b200.kernel_bench).

CPU: the sweep arithmetic and the line format of the reference's
``kernel_bench/bench.py:293-314`` on stub timings, and the CLI.  GPU: one
short ``compare sparse`` sweep and ``single sparse-marlin`` through the
library.
"""
import re

import pytest

from csed499ii_b200 import kernel_bench as kb

LINE = re.compile(r"^\[(.+)\] batch=(\d{4}): s=(\d+\.\d{5}), TFLOP/s=(\d{3}\.\d{3}), "
                  r"GB/s=(\d{4}\.\d{3}), speedup=(\d+\.\d{2})$")


def test_sweep_totals_and_line_format():
    # two layers; baseline 1 s and 3 s, candidate twice as fast on each
    times = {(2, 8): (1.0, 0.5), (4, 8): (3.0, 1.5)}

    def run_case(m, n, k):
        base, ours = times[(k, n)]
        return {"base": {"s": base, "TFLOP/s": 1.0, "GB/s": 10.0},
                "ours": {"s": ours, "TFLOP/s": 2.0, "GB/s": 20.0}}

    lines = []
    kb.run_sweep({"Toy": [(2, 8), (4, 8)]}, [16], run_case, out=lines.append)
    assert lines[0] == "Toy" and lines[-1] == ""
    parsed = {LINE.match(l).group(1): LINE.match(l).groups() for l in lines[1:-1]}
    assert parsed["base"][2] == "4.00000" and parsed["base"][5] == "1.00"
    assert parsed["ours"][2] == "2.00000" and parsed["ours"][5] == "2.00"
    assert parsed["ours"][3] == "002.000" and parsed["ours"][4] == "0020.000"
    assert parsed["ours"][1] == "0016"


def test_cli_parsing():
    a = kb.parse_args(["compare", "sparse", "--models", "Llama7B", "--batchsizes", "1", "16"])
    assert a.mode == "compare" and a.models == ["Llama7B"] and a.batchsizes == [1, 16]
    a = kb.parse_args(["single", "sparse-marlin", "-m", "16", "-n", "4096", "-k", "4096"])
    assert (a.kernel, a.m, a.n, a.k) == ("sparse-marlin", 16, 4096, 4096)
    with pytest.raises(SystemExit):
        kb.parse_args(["single", "sparse-marlin", "-m", "0", "-n", "4096", "-k", "4096"])


@pytest.mark.gpu
def test_compare_sparse_and_single_on_gpu():
    lines = []
    kb.benchmark_sparse_kernels({"Llama7B": kb.MODELS["Llama7B"]}, [1, 16], iter=3,
                                out=lines.append, cooldown=0.0)
    rows = [LINE.match(l) for l in lines if l.startswith("[")]
    assert len(rows) == 4 and all(rows)
    names = {r.group(1) for r in rows}
    assert names == {"cuSPARSELt", "2:4"}
    res = kb.benchmark_kernel("sparse-marlin", 16, 4096, 4096, iter=3)
    assert set(res) == {"s", "TFLOP/s", "GB/s"} and res["s"] > 0
