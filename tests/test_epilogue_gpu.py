"""Fused epilogue (bias + activation) on the GPU, through the C ABI.

``mul_2_4_epilogue`` computes ``act(A @ W + bias)`` in the GEMM's store.  The
reference has no such entry (its ``Layer_2_4`` is "without bias"); the check
is the plain PyTorch fp32 composition of the same steps on the oracle's
dequantised weights, with the same tolerances as the GEMM itself.  Every
kernel's epilogue is covered: decode (batch <= 64, both scale modes, 3-bit
metadata), the CTA-pair prefill kernel, the dense-expansion prefill kernel
(K not a multiple of 128) and the chunked 3-bit path above 64 rows.
"""
import io

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import marlin24_oracle as O
from problems import REL_FRO_TOL, REL_MAE_TOL, activations, errors, quantized_problem, random_packed_problem

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

ACTS = {"none": lambda x: x, "relu": F.relu, "silu": F.silu,
        "gelu_tanh": lambda x: F.gelu(x, approximate="tanh")}


@pytest.fixture(scope="module", autouse=True)
def _setup():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    import csed499ii_b200 as m

    assert m.device_status(0) == 0


def _run(A, B, meta, s, N, bias, act, meta_bits=4):
    import csed499ii_b200 as m
    from csed499ii_b200 import metadata_decode as md

    A_d = torch.from_numpy(A).to(DEV)
    meta_d = torch.from_numpy(meta).to(DEV)
    if meta_bits == 3:
        meta_d = md.pack(meta_d)
    C = torch.zeros((A.shape[0], N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    m.mul_2_4_epilogue(A_d, torch.from_numpy(B).to(DEV), meta_d, C, torch.from_numpy(s).to(DEV), ws,
                       bias=bias, activation=act, meta_bits=meta_bits)
    torch.cuda.synchronize()
    assert int(ws.abs().sum().item()) == 0
    return C


def _ref(A, W, bias, act):
    x = torch.from_numpy(A).to(DEV).float() @ torch.from_numpy(W).to(DEV).float()
    if bias is not None:
        x = x + bias.float()
    return ACTS[act](x)


def _check(C, ref):
    rel_mae, rel_fro, _ = errors(C, ref)
    assert torch.isfinite(C).all()
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL, (rel_mae, rel_fro)


def _bias(N, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    return torch.randn((N,), dtype=torch.half, device=DEV, generator=g) * 2


# (K, N, M, groupsize): decode (M <= 64), CTA-pair prefill (K % 128 == 0),
# dense-expansion prefill (K % 128 != 0, per-column scales)
SHAPES = [(4096, 4096, 1, 128), (1024, 384, 16, -1), (2048, 1024, 64, 128),
          (1024, 1024, 300, 128), (512, 512, 200, -1), (704, 512, 160, -1)]


@pytest.mark.parametrize("act", list(ACTS))
@pytest.mark.parametrize("with_bias", [True, False])
@pytest.mark.parametrize("K,N,M,g", SHAPES)
def test_epilogue_matches_composition(K, N, M, g, act, with_bias):
    if act == "none" and not with_bias:
        pytest.skip("plain GEMM: covered by the GEMM parity tests")
    if g == -1:
        W, B, s, meta = quantized_problem(N, K, -1, seed=K + N + M)
    else:
        W, B, s, meta = random_packed_problem(N, K, 128, seed=K + N + M)
    A = activations(M, K, seed=M + 3)
    bias = _bias(N, K + M) if with_bias else None
    _check(_run(A, B, meta, s, N, bias, act), _ref(A, W, bias, act))


@pytest.mark.parametrize("M", [16, 100])
def test_epilogue_three_bit_metadata(M):
    K, N = 2048, 1024
    W, B, s, meta = random_packed_problem(N, K, 128, seed=M + 11)
    A = activations(M, K, seed=M + 4)
    bias = _bias(N, M)
    _check(_run(A, B, meta, s, N, bias, "silu", meta_bits=3), _ref(A, W, bias, "silu"))


def test_epilogue_argument_errors():
    import csed499ii_b200 as m

    K, N, M = 256, 256, 4
    W, B, s, meta = random_packed_problem(N, K, 128, seed=1)
    A = torch.from_numpy(activations(M, K, seed=1)).to(DEV)
    C = torch.zeros((M, N), dtype=torch.half, device=DEV)
    ws = torch.zeros(N // 128 * 16, dtype=torch.int32, device=DEV)
    args = (A, torch.from_numpy(B).to(DEV), torch.from_numpy(meta).to(DEV), C,
            torch.from_numpy(s).to(DEV), ws)
    with pytest.raises(ValueError, match="activation"):
        m.mul_2_4_epilogue(*args, activation="tanh")
    with pytest.raises(RuntimeError, match="bias must have"):
        m.mul_2_4_epilogue(*args, bias=torch.zeros(N - 8, dtype=torch.half, device=DEV))
    lib = m._ext.load()
    # unknown activation code and unaligned bias through the C ABI
    assert lib.sm100_marlin_mul_2_4_epilogue(A.data_ptr(), args[1].data_ptr(), args[2].data_ptr(),
                                             C.data_ptr(), args[4].data_ptr(), N, M, K,
                                             ws.data_ptr(), 64, 0, None, -1, -1, -1, 16, 4, None,
                                             7) == m._ext.ERR_ARGUMENT
    bias = torch.zeros(N + 8, dtype=torch.half, device=DEV)
    assert lib.sm100_marlin_mul_2_4_epilogue(A.data_ptr(), args[1].data_ptr(), args[2].data_ptr(),
                                             C.data_ptr(), args[4].data_ptr(), N, M, K,
                                             ws.data_ptr(), 64, 0, None, -1, -1, -1, 16, 4,
                                             bias.data_ptr() + 2, 1) == m._ext.ERR_ALIGNMENT


class _Lin:
    def __init__(self, w, b):
        self.weight = nn.Parameter(w, requires_grad=False)
        self.bias = nn.Parameter(b, requires_grad=False)


@pytest.mark.parametrize("M", [8, 300])
def test_layer_with_bias_and_activation(M):
    from csed499ii_b200 import Layer_2_4

    K, N, g = 1024, 512, 128
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    s = O.group_scales(w, g)
    b = torch.randn((N,), dtype=torch.half, device=DEV)
    layer = Layer_2_4(K, N, groupsize=g, bias=True, activation="gelu_tanh").to(DEV)
    layer.pack(_Lin(torch.from_numpy(w).to(DEV), b), torch.from_numpy(s).to(DEV))
    A = torch.randn((M, K), dtype=torch.half, device=DEV)
    C = layer(A)
    W = torch.from_numpy(O.dequant_2_4(*O.pack_2_4(w, s, g), K, N, g)).to(DEV).float()
    ref = F.gelu(A.float() @ W + b.float(), approximate="tanh")
    rel_mae, rel_fro, _ = errors(C, ref)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL
    # the bias is a buffer: it survives a state_dict round trip
    buf = io.BytesIO()
    torch.save(layer.state_dict(), buf)
    buf.seek(0)
    fresh = Layer_2_4(K, N, groupsize=g, bias=True, activation="gelu_tanh").to(DEV)
    fresh.load_state_dict(torch.load(buf))
    assert torch.equal(fresh(A), C)
