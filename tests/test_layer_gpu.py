"""GPU packer and Layer_2_4 end to end.

``sm100_marlin_pack_2_4`` must produce the reference packer's bytes: checked
against the oracle restatement (pinned to the reference) on random weights and
against the golden fixtures written by the reference's own ``Layer_2_4.pack``.
Then a packed layer must multiply like the oracle and survive a state_dict
round trip.
"""
import io
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

import marlin24_oracle as O
from conftest import GOLDEN, golden_cases
from csed499ii_b200 import Layer_2_4, replace_linear
from problems import REL_FRO_TOL, REL_MAE_TOL, errors

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


class _Lin:
    def __init__(self, w):
        self.weight = nn.Parameter(w, requires_grad=False)


def _pack_gpu(w_kn, s, g):
    K, N = w_kn.shape
    layer = Layer_2_4(K, N, groupsize=g).to(DEV)
    layer.pack(_Lin(torch.from_numpy(w_kn).to(DEV)), torch.from_numpy(s).to(DEV))
    torch.cuda.synchronize()
    return layer


@pytest.mark.parametrize("K,N,g", [(256, 256, 128), (512, 768, -1), (1024, 512, 128),
                                   (4096, 4096, 128)])
def test_pack_matches_oracle(K, N, g):
    rng = np.random.default_rng(K + N)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    s = O.group_scales(w, g)
    B, meta, s_p = O.pack_2_4(w, s, g)
    layer = _pack_gpu(w, s, g)
    np.testing.assert_array_equal(layer.B.cpu().numpy(), B)
    np.testing.assert_array_equal(layer.meta.cpu().numpy(), meta)
    np.testing.assert_array_equal(layer.s.cpu().numpy().view(np.uint16), s_p.view(np.uint16))


@pytest.mark.parametrize("name", [n for n in golden_cases() if "k192" not in n])
def test_pack_matches_reference_fixtures(name):
    # the fixtures hold the reference's pack of the fake-quantised weight
    z = np.load(os.path.join(GOLDEN, name))
    K, N, g = int(z["K"]), int(z["N"]), int(z["groupsize"])
    codes = O.quantize_codes(z["w"], z["s_raw"], g)
    ref_w = O.dequant_codes(codes, z["s_raw"], g)
    layer = _pack_gpu(ref_w, z["s_raw"].reshape(-1, N).astype(np.float16), g)
    np.testing.assert_array_equal(layer.B.cpu().numpy(), z["B"])
    np.testing.assert_array_equal(layer.meta.cpu().numpy(), z["meta"])
    np.testing.assert_array_equal(layer.s.cpu().numpy().view(np.uint16), z["s"].view(np.uint16))


@pytest.mark.parametrize("M", [1, 16, 200])
def test_layer_forward_and_state_dict_round_trip(M):
    K, N, g = 1024, 512, 128
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    s = O.group_scales(w, g)
    layer = _pack_gpu(w, s, g)
    A = torch.randn((2, M, K), dtype=torch.half, device=DEV)
    C = layer(A)
    assert C.shape == (2, M, N)
    W = torch.from_numpy(O.dequant_2_4(*O.pack_2_4(w, s, g), K, N, g)).to(DEV).float()
    rel_mae, rel_fro, _ = errors(C.view(-1, N), A.view(-1, K).float() @ W)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL
    buf = io.BytesIO()
    torch.save(layer.state_dict(), buf)
    buf.seek(0)
    fresh = Layer_2_4(K, N, groupsize=g).to(DEV)
    fresh.load_state_dict(torch.load(buf))
    assert torch.equal(fresh(A), C)


def test_replace_then_pack_a_block():
    torch.manual_seed(0)
    block = nn.Module()
    block.up = nn.Linear(512, 1024, bias=False)
    block.down = nn.Linear(1024, 512, bias=False)
    w_up = (block.up.weight.data.t().contiguous() * 0.5).half().numpy()
    w_dn = (block.down.weight.data.t().contiguous() * 0.5).half().numpy()
    replace_linear(block, groupsize=128)
    for lay, w in ((block.up, w_up), (block.down, w_dn)):
        lay.to(DEV)
        s = O.group_scales(w, 128)
        lay.pack(_Lin(torch.from_numpy(w).to(DEV)), torch.from_numpy(s).to(DEV))
    x = torch.randn((8, 512), dtype=torch.half, device=DEV)
    y = block.down(torch.relu(block.up(x)))
    ref_up = torch.from_numpy(O.dequant_2_4(*O.pack_2_4(w_up, O.group_scales(w_up, 128), 128),
                                            512, 1024, 128)).to(DEV).float()
    ref_dn = torch.from_numpy(O.dequant_2_4(*O.pack_2_4(w_dn, O.group_scales(w_dn, 128), 128),
                                            1024, 512, 128)).to(DEV).float()
    h = torch.relu((x.float() @ ref_up).half().float())
    rel_mae, rel_fro, _ = errors(y, h @ ref_dn)
    assert rel_mae < REL_MAE_TOL and rel_fro <= REL_FRO_TOL
