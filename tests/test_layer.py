"""Layer_2_4 / replace_linear module surface (CPU): construction checks,
buffers and state_dict keys, and the reference's replacement traversal
(``kernel_experiments/sparse_marlin/src/marlin/__init__.py:274-415``)."""
import pytest
import torch
import torch.nn as nn

from csed499ii_b200 import Layer_2_4, replace_linear


def test_constructor_checks():
    with pytest.raises(ValueError, match="groupsize"):
        Layer_2_4(256, 256, groupsize=64)
    with pytest.raises(ValueError, match="divisible"):
        Layer_2_4(200, 256)
    with pytest.raises(ValueError, match="divisible"):
        Layer_2_4(256, 320)


@pytest.mark.parametrize("g", [-1, 128])
def test_buffers_and_state_dict(g):
    layer = Layer_2_4(512, 768, groupsize=g)
    assert layer.B.shape == (512 // 32, 2 * 768) and layer.B.dtype == torch.int32
    assert layer.meta.shape == (768, 512 // 16) and layer.meta.dtype == torch.int16
    assert layer.s.shape == ((1 if g == -1 else 512 // 128), 768) and layer.s.dtype == torch.half
    assert set(layer.state_dict()) == {"B", "meta", "s"}  # workspace is not persistent
    assert layer.workspace.numel() == 768 // 128 * 16 and int(layer.workspace.abs().sum()) == 0


class Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(256, 512, bias=False)
        self.o_proj = nn.Linear(512, 256, bias=False)
        self.inner = nn.Module()
        self.inner.up = nn.Linear(256, 1024, bias=False)
        self.norm = nn.LayerNorm(256)


def test_replace_linear_traversal_and_filter():
    net = Block()
    replace_linear(net, name_filter=lambda n: n != "o_proj", groupsize=128)
    assert isinstance(net.q_proj, Layer_2_4) and (net.q_proj.k, net.q_proj.n) == (256, 512)
    assert isinstance(net.o_proj, nn.Linear)
    assert isinstance(net.inner.up, Layer_2_4) and net.inner.up.groupsize == 128
    assert isinstance(net.norm, nn.LayerNorm)
    replace_linear(net)  # idempotent on already replaced layers
    assert isinstance(net.q_proj, Layer_2_4)
