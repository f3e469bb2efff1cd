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


# Extension (not in the reference): a bias buffer and a fused activation.
def test_bias_and_activation_options():
    with pytest.raises(ValueError, match="activation"):
        Layer_2_4(256, 256, activation="tanh")
    plain = Layer_2_4(256, 256)
    assert plain.bias is None and plain.activation == "none"
    layer = Layer_2_4(256, 512, groupsize=128, bias=True, activation="silu")
    assert layer.bias.shape == (512,) and layer.bias.dtype == torch.half
    assert set(layer.state_dict()) == {"B", "meta", "s", "bias"}


def test_replace_linear_keep_bias():
    m = nn.Module()
    m.a = nn.Linear(256, 512, bias=True)
    m.b = nn.Linear(256, 512, bias=False)
    replace_linear(m, keep_bias=True)
    assert m.a.bias is not None and m.b.bias is None
    m2 = nn.Module()
    m2.a = nn.Linear(256, 512, bias=True)
    replace_linear(m2)  # the reference's behaviour: biases are dropped
    assert m2.a.bias is None


def test_epilogue_argument_checks_before_the_gpu():
    import csed499ii_b200 as marlin

    assert marlin.ACTIVATIONS == {"none": 0, "relu": 1, "silu": 2, "gelu_tanh": 3}
    t = torch.zeros(1)
    with pytest.raises(ValueError, match="activation"):
        marlin.mul_2_4_epilogue(t, t, t, t, t, t, activation="swish")
    with pytest.raises(ValueError, match="meta_bits"):
        marlin.mul_2_4_epilogue(t, t, t, t, t, t, meta_bits=2)
