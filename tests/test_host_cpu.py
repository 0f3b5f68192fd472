"""Host-side logic that needs no GPU: module API parity and error behaviour."""
import sys
import types

import pytest
import torch

from _helpers import package


def test_module_parameter_layout_matches_reference():
    layers = package().layers
    m = layers.SparseMoESwiGLU(1536, 512, 64, 8, True, implementation="grouped_b200")
    sd = m.state_dict()
    assert tuple(sd["gate.weight"].shape) == (64, 1536)
    assert tuple(sd["experts.gate_up_weight"].shape) == (64, 1024, 1536)
    assert tuple(sd["experts.down_weight"].shape) == (64, 1536, 512)
    assert set(sd) == {"gate.weight", "experts.gate_up_weight", "experts.down_weight"}


def test_module_config_errors():
    layers = package().layers
    with pytest.raises(ValueError):
        layers.SparseMoESwiGLU(16, 32, 0, 1, True)
    with pytest.raises(ValueError):
        layers.SparseMoESwiGLU(16, 32, 8, 9, True)
    with pytest.raises(ValueError):
        layers.SparseMoESwiGLU(16, 32, 8, 2, True, expert_in_one_shard=3)
    with pytest.raises(ValueError):
        layers.SparseMoESwiGLU(16, 32, 8, 2, True, implementation="grouped_triton")


def test_no_cpu_path():
    ops = package().ops
    x = torch.zeros((4, 16))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.ffn_forward(x, torch.zeros((8, 16)), torch.zeros((8, 64, 16)), torch.zeros((8, 16, 32)),
                        2, True)
    with pytest.raises(TypeError):
        ops.dtype_code(torch.float16)


def test_forward_has_no_cpu_path_for_training():
    """With autograd recording the module runs the native training path; on
    CPU tensors that fails loudly (there is no CPU fallback)."""
    layers = package().layers
    m = layers.SparseMoESwiGLU(16, 32, 8, 2, True)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros((3, 16)))
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros((3, 16)), moe_context={})


def test_reference_state_dict_loads(tmp_path):
    """Weights laid out like the reference's grouped layer load unchanged."""
    layers = package().layers
    src = {"gate.weight": torch.randn(8, 16), "experts.gate_up_weight": torch.randn(8, 64, 16),
           "experts.down_weight": torch.randn(8, 16, 32)}
    m = layers.SparseMoESwiGLU(16, 32, 8, 2, True)
    m.load_state_dict(src)
    assert torch.equal(m.experts.down_weight, src["experts.down_weight"])


def test_init_matches_reference_distribution():
    """Parameters are drawn like the reference's trunc_normal_init_
    (models/common.py:10-13): N(0,1) folded into (-3, 3) by fmod, scaled to
    the requested std, so fresh layers have the reference's weight scale."""
    import torch
    layers = package().layers
    torch.manual_seed(0)
    mod = layers.SparseMoESwiGLU(256, 128, 16, 4, True, implementation="grouped_b200")
    for t, std in ((mod.gate.weight, 256 ** -0.5), (mod.experts.gate_up_weight, 256 ** -0.5),
                   (mod.experts.down_weight, 128 ** -0.5)):
        assert abs(float(t.std()) / std - 1.0) < 0.02
        assert float(t.abs().max()) <= 3.0 * 1.014762601732121 * std * (1 + 1e-6)
