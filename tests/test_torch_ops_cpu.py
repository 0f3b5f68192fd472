"""torch.ops.hrm_moe.* registration: schema, fake (meta) shapes, no CPU path."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from _helpers import package


@pytest.fixture(scope="module")
def tops():
    package()
    import importlib
    return importlib.import_module("hrm-moe_b200.torch_ops")


def test_ops_are_registered(tops):
    assert hasattr(torch.ops.hrm_moe, "ffn_forward")
    assert hasattr(torch.ops.hrm_moe, "grouped_linear")
    schema = str(torch.ops.hrm_moe.ffn_forward.default._schema)
    assert "top_k" in schema and "router_bias" in schema


def test_fake_shapes(tops):
    T, d, E, I, k = 96, 64, 16, 32, 4
    with FakeTensorMode():
        x = torch.empty(T, d, dtype=torch.bfloat16)
        y, idx, w, counts, perm = torch.ops.hrm_moe.ffn_forward(
            x, torch.empty(E, d, dtype=torch.bfloat16), torch.empty(E, 2 * I, d, dtype=torch.bfloat16),
            torch.empty(E, d, I, dtype=torch.bfloat16), k, True, None)
        assert y.shape == (T, d) and y.dtype == torch.bfloat16
        assert idx.shape == (T, k) and idx.dtype == torch.int32
        assert w.shape == (T, k) and w.dtype == torch.bfloat16
        assert counts.shape == (E,) and perm.shape == (T * k,)
        out = torch.ops.hrm_moe.grouped_linear(torch.empty(T, d, dtype=torch.bfloat16),
                                               torch.empty(E, I, d, dtype=torch.bfloat16),
                                               torch.empty(E, dtype=torch.int64))
        assert out.shape == (T, I)


def test_cpu_tensors_are_refused(tops):
    T, d, E, I, k = 8, 16, 4, 8, 2
    x = torch.randn(T, d)
    with pytest.raises(RuntimeError):
        torch.ops.hrm_moe.ffn_forward(x, torch.randn(E, d), torch.randn(E, 2 * I, d),
                                      torch.randn(E, d, I), k, True, None)
