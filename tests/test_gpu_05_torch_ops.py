"""torch.ops.hrm_moe.* on the GPU: same bits as the ops they wrap, and the
oracle's routing."""
import importlib

import numpy as np
import pytest
import torch

from _helpers import synthetic
from gpu_util import get_ops, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def test_ffn_forward_op_matches_ops_and_oracle():
    importlib.import_module("hrm-moe_b200.torch_ops")
    ops = get_ops()
    syn = synthetic()
    shape = syn.MoEShape(700, 1536, 64, 512, 8, True, "bf16")
    inp = syn.make_inputs(shape, seed=31)
    args = [to_dev(a, "bf16") for a in (inp.x, inp.w_router, inp.w_gate_up, inp.w_down)]
    y, idx, w, counts, perm = torch.ops.hrm_moe.ffn_forward(*args, 8, True, None)
    y2, r = ops.ffn_forward(*args, 8, True, return_routing=True)
    assert torch.equal(y, y2)
    assert torch.equal(idx, r["topk_idx"]) and torch.equal(w, r["topk_weight"])
    assert torch.equal(counts, r["counts"]) and torch.equal(perm, r["sort_idx"])
    ol = O.router_logits(inp.x, inp.w_router, None, "bf16")
    oidx, _, _ = O.route(ol, 8, True, "bf16")
    assert np.array_equal(to_np(idx).astype(np.int64), oidx)
    operm, _, ocounts = O.dispatch(oidx, 64)
    assert np.array_equal(to_np(perm).astype(np.int64), operm)
    assert np.array_equal(to_np(counts).astype(np.int64), ocounts)


def test_grouped_linear_op_matches_ops():
    importlib.import_module("hrm-moe_b200.torch_ops")
    ops = get_ops()
    g = torch.Generator(device="cuda").manual_seed(3)
    counts = torch.tensor([0, 130, 7, 300], dtype=torch.int64, device="cuda")
    M = int(counts.sum())
    a = torch.randn(M, 256, generator=g, device="cuda").bfloat16()
    wt = (torch.randn(4, 384, 256, generator=g, device="cuda") * 0.05).bfloat16()
    assert torch.equal(torch.ops.hrm_moe.grouped_linear(a, wt, counts), ops.grouped_linear(a, wt, counts))


def test_captured_forward_replays_the_same_kernels():
    ops = get_ops()
    syn = synthetic()
    shape = syn.MoEShape(1000, 1536, 64, 512, 8, True, "bf16")
    a = syn.make_inputs(shape, seed=41)
    b = syn.make_inputs(shape, seed=42)
    w = [to_dev(t, "bf16") for t in (a.w_router, a.w_gate_up, a.w_down)]
    xa, xb = to_dev(a.x, "bf16"), to_dev(b.x, "bf16")
    cap = ops.CapturedFfn(xa, *w, 8, True)
    ya = cap().clone()
    yb = cap(xb).clone()
    ya2 = cap(xa).clone()
    assert torch.equal(ya, ops.ffn_forward(xa, *w, 8, True))
    assert torch.equal(yb, ops.ffn_forward(xb, *w, 8, True))
    assert torch.equal(ya2, ya)
    with pytest.raises(ValueError):
        cap(xa[:10])
