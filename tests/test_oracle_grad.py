"""The oracle's backward restatement against gradients the reference computed.

The fixtures (tests/golden/grad_*.npz, made by ``make_golden.py --grad``)
hold what autograd gave through the reference's own SparseMoESwiGLU on CPU
with the loss of its equivalence test (scripts/test_moe_shard_equivalence.py
:227-232: sum(y * grad_y) + sum(aux_losses)): the gradients of x, of the
router weight (and bias) and of both expert weights, the aux loss and the
expert counts.  ``oracle.moe_backward`` must reproduce them: fp32 within
1e-4 max-relative per tensor, bf16 within 1e-2 (the task's tolerances).
"""
import json

import numpy as np
import pytest

from _helpers import GOLDEN, synthetic
from oracle import moe_oracle as O

import make_golden

TOL = {"f32": 1e-4, "bf16": 1e-2}


def _load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    ref = {}
    for key in z.files:
        if key == "meta":
            continue
        a = z[key]
        ref[key] = synthetic().from_bf16_bits(a) if a.dtype == np.uint16 else a.astype(np.float32)
    return ref, meta


@pytest.mark.parametrize("name", list(make_golden.GRAD_CASES))
def test_oracle_backward_matches_reference_autograd(name):
    ref, meta = _load(name)
    inp, grad_y = make_golden.grad_case_inputs(name)
    for key, val in make_golden.checksums(inp).items():
        assert val == pytest.approx(meta["checksums"][key], rel=1e-12), key
    dtype = meta["dtype"]
    o = O.moe_backward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, meta["k"], meta["norm"],
                       dtype, grad_y, router_bias=inp.router_bias, aux_grad=1.0,
                       valid_tokens=meta["valid_tokens"])
    fwd = O.moe_forward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, meta["k"], meta["norm"],
                        dtype, inp.router_bias)
    assert O.max_rel(fwd["y"], ref["y"]) <= TOL[dtype]
    assert o["aux"] == pytest.approx(float(ref["aux"][0]), rel=1e-5)
    _, counts = O.aux_loss(o["probs"], o["topk_idx"], meta["E"], meta["valid_tokens"])
    assert np.array_equal(counts, ref["expert_counts"][0])
    keys = ["dx", "d_w_router", "d_w_gate_up", "d_w_down"]
    if inp.router_bias is not None:
        keys.append("d_bias")
    for key in keys:
        err = O.max_rel(o[key], ref[key])
        assert err <= TOL[dtype], (key, err)
