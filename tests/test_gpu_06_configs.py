"""The stress configurations at their full sizes, on one GPU.

* cfg3: the XL 128x8 layer (E = 128) at T = 32768 tokens (the per-rank size
  of the reference's expert-parallel configuration, run here on one GPU).
* cfg4: the XL 64x8 layer at T = 65536 tokens with a router bias that makes
  expected expert selection follow Zipf(1.2) over a seeded permutation, with
  and without 4 dead experts (bias -inf: no token may reach them).

Routing indices, per-expert counts and the permutation are checked bit for
bit against the CPU oracle on every token (models/layers.py:605-610 and
:311-322); the layer output, which is independent per token, is checked on
a seeded token sample against the oracle's expert path (max-relative 1e-2,
the bf16 tolerance).
"""
import numpy as np
import pytest

from _helpers import synthetic
from gpu_util import get_ops, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _shape(cfg, T=None):
    base = synthetic().CONFIGS[cfg]
    return synthetic().MoEShape(T or base.tokens, base.hidden, base.experts, base.intermediate,
                                base.top_k, base.norm_topk_prob, base.dtype)


def _check_full(shape, seed, bias=None, sample=384):
    inp = synthetic().make_inputs(shape, seed=seed, router_bias=bias)
    ops = get_ops()
    y, r = ops.ffn_forward(to_dev(inp.x, "bf16"), to_dev(inp.w_router, "bf16"),
                           to_dev(inp.w_gate_up, "bf16"), to_dev(inp.w_down, "bf16"),
                           shape.top_k, True,
                           router_bias=None if bias is None else to_dev(bias, "bf16"),
                           return_routing=True)
    y = to_np(y)
    r = {key: to_np(v) for key, v in r.items()}
    logits = O.router_logits(inp.x, inp.w_router, bias, "bf16")
    oidx, ow, _ = O.route(logits, shape.top_k, True, "bf16")
    assert np.array_equal(r["topk_idx"].astype(np.int64), oidx)
    sort_idx, _, counts = O.dispatch(oidx, shape.experts)
    assert np.array_equal(r["counts"].astype(np.int64), counts)
    assert np.array_equal(r["sort_idx"].astype(np.int64), sort_idx)
    pick = np.random.default_rng(seed).choice(shape.tokens, sample, replace=False)
    ys = O.experts_forward(inp.x[pick], oidx[pick], ow[pick], inp.w_gate_up, inp.w_down, "bf16")
    assert O.max_rel(y[pick], ys) <= 1e-2
    assert np.isfinite(y).all()
    return counts


def test_cfg3_xl128_full_size_single_gpu():
    shape = _shape("cfg3_xl128_ep_bf16")
    assert (shape.tokens, shape.experts) == (32768, 128)
    counts = _check_full(shape, seed=3)
    assert counts.sum() == shape.assignments


@pytest.mark.parametrize("dead", [0, 4])
def test_cfg4_zipf_full_size(dead):
    shape = _shape("cfg4_xl64_zipf_bf16")
    assert shape.tokens == 65536
    bias = O.round_to_bf16(synthetic().zipf_router_bias(shape.experts, 4, dead_experts=dead))
    counts = _check_full(shape, seed=4, bias=bias)
    if dead:
        assert (counts[np.isinf(bias)] == 0).all()
        assert int((counts == 0).sum()) >= dead
    # the bias skews the load: the busiest expert gets several times the mean
    assert counts.max() > 3 * counts.mean()
