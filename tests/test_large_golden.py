"""The full-size XL 64x8 layer (T = 16384) against the reference on a B200.

tests/golden/xl64_t16384_gpu_bf16.npz was made by running the reference's
own SparseMoESwiGLU(implementation="grouped_triton") on a B200
(``make_golden.py --large``): its cuBLAS router logits, its routing and
counts, and its output on a seeded sample of tokens.

bf16 logits tie often at this size: about one row in eight has its k-th and
(k+1)-th logits equal, and torch.topk then picks either expert, while this
build (and the oracle) pick the lower index.  Such rows are "tie-only": the
selected logit values are the same on both sides.  A row may also differ
because cuBLAS and the fixed-order sum round one logit to neighbouring bf16
values; that is only possible where the two boundary logits are within a
bf16 step or two, so every such row must be one of the fixture's near-tie
rows.  Every other row must match exactly, and the output of sample tokens
with the same routing must be within the bf16 tolerance (1e-2 max-relative).
"""
import json

import numpy as np
import pytest

from _helpers import GOLDEN, synthetic
from oracle import moe_oracle as O

import make_golden

NAME = "xl64_t16384_gpu_bf16"


def _load():
    z = np.load(GOLDEN / f"{NAME}.npz")
    meta = json.loads(str(z["meta"]))
    syn = synthetic()
    ref = {"topk_idx": z["topk_idx"].astype(np.int64), "counts": z["counts"].astype(np.int64),
           "topk_weight": syn.from_bf16_bits(z["topk_weight"]), "sample": z["sample"].astype(np.int64),
           "y_sample": syn.from_bf16_bits(z["y_sample"]),
           "near_tie_rows": z["near_tie_rows"].astype(np.int64),
           "near_tie_logits": syn.from_bf16_bits(z["near_tie_logits"])}
    return ref, meta


def _classify(ours_idx, ours_logits, ref):
    """Rows differing from the reference, split into (order-only, tie-only,
    near-tie); anything else fails.

    order-only: the same experts in another order (equal logits inside the
    top k, which torch.topk orders either way); tie-only: equal logits at the
    k / k+1 boundary, resolved to the other expert; near-tie: the reference's
    logits of the two picks within two bf16 steps.
    """
    diff = np.nonzero((ours_idx != ref["topk_idx"]).any(axis=1))[0]
    pos = {int(r): i for i, r in enumerate(ref["near_tie_rows"])}
    order_only, tie_only, near = 0, 0, 0
    for r in diff:
        if np.array_equal(np.sort(ours_idx[r]), np.sort(ref["topk_idx"][r])):
            # same set: our order is by logit, then lower index; the swapped
            # experts must carry equal logits
            lv = ours_logits[r][ours_idx[r]]
            assert (np.diff(lv) <= 0).all(), r
            order_only += 1
            continue
        assert int(r) in pos, f"row {r} picks other experts but is not a near-tie row"
        rl = ref["near_tie_logits"][pos[int(r)]]
        ours_vals = np.sort(rl[ours_idx[r]])
        ref_vals = np.sort(rl[ref["topk_idx"][r]])
        if np.array_equal(ours_vals, ref_vals):
            tie_only += 1
        else:
            # a logit rounded to the neighbouring bf16 value: the two picks
            # differ by at most two bf16 steps in the reference's own logits
            step = np.spacing(np.abs(ref_vals).max()).astype(np.float32) * 65536
            assert np.abs(ours_vals - ref_vals).max() <= 2 * step, r
            near += 1
    return order_only, tie_only, near


def _inputs(meta):
    inp = make_golden.large_case_inputs(NAME)
    for key, val in make_golden.checksums(inp).items():
        assert val == pytest.approx(meta["checksums"][key], rel=1e-12), key
    return inp


def test_oracle_matches_reference_on_gpu_at_full_size():
    ref, meta = _load()
    inp = _inputs(meta)
    logits = O.router_logits(inp.x, inp.w_router, None, "bf16")
    idx, w, _ = O.route(logits, meta["k"], True, "bf16")
    order_only, tie_only, near = _classify(idx.astype(np.int64), logits, ref)
    assert near <= 0.01 * meta["T"], (order_only, tie_only, near)
    same = (idx == ref["topk_idx"]).all(axis=1)
    pick = ref["sample"][same[ref["sample"]]]
    y = O.experts_forward(inp.x[pick], idx[pick], w[pick], inp.w_gate_up, inp.w_down, "bf16")
    sel = np.isin(ref["sample"], pick)
    assert O.max_rel(y, ref["y_sample"][sel]) <= 1e-2


@pytest.mark.gpu
def test_layer_matches_reference_on_gpu_at_full_size():
    from gpu_util import get_ops, to_dev, to_np
    ref, meta = _load()
    inp = _inputs(meta)
    y, r = get_ops().ffn_forward(to_dev(inp.x, "bf16"), to_dev(inp.w_router, "bf16"),
                                 to_dev(inp.w_gate_up, "bf16"), to_dev(inp.w_down, "bf16"),
                                 meta["k"], True, return_routing=True)
    idx = to_np(r["topk_idx"]).astype(np.int64)
    logits = O.router_logits(inp.x, inp.w_router, None, "bf16")
    order_only, tie_only, near = _classify(idx, logits, ref)
    assert near <= 0.01 * meta["T"], (order_only, tie_only, near)
    same = (idx == ref["topk_idx"]).all(axis=1)
    # the oracle's routing is exact on every row (the other tests pin it),
    # so counts differ from the reference's only through tie and near-tie rows
    if tie_only + near == 0:
        assert np.array_equal(to_np(r["counts"]).astype(np.int64), ref["counts"])
    sel = same[ref["sample"]]
    ys = to_np(y)[ref["sample"][sel]]
    assert O.max_rel(ys, ref["y_sample"][sel]) <= 1e-2
