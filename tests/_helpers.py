"""Shared test helpers: package import, golden fixtures, tie-aware comparison."""
from __future__ import annotations

import functools
import importlib
import json
import pathlib

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"


def package():
    return importlib.import_module("hrm-moe_b200")


def synthetic():
    return importlib.import_module("hrm-moe_b200.synthetic")


def golden_names():
    import make_golden
    return list(make_golden.CASES)


@functools.lru_cache(maxsize=None)
def load_golden(name: str):
    """(inputs, reference outputs as float32/int arrays, meta)."""
    import make_golden
    syn = synthetic()
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    inp = make_golden.case_inputs(name)
    ref = {}
    for key in ("logits", "topk_weight", "y"):
        ref[key] = syn.from_bf16_bits(z[key]) if meta["dtype"] == "bf16" else z[key].astype(np.float32)
    for key in ("topk_idx", "sort_idx", "counts"):
        ref[key] = z[key].astype(np.int64)
    return inp, ref, meta


def routing_agrees(ours_idx, ours_logits, ref_idx, ref_logits, k):
    """Tie-aware routing comparison.

    Returns (exact_rows, tie_only_rows, real_mismatch_rows) boolean masks.
    A row is tie-only when the selected logit values, in selection order,
    are identical on both sides although the indices differ: the two sides
    broke an exact tie differently (the reference uses torch.topk's
    unspecified order, this build the lower expert index).
    """
    ours_idx = np.asarray(ours_idx, np.int64)
    ref_idx = np.asarray(ref_idx, np.int64)
    exact = (ours_idx == ref_idx).all(axis=1)
    ov = np.take_along_axis(ours_logits, ours_idx, axis=1)
    rv = np.take_along_axis(ref_logits, ref_idx, axis=1)
    same_values = (ov == rv).all(axis=1)
    tie_only = ~exact & same_values
    return exact, tie_only, ~exact & ~same_values
