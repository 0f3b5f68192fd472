"""Dispatch (stable permutation, counts, gather) vs the oracle: bit-exact."""
import numpy as np
import pytest
import torch

from _helpers import golden_names, load_golden
from gpu_util import get_ops, random_topk, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _check(idx: np.ndarray, E: int, x: np.ndarray, w: np.ndarray, dtype: str):
    ops = get_ops()
    out = ops.dispatch(torch.from_numpy(idx).cuda(), E, to_dev(x, dtype), to_dev(w, dtype))
    sort_idx, sorted_token, counts = O.dispatch(idx, E)
    assert np.array_equal(to_np(out["sort_idx"]).astype(np.int64), sort_idx)
    assert np.array_equal(to_np(out["counts"]).astype(np.int64), counts)
    assert np.array_equal(to_np(out["sorted_token"]).astype(np.int64), sorted_token)
    assert np.array_equal(to_np(out["x_sorted"]), x[sorted_token])
    assert np.array_equal(to_np(out["sorted_weight"]), w.reshape(-1)[sort_idx])


@pytest.mark.parametrize("name", golden_names())
def test_dispatch_reference_routing(name):
    inp, ref, meta = load_golden(name)
    idx = ref["topk_idx"].astype(np.int32)
    _check(idx, meta["E"], inp.x, ref["topk_weight"], meta["dtype"])
    # the reference's own permutation and counts
    out = get_ops().dispatch(torch.from_numpy(idx).cuda(), meta["E"])
    assert np.array_equal(to_np(out["sort_idx"]).astype(np.int64), ref["sort_idx"])
    assert np.array_equal(to_np(out["counts"]).astype(np.int64), ref["counts"])


@pytest.mark.parametrize("T,E,k,d,dtype", [
    (1, 64, 8, 64, "bf16"),
    (129, 64, 8, 1536, "bf16"),
    (1000, 128, 8, 256, "bf16"),
    (5000, 64, 8, 128, "f32"),
    (333, 8, 3, 16, "bf16"),
    (20000, 64, 1, 64, "bf16"),
    (300, 64, 32, 64, "f32"),
])
def test_dispatch_random(T, E, k, d, dtype):
    rng = np.random.default_rng(T + E + k)
    idx = random_topk(T, E, k, seed=T)
    x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w = O.round_to_bf16(rng.random((T, k), dtype=np.float32))
    _check(idx, E, x, w, dtype)


def test_dispatch_skewed_and_duplicates():
    # every token on the same two experts (huge groups, most experts empty),
    # and rows naming one expert twice: the result is still the stable sort
    T, E, k = 4096, 64, 4
    idx = np.zeros((T, k), np.int32)
    idx[:, 1] = 63
    idx[:, 2] = 0
    idx[:, 3] = np.arange(T) % 7
    x = O.round_to_bf16(np.random.default_rng(0).standard_normal((T, 64), dtype=np.float32))
    w = np.ones((T, k), np.float32)
    _check(idx, E, x, w, "bf16")


def test_dispatch_full_size_properties():
    # XL 64x8 at 16K tokens: permutation is a bijection sorted by expert
    T, E, k = 16384, 64, 8
    idx = random_topk(T, E, k, seed=99)
    out = get_ops().dispatch(torch.from_numpy(idx).cuda(), E)
    s = to_np(out["sort_idx"]).astype(np.int64)
    assert np.array_equal(np.sort(s), np.arange(T * k))
    flat = idx.reshape(-1)
    assert (np.diff(flat[s]) >= 0).all()
    same = np.diff(flat[s]) == 0
    assert (np.diff(s)[same] > 0).all()
    assert np.array_equal(to_np(out["counts"]), np.bincount(flat, minlength=E))
