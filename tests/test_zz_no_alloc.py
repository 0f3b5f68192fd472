"""hmoe_dispatch_noalloc: the dispatch stage for callers that cannot allocate.

Some embedding hosts cannot give this library device memory for scratch (a
plugin host without a CUDA allocator binding, a process whose device memory
another framework has already reserved, a serving loop that must not
allocate after start-up).  For them the library offers one entry point whose
scratch is a fixed __device__ array inside the library.  These tests call it
through the C ABI and check that calls in a row give exactly what the
workspace-based hmoe_dispatch gives and what the CPU oracle's stable sort
gives (integer and byte outputs: bit-exact), including top_k other than 8,
expert ids outside [0, E) (dropped: counts leave them out and only the
first sum(counts) sorted entries are written), an empty call (counts become
E zeros) and a call beyond the array's capacity (refused).  The file is
collected last so a failure here leaves every other test already run.
"""
import ctypes
import errno
import importlib

import numpy as np
import pytest
import torch

from gpu_util import get_ops, random_topk, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    return importlib.import_module("hrm-moe_b200._lib")


def _noalloc(lib, idx, w, x, E):
    T, k = idx.shape
    d = x.shape[1]
    shape = lib.HmoeShape(T, d, E, 8, k, 0, 1)
    dev = idx.device
    out = {
        "sort_idx": torch.full((T * k,), -7, dtype=torch.int32, device=dev),
        "counts": torch.full((E,), -7, dtype=torch.int32, device=dev),
        "sorted_token": torch.full((T * k,), -7, dtype=torch.int32, device=dev),
        "sorted_weight": torch.zeros(T * k, dtype=torch.bfloat16, device=dev),
        "x_sorted": torch.zeros((T * k, d), dtype=torch.bfloat16, device=dev),
    }
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.load().hmoe_dispatch_noalloc(
        ctypes.byref(shape), p(idx), p(w), p(x), p(out["sort_idx"]), p(out["counts"]),
        p(out["sorted_token"]), p(out["sorted_weight"]), p(out["x_sorted"]),
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == 0, lib.last_error()
    return out


def _inputs(T, E, k, d, seed):
    rng = np.random.default_rng(seed)
    idx_np = random_topk(T, E, k, seed)
    x_np = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w_np = O.round_to_bf16(rng.random((T, k), dtype=np.float32))
    return idx_np, x_np, w_np


def _check_against_oracle(ours, idx_np, x_np, w_np, E):
    sort_idx, sorted_token, counts = O.dispatch(idx_np, E)
    assert np.array_equal(to_np(ours["sort_idx"]).astype(np.int64), sort_idx)
    assert np.array_equal(to_np(ours["sorted_token"]).astype(np.int64), sorted_token)
    assert np.array_equal(to_np(ours["counts"]).astype(np.int64), counts)
    assert np.array_equal(to_np(ours["sorted_weight"]), w_np.reshape(-1)[sort_idx])
    assert np.array_equal(to_np(ours["x_sorted"]), x_np[sorted_token])


def test_dispatch_noalloc_matches_dispatch_and_oracle_on_calls_in_a_row():
    lib = _lib()
    # (T, E, k, d, seed); the 32768 x 8 case fills the array to its limit
    cases = [(3000, 64, 8, 512, 1), (32768, 128, 8, 64, 2), (4000, 64, 2, 256, 3),
             (1000, 16, 6, 128, 4)]
    for T, E, k, d, seed in cases:
        idx_np, x_np, w_np = _inputs(T, E, k, d, seed)
        idx = torch.from_numpy(idx_np).cuda()
        x, w = to_dev(x_np, "bf16"), to_dev(w_np, "bf16")
        first = _noalloc(lib, idx, w, x, E)
        second = _noalloc(lib, idx, w, x, E)
        ref = get_ops().dispatch(idx, E, x, w)
        torch.cuda.synchronize()
        for key in ("sort_idx", "counts", "sorted_token", "sorted_weight", "x_sorted"):
            assert torch.equal(first[key], ref[key]), (T, k, key)
            assert torch.equal(second[key], ref[key]), (T, k, key)
        _check_against_oracle(second, idx_np, x_np, w_np, E)


def test_dispatch_noalloc_drops_out_of_range_ids_like_dispatch():
    lib = _lib()
    T, E, k, d = 2000, 64, 8, 128
    idx_np, x_np, w_np = _inputs(T, E, k, d, 11)
    rng = np.random.default_rng(12)
    bad = rng.choice(T * k, 37, replace=False)
    flat = idx_np.reshape(-1).copy()
    flat[bad[:20]] = E + 5
    flat[bad[20:]] = -3
    idx_np = flat.reshape(T, k)
    idx = torch.from_numpy(idx_np).cuda()
    x, w = to_dev(x_np, "bf16"), to_dev(w_np, "bf16")
    ours = _noalloc(lib, idx, w, x, E)
    ref = get_ops().dispatch(idx, E, x, w)
    torch.cuda.synchronize()
    counts = to_np(ours["counts"]).astype(np.int64)
    valid = (flat >= 0) & (flat < E)
    assert np.array_equal(counts, np.bincount(flat[valid], minlength=E))
    assert torch.equal(ours["counts"], ref["counts"])
    n = int(counts.sum())
    assert n == T * k - 37
    for key in ("sort_idx", "sorted_token", "sorted_weight", "x_sorted"):
        assert torch.equal(ours[key][:n], ref[key][:n]), key
    # the valid assignments in stable expert order
    order = np.argsort(np.where(valid, flat, E + 1000), kind="stable")[:n]
    assert np.array_equal(to_np(ours["sort_idx"][:n]).astype(np.int64), order)


def test_dispatch_noalloc_empty_call_zeroes_counts():
    lib = _lib()
    E = 64
    shape = lib.HmoeShape(0, 128, E, 8, 8, 0, 1)
    counts = torch.full((E,), -7, dtype=torch.int32, device="cuda")
    rc = lib.load().hmoe_dispatch_noalloc(ctypes.byref(shape), None, None, None, None,
                                         ctypes.c_void_p(counts.data_ptr()), None, None, None,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(counts, torch.zeros_like(counts))


def test_dispatch_noalloc_refuses_oversize():
    lib = _lib()
    so = lib.load()
    limit = 262144
    T, k = limit // 8 + 1, 8
    shape = lib.HmoeShape(T, 64, 64, 8, k, 0, 1)
    idx = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    sort_idx = torch.empty(T * k, dtype=torch.int32, device="cuda")
    rc = so.hmoe_dispatch_noalloc(ctypes.byref(shape), ctypes.c_void_p(idx.data_ptr()), None,
                                  None, ctypes.c_void_p(sort_idx.data_ptr()), None, None, None,
                                  None, None)
    assert rc == errno.EINVAL
    assert "at most 262144" in lib.last_error()
