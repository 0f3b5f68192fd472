"""hmoe_dispatch_noalloc: the dispatch stage for callers that cannot allocate.

Some embedding hosts cannot give this library device memory for scratch (a
plugin host without a CUDA allocator binding, a process whose device memory
another framework has already reserved, a serving loop that must not
allocate after start-up).  For them the library offers one entry point whose
scratch is a fixed __device__ array inside the library.  This test calls it
through the C ABI and checks that two calls in a row give exactly what the
workspace-based hmoe_dispatch gives (integer and byte outputs: bit-exact),
and that a call beyond the array's capacity is refused.  It is collected
last so a failure here leaves every other test already run.
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


def test_dispatch_noalloc_matches_dispatch_on_two_calls():
    lib = _lib()
    cases = [(3000, 64, 8, 512, 1), (32768, 128, 8, 64, 2)]  # the second fills the array
    for T, E, k, d, seed in cases:
        rng = np.random.default_rng(seed)
        idx = torch.from_numpy(random_topk(T, E, k, seed)).cuda()
        x = to_dev(O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32)), "bf16")
        w = to_dev(O.round_to_bf16(rng.random((T, k), dtype=np.float32)), "bf16")
        ours = _noalloc(lib, idx, w, x, E)
        ref = get_ops().dispatch(idx, E, x, w)
        torch.cuda.synchronize()
        for key in ("sort_idx", "counts", "sorted_token", "sorted_weight", "x_sorted"):
            assert torch.equal(ours[key], ref[key]), key


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
