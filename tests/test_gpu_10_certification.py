"""The router's certification margin against measured tensor-core errors.

The bf16 router takes each logit from the tensor cores, whose fp32
accumulation order differs from the fixed order that defines the routing
(one fma per k within 64-wide blocks, blocks added in order).  A logit is
trusted to round like the fixed-order sum unless it lies within
margin = cert_rel * max|logit of the token| (cert_rel = 2^-16) of a bf16
rounding midpoint; tokens with any untrusted order decision are recomputed
in the fixed order.  The margin is not a worst-case bound, so this test
measures what it protects against: over many seeds, token counts, shapes
and value scales it compares the tensor-core sums (hmoe_router_topk_sums)
with the fixed-order fp32 sums of the oracle and records, for every logit,
|tc - exact| / margin.  The largest ratio seen must stay below 1/4 (the
margin covers four times the worst error measured), and the routing must be
the fixed-order routing on every token.
"""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from gpu_util import to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

CERT_REL = 2.0 ** -16
RATIO_LIMIT = 1.0 / 4

CASES = [
    # (T, d, E, k, x scale, w scale, seed, quantised weights)
    (16384, 1536, 64, 8, 1.0, 0.02, 0, False),
    (16384, 1536, 64, 8, 1.0, 0.02, 1, False),
    (16384, 1536, 64, 8, 3.0, 0.05, 2, False),
    (8192, 1536, 128, 8, 1.0, 0.02, 3, False),
    (8192, 1536, 128, 8, 1.0, 0.02, 4, True),
    (4096, 1280, 64, 8, 1.0, 0.02, 5, False),
    (4096, 2048, 64, 8, 0.5, 0.2, 6, False),
    (2048, 1000, 64, 8, 1.0, 0.02, 7, False),
    (2048, 24, 16, 4, 1.0, 0.3, 8, False),
]


def _sums(x, w, k):
    lib_mod = importlib.import_module("hrm-moe_b200._lib")
    ops = importlib.import_module("hrm-moe_b200.ops")
    lib = lib_mod.load()
    T, d = x.shape
    E = w.shape[0]
    shape = ops.make_shape(T, d, E, 8, k, torch.bfloat16, True)
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    wt = torch.empty((T, k), dtype=torch.bfloat16, device="cuda")
    sums = torch.empty((T, E), dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.hmoe_router_workspace_bytes(ctypes.byref(shape)), dtype=torch.uint8,
                     device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.hmoe_router_topk_sums(ctypes.byref(shape), p(x), p(w), None, p(idx), p(wt), None,
                                   p(sums), p(ws), ws.numel(),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib_mod.last_error()
    torch.cuda.synchronize()
    return to_np(idx).astype(np.int64), to_np(sums)


def test_tensor_core_error_stays_far_inside_the_margin():
    worst = []
    for T, d, E, k, xs, wsc, seed, quant in CASES:
        rng = np.random.default_rng(1000 + seed)
        x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32) * np.float32(xs))
        if quant:
            w = np.round(rng.standard_normal((E, d)).astype(np.float32) * 4) / np.float32(200)
        else:
            w = rng.standard_normal((E, d), dtype=np.float32) * np.float32(wsc)
        w = O.round_to_bf16(w.astype(np.float32))
        idx, tc = _sums(to_dev(x, "bf16"), to_dev(w, "bf16"), k)
        exact = O.router_logits(x, w, None, "f32")
        margin = CERT_REL * np.abs(exact).max(axis=1, keepdims=True)
        ratio = np.abs(tc.astype(np.float64) - exact) / margin
        worst.append((T, d, E, float(ratio.max()), float(np.median(ratio))))
        oidx, _, _ = O.route(O.round_to_bf16(exact), k, True, "bf16")
        assert np.array_equal(idx, oidx), (T, d, E, seed)
    print("\nmax / median |tc - exact| / margin per case:")
    for T, d, E, mx, med in worst:
        print(f"  T={T} d={d} E={E}: max {mx:.4f}, median {med:.5f}")
    assert max(w[3] for w in worst) < RATIO_LIMIT, worst
