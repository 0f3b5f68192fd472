"""Router kernel vs the oracle (bit-exact) and vs the reference (tie-aware)."""
import numpy as np
import pytest

from _helpers import golden_names, load_golden, routing_agrees, synthetic
from gpu_util import get_ops, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _run(x, w, bias, k, norm, dtype):
    ops = get_ops()
    bt = None if bias is None else to_dev(bias, dtype)
    idx, wt, logits = ops.router_topk(to_dev(x, dtype), to_dev(w, dtype), k, norm, bt,
                                      return_logits=True)
    return to_np(idx).astype(np.int64), to_np(wt), to_np(logits)


def _check_against_oracle(x, w, bias, k, norm, dtype):
    idx, wt, logits = _run(x, w, bias, k, norm, dtype)
    ol = O.router_logits(x, w, bias, dtype)
    oidx, ow, _ = O.route(ol, k, norm, dtype)
    # the routing is the exact-order routing, bit for bit
    assert np.array_equal(idx, oidx)
    fin = np.isfinite(ol)
    assert np.array_equal(fin, np.isfinite(logits))
    if dtype == "bf16":
        # tensor-core sums: a logit may sit one bf16 step away from the
        # exact-order one where the sum is next to a rounding midpoint (the
        # routing above is certified against exactly that)
        a, b = logits[fin].astype(np.float64), ol[fin].astype(np.float64)
        row_max = np.abs(np.where(fin, ol, 0)).max(axis=1, keepdims=True)
        scale = np.broadcast_to(row_max, ol.shape)[fin]
        step = 2.0 ** -7 * np.maximum(np.abs(a), np.abs(b))
        assert (np.abs(a - b) <= step + 2.0 ** -12 * scale).all()
        assert (a != b).sum() <= max(2, 0.01 * a.size)
        np.testing.assert_allclose(wt, ow, rtol=2 ** -6, atol=0)
    else:
        # CUDA cores in the same fma order: identical bits
        assert np.array_equal(logits, ol)
        np.testing.assert_allclose(wt, ow, rtol=2e-6, atol=1e-7)
    return idx, wt, logits


@pytest.mark.parametrize("name", golden_names())
def test_router_golden(name):
    inp, ref, meta = load_golden(name)
    k = meta["k"]
    idx, _, logits = _check_against_oracle(inp.x, inp.w_router, inp.router_bias, k, meta["norm"],
                                           meta["dtype"])
    exact, tie_only, real = routing_agrees(idx, logits, ref["topk_idx"], ref["logits"], k)
    if meta["dtype"] == "bf16":
        assert not real.any()
    else:
        # fp32 logits differ from BLAS in the last bits; a real mismatch may
        # only happen where the k-th and (k+1)-th logits are that close
        near = O.boundary_tie_rows(ref["logits"], k, rel=1e-5)
        assert not (real & ~near).any()


@pytest.mark.parametrize("T,d,E,k,dtype,seed", [
    (1, 1536, 64, 8, "bf16", 1),
    (63, 1536, 64, 8, "bf16", 2),
    (65, 1280, 64, 8, "f32", 3),
    (4096, 1536, 64, 8, "bf16", 4),
    (2048, 1280, 64, 8, "f32", 0),
    (1024, 1536, 128, 8, "bf16", 5),
    (300, 40, 8, 3, "bf16", 6),
    (77, 16, 5, 5, "f32", 7),
    (129, 256, 100, 32, "bf16", 8),
])
def test_router_seeded(T, d, E, k, dtype, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, d), dtype=np.float32)
    w = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02))
    if dtype == "bf16":
        x, w = O.round_to_bf16(x), O.round_to_bf16(w)
    _check_against_oracle(x, w, None, k, True, dtype)


@pytest.mark.parametrize("T,d,E,k,bias,seed", [
    (3000, 2048, 64, 8, False, 21),   # resident weight half of 16 k-blocks, 4 ring stages
    (1000, 2560, 64, 8, False, 22),   # too large to keep resident: the row-split pass
    (700, 1536, 96, 8, True, 23),     # 64 < E < 128: the streamed-weight pair pass
    (513, 1536, 64, 16, False, 24),   # k > 8
    (257, 512, 64, 1, True, 25),      # k = 1
    (129, 256, 128, 32, False, 26),   # E = 128, k = 32
    (5000, 1536, 32, 8, False, 27),   # E below the configuration's 64
    (64, 1536, 64, 8, False, 28),     # one pair tile, the odd CTA without tokens
    (129, 1536, 64, 8, True, 29),     # a second tile of one token
])
def test_router_pair_pass_shapes(T, d, E, k, bias, seed):
    """Shapes at the pair pass's edges: its routing must equal the
    exact-order routing bit for bit, as every pass's."""
    rng = np.random.default_rng(seed)
    x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w = O.round_to_bf16(rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02))
    b = O.round_to_bf16(rng.standard_normal(E).astype(np.float32) * np.float32(0.1)) if bias else None
    _check_against_oracle(x, w, b, k, True, "bf16")


def test_router_norm_false_and_bias():
    rng = np.random.default_rng(11)
    x = O.round_to_bf16(rng.standard_normal((500, 256), dtype=np.float32))
    w = O.round_to_bf16(rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.02))
    bias = O.round_to_bf16(synthetic().zipf_router_bias(64, 3, dead_experts=4))
    idx, _, _ = _check_against_oracle(x, w, bias, 8, False, "bf16")
    dead = np.nonzero(np.isinf(bias))[0]
    assert not np.isin(idx, dead).any()


def test_router_exact_ties_go_to_lower_index():
    rng = np.random.default_rng(12)
    x = O.round_to_bf16(rng.standard_normal((256, 64), dtype=np.float32))
    w = O.round_to_bf16(rng.standard_normal((16, 64), dtype=np.float32) * np.float32(0.02))
    w[7] = w[2]
    w[9] = w[4]
    w[15] = w[0]
    idx, _, logits = _check_against_oracle(x, w, None, 4, True, "bf16")
    vals = np.take_along_axis(logits, idx, axis=1)
    eq = np.diff(vals, axis=1) == 0
    assert eq.any()
    assert (np.diff(idx, axis=1)[eq] > 0).all()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_router_full_size_exact(seed):
    """XL 64x8 at 16K tokens: certified tensor-core routing == exact-order routing."""
    T, d, E, k = 16384, 1536, 64, 8
    rng = np.random.default_rng(100 + seed)
    x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w = O.round_to_bf16(rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02))
    _check_against_oracle(x, w, None, k, True, "bf16")


def test_router_full_size_exact_e128_near_ties():
    """E=128 with quantised weights, which makes many logits collide or sit
    next to each other -- the hard case for certification."""
    T, d, E, k = 8192, 1536, 128, 8
    rng = np.random.default_rng(7)
    x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w = (np.round(rng.standard_normal((E, d)).astype(np.float32) * 4) / np.float32(200)).astype(np.float32)
    w = O.round_to_bf16(w)
    _check_against_oracle(x, w, None, k, True, "bf16")


@pytest.mark.parametrize("mode", ["pair_token", "pair_logit", "fixup_kernels"])
def test_router_fixup_pass_is_exact_order(tmp_path, mode):
    """With HMOE_ROUTER_CERT_REL=1 (child process) no token is certified, so
    every token takes a fix-up path: their logits must be the exact-order
    logits bit for bit, and the routing the oracle's.  Paths: the pair pass's
    in-kernel recompute of a whole token (every logit is uncertain) and the
    separate fix-up kernels behind the other passes (HMOE_ROUTER_PAIR=0).
    pair_logit widens the margin to 2^-12 instead, so that many tokens take
    the pair pass's shared one-logit-at-a-time fixes; only their decisive
    logits are recomputed there, so the routing is compared, not every
    logit."""
    import os
    import subprocess
    import sys

    import torch

    import router_fixup_worker_gpu as W

    path = tmp_path / f"{mode}.pt"
    env = dict(os.environ, HMOE_ROUTER_CERT_REL="1")
    if mode == "pair_logit":
        env["HMOE_ROUTER_CERT_REL"] = str(2.0 ** -12)
    elif mode == "fixup_kernels":
        env["HMOE_ROUTER_PAIR"] = "0"
    subprocess.run([sys.executable, W.__file__, str(path)], env=env, check=True, timeout=600)
    res = torch.load(path)
    for name, x, w, bias, k, norm in W.cases():
        idx, wt, logits = (t.numpy() for t in res[name])
        ol = O.router_logits(x, w, bias, "bf16")
        oidx, ow, _ = O.route(ol, k, norm, "bf16")
        if mode != "pair_logit":
            assert np.array_equal(logits, ol), name
        assert np.array_equal(idx.astype(np.int64), oidx), name
        np.testing.assert_allclose(wt, ow, rtol=2 ** -6 if mode == "pair_logit" else 2 ** -7,
                                   atol=0, err_msg=name)


@pytest.mark.parametrize("mode", ["whole_rows", "rows"])
def test_router_whole_row_pass_is_exact(tmp_path, mode):
    """The tensor-core passes other than the default pair pass, each with its
    separate fix-up kernels, in a child process: the 128-token whole-row pass
    (the one that runs when d is not a multiple of 16), forced for every d
    with HMOE_ROUTER_WHOLE_ROWS=1, and the 64-token row-split pass (the one
    for E > 64), forced for E <= 64 with HMOE_ROUTER_PAIR=0.  Their certified
    routing must equal the exact-order routing too, on the same cases as the
    fix-up test."""
    import os
    import subprocess
    import sys

    import torch

    import router_fixup_worker_gpu as W

    path = tmp_path / f"{mode}.pt"
    env = dict(os.environ)
    if mode == "whole_rows":
        env["HMOE_ROUTER_WHOLE_ROWS"] = "1"
    else:
        env["HMOE_ROUTER_PAIR"] = "0"
    env.pop("HMOE_ROUTER_CERT_REL", None)
    subprocess.run([sys.executable, W.__file__, str(path)], env=env, check=True, timeout=600)
    res = torch.load(path)
    for name, x, w, bias, k, norm in W.cases():
        idx, wt, _ = (t.numpy() for t in res[name])
        ol = O.router_logits(x, w, bias, "bf16")
        oidx, ow, _ = O.route(ol, k, norm, "bf16")
        assert np.array_equal(idx.astype(np.int64), oidx), name
        np.testing.assert_allclose(wt, ow, rtol=2 ** -6, atol=0, err_msg=name)


@pytest.mark.parametrize("T,d,E,k,seed", [(1000, 24, 16, 4, 11), (333, 1000, 64, 8, 12),
                                          (4097, 1536, 128, 8, 13), (129, 40, 8, 8, 14)])
def test_router_odd_shapes_exact(T, d, E, k, seed):
    """d not a multiple of 16 (whole-row pass) or of 128 (a partial k-block in
    each half), E below the kernel's 64 / 128 expert maximum, k = E."""
    rng = np.random.default_rng(seed)
    x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    w = O.round_to_bf16(rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02))
    _check_against_oracle(x, w, None, k, True, "bf16")
