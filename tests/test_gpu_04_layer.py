"""Whole MoE-FFN forward vs the reference goldens and vs the oracle.

Tolerances are the ones the task states for this path: bf16 outputs within
max-relative error 1e-2, fp32 within 1e-4 (max|y - r| / max|r|); routing
indices, counts and the permutation bit-exact on every row whose top-k is
not decided by an exact tie.
"""
import numpy as np
import pytest
import torch

from _helpers import golden_names, load_golden, package, routing_agrees, synthetic
from gpu_util import get_ops, random_topk, to_dev, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = {"bf16": 1e-2, "f32": 1e-4}


def _run_layer(inp, k, norm, dtype, accumulate_into=None):
    ops = get_ops()
    out = None if accumulate_into is None else to_dev(accumulate_into, dtype)
    y, r = ops.ffn_forward(to_dev(inp.x, dtype), to_dev(inp.w_router, dtype),
                           to_dev(inp.w_gate_up, dtype), to_dev(inp.w_down, dtype), k, norm,
                           router_bias=None if inp.router_bias is None else to_dev(inp.router_bias, dtype),
                           out=out, accumulate=accumulate_into is not None, return_routing=True)
    return to_np(y), {key: to_np(v) for key, v in r.items()}


@pytest.mark.parametrize("name", golden_names())
def test_layer_vs_reference_golden(name):
    inp, ref, meta = load_golden(name)
    k, dtype = meta["k"], meta["dtype"]
    y, r = _run_layer(inp, k, meta["norm"], dtype)
    logits = O.router_logits(inp.x, inp.w_router, inp.router_bias, dtype)
    exact, tie_only, real = routing_agrees(r["topk_idx"], logits, ref["topk_idx"], ref["logits"], k)
    if dtype == "bf16":
        assert not real.any()
    else:
        assert not (real & ~O.boundary_tie_rows(ref["logits"], k, rel=1e-5)).any()
    assert O.max_rel(y[exact], ref["y"][exact]) <= TOL[dtype]
    if exact.all():
        assert np.array_equal(r["counts"].astype(np.int64), ref["counts"])
        assert np.array_equal(r["sort_idx"].astype(np.int64), ref["sort_idx"])


@pytest.mark.parametrize("name", golden_names())
def test_layer_vs_oracle_golden_inputs(name):
    inp, _, meta = load_golden(name)
    k, dtype = meta["k"], meta["dtype"]
    y, r = _run_layer(inp, k, meta["norm"], dtype)
    o = O.moe_forward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, k, meta["norm"], dtype,
                      inp.router_bias)
    assert np.array_equal(r["topk_idx"].astype(np.int64), o["topk_idx"])
    assert np.array_equal(r["counts"].astype(np.int64), o["counts"])
    assert np.array_equal(r["sort_idx"].astype(np.int64), o["sort_idx"])
    assert O.max_rel(y, o["y"]) <= TOL[dtype]


@pytest.mark.parametrize("cfg,T", [("cfg2_xl64_bf16", 2048), ("cfg1_l_f32", 2048),
                                   ("cfg3_xl128_ep_bf16", 1024)])
def test_layer_vs_oracle_config_shapes(cfg, T):
    base = synthetic().CONFIGS[cfg]
    shape = synthetic().MoEShape(T, base.hidden, base.experts, base.intermediate, base.top_k,
                                 base.norm_topk_prob, base.dtype)
    inp = synthetic().make_inputs(shape, seed=0)
    y, r = _run_layer(inp, shape.top_k, True, shape.dtype)
    o = O.moe_forward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, shape.top_k, True,
                      shape.dtype)
    assert np.array_equal(r["topk_idx"].astype(np.int64), o["topk_idx"])
    assert np.array_equal(r["sort_idx"].astype(np.int64), o["sort_idx"])
    assert O.max_rel(y, o["y"]) <= TOL[shape.dtype]


def test_layer_full_size_xl_properties():
    """XL 64x8 at 16K tokens: exact routing, a valid stable permutation, and
    the output of a token sample against the oracle (per-token independent)."""
    shape = synthetic().CONFIGS["cfg2_xl64_bf16"]
    inp = synthetic().make_inputs(shape, seed=0)
    y, r = _run_layer(inp, shape.top_k, True, "bf16")
    logits = O.router_logits(inp.x, inp.w_router, None, "bf16")
    oidx, ow, _ = O.route(logits, shape.top_k, True, "bf16")
    assert np.array_equal(r["topk_idx"].astype(np.int64), oidx)
    s = r["sort_idx"].astype(np.int64)
    assert np.array_equal(np.sort(s), np.arange(shape.assignments))
    flat = oidx.reshape(-1)
    assert (np.diff(flat[s]) >= 0).all()
    assert (np.diff(s)[np.diff(flat[s]) == 0] > 0).all()
    assert np.array_equal(r["counts"], np.bincount(flat, minlength=shape.experts))
    sample = np.random.default_rng(0).choice(shape.tokens, 256, replace=False)
    ys = O.experts_forward(inp.x[sample], oidx[sample], ow[sample], inp.w_gate_up, inp.w_down, "bf16")
    assert O.max_rel(y[sample], ys) <= TOL["bf16"]


def test_layer_zipf_with_dead_experts():
    base = synthetic().CONFIGS["cfg4_xl64_zipf_bf16"]
    shape = synthetic().MoEShape(4096, base.hidden, base.experts, base.intermediate, base.top_k,
                                 True, "bf16")
    bias = O.round_to_bf16(synthetic().zipf_router_bias(shape.experts, 4, dead_experts=4))
    inp = synthetic().make_inputs(shape, seed=4, router_bias=bias)
    y, r = _run_layer(inp, shape.top_k, True, "bf16")
    o = O.moe_forward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, shape.top_k, True, "bf16",
                      bias)
    assert np.array_equal(r["topk_idx"].astype(np.int64), o["topk_idx"])
    assert np.array_equal(r["counts"].astype(np.int64), o["counts"]), (r["counts"], o["counts"])
    assert (r["counts"][np.isinf(bias)] == 0).all()
    err = O.max_rel(y, o["y"])
    bad = np.argmax(np.abs(y - o["y"]).max(axis=1))
    assert err <= TOL["bf16"], (err, bad, r["topk_idx"][bad], y[bad][:4], o["y"][bad][:4])


def test_layer_accumulate_and_edges():
    ops = get_ops()
    shape = synthetic().MoEShape(37, 128, 8, 64, 2, True, "bf16")
    inp = synthetic().make_inputs(shape, seed=3)
    base = O.round_to_bf16(np.random.default_rng(1).standard_normal((37, 128), dtype=np.float32))
    y_acc, _ = _run_layer(inp, 2, True, "bf16", accumulate_into=base)
    y, _ = _run_layer(inp, 2, True, "bf16")
    assert O.max_rel(y_acc, O.round_to_bf16(base + y)) <= 1e-2
    empty = ops.ffn_forward(torch.zeros((0, 128), device="cuda", dtype=torch.bfloat16),
                            to_dev(inp.w_router, "bf16"), to_dev(inp.w_gate_up, "bf16"),
                            to_dev(inp.w_down, "bf16"), 2, True)
    assert tuple(empty.shape) == (0, 128)


@pytest.mark.parametrize("name", ["xl64_t32_bf16", "cfg1_t32_f32", "zipf_dead_bf16", "ties_bf16"])
def test_experts_module_on_reference_routing(name):
    """SparseMoEGroupedExperts.forward with the reference's own routing (int64 ids)."""
    inp, ref, meta = load_golden(name)
    dtype = meta["dtype"]
    final = torch.zeros((meta["T"], meta["d"]), device="cuda",
                        dtype=torch.bfloat16 if dtype == "bf16" else torch.float32)
    get_ops().experts_forward(to_dev(inp.x, dtype), torch.from_numpy(ref["topk_idx"]).cuda(),
                              to_dev(ref["topk_weight"], dtype), final,
                              to_dev(inp.w_gate_up, dtype), to_dev(inp.w_down, dtype))
    assert O.max_rel(to_np(final), ref["y"]) <= TOL[dtype]


def test_module_mirror_matches_ops():
    pkg = package()
    layers = pkg.layers
    shape = synthetic().MoEShape(64, 256, 16, 128, 4, True, "bf16")
    inp = synthetic().make_inputs(shape, seed=9)
    mod = layers.SparseMoESwiGLU(256, 128, 16, 4, True, implementation="grouped_b200").cuda().bfloat16()
    with torch.no_grad():
        mod.gate.weight.copy_(to_dev(inp.w_router, "bf16"))
        mod.experts.gate_up_weight.copy_(to_dev(inp.w_gate_up, "bf16"))
        mod.experts.down_weight.copy_(to_dev(inp.w_down, "bf16"))
        y = mod(to_dev(inp.x, "bf16").reshape(4, 16, 256))
    assert tuple(y.shape) == (4, 16, 256)
    o = O.moe_forward(inp.x, inp.w_router, inp.w_gate_up, inp.w_down, 4, True, "bf16")
    assert O.max_rel(to_np(y).reshape(64, 256), o["y"]) <= 1e-2


def test_combine_op_matches_reference_rounding():
    """hmoe_combine reproduces index_add_'s rounding sequence bit for bit:
    bf16(w * y) added one at a time in ascending sorted position."""
    T, E, k, d = 500, 16, 4, 256
    rng = np.random.default_rng(5)
    idx = random_topk(T, E, k, seed=5)
    w = O.round_to_bf16(rng.random((T, k), dtype=np.float32))
    sort_idx, sorted_token, _ = O.dispatch(idx, E)
    expert_out = O.round_to_bf16(rng.standard_normal((T * k, d), dtype=np.float32))
    final0 = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
    final = to_dev(final0, "bf16")
    get_ops().combine(to_dev(expert_out, "bf16"), torch.from_numpy(sort_idx).cuda(),
                      to_dev(w, "bf16"), final)
    ref = final0.copy()
    flat_w = w.reshape(-1)[sort_idx]
    for p in range(T * k):  # index_add_ order: ascending sorted position
        t = sorted_token[p]
        ref[t] = O.round_to_bf16(ref[t] + O.round_to_bf16(expert_out[p] * flat_w[p]))
    assert np.array_equal(to_np(final), ref)


@pytest.mark.parametrize("T,chunk", [(10000, 4096), (300, 4096), (4096, 1000)])
def test_host_buffer_pipeline_matches_device_path(T, chunk):
    """hmoe_ffn_forward_host (chunked, copies overlapped) == the device path, bit for bit."""
    ops = get_ops()
    shape = synthetic().MoEShape(T, 1536, 64, 512, 8, True, "bf16")
    inp = synthetic().make_inputs(shape, seed=13)
    w = [to_dev(a, "bf16") for a in (inp.w_router, inp.w_gate_up, inp.w_down)]
    x_host = torch.from_numpy(inp.x).bfloat16().pin_memory()
    y_host = ops.ffn_forward_host(x_host, *w, 8, True, chunk_tokens=chunk)
    torch.cuda.synchronize()
    y_dev = ops.ffn_forward(x_host.cuda(), *w, 8, True).cpu()
    assert torch.equal(y_host, y_dev)


@pytest.mark.parametrize("T,E", [(64, 64), (1000, 64), (16384, 64), (3000, 128)])
def test_programmatic_launch_same_bits(T, E):
    """Kernels launched with programmatic dependent launch (every class, the
    combine included) give the bits of plain launches, eagerly and replayed
    from a captured CUDA graph; the layer at small T runs the single-CTA
    GEMM, at large T the CTA-pair GEMM."""
    import importlib

    ops = get_ops()
    lib = importlib.import_module("hrm-moe_b200._lib").load()
    shape = synthetic().MoEShape(T, 1536, E, 512, 8, True, "bf16")
    inp = synthetic().make_inputs(shape, seed=17)
    x, wr, wgu, wd = (to_dev(a, "bf16") for a in (inp.x, inp.w_router, inp.w_gate_up, inp.w_down))
    old = lib.hmoe_set_pdl_mask(0)
    try:
        ref, r0 = ops.ffn_forward(x, wr, wgu, wd, 8, True, return_routing=True)
        lib.hmoe_set_pdl_mask(15)
        y, r1 = ops.ffn_forward(x, wr, wgu, wd, 8, True, return_routing=True)
        out = torch.empty_like(ref)
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap, capture_error_mode="relaxed"):
            ops.ffn_forward(x, wr, wgu, wd, 8, True, out=out)
        torch.cuda.current_stream().wait_stream(cap)
        for _ in range(3):
            out.zero_()
            g.replay()
        torch.cuda.synchronize()
        del g
    finally:
        lib.hmoe_set_pdl_mask(old)
    assert torch.equal(y, ref)
    assert torch.equal(out, ref)
    for key in r0:
        assert torch.equal(r1[key], r0[key]), key
