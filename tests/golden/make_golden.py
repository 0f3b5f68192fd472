#!/usr/bin/env python
"""Generate the golden fixtures in this folder from the reference itself.

Runs XiaoYee/HRM-MoE's own ``SparseMoESwiGLU`` (``models/layers.py:518-634``,
``implementation="grouped_triton"``, whose CPU path is the per-expert
``F.linear`` loop of ``models/moe_triton_grouped_gemm.py:55-65``) on seeded
inputs from ``synthetic.make_inputs`` and records what it computes:

* ``logits``       -- output of ``self.gate`` (forward hook on the gate),
* ``topk_idx``/``topk_weight`` -- the ``selected_experts``/``routing_weights``
  the layer hands to its experts module (forward pre-hook),
* ``sort_idx``/``counts`` -- ``torch.sort(flat, stable=True)`` and
  ``bincount`` of those selections, the expressions of layers.py:313-322,
  cross-checked against the ``tokens_per_expert`` the layer passes to its
  grouped GEMM (captured by wrapping ``models.layers.triton_grouped_linear``),
* ``y``            -- the layer output.

The reference imports FlashAttention at module scope; like its own test
(``scripts/test_moe_shard_equivalence.py:12-18``) we stub those two modules.

Inputs are not stored: every case records its seed and shape and the tests
regenerate them with ``synthetic.make_inputs`` (plus checksums to catch a
generator drift).  Usage::

    python tests/golden/make_golden.py --reference /path/to/HRM-MoE [--only NAME ...]
"""
from __future__ import annotations

import argparse
import importlib
import json
import pathlib
import sys
import types

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
synthetic = importlib.import_module("hrm-moe_b200.synthetic")

# name: (T, d, E, I, k, norm, dtype, seed, bias)  bias in {None, "zipf", "zipf_dead", "ties"}
CASES = {
    # the reference equivalence test's CPU default shape (test_moe_shard_equivalence.py:102-108)
    "refcpu_default_f32": (35, 16, 8, 32, 3, True, "f32", 0, None),
    "refcpu_default_bf16": (35, 16, 8, 32, 3, True, "bf16", 0, None),
    # the EP equivalence test's shape (test_moe_ep_distributed_equivalence.py:72-81)
    "ep_shape_f32": (16, 128, 8, 64, 2, True, "f32", 1234, None),
    "ep_shape_bf16": (16, 128, 8, 64, 2, True, "bf16", 1234, None),
    # config 1 (L-scale) and config 2/3 (XL) layer shapes at a few tokens
    "cfg1_t32_f32": (32, 1280, 64, 448, 8, True, "f32", 0, None),
    "xl64_t32_bf16": (32, 1536, 64, 512, 8, True, "bf16", 0, None),
    "xl128_t16_bf16": (16, 1536, 128, 512, 8, True, "bf16", 3, None),
    # variants: no renormalisation, top-1, fewer tokens than experts
    "norm_false_f32": (24, 64, 16, 32, 4, False, "f32", 5, None),
    "norm_false_bf16": (24, 64, 16, 32, 4, False, "bf16", 5, None),
    "top1_f32": (20, 32, 4, 16, 1, True, "f32", 6, None),
    "tiny_tokens_f32": (3, 64, 16, 32, 4, True, "f32", 7, None),
    # load imbalance: Zipf(1.2) router bias, and with 2 experts receiving nothing
    "zipf_bf16": (64, 128, 16, 64, 4, True, "bf16", 8, "zipf"),
    "zipf_dead_bf16": (64, 128, 16, 64, 4, True, "bf16", 9, "zipf_dead"),
    # exact logit ties: duplicated router rows
    "ties_bf16": (32, 64, 16, 32, 4, True, "bf16", 10, "ties"),
    "ties_f32": (32, 64, 16, 32, 4, True, "f32", 10, "ties"),
}

TIE_PAIRS = ((3, 5), (2, 9), (11, 12), (0, 15))


def case_inputs(name: str):
    """Regenerate a case's inputs (also used by the tests)."""
    T, d, E, I, k, norm, dtype, seed, bias_kind = CASES[name]
    shape = synthetic.MoEShape(T, d, E, I, k, norm, dtype)
    bias = None
    if bias_kind == "zipf":
        bias = synthetic.zipf_router_bias(E, seed)
    elif bias_kind == "zipf_dead":
        bias = synthetic.zipf_router_bias(E, seed, dead_experts=2)
    if bias is not None and dtype == "bf16":
        # the gate bias is a parameter of the layer, so it lives in the layer dtype
        bias = synthetic.round_to_bf16(bias)
    inp = synthetic.make_inputs(shape, seed, router_bias=bias)
    if bias_kind == "ties":
        for a, b in TIE_PAIRS:
            inp.w_router[b] = inp.w_router[a]
    return inp


def checksums(inp) -> dict:
    return {k: float(np.float64(getattr(inp, k)).sum())
            for k in ("x", "w_router", "w_gate_up", "w_down")}


def import_reference(path: pathlib.Path):
    sys.path.insert(0, str(path))
    stub = types.ModuleType("models.flash_attention_prefixlm_v2")
    stub.flash_attn_varlen_prefixlm = None
    sys.modules.setdefault("models.flash_attention_prefixlm_v2", stub)
    stub2 = types.ModuleType("flash_attn_interface")
    stub2.flash_attn_with_kvcache = None
    sys.modules.setdefault("flash_attn_interface", stub2)
    return importlib.import_module("models.layers")


def run_reference(layers, inp):
    s = inp.shape
    tdt = torch.bfloat16 if s.dtype == "bf16" else torch.float32
    mod = layers.SparseMoESwiGLU(s.hidden, s.intermediate, s.experts, s.top_k,
                                 s.norm_topk_prob, implementation="grouped_triton")
    if inp.router_bias is not None:
        # the reference gate has no bias; swap in its own LinearInit with one
        # (layers.py:66-90); forward calls self.gate generically (layers.py:605)
        mod.gate = layers.LinearInit(s.hidden, s.experts, bias=True)
    mod = mod.to(tdt)
    with torch.no_grad():
        mod.gate.weight.copy_(torch.from_numpy(inp.w_router))
        if inp.router_bias is not None:
            mod.gate.bias.copy_(torch.from_numpy(inp.router_bias))
        mod.experts.gate_up_weight.copy_(torch.from_numpy(inp.w_gate_up))
        mod.experts.down_weight.copy_(torch.from_numpy(inp.w_down))
    cap = {}
    h1 = mod.gate.register_forward_hook(lambda m, a, o: cap.__setitem__("logits", o.detach().clone()))
    h2 = mod.experts.register_forward_pre_hook(
        lambda m, a: cap.update(selected=a[1].detach().clone(), weights=a[2].detach().clone()))
    orig = layers.triton_grouped_linear
    seen = []

    def wrapped(inp_, weight, tokens_per_expert):
        seen.append(tokens_per_expert.detach().clone())
        return orig(inp_, weight, tokens_per_expert)

    layers.triton_grouped_linear = wrapped
    try:
        with torch.no_grad():
            y = mod(torch.from_numpy(inp.x).to(tdt))
    finally:
        layers.triton_grouped_linear = orig
        h1.remove()
        h2.remove()
    sel = cap["selected"]
    flat = sel.reshape(-1)
    _, sort_idx = torch.sort(flat, stable=True)                      # layers.py:317
    counts = torch.bincount(flat, minlength=s.experts)               # layers.py:322
    if seen:
        assert torch.equal(seen[0].cpu(), counts), "captured tokens_per_expert differs"
    return {
        "logits": cap["logits"].float().numpy(),
        "topk_idx": sel.numpy().astype(np.int32),
        "topk_weight": cap["weights"].float().numpy(),
        "sort_idx": sort_idx.numpy().astype(np.int32),
        "counts": counts.numpy().astype(np.int32),
        "y": y.float().numpy(),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (XiaoYee/HRM-MoE) to import models/layers.py from")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    layers = import_reference(pathlib.Path(args.reference))
    for name in CASES:
        if args.only and name not in args.only:
            continue
        inp = case_inputs(name)
        out = run_reference(layers, inp)
        T, d, E, I, k, norm, dtype, seed, bias_kind = CASES[name]
        arrays = {}
        for key, val in out.items():
            if dtype == "bf16" and key in ("logits", "topk_weight", "y"):
                arrays[key] = synthetic.bf16_bits(val)
            else:
                arrays[key] = val
        meta = {"case": name, "T": T, "d": d, "E": E, "I": I, "k": k, "norm": norm,
                "dtype": dtype, "seed": seed, "bias": bias_kind,
                "checksums": checksums(inp), "torch": torch.__version__,
                "generator": "tests/golden/make_golden.py"}
        np.savez_compressed(HERE / f"{name}.npz", meta=np.array(json.dumps(meta)), **arrays)
        print(f"{name}: y {out['y'].shape} counts {out['counts'].tolist()[:8]}...")


if __name__ == "__main__":
    main()
