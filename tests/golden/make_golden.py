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

``--grad`` runs the backward cases of ``GRAD_CASES``: autograd through the
reference module on CPU with the loss of its own equivalence test
(``sum(y * grad_y) + sum(aux_losses)``), keeping the gradients of x and of
every parameter, the aux losses and the expert counts::

    python tests/golden/make_golden.py --reference /path/to/HRM-MoE --grad

``--large`` runs the full-size cases of ``LARGE_CASES`` instead, on a CUDA
device with the reference's Triton grouped GEMMs (the reference must be
importable there, e.g. the copy ``bench.py --prepare-reference`` makes under
``baseline/_ref``).  Those fixtures keep the routing, the counts, the output
of a seeded token sample and the reference's own logits of every row whose
k-th and (k+1)-th logits are within two bf16 steps (where a different
accumulation order may legitimately pick the other expert)::

    python tests/golden/make_golden.py --reference baseline/_ref --large --out DIR
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

# Backward cases (CPU autograd through the reference module, loss =
# sum(y * grad_y) + sum(aux_losses) as in test_moe_shard_equivalence.py:227-232):
# name: (T, d, E, I, k, norm, dtype, seed, bias, valid_tokens or None)
GRAD_CASES = {
    "grad_refcpu_f32": (35, 16, 8, 32, 3, True, "f32", 0, None, None),
    "grad_refcpu_bf16": (35, 16, 8, 32, 3, True, "bf16", 0, None, None),
    "grad_mid_bf16": (64, 64, 16, 32, 4, True, "bf16", 21, None, None),
    "grad_norm_false_f32": (24, 32, 16, 16, 4, False, "f32", 22, None, None),
    # seed picked so that no row's 4th and 5th logits are within two bf16
    # steps: a near tie there can route differently in another summation
    # order, and a gradient fixture needs the reference's routing
    "grad_zipf_bias_bf16": (48, 64, 16, 32, 4, True, "bf16", 36, "zipf", None),
    "grad_valid_tokens_f32": (40, 32, 8, 16, 2, True, "f32", 24, None, 29),
}


def grad_case_inputs(name: str):
    T, d, E, I, k, norm, dtype, seed, bias_kind, _ = GRAD_CASES[name]
    shape = synthetic.MoEShape(T, d, E, I, k, norm, dtype)
    bias = None
    if bias_kind == "zipf":
        bias = synthetic.zipf_router_bias(E, seed)
        if dtype == "bf16":
            bias = synthetic.round_to_bf16(bias)
    inp = synthetic.make_inputs(shape, seed, router_bias=bias)
    rng = np.random.default_rng([seed, 7])
    grad_y = rng.standard_normal((T, d), dtype=np.float32)
    if dtype == "bf16":
        grad_y = synthetic.round_to_bf16(grad_y)
    return inp, grad_y


def run_reference_grad(layers, inp, grad_y, valid_tokens=None):
    """Forward + backward of the reference module on CPU; returns the grads."""
    s = inp.shape
    tdt = torch.bfloat16 if s.dtype == "bf16" else torch.float32
    mod = layers.SparseMoESwiGLU(s.hidden, s.intermediate, s.experts, s.top_k,
                                 s.norm_topk_prob, implementation="grouped_triton")
    if inp.router_bias is not None:
        mod.gate = layers.LinearInit(s.hidden, s.experts, bias=True)
    mod = mod.to(tdt)
    with torch.no_grad():
        mod.gate.weight.copy_(torch.from_numpy(inp.w_router))
        if inp.router_bias is not None:
            mod.gate.bias.copy_(torch.from_numpy(inp.router_bias))
        mod.experts.gate_up_weight.copy_(torch.from_numpy(inp.w_gate_up))
        mod.experts.down_weight.copy_(torch.from_numpy(inp.w_down))
    x = torch.from_numpy(inp.x).to(tdt).requires_grad_(True)
    ctx = {"aux_losses": [], "expert_counts": []}
    kw = {}
    if valid_tokens is not None:
        kw["total_seqlen"] = torch.tensor(valid_tokens)
    y = mod(x, moe_context=ctx, **kw)
    aux = torch.stack(ctx["aux_losses"])
    loss = (y * torch.from_numpy(grad_y).to(tdt)).sum() + aux.sum()
    loss.backward()
    out = {
        "y": y.detach().float().numpy(),
        "aux": aux.detach().float().numpy(),
        "expert_counts": torch.stack(ctx["expert_counts"]).float().numpy(),
        "dx": x.grad.float().numpy(),
        "d_w_router": mod.gate.weight.grad.float().numpy(),
        "d_w_gate_up": mod.experts.gate_up_weight.grad.float().numpy(),
        "d_w_down": mod.experts.down_weight.grad.float().numpy(),
    }
    if inp.router_bias is not None:
        out["d_bias"] = mod.gate.bias.grad.float().numpy()
    return out


def make_grad(layers, out_dir: pathlib.Path, only=None):
    for name, (T, d, E, I, k, norm, dtype, seed, bias_kind, valid) in GRAD_CASES.items():
        if only and name not in only:
            continue
        inp, grad_y = grad_case_inputs(name)
        out = run_reference_grad(layers, inp, grad_y, valid)
        arrays = {}
        for key, val in out.items():
            if dtype == "bf16" and key not in ("aux", "expert_counts"):
                arrays[key] = synthetic.bf16_bits(val)
            else:
                arrays[key] = np.asarray(val, np.float32)
        meta = {"case": name, "T": T, "d": d, "E": E, "I": I, "k": k, "norm": norm,
                "dtype": dtype, "seed": seed, "bias": bias_kind, "valid_tokens": valid,
                "checksums": checksums(inp), "torch": torch.__version__,
                "generator": "tests/golden/make_golden.py --grad"}
        np.savez_compressed(out_dir / f"{name}.npz", meta=np.array(json.dumps(meta)), **arrays)
        print(f"{name}: aux {out['aux'].tolist()} |dx| {np.abs(out['dx']).max():.3e}")


# Full-size cases run on the GPU (the reference's grouped_triton path):
# name: (T, d, E, I, k, norm, dtype, seed, bias, output sample size)
LARGE_CASES = {
    "xl64_t16384_gpu_bf16": (16384, 1536, 64, 512, 8, True, "bf16", 0, None, 96),
}


def large_case_inputs(name: str):
    T, d, E, I, k, norm, dtype, seed, bias_kind, _ = LARGE_CASES[name]
    return synthetic.make_inputs(synthetic.MoEShape(T, d, E, I, k, norm, dtype), seed)


def near_tie_rows(logits: np.ndarray, k: int, steps: int = 2) -> np.ndarray:
    """Rows whose k-th and (k+1)-th largest bf16 logits are within ``steps`` bf16 steps."""
    s = -np.sort(-logits, axis=1)
    a, b = s[:, k - 1], s[:, k]
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32)) * np.float32(65536)
    return np.abs(a - b) <= steps * ulp


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


def run_reference(layers, inp, device: str = "cpu"):
    s = inp.shape
    tdt = torch.bfloat16 if s.dtype == "bf16" else torch.float32
    mod = layers.SparseMoESwiGLU(s.hidden, s.intermediate, s.experts, s.top_k,
                                 s.norm_topk_prob, implementation="grouped_triton")
    if inp.router_bias is not None:
        # the reference gate has no bias; swap in its own LinearInit with one
        # (layers.py:66-90); forward calls self.gate generically (layers.py:605)
        mod.gate = layers.LinearInit(s.hidden, s.experts, bias=True)
    mod = mod.to(device=device, dtype=tdt)
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
            y = mod(torch.from_numpy(inp.x).to(device=device, dtype=tdt))
    finally:
        layers.triton_grouped_linear = orig
        h1.remove()
        h2.remove()
    sel = cap["selected"].cpu()
    cap = {key: v.cpu() for key, v in cap.items()}
    y = y.cpu()
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


def make_large(layers, out_dir: pathlib.Path, only=None):
    for name, (T, d, E, I, k, norm, dtype, seed, bias_kind, n_sample) in LARGE_CASES.items():
        if only and name not in only:
            continue
        inp = large_case_inputs(name)
        out = run_reference(layers, inp, device="cuda")
        sample = np.sort(np.random.default_rng(seed).choice(T, 512, replace=False)[:n_sample])
        ties = np.nonzero(near_tie_rows(out["logits"], k))[0]
        meta = {"case": name, "T": T, "d": d, "E": E, "I": I, "k": k, "norm": norm,
                "dtype": dtype, "seed": seed, "bias": bias_kind, "device": "cuda",
                "gpu": torch.cuda.get_device_name(), "checksums": checksums(inp),
                "torch": torch.__version__, "generator": "tests/golden/make_golden.py --large",
                "sample_note": f"first {n_sample} of rng.choice(T, 512) sorted"}
        np.savez_compressed(
            out_dir / f"{name}.npz", meta=np.array(json.dumps(meta)),
            topk_idx=out["topk_idx"].astype(np.uint8),
            topk_weight=synthetic.bf16_bits(out["topk_weight"]),
            counts=out["counts"], sample=sample.astype(np.int32),
            y_sample=synthetic.bf16_bits(out["y"][sample]),
            near_tie_rows=ties.astype(np.int32),
            near_tie_logits=synthetic.bf16_bits(out["logits"][ties]))
        print(f"{name}: counts {out['counts'].tolist()[:8]}... near-tie rows {ties.size}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (XiaoYee/HRM-MoE) to import models/layers.py from")
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--large", action="store_true",
                    help="the full-size LARGE_CASES, on the GPU")
    ap.add_argument("--grad", action="store_true",
                    help="the backward cases of GRAD_CASES (CPU autograd)")
    ap.add_argument("--out", default=str(HERE), help="output folder")
    args = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    layers = import_reference(pathlib.Path(args.reference))
    if args.grad:
        make_grad(layers, pathlib.Path(args.out), args.only)
        return
    if args.large:
        out_dir = pathlib.Path(args.out)
        out_dir.mkdir(parents=True, exist_ok=True)
        make_large(layers, out_dir, args.only)
        return
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
