#!/usr/bin/env python
"""Benchmark: routed MoE-FFN forward tokens/s (XL 64x8 layer, bf16) on B200.

A step is one forward of the MoE FFN layer over one batch of T tokens
(default: the XL 64x8 layer at T = 16384 per GPU, d = 1536, 64 experts of
width 512, top-8).  `value` is the whole-job tokens/s with inputs resident in
HBM; `e2e` is the same through the public module API with the hidden states
copied in from pinned host memory and the output read back every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events
on the launching stream; before every step, outside the events, a 256 MiB
buffer (2x the L2) is rewritten and a second one read, so that the step
starts with no input in L2 and no dirty line of the flush left to write
back.  Per-stage times come from events the C ABI records between its
kernels (hmoe_ffn_forward_marked): at N=1 from the
marked layer captured as one CUDA graph like the timed steps (the events
become graph nodes; read after each of up to 50 replays, untimed), with the
eager steps' per-stage times beside them; at N>1 from the timed steps.
Multi-GPU runs take the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import importlib
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-FFN fwd tokens/s (XL 64x8 bf16)"
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = ("256 MiB buffer rewritten, then another 256 MiB read, before every step "
           "(outside the timed events)")


class L2Flush:
    """Evicts the L2 before a step: writes one buffer twice the L2, then
    reads another, so the lines left in L2 are clean and the step's first
    kernel does not pay for writing the flush's own lines back to HBM."""

    def __init__(self, torch, dev):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.max()


# measured peer copy bandwidth per direction per GPU on this pool (NVLink 5)
NVLINK_GBS = 770.0
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per forward of
# each phase's kernels, from one ncu capture of this workload on one B200
# (profiles/grouped_gemm_pair_xl64_t16384_full.md, profiles/hbm_kernels_xl64_t16384.md,
# profiles/router_pair_xl64_t16384.md).
# Keyed by (config, tokens per GPU); other workloads report null.
NCU_TRAFFIC_BYTES = {
    ("cfg2_xl64_bf16", 16384): {
        "router": 50.606e6 + 0.041e6,  # router_pair
        "dispatch": 0.534e6 + 0.039e6 + 51.425e6 + 344.146e6,  # hist + scan + permute
        "gate_up_gemm": 604.140e6 + 123.425e6,
        "down_gemm": 235.043e6 + 354.587e6,
        "combine": 403.712e6 + 42.690e6,
    },
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)  # >= one 200 ms clock sample at N=1
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-gpu"],
                    help="b200: this build; reference: the reference's CPU path (oracle port) "
                         "on the host cores; reference-gpu: the reference's own grouped_triton "
                         "module on this GPU, imported from baseline/_ref (see "
                         "--prepare-reference)")
    ap.add_argument("--prepare-reference", metavar="CHECKOUT",
                    help="copy CHECKOUT/models (the reference's MoE layer and its Triton "
                         "grouped GEMM) into baseline/_ref/ for --impl reference-gpu, and exit")
    ap.add_argument("--config", default="cfg2_xl64_bf16")
    ap.add_argument("--dead-experts", type=int, default=0,
                    help="cfg4: experts whose router bias is -inf (no token reaches them)")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per GPU (default: the config's)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target duration of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-train", action="store_true",
                    help="N=1: skip the training-step measurement (forward that keeps its "
                         "activations + the full backward with the aux loss)")
    ap.add_argument("--train-steps", type=int, default=50)
    ap.add_argument("--e2e-chunk", type=int, default=0,
                    help="tokens per host-copy chunk of the end-to-end measurement (default: "
                         "3584 at N=1, the best of 2560-4096 measured for 16K tokens; 4096 for "
                         "the expert-parallel layer, whose every call repeats the exchange)")
    ap.add_argument("--no-graph", action="store_true",
                    help="N=1: time eager launches instead of one CUDA graph per step")
    ap.add_argument("--ep-impl", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel transport for --gpus > 1: peer memory (the product "
                         "path) or NCCL all_to_all")
    return ap.parse_args()


def workload_name(config: str, shape, tokens: int, dead_experts: int = 0) -> str:
    bias = ""
    if config.startswith("cfg4"):
        bias = ", router bias for Zipf(1.2) expert load" + (
            f", {dead_experts} dead experts" if dead_experts else "")
    return (f"{config}: XL {shape.experts}x{shape.top_k} MoE-FFN layer forward "
            f"(T={tokens} tokens per GPU, d={shape.hidden}, E={shape.experts}, "
            f"I={shape.intermediate}, top-{shape.top_k}{bias})")


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi samples of one GPU while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = pathlib.Path(os.environ.get("TMPDIR", "/tmp")) / f"hmoe_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.gpu_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return self
        # nvidia-smi takes a while to start on a many-GPU box: begin the timed
        # region only once it is sampling.  (Sampling much faster than every
        # 200 ms delays kernel launches and shows up in the step time.)
        deadline = time.time() + 10.0
        while time.time() < deadline and self.proc.poll() is None:
            self.f.flush()
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.01)
        self.skip = self.path.read_text().count("\n")  # samples taken before the region
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.f.flush()
            self.stop = self.path.read_text().count("\n")  # samples up to the region's end
            time.sleep(0.3)  # one more interval: the fallback sample for a short region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()
        return False

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.path.read_text().splitlines()
        skip, stop = getattr(self, "skip", 0), getattr(self, "stop", len(lines))
        # the region's own samples; a region shorter than one interval gets the
        # first sample after it (still this workload's clocks), and says so
        inside = lines[skip:stop]
        after = not inside
        for line in (inside or lines[stop:stop + 1]):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        out = {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
               "power_w_max": max(power), "samples": len(sm), "reasons": sorted(reasons)}
        if after:
            out["sampled_after_region"] = True
        return out


def gpu_uuid(torch, dev: int) -> str:
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return str(dev)


# ------------------------------------------------------------- CPU timing --
def config_router_bias(syn, config: str, shape, dead_experts: int):
    """cfg4's Zipf(1.2) router bias in the layer dtype (float32 array), else None."""
    if not config.startswith("cfg4"):
        return None
    b = syn.zipf_router_bias(shape.experts, 4, dead_experts=dead_experts)
    return syn.round_to_bf16(b) if shape.dtype == "bf16" else b


def cpu_oracle_tokens_per_s(shape, target_s: float, seed: int = 0, max_tokens: int = 16384,
                            bias=None):
    """Time the CPU port of the reference path (oracle) on a bounded sample."""
    from oracle import moe_oracle as O
    syn = importlib.import_module("hrm-moe_b200.synthetic")
    w_r, w_gu, w_d = syn.make_weights(shape, seed)

    def run(T):
        sub = syn.MoEShape(T, shape.hidden, shape.experts, shape.intermediate, shape.top_k,
                           shape.norm_topk_prob, shape.dtype)
        x = syn.make_hidden(sub, seed)
        t0 = time.perf_counter()
        O.moe_forward(x, w_r, w_gu, w_d, shape.top_k, shape.norm_topk_prob, shape.dtype, bias)
        return time.perf_counter() - t0

    run(64)  # warm-up (threads, BLAS)
    T, dt = 128, run(128)
    while dt < target_s / 2 and T < max_tokens:
        T = min(max_tokens, int(T * min(8.0, max(2.0, target_s / max(dt, 1e-3)))))
        dt = run(T)
    return T / dt, T, dt


# --------------------------------------------------------- reference arm --
def reference_arm(args, rank, world):
    """The reference's CPU path (the oracle port of it) on the host cores."""
    if rank != 0:
        return 0
    syn = importlib.import_module("hrm-moe_b200.synthetic")
    shape = syn.CONFIGS[args.config]
    from oracle import moe_oracle as O
    w_r, w_gu, w_d = syn.make_weights(shape, 0)
    sample_T = 256
    sub = syn.MoEShape(sample_T, shape.hidden, shape.experts, shape.intermediate, shape.top_k,
                       shape.norm_topk_prob, shape.dtype)
    x = syn.make_hidden(sub, 0)
    bias = config_router_bias(syn, args.config, shape, args.dead_experts)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.moe_forward(x, w_r, w_gu, w_d, shape.top_k, shape.norm_topk_prob, shape.dtype, bias)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = sample_T / (ms * 1e-3)
    cores = os.cpu_count()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": shape.dtype,
        "data": "synthetic: x~N(0,1), weights~N(0,0.02), numpy PCG64 seed 0",
        "impl": "reference",
        "config": {"workload": workload_name(args.config, shape, sample_T, args.dead_experts)
                               + f", a sample of {sample_T} tokens per step on the host CPU",
                   "tokens_per_step": sample_T, "hidden": shape.hidden,
                   "experts": shape.experts, "intermediate": shape.intermediate,
                   "top_k": shape.top_k},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{sample_T} tokens of the {args.config} layer per step "
                                   f"(numpy/OpenBLAS + C, all {cores} host threads)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------- reference module on the GPU --
REF_DIR = ROOT / "baseline" / "_ref"


def prepare_reference(checkout: str) -> int:
    """Copy the reference's models/ package into baseline/_ref/ (git-ignored)."""
    import shutil
    src = pathlib.Path(checkout) / "models"
    if not (src / "layers.py").exists():
        print(f"no models/layers.py under {checkout}", file=sys.stderr)
        return 2
    dst = REF_DIR / "models"
    if dst.exists():
        shutil.rmtree(dst)
    shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__"))
    print(f"copied {src} -> {dst}")
    return 0


def import_reference_layers():
    """models.layers from baseline/_ref, with the two FlashAttention modules it
    imports at module scope stubbed out, as the reference's own equivalence
    test does (scripts/test_moe_shard_equivalence.py:12-18)."""
    import types
    stub = types.ModuleType("models.flash_attention_prefixlm_v2")
    stub.flash_attn_varlen_prefixlm = None
    sys.modules.setdefault("models.flash_attention_prefixlm_v2", stub)
    stub2 = types.ModuleType("flash_attn_interface")
    stub2.flash_attn_with_kvcache = None
    sys.modules.setdefault("flash_attn_interface", stub2)
    sys.path.insert(0, str(REF_DIR))
    return importlib.import_module("models.layers"), importlib.import_module("models.moe_profile")


def reference_gpu_arm(args, rank, world, local_rank):
    """The reference's own SparseMoESwiGLU(implementation="grouped_triton") on
    this GPU (its Triton grouped GEMMs, models/moe_triton_grouped_gemm.py:113-184,
    autotuned, 16 SMs of margin as its README runs them), same workload and
    weights as the b200 arm, and the same tokens through this build for a
    same-box comparison of routing and output."""
    if rank != 0:
        return 0
    if not (REF_DIR / "models" / "layers.py").exists():
        print(json.dumps({"impl": "reference-gpu", "unavailable":
                          "baseline/_ref/models is absent (bench.py --prepare-reference CHECKOUT)"}))
        return 0
    os.environ.setdefault("HRM_MOE_TRITON_AUTOTUNE", "1")
    os.environ.setdefault("HRM_MOE_TRITON_SM_MARGIN", "16")
    import torch
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    layers, prof = import_reference_layers()
    ops = importlib.import_module("hrm-moe_b200.ops")
    syn = importlib.import_module("hrm-moe_b200.synthetic")
    base = syn.CONFIGS[args.config]
    T = args.tokens or base.tokens
    shape = syn.MoEShape(T, base.hidden, base.experts, base.intermediate, base.top_k,
                         base.norm_topk_prob, base.dtype)
    d, E, I, k = shape.hidden, shape.experts, shape.intermediate, shape.top_k
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1234)
    wg = torch.Generator(device=dev).manual_seed(1000)
    w_router = (torch.randn((E, d), generator=g, device=dev) * 0.02).to(dt)
    w_gate_up = (torch.randn((E, 2 * I, d), generator=g, device=dev) * 0.02).to(dt)
    w_down = (torch.randn((E, d, I), generator=g, device=dev) * 0.02).to(dt)
    x = torch.randn((T, d), generator=wg, device=dev).to(dt)
    zb = config_router_bias(syn, args.config, shape, args.dead_experts)
    bias = None if zb is None else torch.from_numpy(zb).to(dev).to(dt)
    mod = layers.SparseMoESwiGLU(d, I, E, k, shape.norm_topk_prob,
                                 implementation="grouped_triton")
    if bias is not None:
        mod.gate = layers.LinearInit(d, E, bias=True)
    mod = mod.to(device=dev, dtype=dt)
    with torch.no_grad():
        mod.gate.weight.copy_(w_router)
        if bias is not None:
            mod.gate.bias.copy_(bias)
        mod.experts.gate_up_weight.copy_(w_gate_up)
        mod.experts.down_weight.copy_(w_down)
    flush = L2Flush(torch, dev)
    stream = torch.cuda.current_stream(dev)
    prof._MOE_PROFILE_ENABLED = False
    with torch.no_grad():
        for _ in range(max(1, args.warmup)):  # the first call autotunes the Triton kernels
            flush()
            mod(x)
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        with ClockSampler(gpu_uuid(torch, local_rank)) as clocks:
            for i in range(args.steps):
                flush()
                starts[i].record(stream)
                y_ref = mod(x)
                ends[i].record(stream)
            torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends))
        # per-phase times from the reference's own profiler (it synchronises
        # after each phase, so these steps are not the timed ones above)
        prof._MOE_PROFILE_ENABLED = True
        prof.reset_moe_profile()
        n_prof = min(20, args.steps)
        for _ in range(n_prof):
            flush()
            mod(x)
        phases = {n: 1e3 * v / n_prof for n, v in prof.pop_moe_profile().items()}
        prof._MOE_PROFILE_ENABLED = False
        # same tokens through this build: routing and output agreement
        cap = {}
        h = mod.experts.register_forward_pre_hook(
            lambda m, a: cap.update(selected=a[1].detach().clone()))
        y_ref = mod(x)
        h.remove()
        y_b200, r = ops.ffn_forward(x, w_router, w_gate_up, w_down, k, shape.norm_topk_prob,
                                    router_bias=bias, return_routing=True)
        torch.cuda.synchronize()
    same_rows = (r["topk_idx"].long() == cap["selected"].long()).all(dim=1)
    diff = (y_b200.float() - y_ref.float()).abs()[same_rows]
    max_rel = float(diff.max() / y_ref.float().abs()[same_rows].max()) if same_rows.any() else None
    gu_flops, dn_flops = shape.gemm_flops()
    gemm = {}
    for name, flops in (("gate_up_gemm", gu_flops), ("down_gemm", dn_flops)):
        if name in phases:
            gemm[name] = {"ms": phases[name], "tflops": flops / (phases[name] * 1e-3) / 1e12}
    line = {
        "metric": METRIC, "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "impl": "reference-gpu",
        "data": "synthetic: x~N(0,1), weights~N(0,0.02) (seeded torch.Generator on device)",
        "config": {"workload": workload_name(args.config, shape, T, args.dead_experts),
                   "module": "models.layers.SparseMoESwiGLU(implementation='grouped_triton')",
                   "env": {k_: os.environ[k_] for k_ in ("HRM_MOE_TRITON_AUTOTUNE",
                                                         "HRM_MOE_TRITON_SM_MARGIN")},
                   "l2": L2_NOTE},
        "phases_ms": phases,
        "gemms": gemm,
        "vs_b200_same_inputs": {
            "rows": T, "rows_same_routing": int(same_rows.sum()),
            "max_rel_y_on_same_rows": max_rel,
        },
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------- training step --
TRAIN_PHASES = ["forward_train", "combine_router_bwd", "down_dgrad_swiglu_bwd", "down_wgrad",
                "gate_up_dgrad", "gate_up_wgrad", "router_dgrad_and_dx", "router_wgrad"]


def measure_train_step(torch, lib, _lib, ops, shape, x, w_router, bias, w_gate_up, w_down, flush,
                       stream, warmup, steps, peaks):
    """One training step of the layer per iteration: the forward that keeps
    its activations (with the aux loss over all tokens) and the whole
    backward (grad of sum(y * g) + aux), each phase between CUDA events."""
    T, d = x.shape
    E, I, k = shape.experts, shape.intermediate, shape.top_k
    dev = x.device
    cs = ops.make_shape(T, d, E, I, k, torch.bfloat16, shape.norm_topk_prob)
    saved = torch.empty(lib.hmoe_ffn_train_saved_bytes(ctypes.byref(cs)), dtype=torch.uint8,
                        device=dev)
    ws = torch.empty(lib.hmoe_ffn_train_workspace_bytes(ctypes.byref(cs)), dtype=torch.uint8,
                     device=dev)
    y = torch.empty_like(x)
    gy = (torch.randn((T, d), generator=torch.Generator(device=dev).manual_seed(77), device=dev)
          .to(torch.bfloat16))
    aux = torch.zeros((), dtype=torch.float32, device=dev)
    counts = torch.zeros(E, dtype=torch.float32, device=dev)
    aux_grad = torch.ones((), dtype=torch.float32, device=dev)
    gx, gwr = torch.empty_like(x), torch.empty_like(w_router)
    gb = torch.empty_like(bias) if bias is not None else None
    gwgu, gwd = torch.empty_like(w_gate_up), torch.empty_like(w_down)
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(stream.cuda_stream)

    def events(n):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for e in ev:
            e.record(stream)
        return ev

    def step(ev):
        ev[0].record(stream)
        _lib.check(lib.hmoe_ffn_forward_train(
            ctypes.byref(cs), p(x), p(w_router), p(bias), p(w_gate_up), p(w_down), p(y), T,
            p(aux), p(counts), p(saved), saved.numel(), p(ws), ws.numel(), st))
        arr = (ctypes.c_void_p * 8)(*[ctypes.c_void_p(e.cuda_event) for e in ev[1:]])
        _lib.check(lib.hmoe_ffn_backward_marked(
            ctypes.byref(cs), p(gy), p(aux_grad), T, p(x), p(w_router), p(bias), p(w_gate_up),
            p(w_down), p(saved), saved.numel(), p(gx), p(gwr), p(gb), p(gwgu), p(gwd), p(ws),
            ws.numel(), st, arr))

    warm = events(9)
    for _ in range(max(3, warmup)):
        flush()
        step(warm)
    torch.cuda.synchronize()
    ops.workspace_status(ws)
    evs = [events(9) for _ in range(steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        flush()
        step(evs[i])
    torch.cuda.synchronize()
    ops.workspace_status(ws)
    ms = {n: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs)
          for i, n in enumerate(TRAIN_PHASES)}
    total = statistics.mean(e[0].elapsed_time(e[8]) for e in evs)
    A = T * k
    gflop = {"down_dgrad_swiglu_bwd": 2.0 * A * d * I, "down_wgrad": 2.0 * A * d * I,
             "gate_up_dgrad": 4.0 * A * d * I, "gate_up_wgrad": 4.0 * A * d * I,
             "router_wgrad": 2.0 * T * E * d}
    hbm = {"combine_router_bwd": T * d * 2 + 2 * A * d * 2 + 2 * T * E * 2 + A * 12,
           "router_dgrad_and_dx": A * d * 2 + 2 * T * d * 2 + A * 4}
    phases = {}
    for n in TRAIN_PHASES:
        sec = ms[n] * 1e-3
        if n in gflop:
            ach = gflop[n] / sec / 1e12
            phases[n] = {"ms": ms[n], "bound": "tensor", "achieved": ach, "unit": "TFLOP/s",
                         "frac": ach / peaks["bf16_tflops"]}
        elif n in hbm:
            ach = hbm[n] / sec / 1e9
            phases[n] = {"ms": ms[n], "bound": "hbm", "achieved": ach, "unit": "GB/s",
                         "frac": ach / peaks["hbm_gbs"]}
        else:
            phases[n] = {"ms": ms[n]}
    flops = 3 * sum(shape.gemm_flops())  # forward + dgrad + wgrad of both expert GEMMs
    return {"tokens_per_s": T / (total * 1e-3), "ms_per_step": total, "steps": steps,
            "what": "forward that keeps activations (aux loss over all tokens) + backward of "
                    "sum(y * grad_y) + aux: grads of x, router weight, both expert weights",
            "expert_gemm_tflops": flops / (total * 1e-3) / 1e12, "phases": phases,
            "gpu_launches_per_step": 17 if bias is None else 19}


# ------------------------------------------------------------- B200 arm --
def b200_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)
    pkg = importlib.import_module("hrm-moe_b200")
    _lib = importlib.import_module("hrm-moe_b200._lib")
    ops = importlib.import_module("hrm-moe_b200.ops")
    layers = importlib.import_module("hrm-moe_b200.layers")
    syn = pkg.synthetic
    base = syn.CONFIGS[args.config]
    T = args.tokens or base.tokens
    shape = syn.MoEShape(T, base.hidden, base.experts, base.intermediate, base.top_k,
                         base.norm_topk_prob, base.dtype)
    d, E, I, k = shape.hidden, shape.experts, shape.intermediate, shape.top_k
    dt = torch.bfloat16 if shape.dtype == "bf16" else torch.float32
    es = 2 if shape.dtype == "bf16" else 4

    g = torch.Generator(device=dev).manual_seed(1234)
    wg = torch.Generator(device=dev).manual_seed(1000 + rank)
    w_router = (torch.randn((E, d), generator=g, device=dev) * 0.02).to(dt)
    w_gate_up = (torch.randn((E, 2 * I, d), generator=g, device=dev) * 0.02).to(dt)
    w_down = (torch.randn((E, d, I), generator=g, device=dev) * 0.02).to(dt)
    x = torch.randn((T, d), generator=wg, device=dev).to(dt)
    y = torch.empty_like(x)
    # cfg4: a router bias that makes expected expert selection follow
    # Zipf(1.2) over a seeded permutation (optionally with dead experts)
    bias = None
    if args.config.startswith("cfg4"):
        zb = syn.zipf_router_bias(E, 4, dead_experts=args.dead_experts)
        bias = torch.from_numpy(zb).to(dev).to(dt)
    bias_p = ctypes.c_void_p(bias.data_ptr()) if bias is not None else None
    flush = L2Flush(torch, dev)

    lib = _lib.load()
    cshape = ops.make_shape(T, d, E, I, k, dt, shape.norm_topk_prob)
    ws_bytes = lib.hmoe_ffn_workspace_bytes(ctypes.byref(cshape))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    n_marks = 6

    def make_events(n):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for e in evs:
            e.record(stream)  # create the underlying cudaEvent_t
        return evs

    def step(marks):
        arr = (ctypes.c_void_p * n_marks)(*[ctypes.c_void_p(m.cuda_event) for m in marks])
        _lib.check(lib.hmoe_ffn_forward_marked(
            ctypes.byref(cshape), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w_router.data_ptr()),
            bias_p, ctypes.c_void_p(w_gate_up.data_ptr()), ctypes.c_void_p(w_down.data_ptr()),
            ctypes.c_void_p(y.data_ptr()), 0, ctypes.c_void_p(ws.data_ptr()), ws.numel(),
            ctypes.c_void_p(stream.cuda_stream), arr))

    ep = None
    peer = None
    if world > 1:
        # expert parallel: this rank keeps experts [rank*E/N, (rank+1)*E/N)
        ep = importlib.import_module("hrm-moe_b200.ep")
        el = E // world
        # every rank drew all experts' weights from the same seed; the full
        # set stays until the parity check below has run
        w_gate_up_full, w_down_full = w_gate_up, w_down
        w_gate_up = w_gate_up[rank * el:(rank + 1) * el].contiguous()
        w_down = w_down[rank * el:(rank + 1) * el].contiguous()
        # rows per (source rank, expert), from one untimed routing pass
        idx, _ = ops.router_topk(x, w_router, k, shape.norm_topk_prob, bias)
        cnt = torch.bincount(idx.reshape(-1).long(), minlength=E).to(torch.int64)
        cnt_all = [torch.empty_like(cnt) for _ in range(world)]
        dist.all_gather(cnt_all, cnt)
        cnt_all = torch.stack(cnt_all).view(world, world, el).cpu()  # [src, owner, el]
        own = cnt_all.sum(2)  # [src, owner]
        send_rows = float(own[rank].sum() - own[rank, rank])
        recv_rows = float(own[:, rank].sum() - own[rank, rank])
        gemm_rows = float(own[:, rank].sum())
        if args.ep_impl == "peer":
            peer = ep.PeerExpertParallel(d, I, E, k, shape.norm_topk_prob, max_tokens=T, dtype=dt)

            def step(marks):  # noqa: F811  (EP replaces the single-GPU step)
                peer.forward(x, w_router, w_gate_up, w_down, router_bias=bias, y=y, marks=marks)
        else:
            def step(marks):  # noqa: F811
                y.copy_(ep.ep_forward(x, w_router, w_gate_up, w_down, E, k,
                                      shape.norm_topk_prob, router_bias=bias, marks=marks))

    warm_marks = make_events(n_marks)
    for _ in range(args.warmup):
        flush()
        step(warm_marks)
    torch.cuda.synchronize()
    ops.workspace_status(ws)
    if peer is not None:
        peer.status()

    # ------------------------------------- expert-parallel parity (untimed)
    # One more expert-parallel step, then each rank runs the single-GPU layer
    # (all experts, same tokens, same router) and compares: the EP output
    # must be bit-identical (same kernels, same order per row).
    ep_parity = None
    if world > 1:
        y.zero_()
        step(warm_marks)
        y_ref = ops.ffn_forward(x, w_router, w_gate_up_full, w_down_full, k,
                                shape.norm_topk_prob, router_bias=bias)
        torch.cuda.synchronize()
        yd, rd = y.float(), y_ref.float()
        t = torch.tensor([0.0 if torch.equal(y, y_ref) else 1.0,
                          float((yd - rd).abs().max()),
                          float((yd - rd).abs().max() / rd.abs().max().clamp_min(1e-30)),
                          0.0 if bool(torch.isfinite(yd).all()) else 1.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ep_parity = {"bit_exact": bool(t[0].item() == 0.0), "max_abs_diff": float(t[1].item()),
                     "max_rel": float(t[2].item()), "all_finite": bool(t[3].item() == 0.0),
                     "tokens_checked": world * T,
                     "against": "the single-GPU layer (hmoe_ffn_forward, all experts) on each "
                                "rank's own tokens"}
        del y_ref, yd, rd, w_gate_up_full, w_down_full
        torch.cuda.empty_cache()

    marks = [make_events(n_marks) for _ in range(args.steps)]
    starts = make_events(args.steps)
    ends = make_events(args.steps)
    torch.cuda.synchronize()
    with ClockSampler(gpu_uuid(torch, local_rank)) as clocks:
        # the barrier comes after each rank's sampler has started (that waits
        # for its first sample), so that the ranks enter the timed steps
        # together: an expert-parallel step waits for its peers' rows
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush()
            starts[i].record(stream)
            step(marks[i])
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ops.workspace_status(ws)
    if peer is not None:
        peer.status()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if ep is None:
        phase_names = ["router", "dispatch", "gate_up_gemm", "down_gemm", "combine"]
    elif peer is not None:
        phase_names = ["router_dispatch", "exchange", "dispatch_and_gate_up",
                       "down_gemm_and_return", "combine"]
    else:
        phase_names = ["router_dispatch", "a2a_dispatch", "local_experts", "a2a_combine",
                       "combine"]
    phase_ms = {n: statistics.mean(m[i].elapsed_time(m[i + 1]) for m in marks)
                for i, n in enumerate(phase_names)}
    ms = statistics.mean(step_ms)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_eager = ms

    # ------------------------------------------ one CUDA graph per step (N=1)
    # The C ABI is capture-safe (no host sync, no allocation, setup done on
    # the first call), so a serving loop captures the layer once and replays
    # it; the K timed steps are K replays, each after the L2 flush.
    graph_used = False
    phases_eager_ms = None
    if world == 1 and not args.no_graph:
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="relaxed"):
            _lib.check(lib.hmoe_ffn_forward(
                ctypes.byref(cshape), ctypes.c_void_p(x.data_ptr()),
                ctypes.c_void_p(w_router.data_ptr()), bias_p, ctypes.c_void_p(w_gate_up.data_ptr()),
                ctypes.c_void_p(w_down.data_ptr()), ctypes.c_void_p(y.data_ptr()), 0, None, None,
                None, None, ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                ctypes.c_void_p(cap.cuda_stream)))
        stream.wait_stream(cap)
        for _ in range(args.warmup):
            flush()
            graph.replay()
        g_s, g_e = make_events(args.steps), make_events(args.steps)
        torch.cuda.synchronize()
        with ClockSampler(gpu_uuid(torch, local_rank)) as clocks:
            for i in range(args.steps):
                flush()
                g_s[i].record(stream)
                graph.replay()
                g_e[i].record(stream)
            torch.cuda.synchronize()
        ops.workspace_status(ws)
        ms = statistics.mean(a.elapsed_time(b) for a, b in zip(g_s, g_e))
        graph_used = True
        del graph
        # Per-stage times of the same graph form: the marked layer captured
        # once (its events become event-record nodes of the graph) and
        # replayed after the L2 flush, read after each replay (untimed).
        gm = make_events(n_marks)
        mgraph = torch.cuda.CUDAGraph()
        cap.wait_stream(stream)
        with torch.cuda.graph(mgraph, stream=cap, capture_error_mode="relaxed"):
            arr = (ctypes.c_void_p * n_marks)(*[ctypes.c_void_p(m.cuda_event) for m in gm])
            _lib.check(lib.hmoe_ffn_forward_marked(
                ctypes.byref(cshape), ctypes.c_void_p(x.data_ptr()),
                ctypes.c_void_p(w_router.data_ptr()), bias_p, ctypes.c_void_p(w_gate_up.data_ptr()),
                ctypes.c_void_p(w_down.data_ptr()), ctypes.c_void_p(y.data_ptr()), 0,
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(cap.cuda_stream), arr))
        stream.wait_stream(cap)
        graph_phase = {n: [] for n in phase_names}
        for r in range(max(3, min(args.steps, 50)) + 2):
            flush()
            mgraph.replay()
            torch.cuda.synchronize()
            if r >= 2:
                for i, n in enumerate(phase_names):
                    graph_phase[n].append(gm[i].elapsed_time(gm[i + 1]))
        ops.workspace_status(ws)
        del mgraph
        phases_eager_ms = phase_ms
        phase_ms = {n: statistics.mean(v) for n, v in graph_phase.items()}

    # ------------------------------------------------- end to end (public API)
    # The C ABI on pinned HOST buffers (hmoe_ffn_forward_host): every step
    # copies the tokens in and the layer output out; the copies of one chunk
    # overlap the layer on the next.
    e2e = None
    if not args.no_e2e and ep is None:
        x_host = x.cpu().pin_memory()
        y_host = torch.empty_like(x_host).pin_memory()
        chunk = min(T, args.e2e_chunk or 3584)
        cs = ops.make_shape(T, d, E, I, k, dt, shape.norm_topk_prob)
        hws = torch.empty(lib.hmoe_ffn_host_workspace_bytes(ctypes.byref(cs), chunk),
                          dtype=torch.uint8, device=dev)
        e_s, e_e = make_events(args.steps), make_events(args.steps)
        for i in range(args.warmup + args.steps):
            flush()
            if i >= args.warmup:
                e_s[i - args.warmup].record(stream)
            ops.ffn_forward_host(x_host, w_router, w_gate_up, w_down, k, shape.norm_topk_prob,
                                 router_bias=bias, y_host=y_host, chunk_tokens=chunk,
                                 workspace=hws)
            if i >= args.warmup:
                e_e[i - args.warmup].record(stream)
        torch.cuda.synchronize()
        e2e_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(e_s, e_e))
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": T * d * es,
               "d2h_bytes_per_step": T * d * es,
               "api": f"hmoe_ffn_forward_host (C ABI, pinned host buffers, {chunk}-token chunks)"}
    elif not args.no_e2e and peer is not None:
        # every step: pinned host tokens in, the peer-memory EP layer, output
        # back to pinned host memory, in chunks whose copies overlap the layer
        x_host = x.cpu().pin_memory()
        y_host = torch.empty_like(x_host).pin_memory()
        chunk = min(T, args.e2e_chunk or 4096)
        e_s, e_e = make_events(args.steps), make_events(args.steps)
        dist.barrier()
        for i in range(args.warmup + args.steps):
            flush()
            if i >= args.warmup:
                e_s[i - args.warmup].record(stream)
            peer.forward_host(x_host, w_router, w_gate_up, w_down, y_host=y_host,
                              chunk_tokens=chunk, router_bias=bias)
            if i >= args.warmup:
                e_e[i - args.warmup].record(stream)
        torch.cuda.synchronize()
        peer.status()
        e2e_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(e_s, e_e))
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
        e2e = {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": T * d * es,
               "d2h_bytes_per_step": T * d * es,
               "api": f"PeerExpertParallel.forward_host (pinned host buffers, {chunk}-token "
                      "chunks, copies overlapped with the layer)"}

    # ------------------------------------------------------------ roofline
    peaks = measured_peaks()
    train = None
    if world == 1 and not args.no_train and shape.dtype == "bf16":
        train = measure_train_step(torch, lib, _lib, ops, shape, x, w_router, bias, w_gate_up,
                                   w_down, flush, stream, args.warmup, args.train_steps, peaks)
    A = T * k
    gu_flops, dn_flops = shape.gemm_flops()
    if ep is None:
        algo = {
            "router": ("hbm", T * d * es + E * d * es + T * k * (4 + es)),
            "dispatch": ("hbm", T * d * es + A * d * es + A * 8),
            "gate_up_gemm": ("tensor", gu_flops),
            "down_gemm": ("tensor", dn_flops),
            "combine": ("hbm", A * d * es + A * (4 + es) + T * d * es),
        }
    else:
        # NVLink bytes: the rows that leave this rank (or arrive), whichever is larger
        link_rows = max(send_rows, recv_rows)
        gemm_flops = 2.0 * gemm_rows * d * 2 * I + 2.0 * gemm_rows * I * d
        combine_bytes = A * d * es + A * (4 + es) + T * d * es
        if peer is not None:
            algo = {
                "router_dispatch": ("hbm", T * d * es + E * d * es + A * 20),
                "exchange": ("latency", 0),
                # one kernel each: the gate_up GEMM whose sender warps push the
                # rows out over NVLink, and the down GEMM whose epilogue stores
                # them back; each targets the slower of its GEMM and its link
                "dispatch_and_gate_up": ("fused", (2.0 * gemm_rows * d * 2 * I, link_rows * d * es)),
                "down_gemm_and_return": ("fused", (2.0 * gemm_rows * I * d, link_rows * d * es)),
                "combine": ("hbm", combine_bytes),
            }
        else:
            algo = {
                "router_dispatch": ("hbm", T * d * es + E * d * es + T * d * es + A * d * es),
                "a2a_dispatch": ("nvlink", link_rows * d * es),
                "local_experts": ("tensor", gemm_flops),
                "a2a_combine": ("nvlink", link_rows * d * es),
                "combine": ("hbm", combine_bytes),
            }
    phases = {}
    for n in phase_names:
        bound, work = algo[n]
        sec = phase_ms[n] * 1e-3
        if bound == "tensor":
            ach = work / sec / 1e12
            phases[n] = {"ms": phase_ms[n], "bound": "tensor", "achieved": ach,
                         "unit": "TFLOP/s", "frac": ach / peaks["bf16_tflops"]}
            if peaks.get("bf16_tflops_sustained"):
                # the timed steps run back to back under the power cap: the
                # measured sustained cuBLAS figure, beside the burst one
                phases[n]["frac_of_sustained"] = ach / peaks["bf16_tflops_sustained"]
        elif bound == "latency":
            phases[n] = {"ms": phase_ms[n], "bound": "latency", "achieved": None, "unit": None,
                         "frac": None}
        elif bound == "fused":
            flops, link_bytes = work
            target = max(flops / (peaks["bf16_tflops"] * 1e12), link_bytes / (NVLINK_GBS * 1e9))
            phases[n] = {"ms": phase_ms[n], "bound": "tensor+nvlink",
                         "achieved": target / sec, "unit": "fraction of max(GEMM, NVLink) time",
                         "frac": target / sec, "tflops": flops / sec / 1e12,
                         "nvlink_gbs": link_bytes / sec / 1e9}
        elif bound == "nvlink":
            ach = work / sec / 1e9
            phases[n] = {"ms": phase_ms[n], "bound": "nvlink", "achieved": ach, "unit": "GB/s",
                         "frac": ach / NVLINK_GBS}
        else:
            ach = work / sec / 1e9
            phases[n] = {"ms": phase_ms[n], "bound": "hbm", "achieved": ach, "unit": "GB/s",
                         "frac": ach / peaks["hbm_gbs"]}
    dom = max((n for n in phase_names if phases[n]["bound"] != "latency"), key=lambda n: phase_ms[n])
    dp = phases[dom]
    peak_of = {"tensor": peaks["bf16_tflops"], "hbm": peaks["hbm_gbs"], "nvlink": NVLINK_GBS,
               "tensor+nvlink": 1.0}
    roofline = {"kernel": dom, "bound": dp["bound"], "achieved": dp["achieved"],
                "peak": peak_of[dp["bound"]],
                "unit": dp["unit"], "frac": dp["frac"],
                "peak_source": f"{peaks['source']} (burst)" if dp["bound"] == "tensor" else peaks["source"],
                "peak_sustained": peaks.get("bf16_tflops_sustained") if dp["bound"] == "tensor" else None,
                "frac_of_sustained": dp.get("frac_of_sustained"),
                "traffic": (NCU_TRAFFIC_BYTES.get((args.config, T), {}).get(dom)
                            if world == 1 else None),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, "
                                  "one capture of this workload (profiles/)",
                "algorithmic": algo[dom][1]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, Ts, secs = cpu_oracle_tokens_per_s(
            shape, args.cpu_seconds,
            bias=config_router_bias(syn, args.config, shape, args.dead_experts))
        cpu = {"value": tps, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{Ts} tokens of the {args.config} layer in {secs:.1f} s "
                         f"(numpy/OpenBLAS + C router, {os.cpu_count()} host threads)"}

    clk = clocks.summary()
    if peer is not None:
        peer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": world * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": shape.dtype,
        "data": "synthetic: x~N(0,1), weights~N(0,0.02) (seeded torch.Generator on device)",
        "config": {"workload": workload_name(args.config, shape, T, args.dead_experts),
                   "tokens_per_gpu": T, "global_tokens": world * T,
                   "parallelism": ("single GPU" if world == 1 else
                                   f"expert parallel x{world} ({E // world} experts per GPU, "
                                   + ("rows over NVLink peer memory, no host sync)"
                                      if peer is not None else "NCCL all_to_all)")),
                   "l2": L2_NOTE},
        "roofline": roofline,
        "phases": phases,
        "launch": ("one CUDA graph per step (the layer captured once, replayed K times)"
                   if graph_used else "eager launches"),
        "phases_source": ("the marked layer as one CUDA graph, events recorded by graph nodes, "
                          "mean over replays after the L2 flush" if graph_used
                          else "events between the kernels of the timed steps"),
        "ms_per_step_eager": ms_eager,
        "phases_eager_ms": phases_eager_ms,
        "cpu_baseline": cpu,
        "e2e": e2e,
        # ours per step: router (1: the pair pass fixes its tokens itself),
        # dispatch (3), 2 GEMMs, combine; the peer path adds the exchange and
        # one wait (the row push runs inside the gate_up GEMM, the return
        # inside the down GEMM); NCCL's own kernels are not counted
        "gpu_launches": (9 if peer is not None else 7) * args.steps,
        "clocks": clk,
    }
    if ep_parity is not None:
        line["ep_parity"] = ep_parity
    if train is not None:
        line["train"] = train
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.prepare_reference:
        return prepare_reference(args.prepare_reference)
    rank, world, local_rank = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.impl == "reference-gpu":
        return reference_gpu_arm(args, rank, world, local_rank)
    return b200_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
