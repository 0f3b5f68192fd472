"""Seeded synthetic inputs for the routed MoE-FFN forward.

The reference measures this layer on synthetic data only: hidden states are
N(0, 1) and every weight (router [E, d], expert gate/up [E, 2I, d], expert
down [E, d, I]) is N(0, 0.02), all drawn from one seed.  The generator here
is numpy's PCG64 so the same arrays come out on any machine with numpy >= 2,
independently of torch's RNG.

Arrays are returned as float32.  For a bf16 workload every value is rounded
to bf16 (round-to-nearest-even) first, so the float32 array holds exactly the
bf16 values the GPU sees; converting it with ``torch.from_numpy(a).bfloat16()``
is lossless.

Parameter layout follows ``models/layers.py:272-283`` of the reference:
``gate_up_weight[e]`` rows ``0..I-1`` are the gate projection and rows
``I..2I-1`` the up projection (``models/layers.py:328`` chunks them in that
order); ``down_weight[e]`` is ``[d, I]``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

WEIGHT_STD = 0.02


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    # uint32 wrap-around only happens for NaN bit patterns, restored below
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    out = rounded.view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of bf16-exact float32 values (for compact fixtures)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


@dataclass(frozen=True)
class MoEShape:
    tokens: int
    hidden: int
    experts: int
    intermediate: int
    top_k: int
    norm_topk_prob: bool = True
    dtype: str = "bf16"  # "bf16" or "f32"

    @property
    def assignments(self) -> int:
        return self.tokens * self.top_k

    def gemm_flops(self) -> tuple[float, float]:
        """Algorithmic FLOPs of (gate_up, down) for one forward."""
        a = self.assignments
        return (2.0 * a * self.hidden * 2 * self.intermediate,
                2.0 * a * self.intermediate * self.hidden)


@dataclass
class MoEInputs:
    shape: MoEShape
    x: np.ndarray
    w_router: np.ndarray
    w_gate_up: np.ndarray
    w_down: np.ndarray
    router_bias: Optional[np.ndarray] = None
    meta: dict = field(default_factory=dict)


def _normal(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    out = rng.standard_normal(shape, dtype=np.float32)
    if scale != 1.0:
        out *= np.float32(scale)
    return out


def make_weights(shape: MoEShape, seed: int):
    """Router, gate/up and down weights drawn from one seed."""
    rng = np.random.default_rng([seed, 0])
    E, d, I = shape.experts, shape.hidden, shape.intermediate
    w_router = _normal(rng, (E, d), WEIGHT_STD)
    w_gate_up = _normal(rng, (E, 2 * I, d), WEIGHT_STD)
    w_down = _normal(rng, (E, d, I), WEIGHT_STD)
    if shape.dtype == "bf16":
        w_router, w_gate_up, w_down = (round_to_bf16(w) for w in (w_router, w_gate_up, w_down))
    return w_router, w_gate_up, w_down


def make_hidden(shape: MoEShape, seed: int, rank: int = 0) -> np.ndarray:
    """Hidden states [T, d] ~ N(0, 1); expert-parallel ranks use their own stream."""
    rng = np.random.default_rng([seed, 1, rank])
    x = _normal(rng, (shape.tokens, shape.hidden))
    return round_to_bf16(x) if shape.dtype == "bf16" else x


def zipf_router_bias(experts: int, seed: int, s: float = 1.2,
                     dead_experts: int = 0) -> np.ndarray:
    """Router bias b_e = log q_{pi(e)} with q proportional to rank^-s.

    Expected expert selection then follows Zipf(s) over a seeded random
    permutation pi of the experts.  ``dead_experts`` experts (chosen by the
    same seed) get b = -inf so no token is ever routed to them.
    """
    rng = np.random.default_rng([seed, 2])
    perm = rng.permutation(experts)
    ranks = np.arange(1, experts + 1, dtype=np.float64)
    q = ranks ** (-s)
    q /= q.sum()
    bias = np.empty(experts, dtype=np.float32)
    bias[perm] = np.log(q).astype(np.float32)
    if dead_experts:
        dead = rng.choice(experts, size=dead_experts, replace=False)
        bias[dead] = -np.inf
    return bias


def make_inputs(shape: MoEShape, seed: int, rank: int = 0,
                router_bias: Optional[np.ndarray] = None) -> MoEInputs:
    w_router, w_gate_up, w_down = make_weights(shape, seed)
    x = make_hidden(shape, seed, rank)
    return MoEInputs(shape=shape, x=x, w_router=w_router, w_gate_up=w_gate_up,
                     w_down=w_down, router_bias=router_bias,
                     meta={"seed": seed, "rank": rank})


# The reference's benchmark configurations (single MoE-FFN layer forward).
CONFIGS = {
    # L-scale layer in fp32 (the reference's CPU-runnable case).
    "cfg1_l_f32": MoEShape(2048, 1280, 64, 448, 8, True, "f32"),
    # XL 64x8 layer at 16K tokens in bf16: the headline single-GPU workload.
    "cfg2_xl64_bf16": MoEShape(16384, 1536, 64, 512, 8, True, "bf16"),
    # XL 128x8 layer, 32K tokens per rank, expert parallel.
    "cfg3_xl128_ep_bf16": MoEShape(32768, 1536, 128, 512, 8, True, "bf16"),
    # Load-imbalance stress: 64K tokens with a Zipf(1.2) router bias.
    "cfg4_xl64_zipf_bf16": MoEShape(65536, 1536, 64, 512, 8, True, "bf16"),
}


def tokens_per_second(tokens: int, ms: float) -> float:
    return tokens / (ms * 1e-3) if ms > 0 else math.inf
