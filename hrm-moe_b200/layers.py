"""nn.Module mirror of HRM-MoE's MoE layer with the B200 expert backend.

``SparseMoESwiGLU(..., implementation="grouped_b200")`` keeps the
reference's constructor, forward signature and parameter layout
(models/layers.py:518-634), so ``state_dict`` keys and shapes are
unchanged: ``gate.weight`` [E, d] (+ optional ``gate.bias``),
``experts.gate_up_weight`` [E, 2I, d] and ``experts.down_weight`` [E, d, I].
Weights copied from the reference's ``origin`` / ``grouped`` /
``grouped_triton`` layers (e.g. scripts/test_moe_shard_equivalence.py:23-37)
load as they are.

The backend is forward-only: calling it where autograd would need a
backward raises instead of silently dropping gradients.
"""
from __future__ import annotations

import math
from typing import Any, Literal, Optional, Sequence

import torch
from torch import Tensor, nn

from . import ops

IMPLEMENTATIONS = ("grouped_b200",)


# std of a standard normal folded into (-3, 3) by fmod is 1 / 1.0147626...;
# the reference scales by this factor so the folded values have std 1.
_FOLDED_NORMAL_STD_FIX = 1.014762601732121


def trunc_normal_(t: Tensor, std: float) -> Tensor:
    """The reference's weight init (models/common.py:10-13): draw N(0, 1), fold
    values beyond +-3 back with fmod(3), and scale so the result has the given
    std.  Same distribution as the reference's parameters, so a randomly
    initialised layer here matches one built there."""
    with torch.no_grad():
        return t.normal_().fmod_(3.0).mul_(_FOLDED_NORMAL_STD_FIX * std)


class LinearInit(nn.Module):
    """Same parameters as the reference's LinearInit (models/layers.py:66-90)."""

    def __init__(self, in_features: int, out_features: int, bias: bool,
                 batch_out_features: Sequence[int] = (), init_std: Optional[float] = None,
                 **kwargs):
        super().__init__()
        self.in_features = in_features
        if init_std is None:
            init_std = 1.0 / (in_features ** 0.5)
        rows = math.prod(batch_out_features) * out_features
        self.weight = nn.Parameter(trunc_normal_(torch.empty((rows, in_features), **kwargs), init_std))
        self.bias = nn.Parameter(torch.zeros((rows,), **kwargs)) if bias else None

    def forward(self, input: Tensor) -> Tensor:
        return nn.functional.linear(input, self.weight, self.bias)


def _check_no_grad(*tensors: Optional[Tensor]) -> None:
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise NotImplementedError(
            "the grouped_b200 MoE backend implements the forward pass only; run it under "
            "torch.no_grad() / torch.inference_mode() or detach the parameters")


class SparseMoEGroupedExperts(nn.Module):
    """Experts backend with the reference's layout (models/layers.py:248-335)."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int,
                 init_std_in=None, init_std_out=None, **kwargs):
        super().__init__()
        if num_experts <= 0:
            raise ValueError(f"num_experts must be positive, got {num_experts}")
        if init_std_in is None:
            init_std_in = 1.0 / (hidden_size ** 0.5)
        if init_std_out is None:
            init_std_out = 1.0 / (intermediate_size ** 0.5)
        self.num_experts = num_experts
        self.expert_in_one_shard = num_experts
        self.gate_up_weight = nn.Parameter(trunc_normal_(
            torch.empty((num_experts, 2 * intermediate_size, hidden_size), **kwargs), init_std_in))
        self.down_weight = nn.Parameter(trunc_normal_(
            torch.empty((num_experts, hidden_size, intermediate_size), **kwargs), init_std_out))

    def forward(self, hidden_states: Tensor, selected_experts: Tensor, routing_weights: Tensor,
                final_hidden_states: Tensor) -> Tensor:
        """Adds the experts' weighted outputs into final_hidden_states (in place)."""
        if hidden_states.shape[0] == 0:
            return final_hidden_states
        _check_no_grad(hidden_states, routing_weights, self.gate_up_weight, self.down_weight)
        dt = hidden_states.dtype
        return ops.experts_forward(hidden_states, selected_experts, routing_weights,
                                   final_hidden_states, self.gate_up_weight.to(dt),
                                   self.down_weight.to(dt))


class SparseMoESwiGLU(nn.Module):
    """Routed MoE FFN with the reference's API (models/layers.py:518-634)."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool,
                 implementation: Literal["grouped_b200"] = "grouped_b200",
                 expert_in_one_shard: int = 1, init_std_in=None, init_std_out=None,
                 router_bias: bool = False, **kwargs):
        super().__init__()
        if num_experts <= 0:
            raise ValueError(f"num_experts must be positive, got {num_experts}")
        if top_k <= 0 or top_k > num_experts:
            raise ValueError(f"top_k must be in [1, num_experts], got top_k={top_k}, "
                             f"num_experts={num_experts}")
        if expert_in_one_shard <= 0 or num_experts % expert_in_one_shard != 0:
            raise ValueError(
                f"expert_in_one_shard must divide num_experts, got "
                f"expert_in_one_shard={expert_in_one_shard}, num_experts={num_experts}")
        if implementation not in IMPLEMENTATIONS:
            raise ValueError(f"implementation must be one of {IMPLEMENTATIONS}, got {implementation!r}")
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.implementation = implementation
        self.expert_in_one_shard = expert_in_one_shard
        self.gate = LinearInit(hidden_size, num_experts, bias=router_bias, init_std=init_std_in,
                               **kwargs)
        self.experts = SparseMoEGroupedExperts(hidden_size, intermediate_size, num_experts,
                                               init_std_in=init_std_in, init_std_out=init_std_out,
                                               **kwargs)

    def forward(self, x: Tensor, moe_context: Optional[dict[str, Any]] = None,
                total_seqlen: Optional[Tensor] = None, **_seq_info) -> Tensor:
        original_shape = x.shape
        hidden_states = x.reshape(-1, self.hidden_size)
        _check_no_grad(x, self.gate.weight, self.gate.bias, self.experts.gate_up_weight,
                       self.experts.down_weight)
        want_counts = moe_context is not None
        res = ops.ffn_forward(
            hidden_states, self.gate.weight, self.experts.gate_up_weight,
            self.experts.down_weight, self.top_k, self.norm_topk_prob,
            router_bias=self.gate.bias, return_routing=want_counts)
        y, routing = res if want_counts else (res, None)
        if routing is not None:
            # the reference records aux losses only when gradients flow
            # (layers.py:619); without them it keeps nothing, and the expert
            # counts are exposed here for monitoring
            moe_context.setdefault("expert_counts_b200", []).append(routing["counts"].float())
        return y.reshape(original_shape)
