"""nn.Module mirror of HRM-MoE's MoE layer with the B200 expert backend.

``SparseMoESwiGLU(..., implementation="grouped_b200")`` keeps the
reference's constructor, forward signature and parameter layout
(models/layers.py:518-634), so ``state_dict`` keys and shapes are
unchanged: ``gate.weight`` [E, d] (+ optional ``gate.bias``),
``experts.gate_up_weight`` [E, 2I, d] and ``experts.down_weight`` [E, d, I].
Weights copied from the reference's ``origin`` / ``grouped`` /
``grouped_triton`` layers (e.g. scripts/test_moe_shard_equivalence.py:23-37)
load as they are.

Training works as in the reference: with autograd recording and any of x
or the parameters requiring grad, ``SparseMoESwiGLU`` runs the training
forward and its native backward (one autograd node for the layer), and with
a ``moe_context`` it appends the aux load-balancing loss and the expert
counts under the reference's keys (models/layers.py:619-632).
``SparseMoEGroupedExperts`` under autograd composes the reference's own
expert steps (layers.py:311-334) around the differentiable grouped GEMM.
Training is bf16 only, as the reference's Triton backend.
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


def _needs_grad(*tensors: Optional[Tensor]) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _valid_tokens(total_seqlen, tokens: int) -> int:
    """int(unwrap_tensor(total_seqlen).item()) (models/layers.py:622), at most tokens."""
    v = getattr(total_seqlen, "value", total_seqlen)  # a WrappedTensor holds .value
    v = int(v.item()) if hasattr(v, "item") else int(v)
    return max(0, min(v, tokens))


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
        dt = hidden_states.dtype
        w_gate_up, w_down = self.gate_up_weight.to(dt), self.down_weight.to(dt)
        if _needs_grad(hidden_states, routing_weights, w_gate_up, w_down, final_hidden_states):
            return self._forward_autograd(hidden_states, selected_experts, routing_weights,
                                          final_hidden_states, w_gate_up, w_down)
        return ops.experts_forward(hidden_states, selected_experts, routing_weights,
                                   final_hidden_states, w_gate_up, w_down)

    def _forward_autograd(self, hidden_states, selected_experts, routing_weights,
                          final_hidden_states, w_gate_up, w_down):
        """The reference's expert steps (layers.py:311-334) with the native
        dispatch (integer work, no gradient) and the differentiable grouped
        GEMM; the gathers, SiLU * up, weighting and index_add_ are the same
        torch ops the reference uses, so autograd differentiates them alike."""
        k = selected_experts.shape[-1]
        r = ops.dispatch(selected_experts.reshape(-1, k).to(torch.int32), self.num_experts)
        sort_idx, sorted_token = r["sort_idx"].long(), r["sorted_token"].long()
        sorted_weights = routing_weights.reshape(-1).index_select(0, sort_idx)
        sorted_hidden = hidden_states.index_select(0, sorted_token)
        gate_up = ops.grouped_linear(sorted_hidden, w_gate_up, r["counts"])
        gate, up = gate_up.chunk(2, dim=-1)
        activated = nn.functional.silu(gate) * up
        expert_output = ops.grouped_linear(activated, w_down, r["counts"])
        expert_output = expert_output * sorted_weights[:, None]
        final_hidden_states.index_add_(0, sorted_token, expert_output.to(hidden_states.dtype))
        return final_hidden_states


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
        dt = hidden_states.dtype
        w_router, bias = self.gate.weight, self.gate.bias
        w_gate_up = self.experts.gate_up_weight.to(dt)
        w_down = self.experts.down_weight.to(dt)
        # the reference records the aux loss and the expert counts only while
        # autograd records (layers.py:619)
        want_aux = moe_context is not None and torch.is_grad_enabled()
        if want_aux or _needs_grad(x, w_router, bias, w_gate_up, w_down):
            T = hidden_states.shape[0]
            aux_tokens = -1
            if want_aux:
                aux_tokens = T if total_seqlen is None else _valid_tokens(total_seqlen, T)
            if T == 0:
                y = hidden_states * 0
                aux = torch.zeros((), dtype=torch.float32, device=x.device)
                counts = torch.zeros(self.num_experts, dtype=torch.float32, device=x.device)
            else:
                y, aux, counts = ops.ffn_forward_autograd(
                    hidden_states, w_router, w_gate_up, w_down, self.top_k, self.norm_topk_prob,
                    router_bias=bias, aux_tokens=aux_tokens)
            if want_aux:
                moe_context.setdefault("aux_losses", []).append(aux)
                moe_context.setdefault("expert_counts", []).append(counts)
            return y.reshape(original_shape)
        y = ops.ffn_forward(hidden_states, w_router, w_gate_up, w_down, self.top_k,
                            self.norm_topk_prob, router_bias=bias)
        return y.reshape(original_shape)
