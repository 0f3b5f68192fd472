"""torch custom ops over the C ABI: ``torch.ops.hrm_moe.*``.

Registers, on import of this module:

* ``hrm_moe::ffn_forward(x[T,d], w_router[E,d], w_gate_up[E,2I,d],
  w_down[E,d,I], top_k, norm_topk_prob, router_bias[E]?) ->
  (y[T,d], topk_idx[T,k] int32, topk_weight[T,k], counts[E] int32,
  perm[T*k] int32)``: the layer of models/layers.py:596-634 with the routing
  outputs the parity checks read (perm is the stable expert sort of the
  flattened selection, models/layers.py:317);
* ``hrm_moe::grouped_linear(input[M,K], weight[G,N,K],
  tokens_per_expert[G]) -> [M,N]``: models/moe_triton_grouped_gemm.py:478.

Each op runs the same kernels as ``ops.ffn_forward`` / ``ops.grouped_linear``
on the current stream, and carries a fake (meta) implementation so shape
propagation and graph capture see it as one opaque node.  Forward only, like
the rest of the backend.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops

_LIB = "hrm_moe"


@torch.library.custom_op(f"{_LIB}::ffn_forward", mutates_args=())
def ffn_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                router_bias: Optional[torch.Tensor] = None
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    T, d = x.shape
    E = w_router.shape[0]
    if T == 0:
        dev = x.device
        return (x.new_empty((0, d)), torch.empty((0, top_k), dtype=torch.int32, device=dev),
                x.new_empty((0, top_k)), torch.zeros(E, dtype=torch.int32, device=dev),
                torch.empty(0, dtype=torch.int32, device=dev))
    y, r = ops.ffn_forward(x, w_router, w_gate_up, w_down, top_k, norm_topk_prob, router_bias,
                           return_routing=True)
    return y, r["topk_idx"], r["topk_weight"], r["counts"], r["sort_idx"]


@ffn_forward.register_fake
def _ffn_forward_fake(x, w_router, w_gate_up, w_down, top_k, norm_topk_prob, router_bias=None):
    T, d = x.shape
    E = w_router.shape[0]
    return (x.new_empty((T, d)), x.new_empty((T, top_k), dtype=torch.int32),
            x.new_empty((T, top_k)), x.new_empty((E,), dtype=torch.int32),
            x.new_empty((T * top_k,), dtype=torch.int32))


@torch.library.custom_op(f"{_LIB}::grouped_linear", mutates_args=())
def grouped_linear(input: torch.Tensor, weight: torch.Tensor,
                   tokens_per_expert: torch.Tensor) -> torch.Tensor:
    return ops.grouped_linear(input, weight, tokens_per_expert)


@grouped_linear.register_fake
def _grouped_linear_fake(input, weight, tokens_per_expert):
    return input.new_empty((input.shape[0], weight.shape[1]))
