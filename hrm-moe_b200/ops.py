"""Functional API on torch tensors, one function per reference operator.

Each function mirrors a piece of XiaoYee/HRM-MoE's MoE path (argument
meaning, dtypes, error types) and runs the matching C-ABI entry point on the
current CUDA stream.  torch provides device memory and the stream only; all
arithmetic runs in the native sm_100a kernels.  Scratch workspaces come from
torch's caching allocator on the current stream.

Errors follow the reference: ``ValueError`` for bad shapes
(models/layers.py:531-539, models/moe_triton_grouped_gemm.py:367-368),
``TypeError`` for an unsupported dtype (moe_triton_grouped_gemm.py:350-355),
``RuntimeError`` when the backend cannot run.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"B200 MoE kernels support bf16 and fp32, got {dtype}") from None


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("B200 MoE kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _contig(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if t is None else t.contiguous()


def make_shape(tokens: int, hidden: int, experts: int, intermediate: int, top_k: int,
               dtype: torch.dtype, norm_topk_prob: bool = True) -> _lib.HmoeShape:
    return _lib.HmoeShape(int(tokens), int(hidden), int(experts), int(intermediate), int(top_k),
                          dtype_code(dtype), 1 if norm_topk_prob else 0)


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1024), dtype=torch.uint8, device=device)


# ------------------------------------------------------------------ router --
def router_topk(x: torch.Tensor, w_router: torch.Tensor, top_k: int, norm_topk_prob: bool,
                router_bias: Optional[torch.Tensor] = None, return_logits: bool = False):
    """Router of SparseMoESwiGLU.forward (models/layers.py:604-610).

    Returns (topk_idx int32 [T, k], topk_weight [T, k] in x.dtype) and, with
    ``return_logits``, the rounded logits [T, E] in x.dtype.
    """
    dev = _require_cuda(x, w_router, router_bias)
    T, d = x.shape
    E = w_router.shape[0]
    if w_router.shape[1] != d:
        raise ValueError(f"router weight is {tuple(w_router.shape)}, hidden size is {d}")
    shape = make_shape(T, d, E, 8, top_k, x.dtype, norm_topk_prob)
    x, w_router, router_bias = _contig(x), _contig(w_router.to(x.dtype)), _contig(
        None if router_bias is None else router_bias.to(x.dtype))
    idx = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, top_k), dtype=x.dtype, device=dev)
    logits = torch.empty((T, E), dtype=x.dtype, device=dev) if return_logits else None
    lib = _lib.load()
    ws_bytes = lib.hmoe_router_workspace_bytes(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError(_lib.last_error())
    ws = _workspace(ws_bytes, dev)
    _lib.check(lib.hmoe_router_topk(ctypes.byref(shape), _ptr(x), _ptr(w_router), _ptr(router_bias),
                                    _ptr(idx), _ptr(w), _ptr(logits), _ptr(ws), ws.numel(),
                                    _stream(dev)))
    return (idx, w, logits) if return_logits else (idx, w)


# ---------------------------------------------------------------- dispatch --
def dispatch(topk_idx: torch.Tensor, num_experts: int, x: Optional[torch.Tensor] = None,
             topk_weight: Optional[torch.Tensor] = None, gather: bool = True):
    """Dispatch of SparseMoEGroupedExperts.forward (models/layers.py:311-322).

    Returns a dict with ``sort_idx`` (int32 [T*k], the stable sort order of
    the flattened assignments), ``counts`` (int32 [E]), ``sorted_token``
    (int32 [T*k]) and, when given, ``sorted_weight`` and ``x_sorted``.
    """
    dev = _require_cuda(topk_idx, x, topk_weight)
    T, k = topk_idx.shape
    dtype = x.dtype if x is not None else (topk_weight.dtype if topk_weight is not None else torch.bfloat16)
    d = x.shape[1] if x is not None else 8
    shape = make_shape(T, d, num_experts, 8, k, dtype)
    idx32 = topk_idx.to(torch.int32).contiguous()
    out = {
        "sort_idx": torch.empty(T * k, dtype=torch.int32, device=dev),
        "counts": torch.zeros(num_experts, dtype=torch.int32, device=dev),
        "sorted_token": torch.empty(T * k, dtype=torch.int32, device=dev),
    }
    if topk_weight is not None:
        topk_weight = topk_weight.to(dtype).contiguous()
        out["sorted_weight"] = torch.empty(T * k, dtype=dtype, device=dev)
    if x is not None and gather:
        x = x.contiguous()
        out["x_sorted"] = torch.empty((T * k, d), dtype=dtype, device=dev)
    lib = _lib.load()
    ws_bytes = lib.hmoe_dispatch_workspace_bytes(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError(_lib.last_error())
    ws = _workspace(ws_bytes, dev)
    _lib.check(lib.hmoe_dispatch(ctypes.byref(shape), _ptr(idx32), _ptr(topk_weight), _ptr(x),
                                 _ptr(out["sort_idx"]), _ptr(out["counts"]),
                                 _ptr(out["sorted_token"]), _ptr(out.get("sorted_weight")),
                                 _ptr(out.get("x_sorted")), _ptr(ws), ws.numel(), _stream(dev)))
    return out


# ------------------------------------------------------------ grouped GEMM --
def _grouped(input: torch.Tensor, weight: torch.Tensor, tokens_per_expert: torch.Tensor,
             swiglu: bool) -> torch.Tensor:
    if input.shape[0] == 0:
        n = weight.shape[1] // (2 if swiglu else 1)
        return input.new_empty((0, n))
    dev = _require_cuda(input, weight, tokens_per_expert)
    M, K = input.shape
    G, NW, WK = weight.shape
    if WK != K:
        raise ValueError(f"grouped GEMM K mismatch: input K={K}, weight K={WK}")
    if tokens_per_expert.numel() != G:
        raise ValueError(f"tokens_per_expert has {tokens_per_expert.numel()} entries, weight has {G} groups")
    code = dtype_code(input.dtype)
    if weight.dtype != input.dtype:
        raise TypeError(f"input is {input.dtype} but weight is {weight.dtype}")
    if swiglu and NW % 2:
        raise ValueError("gate_up weight needs an even number of rows")
    N = NW // 2 if swiglu else NW
    input, weight = input.contiguous(), weight.contiguous()
    tpe = tokens_per_expert.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty((M, N), dtype=input.dtype, device=dev)
    lib = _lib.load()
    ws = _workspace(lib.hmoe_grouped_linear_workspace_bytes(G), dev)
    fn = lib.hmoe_grouped_swiglu if swiglu else lib.hmoe_grouped_linear
    _lib.check(fn(_ptr(input), _ptr(weight), _ptr(tpe), M, N, K, G, code, _ptr(out), _ptr(ws),
                  ws.numel(), _stream(dev)))
    return out


def grouped_linear_backward(grad_out: torch.Tensor, input: torch.Tensor, weight: torch.Tensor,
                            tokens_per_expert: torch.Tensor, need_input: bool = True,
                            need_weight: bool = True):
    """_TritonGroupedLinear.backward (models/moe_triton_grouped_gemm.py:427-456).

    grad_out [M, N], input [M, K], weight [G, N, K] -> (grad_input [M, K] or
    None, grad_weight [G, N, K] or None), bf16 on the tensor cores (the
    reference's Triton backward raises TypeError for other dtypes).
    """
    dev = _require_cuda(grad_out, input, weight, tokens_per_expert)
    M, K = input.shape
    G, N, WK = weight.shape
    if WK != K or tuple(grad_out.shape) != (M, N):
        raise ValueError(f"grouped GEMM backward shapes: grad_out {tuple(grad_out.shape)}, "
                         f"input {tuple(input.shape)}, weight {tuple(weight.shape)}")
    if tokens_per_expert.numel() != G:
        raise ValueError(f"tokens_per_expert has {tokens_per_expert.numel()} entries, weight has {G} groups")
    if not (grad_out.dtype == input.dtype == weight.dtype == torch.bfloat16):
        raise TypeError(f"grouped GEMM backward supports bf16 only, got {grad_out.dtype}, "
                        f"{input.dtype}, {weight.dtype}")
    grad_out, input, weight = grad_out.contiguous(), input.contiguous(), weight.contiguous()
    tpe = tokens_per_expert.to(device=dev, dtype=torch.int32).contiguous()
    gi = torch.empty((M, K), dtype=input.dtype, device=dev) if need_input else None
    gw = torch.empty((G, N, K), dtype=weight.dtype, device=dev) if need_weight else None
    if gi is None and gw is None:
        return None, None
    lib = _lib.load()
    ws = _workspace(lib.hmoe_grouped_linear_workspace_bytes(G), dev)
    _lib.check(lib.hmoe_grouped_linear_backward(
        _ptr(grad_out), _ptr(input), _ptr(weight), _ptr(tpe), M, N, K, G, _lib.DTYPE_BF16,
        _ptr(gi), _ptr(gw), _ptr(ws), ws.numel(), _stream(dev)))
    return gi, gw


def grouped_swiglu_backward(grad_out: torch.Tensor, w_down: torch.Tensor, gate_up: torch.Tensor,
                            tokens_per_expert: torch.Tensor) -> torch.Tensor:
    """Backward through the down projection and SiLU(gate) * up
    (models/layers.py:327-331) in one GEMM: grad_out [M, d] = d(expert
    output), w_down [G, d, I], gate_up [M, 2I] saved by the forward ->
    d_gate_up [M, 2I].  bf16 only."""
    dev = _require_cuda(grad_out, w_down, gate_up, tokens_per_expert)
    M, d = grad_out.shape
    G, wd, I = w_down.shape
    if wd != d or tuple(gate_up.shape) != (M, 2 * I):
        raise ValueError(f"swiglu backward shapes: grad_out {tuple(grad_out.shape)}, "
                         f"w_down {tuple(w_down.shape)}, gate_up {tuple(gate_up.shape)}")
    if not (grad_out.dtype == w_down.dtype == gate_up.dtype == torch.bfloat16):
        raise TypeError("swiglu backward supports bf16 only")
    grad_out, w_down, gate_up = grad_out.contiguous(), w_down.contiguous(), gate_up.contiguous()
    tpe = tokens_per_expert.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty((M, 2 * I), dtype=grad_out.dtype, device=dev)
    if M == 0:
        return out
    lib = _lib.load()
    ws = _workspace(lib.hmoe_grouped_linear_workspace_bytes(G), dev)
    _lib.check(lib.hmoe_grouped_swiglu_backward(
        _ptr(grad_out), _ptr(w_down), _ptr(gate_up), _ptr(tpe), M, d, I, G, _ptr(out), _ptr(ws),
        ws.numel(), _stream(dev)))
    return out


class _GroupedLinearFn(torch.autograd.Function):
    """Autograd wrapper of the grouped linear, as _TritonGroupedLinear
    (models/moe_triton_grouped_gemm.py:420-456): saves input and weight,
    backward runs the dgrad and wgrad grouped GEMMs."""

    @staticmethod
    def forward(ctx, input, weight, tokens_per_expert):
        out = _grouped(input, weight, tokens_per_expert, swiglu=False)
        ctx.save_for_backward(input, weight, tokens_per_expert)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        input, weight, tpe = ctx.saved_tensors
        gi, gw = grouped_linear_backward(grad_out.to(input.dtype), input, weight, tpe,
                                         ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return gi, gw, None


def grouped_linear(input: torch.Tensor, weight: torch.Tensor,
                   tokens_per_expert: torch.Tensor) -> torch.Tensor:
    """triton_grouped_linear (models/moe_triton_grouped_gemm.py:478-485).

    input [M, K], weight [G, N, K], tokens_per_expert [G] (rows per group,
    contiguous in order) -> [M, N].  Differentiable for bf16 (the backward
    of _TritonGroupedLinear, :420-456): with autograd recording and input or
    weight requiring grad, the backward runs grouped_linear_backward.
    """
    if (torch.is_grad_enabled() and input.shape[0] > 0
            and (input.requires_grad or weight.requires_grad)):
        return _GroupedLinearFn.apply(input, weight, tokens_per_expert)
    return _grouped(input, weight, tokens_per_expert, swiglu=False)


def grouped_swiglu(input: torch.Tensor, w_gate_up: torch.Tensor,
                   tokens_per_expert: torch.Tensor) -> torch.Tensor:
    """gate_up GEMM + silu(gate) * up fused (models/layers.py:326-329).

    w_gate_up [G, 2I, K] -> [M, I].
    """
    return _grouped(input, w_gate_up, tokens_per_expert, swiglu=True)


def grouped_gemm_mapped(input: torch.Tensor, weight: torch.Tensor, group_rows: torch.Tensor,
                        group_weight: torch.Tensor, swiglu: bool) -> torch.Tensor:
    """Grouped GEMM where group g uses weight[group_weight[g]].

    The local expert step of the expert-parallel layer
    (models/layers.py:462-468): received rows are grouped by (source rank,
    local expert), so several groups share one expert's weight.
    """
    M, K = input.shape
    NW = weight.shape[1]
    N = NW // 2 if swiglu else NW
    if M == 0:
        return input.new_empty((0, N))
    dev = _require_cuda(input, weight, group_rows, group_weight)
    if weight.shape[2] != K:
        raise ValueError(f"grouped GEMM K mismatch: input K={K}, weight K={weight.shape[2]}")
    code = dtype_code(input.dtype)
    G = group_rows.numel()
    rows = group_rows.to(device=dev, dtype=torch.int32).contiguous()
    gw = group_weight.to(device=dev, dtype=torch.int32).contiguous()
    input, weight = input.contiguous(), weight.contiguous()
    out = torch.empty((M, N), dtype=input.dtype, device=dev)
    lib = _lib.load()
    ws = _workspace(lib.hmoe_grouped_linear_workspace_bytes(G), dev)
    _lib.check(lib.hmoe_grouped_gemm_mapped(_ptr(input), _ptr(weight), _ptr(rows), _ptr(gw), M, N,
                                            K, G, weight.shape[0], code, 1 if swiglu else 0,
                                            _ptr(out), _ptr(ws), ws.numel(), _stream(dev)))
    return out


# ----------------------------------------------------------------- combine --
def combine(expert_out: torch.Tensor, sort_idx: torch.Tensor, topk_weight: torch.Tensor,
            final_hidden_states: torch.Tensor) -> torch.Tensor:
    """Weighted combine (models/layers.py:332-334), in place on final_hidden_states."""
    dev = _require_cuda(expert_out, sort_idx, topk_weight, final_hidden_states)
    T, d = final_hidden_states.shape
    k = topk_weight.shape[1]
    if not final_hidden_states.is_contiguous():
        raise ValueError("final_hidden_states must be contiguous (it is updated in place)")
    shape = make_shape(T, d, max(k, 1), 8, k, final_hidden_states.dtype)
    expert_out = expert_out.to(final_hidden_states.dtype).contiguous()
    sort_idx = sort_idx.to(torch.int32).contiguous()
    topk_weight = topk_weight.to(final_hidden_states.dtype).contiguous()
    lib = _lib.load()
    ws = _workspace(lib.hmoe_combine_workspace_bytes(ctypes.byref(shape)), dev)
    _lib.check(lib.hmoe_combine(ctypes.byref(shape), _ptr(expert_out), _ptr(sort_idx),
                                _ptr(topk_weight), _ptr(final_hidden_states), _ptr(ws), ws.numel(),
                                _stream(dev)))
    return final_hidden_states


# ----------------------------------------------------------------- experts --
def experts_forward(hidden_states: torch.Tensor, selected_experts: torch.Tensor,
                    routing_weights: torch.Tensor, final_hidden_states: torch.Tensor,
                    w_gate_up: torch.Tensor, w_down: torch.Tensor,
                    counts_out: Optional[torch.Tensor] = None,
                    sort_idx_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SparseMoEGroupedExperts.forward (models/layers.py:285-335).

    Adds the routed experts' output into ``final_hidden_states`` in place and
    returns it.  selected_experts [T, k] (any integer dtype), routing_weights
    [T, k], w_gate_up [E, 2I, d], w_down [E, d, I].
    """
    T = hidden_states.shape[0]
    if T == 0:
        return final_hidden_states
    dev = _require_cuda(hidden_states, selected_experts, routing_weights, final_hidden_states,
                        w_gate_up, w_down)
    d = hidden_states.shape[1]
    E, two_i, wd = w_gate_up.shape
    I = two_i // 2
    k = selected_experts.shape[-1]
    if wd != d or tuple(w_down.shape) != (E, d, I):
        raise ValueError(f"expert weights {tuple(w_gate_up.shape)} / {tuple(w_down.shape)} do not "
                         f"match hidden size {d}")
    if not final_hidden_states.is_contiguous():
        raise ValueError("final_hidden_states must be contiguous (it is updated in place)")
    dt = hidden_states.dtype
    shape = make_shape(T, d, E, I, k, dt)
    hs = hidden_states.contiguous()
    idx = selected_experts.reshape(T, k).to(torch.int32).contiguous()
    rw = routing_weights.reshape(T, k).to(dt).contiguous()
    w_gate_up, w_down = w_gate_up.to(dt).contiguous(), w_down.to(dt).contiguous()
    lib = _lib.load()
    ws_bytes = lib.hmoe_experts_workspace_bytes(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError(_lib.last_error())
    ws = _workspace(ws_bytes, dev)
    _lib.check(lib.hmoe_experts_forward(ctypes.byref(shape), _ptr(hs), _ptr(idx), _ptr(rw),
                                        _ptr(w_gate_up), _ptr(w_down), _ptr(final_hidden_states),
                                        _ptr(counts_out), _ptr(sort_idx_out), _ptr(ws), ws.numel(),
                                        _stream(dev)))
    return final_hidden_states


# ------------------------------------------------------------------- layer --
def ffn_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                router_bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                accumulate: bool = False, return_routing: bool = False):
    """SparseMoESwiGLU.forward on a flat [T, d] input (models/layers.py:596-634).

    Returns y [T, d] and, with ``return_routing``, a dict with ``topk_idx``
    (int32 [T, k]), ``topk_weight`` ([T, k]), ``counts`` (int32 [E]) and
    ``sort_idx`` (int32 [T*k]).
    """
    T, d = x.shape
    dt = x.dtype
    code = dtype_code(dt)
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    if tuple(w_gate_up.shape) != (E, 2 * I, d) or tuple(w_down.shape) != (E, d, I):
        raise ValueError(f"expert weights {tuple(w_gate_up.shape)} / {tuple(w_down.shape)} do not "
                         f"match hidden size {d} and {E} experts")
    if out is None:
        out = (torch.zeros if accumulate else torch.empty)((T, d), dtype=dt, device=x.device)
    routing = None
    if T == 0:
        return (out, routing) if return_routing else out
    dev = _require_cuda(x, w_router, w_gate_up, w_down, router_bias, out)
    shape = _lib.HmoeShape(T, d, E, I, top_k, code, 1 if norm_topk_prob else 0)
    x = x.contiguous()
    w_router = w_router.to(dt).contiguous()
    w_gate_up = w_gate_up.to(dt).contiguous()
    w_down = w_down.to(dt).contiguous()
    bias = None if router_bias is None else router_bias.to(dt).contiguous()
    if return_routing:
        routing = {
            "topk_idx": torch.empty((T, top_k), dtype=torch.int32, device=dev),
            "topk_weight": torch.empty((T, top_k), dtype=dt, device=dev),
            "counts": torch.empty(E, dtype=torch.int32, device=dev),
            "sort_idx": torch.empty(T * top_k, dtype=torch.int32, device=dev),
        }
    r = routing or {}
    lib = _lib.load()
    ws_bytes = lib.hmoe_ffn_workspace_bytes(ctypes.byref(shape))
    if ws_bytes == 0:
        raise ValueError(_lib.last_error())
    ws = _workspace(ws_bytes, dev)
    _lib.check(lib.hmoe_ffn_forward(
        ctypes.byref(shape), _ptr(x), _ptr(w_router), _ptr(bias), _ptr(w_gate_up), _ptr(w_down),
        _ptr(out), 1 if accumulate else 0, _ptr(r.get("topk_idx")), _ptr(r.get("topk_weight")),
        _ptr(r.get("counts")), _ptr(r.get("sort_idx")), _ptr(ws), ws.numel(), _stream(dev)))
    return (out, routing) if return_routing else out


# ---------------------------------------------------------------- training --
def _train_shape(x, w_router, w_gate_up, w_down, top_k, norm_topk_prob):
    T, d = x.shape
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    if tuple(w_gate_up.shape) != (E, 2 * I, d) or tuple(w_down.shape) != (E, d, I):
        raise ValueError(f"expert weights {tuple(w_gate_up.shape)} / {tuple(w_down.shape)} do not "
                         f"match hidden size {d} and {E} experts")
    if x.dtype != torch.bfloat16:
        # the reference's Triton backend has no other training dtype
        # (models/moe_triton_grouped_gemm.py:350-355)
        raise TypeError(f"the B200 MoE training path supports bf16 only, got {x.dtype}")
    return _lib.HmoeShape(T, d, E, I, top_k, _lib.DTYPE_BF16, 1 if norm_topk_prob else 0)


def ffn_forward_train(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                      w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                      router_bias: Optional[torch.Tensor] = None, aux_tokens: int = -1):
    """The layer forward keeping what the backward needs (bf16).

    Returns (y [T, d], saved (opaque uint8 buffer), aux_loss (fp32 scalar
    tensor), expert_counts (fp32 [E])).  With ``aux_tokens`` >= 0 the aux
    loss and counts are those of models/layers.py:619-632 over the first
    ``aux_tokens`` tokens; otherwise they are zeros.
    """
    dev = _require_cuda(x, w_router, w_gate_up, w_down, router_bias)
    shape = _train_shape(x, w_router, w_gate_up, w_down, top_k, norm_topk_prob)
    T, d = x.shape
    E = w_router.shape[0]
    lib = _lib.load()
    saved_bytes = lib.hmoe_ffn_train_saved_bytes(ctypes.byref(shape))
    ws_bytes = lib.hmoe_ffn_train_workspace_bytes(ctypes.byref(shape))
    if saved_bytes == 0 or ws_bytes == 0:
        raise ValueError(_lib.last_error())
    saved = _workspace(saved_bytes, dev)
    ws = _workspace(ws_bytes, dev)
    y = torch.empty((T, d), dtype=x.dtype, device=dev)
    aux = torch.zeros((), dtype=torch.float32, device=dev)
    counts = torch.zeros(E, dtype=torch.float32, device=dev)
    x, w_router = x.contiguous(), w_router.contiguous()
    w_gate_up, w_down = w_gate_up.contiguous(), w_down.contiguous()
    bias = None if router_bias is None else router_bias.to(x.dtype).contiguous()
    _lib.check(lib.hmoe_ffn_forward_train(
        ctypes.byref(shape), _ptr(x), _ptr(w_router), _ptr(bias), _ptr(w_gate_up), _ptr(w_down),
        _ptr(y), int(aux_tokens), _ptr(aux), _ptr(counts), _ptr(saved), saved.numel(), _ptr(ws),
        ws.numel(), _stream(dev)))
    return y, saved, aux, counts


def ffn_backward(grad_y: torch.Tensor, saved: torch.Tensor, x: torch.Tensor,
                 w_router: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                 top_k: int, norm_topk_prob: bool, router_bias: Optional[torch.Tensor] = None,
                 aux_grad: Optional[torch.Tensor] = None, aux_tokens: int = -1,
                 needs=(True, True, True, True, True)):
    """Gradients of the layer (models/layers.py:596-634, with the aux loss of
    :619-632 when ``aux_grad`` is given) from a :func:`ffn_forward_train`.

    ``needs`` selects (x, w_router, router_bias, w_gate_up, w_down).  Returns
    the five gradients (None where not needed or not applicable), bf16.
    """
    dev = _require_cuda(grad_y, saved, x, w_router, w_gate_up, w_down, router_bias, aux_grad)
    shape = _train_shape(x, w_router, w_gate_up, w_down, top_k, norm_topk_prob)
    T, d = x.shape
    E, I = w_router.shape[0], w_gate_up.shape[1] // 2

    def make(n, *sz):
        return torch.empty(sz, dtype=torch.bfloat16, device=dev) if n else None

    gx = make(needs[0], T, d)
    gwr = make(needs[1], E, d)
    gb = make(needs[2] and router_bias is not None, E)
    gwgu = make(needs[3], E, 2 * I, d)
    gwd = make(needs[4], E, d, I)
    lib = _lib.load()
    ws = _workspace(lib.hmoe_ffn_train_workspace_bytes(ctypes.byref(shape)), dev)
    grad_y = grad_y.to(torch.bfloat16).contiguous()
    ag = None if aux_grad is None else aux_grad.to(torch.float32).reshape(()).contiguous()
    bias = None if router_bias is None else router_bias.to(x.dtype).contiguous()
    _lib.check(lib.hmoe_ffn_backward(
        ctypes.byref(shape), _ptr(grad_y), _ptr(ag), int(aux_tokens), _ptr(x.contiguous()),
        _ptr(w_router.contiguous()), _ptr(bias), _ptr(w_gate_up.contiguous()),
        _ptr(w_down.contiguous()), _ptr(saved), saved.numel(), _ptr(gx), _ptr(gwr), _ptr(gb),
        _ptr(gwgu), _ptr(gwd), _ptr(ws), ws.numel(), _stream(dev)))
    return gx, gwr, gb, gwgu, gwd


class _FfnFunction(torch.autograd.Function):
    """SparseMoESwiGLU's forward and backward as one autograd node: the
    training forward keeps its activations in one buffer, and the backward
    runs the native backward kernels.  Outputs (y, aux_loss, expert_counts);
    expert_counts is not differentiable (the reference computes it under
    no_grad, models/layers.py:630-631)."""

    @staticmethod
    def forward(ctx, x, w_router, router_bias, w_gate_up, w_down, top_k, norm_topk_prob,
                aux_tokens):
        y, saved, aux, counts = ffn_forward_train(x, w_router, w_gate_up, w_down, top_k,
                                                  norm_topk_prob, router_bias, aux_tokens)
        ctx.save_for_backward(x, w_router, router_bias, w_gate_up, w_down, saved)
        ctx.cfg = (top_k, norm_topk_prob, aux_tokens)
        ctx.mark_non_differentiable(counts)
        return y, aux, counts

    @staticmethod
    def backward(ctx, grad_y, grad_aux, _grad_counts):
        x, w_router, router_bias, w_gate_up, w_down, saved = ctx.saved_tensors
        top_k, norm, aux_tokens = ctx.cfg
        n = ctx.needs_input_grad
        if grad_y is None:
            grad_y = torch.zeros_like(x)
        gx, gwr, gb, gwgu, gwd = ffn_backward(
            grad_y, saved, x, w_router, w_gate_up, w_down, top_k, norm, router_bias,
            aux_grad=grad_aux if aux_tokens >= 0 else None, aux_tokens=aux_tokens,
            needs=(n[0], n[1], n[2], n[3], n[4]))
        return gx, gwr, gb, gwgu, gwd, None, None, None


def ffn_forward_autograd(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                         w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                         router_bias: Optional[torch.Tensor] = None, aux_tokens: int = -1):
    """Differentiable layer forward (bf16): (y, aux_loss, expert_counts).

    Gradients flow to x, the router weight (and bias) and both expert
    weights; aux_loss (when ``aux_tokens`` >= 0) is differentiable too.
    """
    return _FfnFunction.apply(x, w_router, router_bias, w_gate_up, w_down, int(top_k),
                              bool(norm_topk_prob), int(aux_tokens))


class CapturedFfn:
    """The layer forward captured once as a CUDA graph over fixed buffers.

    For serving loops with a fixed token count: the kernels of one forward
    (router, dispatch, the two grouped GEMMs, combine) are replayed as one
    graph launch, which removes the per-kernel launch gaps.  ``x_static`` is
    the graph's input and ``y`` its output; ``__call__(x)`` copies ``x`` into
    the input (same shape and dtype), replays the graph on the current stream
    and returns ``y`` (overwritten by the next call).  Same kernels and
    results as :func:`ffn_forward`.
    """

    def __init__(self, x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                 w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                 router_bias: Optional[torch.Tensor] = None):
        T, d = x.shape
        if T == 0:
            raise ValueError("nothing to capture for 0 tokens")
        dev = _require_cuda(x, w_router, w_gate_up, w_down, router_bias)
        dt = x.dtype
        E = w_router.shape[0]
        I = w_gate_up.shape[1] // 2
        if tuple(w_gate_up.shape) != (E, 2 * I, d) or tuple(w_down.shape) != (E, d, I):
            raise ValueError(f"expert weights {tuple(w_gate_up.shape)} / {tuple(w_down.shape)} do "
                             f"not match hidden size {d} and {E} experts")
        self.x_static = x.detach().clone().contiguous()
        self.y = torch.empty_like(self.x_static)
        self._w = [w_router.to(dt).contiguous(), w_gate_up.to(dt).contiguous(),
                   w_down.to(dt).contiguous(),
                   None if router_bias is None else router_bias.to(dt).contiguous()]
        self._shape = _lib.HmoeShape(T, d, E, I, top_k, dtype_code(dt), 1 if norm_topk_prob else 0)
        lib = _lib.load()
        nbytes = lib.hmoe_ffn_workspace_bytes(ctypes.byref(self._shape))
        if nbytes == 0:
            raise ValueError(_lib.last_error())
        self._ws = _workspace(nbytes, dev)
        self._launch(torch.cuda.current_stream(dev))  # first call: per-device set-up
        torch.cuda.current_stream(dev).synchronize()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=cap, capture_error_mode="relaxed"):
            self._launch(cap)
        torch.cuda.current_stream(dev).wait_stream(cap)

    def _launch(self, stream: torch.cuda.Stream) -> None:
        wr, wgu, wd, b = self._w
        lib = _lib.load()
        _lib.check(lib.hmoe_ffn_forward(
            ctypes.byref(self._shape), _ptr(self.x_static), _ptr(wr), _ptr(b), _ptr(wgu), _ptr(wd),
            _ptr(self.y), 0, None, None, None, None, _ptr(self._ws), self._ws.numel(),
            ctypes.c_void_p(stream.cuda_stream)))

    def __call__(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            if x.shape != self.x_static.shape or x.dtype != self.x_static.dtype:
                raise ValueError(f"captured for {tuple(self.x_static.shape)} {self.x_static.dtype}, "
                                 f"got {tuple(x.shape)} {x.dtype}")
            self.x_static.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.y


def ffn_forward_host(x_host: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
                     w_down: torch.Tensor, top_k: int, norm_topk_prob: bool,
                     router_bias: Optional[torch.Tensor] = None,
                     y_host: Optional[torch.Tensor] = None, chunk_tokens: int = 4096,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The layer on host tensors (pinned for overlap), weights on the GPU.

    Copies in, computes and copies out chunk by chunk with the three
    overlapped (hmoe_ffn_forward_host).  Returns y_host; it is complete when
    the current CUDA stream of the weights' device reaches this point.
    """
    if x_host.is_cuda:
        raise ValueError("x_host must be a host tensor")
    if not x_host.is_contiguous() or (y_host is not None and not y_host.is_contiguous()):
        raise ValueError("x_host and y_host must be contiguous (the copies are asynchronous)")
    if y_host is not None and y_host.dtype != x_host.dtype:
        raise TypeError("y_host must have x_host's dtype")
    T, d = x_host.shape
    dt = x_host.dtype
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    dev = _require_cuda(w_router, w_gate_up, w_down, router_bias)
    if y_host is None:
        y_host = torch.empty((T, d), dtype=dt, pin_memory=True)
    if T == 0:
        return y_host
    shape = _lib.HmoeShape(T, d, E, I, top_k, dtype_code(dt), 1 if norm_topk_prob else 0)
    lib = _lib.load()
    ws_bytes = lib.hmoe_ffn_host_workspace_bytes(ctypes.byref(shape), chunk_tokens)
    if ws_bytes == 0:
        raise ValueError(_lib.last_error())
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = _workspace(ws_bytes, dev)
    bias = None if router_bias is None else router_bias.to(dt).contiguous()
    _lib.check(lib.hmoe_ffn_forward_host(
        ctypes.byref(shape), _ptr(x_host), _ptr(w_router.to(dt).contiguous()),
        _ptr(bias), _ptr(w_gate_up.to(dt).contiguous()), _ptr(w_down.to(dt).contiguous()),
        _ptr(y_host), chunk_tokens, _ptr(workspace), workspace.numel(), _stream(dev)))
    return y_host


def workspace_status(workspace: torch.Tensor) -> None:
    """Raise if kernels flagged an error in ``workspace`` (synchronises)."""
    lib = _lib.load()
    _lib.check(lib.hmoe_workspace_status(_ptr(workspace), _stream(workspace.device)))
