"""Expert parallelism for the routed MoE FFN: peer memory (product) and NCCL.

Mirrors SparseMoEExpertParallel (models/layers.py:383-478): experts are
sharded contiguously (rank r owns [r*E/R, (r+1)*E/R), layers.py:403-405),
every rank routes its own tokens, rows travel to the rank that owns their
expert, the owner runs its local experts, and the outputs travel back.

Differences from the reference, by design:
* dispatch sorts by *global* expert once (the layer's own stable dispatch).
  Experts are contiguous per rank, so the sorted rows are already grouped by
  destination and the send buffer is the gathered row buffer itself;
* the owner runs its experts straight on the received rows, grouped by
  (source rank, local expert), with a group -> weight map instead of a
  second sort (layers.py:462-468 re-sorts);
* returned rows land at the positions the dispatch gave them, so the combine
  is the single-GPU combine and the result is bit-identical to one GPU
  running all experts (the reference re-sorts to match, layers.py:474-476).

Collectives per call: one all_to_all of per-expert counts (E/R per peer),
one host read of the split sizes (NCCL's variable all_to_all takes host
splits, as in the reference, layers.py:363-364), then the row all_to_all
each way.  The compute stages are a parameter so the same orchestration runs
on CPU ranks (gloo) in tests.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import ops


class CudaCompute:
    """The stages on this GPU, through the C ABI."""

    def router(self, x, w_router, bias, top_k, norm):
        return ops.router_topk(x, w_router, top_k, norm, bias)

    def dispatch(self, idx, num_experts, x, w):
        out = ops.dispatch(idx, num_experts, x, w)
        return out["sort_idx"], out["counts"], out["x_sorted"]

    def local_experts(self, rows, w_gate_up, w_down, group_rows, group_weight):
        h = ops.grouped_gemm_mapped(rows, w_gate_up, group_rows, group_weight, swiglu=True)
        return ops.grouped_gemm_mapped(h, w_down, group_rows, group_weight, swiglu=False)

    def combine(self, y_sorted, sort_idx, w, final):
        return ops.combine(y_sorted, sort_idx, w, final)


@dataclass
class EPStats:
    send_rows: list
    recv_rows: list


def ep_forward(x: torch.Tensor, w_router: torch.Tensor, w_gate_up_local: torch.Tensor,
               w_down_local: torch.Tensor, num_experts: int, top_k: int, norm_topk_prob: bool,
               group=None, router_bias: Optional[torch.Tensor] = None, compute=None,
               stats: Optional[list] = None, marks: Optional[list] = None) -> torch.Tensor:
    """Expert-parallel MoE-FFN forward of this rank's tokens x [T, d].

    ``marks`` (optional, 6 CUDA events) are recorded before the router, after
    dispatch, after the row exchange, after the local experts, after the
    return exchange and after the combine.
    """
    compute = compute or CudaCompute()

    def mark(i):
        if marks is not None:
            marks[i].record()

    mark(0)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if num_experts % world:
        raise ValueError(f"num_experts={num_experts} must be divisible by world_size={world}")
    el = num_experts // world
    if w_gate_up_local.shape[0] != el or w_down_local.shape[0] != el:
        raise ValueError(f"rank {rank} holds {w_gate_up_local.shape[0]} experts, expected {el}")
    T, d = x.shape
    dev = x.device
    if T > 0:
        idx, w = compute.router(x, w_router, router_bias, top_k, norm_topk_prob)
        sort_idx, counts, x_sorted = compute.dispatch(idx, num_experts, x, w)
    else:
        idx = torch.empty((0, top_k), dtype=torch.int32, device=dev)
        w = torch.empty((0, top_k), dtype=x.dtype, device=dev)
        sort_idx = torch.empty(0, dtype=torch.int32, device=dev)
        counts = torch.zeros(num_experts, dtype=torch.int32, device=dev)
        x_sorted = x.new_empty((0, d))
    mark(1)
    # counts of my experts from every source: recv_counts[s * el + e]
    counts = counts.to(torch.int32).contiguous()
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    splits = torch.cat([counts.view(world, el).sum(1), recv_counts.view(world, el).sum(1)])
    splits = splits.cpu().tolist()
    send_splits, recv_splits = splits[:world], splits[world:]
    if stats is not None:
        stats.append(EPStats(send_splits, recv_splits))
    recv_rows = x.new_empty((sum(recv_splits), d))
    dist.all_to_all_single(recv_rows, x_sorted.contiguous(), recv_splits, send_splits, group=group)
    mark(2)
    group_weight = torch.arange(world * el, device=dev, dtype=torch.int32) % el
    if recv_rows.shape[0] > 0:
        y_rows = compute.local_experts(recv_rows, w_gate_up_local, w_down_local, recv_counts,
                                       group_weight)
    else:
        y_rows = recv_rows
    mark(3)
    back = x.new_empty((int(sum(send_splits)), d))
    dist.all_to_all_single(back, y_rows.contiguous(), send_splits, recv_splits, group=group)
    mark(4)
    y = torch.zeros_like(x)
    if T > 0:
        compute.combine(back, sort_idx, w, y)
    mark(5)
    return y


class _AllToAllRows(torch.autograd.Function):
    """Row all_to_all with host split sizes whose backward sends the
    gradient rows back the way they came (models/layers.py:360-380)."""

    @staticmethod
    def forward(ctx, rows, send_splits, recv_splits, group):
        out = rows.new_empty((int(sum(recv_splits)), *rows.shape[1:]))
        dist.all_to_all_single(out, rows.contiguous(), list(recv_splits), list(send_splits),
                               group=group)
        ctx.splits = (list(send_splits), list(recv_splits))
        ctx.group = group
        return out

    @staticmethod
    def backward(ctx, grad):
        send, recv = ctx.splits
        out = grad.new_empty((int(sum(send)), *grad.shape[1:]))
        dist.all_to_all_single(out, grad.contiguous(), send, recv, group=ctx.group)
        return out, None, None, None


class _RouterLogits(torch.autograd.Function):
    """The router's rounded logits (computed by the exact-order router, passed
    in) with the backward of the reference's F.linear gate
    (models/layers.py:605): grad_x = g @ W, grad_W = g^T @ x, grad_b = sum g."""

    @staticmethod
    def forward(ctx, x, w, bias, logits):
        ctx.save_for_backward(x, w)
        ctx.has_bias = bias is not None
        return logits.clone()

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        g = g.to(x.dtype)
        gx = g @ w if ctx.needs_input_grad[0] else None
        gw = g.t() @ x if ctx.needs_input_grad[1] else None
        gb = g.float().sum(0).to(x.dtype) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return gx, gw, gb, None


class CudaTrainCompute:
    """The stages of the expert-parallel training forward on this GPU."""

    def route(self, x, w_router, bias, top_k, norm):
        """(topk_idx [T, k] int32, rounded logits [T, E] in x.dtype), no grad."""
        idx, _, logits = ops.router_topk(x.detach(), w_router.detach(), top_k, norm,
                                         None if bias is None else bias.detach(),
                                         return_logits=True)
        return idx, logits

    def sort(self, idx, num_experts):
        """(sort_idx [T*k], counts [E]): the stable sort of the flat assignments."""
        out = ops.dispatch(idx, num_experts)
        return out["sort_idx"].long(), out["counts"]

    def grouped_linear(self, rows, weight, counts):
        return ops.grouped_linear(rows, weight, counts)


def load_balancing_loss(probs: torch.Tensor, selected: torch.Tensor,
                        num_experts: int) -> torch.Tensor:
    """Qwen-style aux loss of the reference (models/layers.py:163-170)."""
    tokens_per_expert = torch.bincount(selected.reshape(-1), minlength=num_experts).to(
        torch.float32) / selected.shape[0]
    return torch.sum(tokens_per_expert * probs.mean(dim=0)) * num_experts


def ep_forward_train(x: torch.Tensor, w_router: torch.Tensor, w_gate_up_local: torch.Tensor,
                     w_down_local: torch.Tensor, num_experts: int, top_k: int,
                     norm_topk_prob: bool, group=None, router_bias: Optional[torch.Tensor] = None,
                     compute=None, aux_tokens: int = -1):
    """Expert-parallel MoE-FFN forward that autograd can differentiate.

    The reference's grouped_ep training step (models/layers.py:596-634 with
    SparseMoEExpertParallel, :427-478): the routing comes from the
    exact-order router; the logits are differentiable as F.linear; softmax,
    top-k gather, renormalisation, the dispatch gather, the SiLU*up product,
    the weighting and the index_add combine are torch operations; the row
    all_to_all each way is an autograd function whose backward sends the
    gradient rows back; the expert GEMMs are the differentiable grouped
    linear (grouped_linear), on the received rows sorted by local expert.
    Returns (y, aux_loss or None, expert_counts or None); aux over the first
    aux_tokens tokens when aux_tokens >= 0.  The backward runs one all_to_all
    each way, so every rank must backpropagate through its y (as with the
    reference's _AllToAllSingle); a rank with no tokens still does.
    """
    compute = compute or CudaTrainCompute()
    world = dist.get_world_size(group)
    if num_experts % world:
        raise ValueError(f"num_experts={num_experts} must be divisible by world_size={world}")
    el = num_experts // world
    if w_gate_up_local.shape[0] != el or w_down_local.shape[0] != el:
        raise ValueError(f"this rank holds {w_gate_up_local.shape[0]} experts, expected {el}")
    T, d = x.shape
    inter = w_gate_up_local.shape[1] // 2
    dev = x.device
    if T > 0:
        idx, logits = compute.route(x, w_router, router_bias, top_k, norm_topk_prob)
        logits = _RouterLogits.apply(x, w_router, router_bias, logits.to(x.dtype))
        probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
        idx = idx.long()
        w = probs.gather(1, idx)
        if norm_topk_prob:
            w = w / w.sum(dim=-1, keepdim=True).clamp_min(1e-12)
        w = w.to(x.dtype)
        sort_idx, counts = compute.sort(idx, num_experts)
        sorted_token = torch.div(sort_idx, top_k, rounding_mode="floor")
        x_sorted = x.index_select(0, sorted_token)
        w_sorted = w.reshape(-1).index_select(0, sort_idx)
    else:
        idx = torch.empty((0, top_k), dtype=torch.long, device=dev)
        probs = torch.empty((0, num_experts), dtype=torch.float32, device=dev)
        counts = torch.zeros(num_experts, dtype=torch.int32, device=dev)
        sorted_token = torch.empty(0, dtype=torch.long, device=dev)
        x_sorted = x[:0]
        w_sorted = x.new_empty(0)
    aux = expert_counts = None
    if aux_tokens >= 0:
        n = min(aux_tokens, T)
        aux = load_balancing_loss(probs[:n], idx[:n], num_experts)
        with torch.no_grad():
            expert_counts = torch.bincount(idx[:n].reshape(-1), minlength=num_experts).to(
                torch.float32)
    # counts of my experts from every source: recv_counts[s * el + e]
    counts = counts.to(torch.int32).contiguous()
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    splits = torch.cat([counts.view(world, el).sum(1), recv_counts.view(world, el).sum(1)])
    splits = splits.cpu().tolist()
    send_splits, recv_splits = splits[:world], splits[world:]
    recv_rows = _AllToAllRows.apply(x_sorted, send_splits, recv_splits, group)
    # received rows come as (source, local expert) blocks: order them by
    # local expert for the grouped GEMMs, and back afterwards
    rc = recv_counts.view(world, el).to(torch.long)
    starts = (torch.cumsum(rc.reshape(-1), 0) - rc.reshape(-1)).view(world, el)
    if recv_rows.shape[0] > 0:
        pieces = [torch.arange(int(starts[s, e]), int(starts[s, e] + rc[s, e]), device=dev)
                  for e in range(el) for s in range(world)]
        perm = torch.cat(pieces)
        rows_e = recv_rows.index_select(0, perm)
        counts_e = rc.sum(0).to(torch.int32)
        gate_up = compute.grouped_linear(rows_e, w_gate_up_local, counts_e)
        h = torch.nn.functional.silu(gate_up[:, :inter]) * gate_up[:, inter:]
        y_e = compute.grouped_linear(h, w_down_local, counts_e)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=dev)
        y_rows = y_e.index_select(0, inv)
    else:
        # no rows here: still a node of the graph (through the rows and the
        # weights), so that every rank runs the backward all_to_all
        y_rows = recv_rows * 0 + 0 * (w_gate_up_local.sum() + w_down_local.sum()).to(recv_rows.dtype)
    back = _AllToAllRows.apply(y_rows, recv_splits, send_splits, group)
    if T > 0:
        y = torch.zeros_like(x).index_add(0, sorted_token, (back * w_sorted[:, None]).to(x.dtype))
    else:
        # no tokens here: y still depends on the returned rows, so that this
        # rank's backward runs the all_to_all its peers' backward waits for
        y = torch.zeros_like(x) + 0 * back.sum()
    return y, aux, expert_counts


class PeerExpertParallel:
    """Expert parallelism over peer memory (hmoe_ep_forward), no host sync per call.

    Set-up (collective, once): every rank allocates its symmetric region in
    the library (cudaMalloc + CUDA IPC handle), the handles are exchanged
    with all_gather_object, and every rank maps its peers' regions (each rank
    on its own GPU).  Each call then runs entirely on the device: counts,
    rows and results move by NVLink stores between the mapped regions,
    ordered by flags carrying the call's epoch.  All ranks must call
    ``forward`` the same number of times (the epochs advance together).
    """

    def __init__(self, hidden: int, intermediate: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool, max_tokens: int, dtype=torch.bfloat16, group=None):
        import ctypes
        from . import _lib
        self._ct = ctypes
        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"num_experts={num_experts} must be divisible by world_size={self.world}")
        if self.world > 8:
            raise ValueError("peer-memory expert parallelism supports up to 8 ranks (one node)")
        self.hidden, self.intermediate, self.num_experts = hidden, intermediate, num_experts
        self.top_k, self.norm = top_k, norm_topk_prob
        self.max_tokens = int(max_tokens)
        self.dtype = dtype
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.epoch = 0
        lib = _lib.load()
        shape = ops.make_shape(self.max_tokens, hidden, num_experts, intermediate, top_k, dtype,
                               norm_topk_prob)
        nbytes = lib.hmoe_ep_symmetric_bytes(ctypes.byref(shape), self.max_tokens, self.world)
        if nbytes == 0:
            raise ValueError(_lib.last_error())
        self.ws = torch.empty(lib.hmoe_ep_workspace_bytes(ctypes.byref(shape), self.max_tokens,
                                                          self.world),
                              dtype=torch.uint8, device=self.device)
        mine = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_lib.EP_HANDLE_BYTES)
        _lib.check(lib.hmoe_ep_symmetric_alloc(nbytes, ctypes.byref(mine), handle))
        self._mine = mine
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        bases = []
        for p, h in enumerate(handles):
            if p == self.rank:
                bases.append(mine.value)
                continue
            ptr = ctypes.c_void_p()
            _lib.check(lib.hmoe_ep_symmetric_open(
                ctypes.create_string_buffer(h, _lib.EP_HANDLE_BYTES), ctypes.byref(ptr)))
            self._opened.append(ptr)
            bases.append(ptr.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def forward(self, x, w_router, w_gate_up_local, w_down_local, router_bias=None, y=None,
                marks=None):
        """y [T, d] for this rank's tokens x [T, d] (T <= max_tokens).

        ``marks`` (optional, 6 torch.cuda.Event) are recorded between the
        stages (see hmoe_ep_forward_marked): for bf16 before the router, after
        the router and index-only dispatch, after the count exchange, after
        the gate_up GEMM with the fused row push, after the down GEMM with the
        fused return, and after the combine.
        """
        ct, lib = self._ct, self._lib.load()
        T, d = x.shape
        el = self.num_experts // self.world
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        if d != self.hidden or x.dtype != self.dtype:
            raise ValueError(f"x must be [T, {self.hidden}] {self.dtype}, got {tuple(x.shape)} {x.dtype}")
        want = {"w_router": (w_router, (self.num_experts, d)),
                "w_gate_up_local": (w_gate_up_local, (el, 2 * self.intermediate, d)),
                "w_down_local": (w_down_local, (el, d, self.intermediate))}
        for name, (t, shp) in want.items():
            if tuple(t.shape) != shp or t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous {shp} {self.dtype}, got "
                                 f"{tuple(t.shape)} {t.dtype}")
        x = x.contiguous()
        if y is None:
            y = torch.empty_like(x)
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        if self.epoch == 0:  # flags start at 0: epoch 0 would pass every wait
            self.epoch = 1
        shape = ops.make_shape(T, d, self.num_experts, self.intermediate, self.top_k, x.dtype,
                               self.norm)
        p = lambda t: None if t is None else ct.c_void_p(t.data_ptr())
        ev = None
        if marks is not None:
            ev = (ct.c_void_p * 6)(*[ct.c_void_p(m.cuda_event) for m in marks])
        self._lib.check(lib.hmoe_ep_forward_marked(
            ct.byref(shape), self.max_tokens, self.rank, self.world, self._bases, self.epoch,
            p(x), p(w_router), p(router_bias), p(w_gate_up_local), p(w_down_local), p(y),
            p(self.ws), self.ws.numel(), ct.c_void_p(torch.cuda.current_stream().cuda_stream), ev))
        return y

    def forward_host(self, x_host, w_router, w_gate_up_local, w_down_local, y_host=None,
                     chunk_tokens: int = 4096, num_chunks: Optional[int] = None,
                     router_bias=None):
        """y_host [T, d] for pinned host tokens x_host [T, d], copies overlapped.

        The tokens go through in chunks of ``chunk_tokens`` (at most
        ``max_tokens``): chunk c+1 is copied in and chunk c-1 copied out on
        side streams while chunk c runs.  Each chunk is one :meth:`forward`,
        so every rank must run the same number of chunks: pass the same
        ``num_chunks`` on all ranks when their token counts differ (a rank
        with fewer tokens runs empty chunks).  Returns once y_host is filled.
        """
        T, d = x_host.shape
        if x_host.is_cuda or not x_host.is_pinned():
            raise ValueError("x_host must be a pinned host tensor")
        if chunk_tokens <= 0 or chunk_tokens > self.max_tokens:
            raise ValueError(f"chunk_tokens must be in [1, max_tokens={self.max_tokens}]")
        n = num_chunks if num_chunks is not None else -(-T // chunk_tokens)
        if n * chunk_tokens < T:
            raise ValueError(f"{n} chunks of {chunk_tokens} tokens cannot hold {T} tokens")
        if y_host is None:
            y_host = torch.empty_like(x_host).pin_memory()
        dev = self.device
        main = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        xb = [torch.empty((chunk_tokens, d), dtype=x_host.dtype, device=dev) for _ in range(2)]
        yb = [torch.empty((chunk_tokens, d), dtype=x_host.dtype, device=dev) for _ in range(2)]
        x_free = [torch.cuda.Event() for _ in range(2)]
        y_free = [torch.cuda.Event() for _ in range(2)]
        for e in x_free + y_free:
            e.record(main)
        for c in range(n):
            i = c & 1
            t0 = min(T, c * chunk_tokens)
            tc = min(T, t0 + chunk_tokens) - t0
            ready = torch.cuda.Event()
            with torch.cuda.stream(s_in):  # the compute of chunk c-2 is done with xb[i]
                s_in.wait_event(x_free[i])
                if tc > 0:
                    xb[i][:tc].copy_(x_host[t0:t0 + tc], non_blocking=True)
                ready.record(s_in)
            main.wait_event(ready)
            main.wait_event(y_free[i])  # the copy-out of chunk c-2 has read yb[i]
            self.forward(xb[i][:tc], w_router, w_gate_up_local, w_down_local, router_bias,
                         y=yb[i][:tc])
            x_free[i].record(main)
            done = torch.cuda.Event()
            done.record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                if tc > 0:
                    y_host[t0:t0 + tc].copy_(yb[i][:tc], non_blocking=True)
                y_free[i].record(s_out)
        main.wait_stream(s_out)
        main.synchronize()
        return y_host

    def status(self):
        """Raise if a device-side wait of an earlier call gave up (synchronises)."""
        ops.workspace_status(self.ws)

    def close(self):
        """Collective: unmap the peers' regions and free this rank's."""
        if self._mine is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = self._lib.load()
        for ptr in self._opened:
            lib.hmoe_ep_symmetric_close(ptr)
        lib.hmoe_ep_symmetric_free(self._mine)
        self._mine = None
        self._opened = []


class SparseMoEExpertParallelSwiGLU(torch.nn.Module):
    """SparseMoESwiGLU(implementation="grouped_ep") with the B200 kernels.

    Parameters follow the reference's expert-parallel layout
    (models/layers.py:406): ``gate.weight`` [E, d] replicated,
    ``experts.local_experts.gate_up_weight`` [E/R, 2I, d] and
    ``experts.local_experts.down_weight`` [E/R, d, I] for this rank's experts.

    ``transport="nccl"`` (default) exchanges rows with NCCL all_to_all, as
    the reference does.  Under autograd (or with a ``moe_context`` while
    gradients are enabled) every transport runs :func:`ep_forward_train`,
    the differentiable NCCL orchestration, and records ``aux_losses`` and
    ``expert_counts`` where the reference does.  ``transport="peer"`` runs the fused peer-memory path
    (:class:`PeerExpertParallel`): it needs ``max_tokens`` (the most tokens any
    rank passes in one call, the same value on every rank), allocates its
    regions collectively on the first forward, and must be released with
    :meth:`close` (collective) before the process group goes away.
    """

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool, group=None, transport: str = "nccl",
                 max_tokens: Optional[int] = None, **kwargs):
        super().__init__()
        from .layers import LinearInit, SparseMoEGroupedExperts
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if num_experts % world:
            raise ValueError(f"num_experts={num_experts} must divide world_size={world}")
        if transport not in ("nccl", "peer"):
            raise ValueError(f"transport must be 'nccl' or 'peer', got {transport!r}")
        if transport == "peer" and not max_tokens:
            raise ValueError("transport='peer' needs max_tokens")
        self.group = group
        self.transport = transport
        self.max_tokens = max_tokens
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.gate = LinearInit(hidden_size, num_experts, bias=False, **kwargs)
        self.experts = torch.nn.Module()
        self.experts.local_experts = SparseMoEGroupedExperts(hidden_size, intermediate_size,
                                                             num_experts // world, **kwargs)
        self._peer = None

    def forward(self, x, moe_context=None, total_seqlen=None, **_seq_info):
        from .layers import _needs_grad, _valid_tokens
        le = self.experts.local_experts
        want_aux = moe_context is not None and torch.is_grad_enabled()
        if want_aux or _needs_grad(x, self.gate.weight, le.gate_up_weight, le.down_weight):
            # training: the differentiable NCCL orchestration (either transport)
            shape = x.shape
            h = x.reshape(-1, self.hidden_size)
            aux_tokens = -1
            if want_aux:
                aux_tokens = (h.shape[0] if total_seqlen is None
                              else _valid_tokens(total_seqlen, h.shape[0]))
            y, aux, counts = ep_forward_train(
                h, self.gate.weight.to(h.dtype), le.gate_up_weight.to(h.dtype),
                le.down_weight.to(h.dtype), self.num_experts, self.top_k, self.norm_topk_prob,
                group=self.group, aux_tokens=aux_tokens)
            if want_aux:
                moe_context.setdefault("aux_losses", []).append(aux)
                moe_context.setdefault("expert_counts", []).append(counts)
            return y.reshape(shape)
        shape = x.shape
        h = x.reshape(-1, self.hidden_size)
        wr, wgu, wd = (self.gate.weight.to(h.dtype), le.gate_up_weight.to(h.dtype),
                       le.down_weight.to(h.dtype))
        if self.transport == "peer":
            if self._peer is None:
                self._peer = PeerExpertParallel(self.hidden_size, self.intermediate_size,
                                                self.num_experts, self.top_k, self.norm_topk_prob,
                                                max_tokens=self.max_tokens, dtype=h.dtype,
                                                group=self.group)
            y = self._peer.forward(h, wr.contiguous(), wgu.contiguous(), wd.contiguous())
        else:
            y = ep_forward(h, wr, wgu, wd, self.num_experts, self.top_k, self.norm_topk_prob,
                           group=self.group)
        return y.reshape(shape)

    def close(self):
        """Release the peer-memory regions (collective; a no-op for NCCL)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None
