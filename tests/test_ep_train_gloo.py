"""Expert-parallel training forward + backward on CPU ranks (gloo).

ep.ep_forward_train (the differentiable orchestration: router logits with
the F.linear backward, softmax / top-k / renormalise in torch, the dispatch
gather, the row all_to_all as an autograd function both ways, the grouped
GEMMs on rows sorted by local expert, the weighted index_add combine) runs on
world_size 2 gloo ranks with CPU stand-ins for the stages (the oracle's
exact-order router, a per-group torch matmul for the grouped linear).  The
result and every gradient must equal one process running the same layer on
all ranks' tokens with all experts (models/layers.py:596-634 with
SparseMoEExpertParallel, :360-478): y and d_x per rank, d_W of each rank's
local experts, and d_W_router summed over ranks (the replicated gate's
gradient, which data parallelism sums), plus the aux loss.
"""
import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class TorchTrainCompute:
    """CPU stand-ins of CudaTrainCompute (tests only)."""

    def route(self, x, w_router, bias, top_k, norm):
        from oracle import moe_oracle as O
        logits = O.router_logits(x.detach().numpy(), w_router.detach().numpy(),
                                 None if bias is None else bias.detach().numpy(), "f32")
        idx, _, _ = O.route(logits, top_k, norm, "f32")
        return torch.from_numpy(idx.astype(np.int64)), torch.from_numpy(logits)

    def sort(self, idx, num_experts):
        flat = idx.reshape(-1)
        sort_idx = torch.sort(flat, stable=True).indices
        return sort_idx, torch.bincount(flat, minlength=num_experts).to(torch.int32)

    def grouped_linear(self, rows, weight, counts):
        out, start = [], 0
        for g, c in enumerate(counts.tolist()):
            out.append(rows[start:start + c] @ weight[g].t())
            start += c
        return torch.cat(out) if out else rows.new_zeros((0, weight.shape[1]))


def _cfg_tensors(cfg):
    T, d, E, I, k, world = cfg
    g = torch.Generator().manual_seed(5)
    xs = [torch.randn(T + 7 * r, d, generator=g) for r in range(world)]  # T = 0: an empty rank
    w_r = torch.randn(E, d, generator=g) * 0.1
    w_gu = torch.randn(E, 2 * I, d, generator=g) * 0.1
    w_d = torch.randn(E, d, I, generator=g) * 0.1
    gys = [torch.randn(x.shape, generator=g) for x in xs]
    return xs, w_r, w_gu, w_d, gys


def _worker(rank, world, port, cfg, outdir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        ep = importlib.import_module("hrm-moe_b200.ep")
        T, d, E, I, k, _ = cfg
        xs, w_r, w_gu, w_d, gys = _cfg_tensors(cfg)
        el = E // world
        x = xs[rank].clone().requires_grad_(True)
        wr = w_r.clone().requires_grad_(True)
        wgu = w_gu[rank * el:(rank + 1) * el].clone().requires_grad_(True)
        wd = w_d[rank * el:(rank + 1) * el].clone().requires_grad_(True)
        n = x.shape[0]
        y, aux, counts = ep.ep_forward_train(x, wr, wgu, wd, E, k, True,
                                             compute=TorchTrainCompute(), aux_tokens=n if n else -1)
        ((y * gys[rank]).sum() + (aux if aux is not None else 0)).backward()
        torch.save({"y": y.detach(), "aux": aux.detach() if aux is not None else None,
                    "counts": counts, "gx": x.grad,
                    "gwr": wr.grad, "gwgu": wgu.grad, "gwd": wd.grad},
                   os.path.join(outdir, f"r{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _reference(cfg):
    """One process, all experts: the same stages without any exchange."""
    sys.path.insert(0, ROOT)
    ep = importlib.import_module("hrm-moe_b200.ep")
    T, d, E, I, k, world = cfg
    xs, w_r, w_gu, w_d, gys = _cfg_tensors(cfg)
    comp = TorchTrainCompute()
    wr = w_r.clone().requires_grad_(True)
    wgu = w_gu.clone().requires_grad_(True)
    wd = w_d.clone().requires_grad_(True)
    xr = [x.clone().requires_grad_(True) for x in xs]
    loss = 0
    outs = []
    for x, gy in zip(xr, gys):
        if x.shape[0] == 0:
            outs.append((torch.zeros_like(x), None))
            continue
        idx, logits = comp.route(x, wr, None, k, True)
        logits = ep._RouterLogits.apply(x, wr, None, logits)
        probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
        w = probs.gather(1, idx)
        w = w / w.sum(dim=-1, keepdim=True).clamp_min(1e-12)
        y = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(k):
                e = int(idx[t, j])
                gu = x[t] @ wgu[e].t()
                h = torch.nn.functional.silu(gu[:I]) * gu[I:]
                y = y.index_add(0, torch.tensor([t]), (w[t, j] * (h @ wd[e].t()))[None])
        aux = ep.load_balancing_loss(probs, idx, E)
        loss = loss + (y * gy).sum() + aux
        outs.append((y.detach(), aux.detach()))
    loss.backward()
    return outs, [x.grad for x in xr], wr.grad, wgu.grad, wd.grad


@pytest.mark.parametrize("cfg", [(12, 16, 8, 8, 2, 2), (9, 24, 8, 12, 3, 2), (0, 16, 8, 8, 2, 2)])
def test_ep_training_gradients_match_one_process(cfg, tmp_path):
    world = cfg[-1]
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, cfg, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    outs, gxs, gwr, gwgu, gwd = _reference(cfg)
    E = cfg[2]
    el = E // world
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(world)]
    for r in range(world):
        torch.testing.assert_close(res[r]["y"], outs[r][0], rtol=1e-5, atol=1e-6)
        if outs[r][1] is not None:
            torch.testing.assert_close(res[r]["aux"], outs[r][1], rtol=1e-5, atol=1e-6)
        if gxs[r] is not None and gxs[r].numel():
            torch.testing.assert_close(res[r]["gx"], gxs[r], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(res[r]["gwgu"], gwgu[r * el:(r + 1) * el], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(res[r]["gwd"], gwd[r * el:(r + 1) * el], rtol=1e-5, atol=1e-6)
    # a rank with no tokens gives the gate no gradient (None)
    gwr_ep = sum(res[r]["gwr"] for r in range(world) if res[r]["gwr"] is not None)
    torch.testing.assert_close(gwr_ep, gwr, rtol=1e-5, atol=1e-6)
