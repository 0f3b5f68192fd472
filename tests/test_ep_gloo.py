"""Expert-parallel orchestration on CPU ranks (gloo), checked against the oracle.

The collective logic of ep.ep_forward (count exchange, split sizes, row
all_to_all both ways, group -> expert map, combine order) runs unchanged on
world_size 2 gloo ranks; the per-rank compute stages are the oracle's
(test-only injection).  Each rank's result must equal the single-process
oracle forward of its tokens bit for bit.
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


class OracleCompute:
    """CPU stages restating the reference (tests only)."""

    def __init__(self, dtype):
        self.dtype = dtype
        from oracle import moe_oracle as O
        self.O = O

    def router(self, x, w_router, bias, top_k, norm):
        O = self.O
        logits = O.router_logits(x.numpy(), w_router.numpy(), None if bias is None else bias.numpy(),
                                 self.dtype)
        idx, w, _ = O.route(logits, top_k, norm, self.dtype)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def dispatch(self, idx, num_experts, x, w):
        sort_idx, sorted_token, counts = self.O.dispatch(idx.numpy(), num_experts)
        return (torch.from_numpy(sort_idx.astype(np.int32)), torch.from_numpy(counts.astype(np.int32)),
                x[torch.from_numpy(sorted_token)])

    def local_experts(self, rows, w_gate_up, w_down, group_rows, group_weight):
        out = torch.empty((rows.shape[0], w_down.shape[1]), dtype=rows.dtype)
        start = 0
        for c, g in zip(group_rows.tolist(), group_weight.tolist()):
            if c:
                out[start:start + c] = torch.from_numpy(self.O.expert_rows(
                    rows[start:start + c].numpy(), w_gate_up[g].numpy(), w_down[g].numpy(), self.dtype))
            start += c
        return out

    def combine(self, y_sorted, sort_idx, w, final):
        O = self.O
        T, k = w.shape
        pos = np.empty(T * k, np.int64)
        pos[sort_idx.numpy().astype(np.int64)] = np.arange(T * k)
        pos = pos.reshape(T, k)
        cast = O.round_to_bf16 if self.dtype == "bf16" else (lambda a: a)
        ys = y_sorted.numpy()
        wn = w.numpy()
        acc = final.numpy().copy()
        order = np.argsort(pos, axis=1)
        rows = np.arange(T)
        for r in range(k):
            j = order[:, r]
            p = pos[rows, j]
            acc = cast(acc + cast(ys[p] * wn[rows, j][:, None]))
        final.copy_(torch.from_numpy(acc))
        return final


def _worker(rank, world, port, cfg, outdir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        syn = importlib.import_module("hrm-moe_b200.synthetic")
        ep = importlib.import_module("hrm-moe_b200.ep")
        T, d, E, I, k, dtype, bias_kind = cfg
        tokens = [T, 0 if bias_kind == "empty_rank" else T // 2 + 3][rank]
        shape = syn.MoEShape(tokens, d, E, I, k, True, dtype)
        inp = syn.make_inputs(shape, seed=11, rank=rank)
        el = E // world
        x = torch.from_numpy(inp.x)
        w_router = torch.from_numpy(inp.w_router)
        if bias_kind == "skew":
            # every token's top picks land on rank 1's experts
            w_router[el:] += torch.from_numpy(np.float32(0.05) * np.ones((E - el, d), np.float32))
            if dtype == "bf16":
                w_router = torch.from_numpy(syn.round_to_bf16(w_router.numpy()))
        wgu = torch.from_numpy(inp.w_gate_up[rank * el:(rank + 1) * el])
        wd = torch.from_numpy(inp.w_down[rank * el:(rank + 1) * el])
        stats = []
        y = ep.ep_forward(x, w_router, wgu, wd, E, k, True, compute=OracleCompute(dtype), stats=stats)
        np.save(os.path.join(outdir, f"y{rank}.npy"), y.numpy())
        np.save(os.path.join(outdir, f"x{rank}.npy"), x.numpy())
        np.save(os.path.join(outdir, f"wr{rank}.npy"), w_router.numpy())
        np.save(os.path.join(outdir, f"splits{rank}.npy"),
                np.array([stats[0].send_rows, stats[0].recv_rows]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg", [
    (40, 64, 8, 32, 2, "f32", None),
    (33, 128, 16, 64, 4, "bf16", None),
    (50, 64, 8, 32, 3, "bf16", "skew"),
    (24, 64, 8, 32, 2, "bf16", "empty_rank"),
])
def test_ep_two_ranks_match_oracle(cfg, tmp_path):
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, cfg, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    from oracle import moe_oracle as O
    syn = importlib.import_module("hrm-moe_b200.synthetic")
    T, d, E, I, k, dtype, bias_kind = cfg
    full = syn.make_weights(syn.MoEShape(T, d, E, I, k, True, dtype), 11)
    total_sent = 0
    for rank in range(world):
        x = np.load(tmp_path / f"x{rank}.npy")
        wr = np.load(tmp_path / f"wr{rank}.npy")
        y = np.load(tmp_path / f"y{rank}.npy")
        ref = O.moe_forward(x, wr, full[1], full[2], k, True, dtype)["y"] if x.shape[0] else y
        assert np.array_equal(y, ref), f"rank {rank}: max diff {np.abs(y - ref).max()}"
        splits = np.load(tmp_path / f"splits{rank}.npy")
        assert splits[0].sum() == x.shape[0] * k
        total_sent += splits[0].sum()
    assert total_sent == sum(np.load(tmp_path / f"splits{r}.npy")[1].sum() for r in range(world))


def _layout_worker(rank, world, port, outdir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        ep = importlib.import_module("hrm-moe_b200.ep")
        m = ep.SparseMoEExpertParallelSwiGLU(16, 32, 8, 2, True)
        sd = m.state_dict()
        shapes = {k: tuple(v.shape) for k, v in sd.items()}
        # the reference's grouped_ep state_dict of this rank loads unchanged
        g = torch.Generator().manual_seed(rank)
        src = {"gate.weight": torch.randn(8, 16, generator=g),
               "experts.local_experts.gate_up_weight": torch.randn(4, 64, 16, generator=g),
               "experts.local_experts.down_weight": torch.randn(4, 16, 32, generator=g)}
        m.load_state_dict(src)
        same = all(torch.equal(m.state_dict()[k], v) for k, v in src.items())
        with open(os.path.join(outdir, f"layout{rank}.txt"), "w") as f:
            f.write(repr((sorted(shapes.items()), same)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep_module_parameter_layout_matches_reference(tmp_path):
    """SparseMoEExpertParallelSwiGLU keeps the reference's grouped_ep layout
    (models/layers.py:395-412): the router replicated, E/R experts per rank
    under experts.local_experts, so its checkpoints load unchanged."""
    world = 2
    port = _free_port()
    mp.start_processes(_layout_worker, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    import ast
    want = sorted({"gate.weight": (8, 16), "experts.local_experts.gate_up_weight": (4, 64, 16),
                   "experts.local_experts.down_weight": (4, 16, 32)}.items())
    for rank in range(world):
        shapes, same = ast.literal_eval((tmp_path / f"layout{rank}.txt").read_text())
        assert shapes == want
        assert same
