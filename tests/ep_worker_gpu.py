"""torchrun worker for the multi-GPU expert-parallel test (tests/test_gpu_ep.py).

Every rank routes its own seeded tokens through ep.ep_forward (NCCL) and
through the single-GPU layer with all experts; the two must agree bit for
bit, because the rows meet the same kernels and the combine sees them in the
same order.  Then the module trains one step under autograd
(ep.ep_forward_train) against the single-GPU trainable layer.  Writes one
line per rank to the file named by argv[1].
"""
import datetime
import importlib
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _max_rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _train_check(rank, world, dev, syn, ep):
    """The expert-parallel module under autograd (ep_forward_train, NCCL)
    against the single-GPU trainable layer with all experts: y, the aux
    loss and d_x of this rank's tokens, d_W_router of its tokens, and its
    local experts' d_W against the single-GPU d_W summed over ranks; bf16,
    max-rel 1e-2 per tensor."""
    layers = importlib.import_module("hrm-moe_b200.layers")
    T, d, E, I, k = 512 + 29 * rank, 256, 8 * world, 128, 4
    inp = syn.make_inputs(syn.MoEShape(T, d, E, I, k, True, "bf16"), seed=31, rank=rank)
    el = E // world
    bf = torch.bfloat16
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(bf)
    one = layers.SparseMoESwiGLU(d, I, E, k, True).to(dev, bf)
    mod = ep.SparseMoEExpertParallelSwiGLU(d, I, E, k, True).to(dev, bf)
    with torch.no_grad():
        one.gate.weight.copy_(t(inp.w_router))
        one.experts.gate_up_weight.copy_(t(inp.w_gate_up))
        one.experts.down_weight.copy_(t(inp.w_down))
        mod.gate.weight.copy_(t(inp.w_router))
        mod.experts.local_experts.gate_up_weight.copy_(t(inp.w_gate_up[rank * el:(rank + 1) * el]))
        mod.experts.local_experts.down_weight.copy_(t(inp.w_down[rank * el:(rank + 1) * el]))
    gy = torch.randn((T, d), generator=torch.Generator(device=dev).manual_seed(rank), device=dev)
    x1 = t(inp.x).requires_grad_(True)
    xe = t(inp.x).requires_grad_(True)
    c1, ce = {}, {}
    y1 = one(x1.unsqueeze(0), moe_context=c1).squeeze(0)
    ye = mod(xe.unsqueeze(0), moe_context=ce).squeeze(0)
    ((y1.float() * gy).sum() + c1["aux_losses"][0]).backward()
    ((ye.float() * gy).sum() + ce["aux_losses"][0]).backward()
    g_gu = one.experts.gate_up_weight.grad.float().clone()
    g_d = one.experts.down_weight.grad.float().clone()
    dist.all_reduce(g_gu)
    dist.all_reduce(g_d)
    errs = {
        "y": _max_rel(ye, y1),
        "aux": _max_rel(ce["aux_losses"][0], c1["aux_losses"][0]),
        "dx": _max_rel(xe.grad, x1.grad),
        "dw_router": _max_rel(mod.gate.weight.grad, one.gate.weight.grad),
        "dw_gate_up": _max_rel(mod.experts.local_experts.gate_up_weight.grad, g_gu[rank * el:(rank + 1) * el]),
        "dw_down": _max_rel(mod.experts.local_experts.down_weight.grad, g_d[rank * el:(rank + 1) * el]),
    }
    counts_ok = torch.equal(ce["expert_counts"][0], c1["expert_counts"][0])
    ok = counts_ok and all(v <= 1e-2 for v in errs.values())
    return ok, ("train " + ("ok" if ok else "BAD") + f" counts {'equal' if counts_ok else 'DIFFER'} "
                + " ".join(f"{k2} {v:.1e}" for k2, v in errs.items()))


def main(out_path):
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    ok = True
    msgs = []
    try:
        syn = importlib.import_module("hrm-moe_b200.synthetic")
        ep = importlib.import_module("hrm-moe_b200.ep")
        ops = importlib.import_module("hrm-moe_b200.ops")
        # T < 0: rank 0 has no tokens (the others have |T| + 37 * rank)
        for (T, d, E, I, k, skew, dtype) in [(1000, 256, 8 * world, 128, 4, False, "bf16"),
                                              (4096, 1536, 64, 512, 8, False, "bf16"),
                                              (777, 256, 4 * world, 64, 2, True, "bf16"),
                                              (300, 128, 2 * world, 64, 2, False, "f32"),
                                              (-200, 256, 4 * world, 64, 4, False, "bf16"),
                                              (-200, 128, 2 * world, 64, 2, False, "f32")]:
            tokens = 0 if (T < 0 and rank == 0) else abs(T) + 37 * rank
            T = abs(T)
            shape = syn.MoEShape(tokens, d, E, I, k, True, dtype)
            tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
            inp = syn.make_inputs(shape, seed=21, rank=rank)
            wr = inp.w_router
            if skew:  # pile the traffic onto the last rank's experts
                el = E // world
                wr = syn.round_to_bf16(wr + np.concatenate(
                    [np.zeros(((world - 1) * el, d), np.float32), np.full((el, d), 0.03, np.float32)]))
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(tdt)
            el = E // world
            y_ep = ep.ep_forward(t(inp.x), t(wr), t(inp.w_gate_up[rank * el:(rank + 1) * el]),
                                 t(inp.w_down[rank * el:(rank + 1) * el]), E, k, True)
            y_1 = ops.ffn_forward(t(inp.x), t(wr), t(inp.w_gate_up), t(inp.w_down), k, True)
            peer = ep.PeerExpertParallel(d, I, E, k, True, max_tokens=T + 37 * (world - 1),
                                         dtype=tdt)
            wgu_l = t(inp.w_gate_up[rank * el:(rank + 1) * el])
            wd_l = t(inp.w_down[rank * el:(rank + 1) * el])
            for _ in range(3):  # repeated calls reuse the regions
                y_p2p = peer.forward(t(inp.x), t(wr), wgu_l, wd_l)
            torch.cuda.synchronize()
            peer.status()
            peer.close()
            same = torch.equal(y_ep, y_1)
            same_p = torch.equal(y_p2p, y_1)
            if T == 4096:  # host buffers in overlapped chunks (every rank runs 5 chunks)
                peer2 = ep.PeerExpertParallel(d, I, E, k, True, max_tokens=1000, dtype=tdt)
                xh = t(inp.x).cpu().pin_memory()
                yh = peer2.forward_host(xh, t(wr), wgu_l, wd_l, chunk_tokens=1000, num_chunks=5)
                peer2.status()
                peer2.close()
                same_p = same_p and torch.equal(yh.to(dev), y_1)
            if T == 4096:  # the module with the peer transport, reference parameter layout
                mod = ep.SparseMoEExpertParallelSwiGLU(d, I, E, k, True, transport="peer",
                                                       max_tokens=T + 37 * (world - 1)).to(dev)
                with torch.no_grad():
                    mod.gate.weight.copy_(t(wr))
                    mod.experts.local_experts.gate_up_weight.copy_(wgu_l)
                    mod.experts.local_experts.down_weight.copy_(wd_l)
                    y_mod = mod(t(inp.x).unsqueeze(0)).squeeze(0)
                torch.cuda.synchronize()
                mod.close()
                same_p = same_p and torch.equal(y_mod, y_1)
            ok &= same and same_p
            msgs.append(f"T={shape.tokens} E={E} {dtype} skew={skew}: nccl {'equal' if same else 'DIFFER'}, "
                        f"p2p {'equal' if same_p else 'DIFFER max %g' % (y_p2p.float() - y_1.float()).abs().max().item()}")
        ok_t, msg_t = _train_check(rank, world, dev, syn, ep)
        ok &= ok_t
        msgs.append(msg_t)
        dist.barrier()
    except Exception as e:  # report, then leave the group cleanly
        ok = False
        msgs.append(f"error {type(e).__name__}: {e}")
    finally:
        dist.destroy_process_group()
    with open(out_path, "a") as f:
        f.write(f"rank {rank}/{world} {'OK' if ok else 'FAIL'} " + "; ".join(msgs) + "\n")


if __name__ == "__main__":
    main(sys.argv[1])
