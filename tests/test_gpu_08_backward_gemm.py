"""Backward grouped GEMMs (tcgen05) against an fp32 PyTorch reference.

_TritonGroupedLinear.backward (models/moe_triton_grouped_gemm.py:427-456):
grad_input = grad_out[rows of g] @ W[g] and grad_weight[g] = grad_out[rows of
g]^T @ input[rows of g], fp32 accumulation, one rounding to bf16.  The fp32
reference is torch on the same bf16 values; the bf16 results must agree
element-wise within one bf16 rounding (2^-8 relative) plus 2^-12 of the
tensor's largest magnitude for the different fp32 summation order, and
within the task's 1e-2 max-relative.  Ragged groups, empty groups, groups of
1, 63, 64 and 65 rows, and sizes that are not multiples of the tiles are
covered.  The SiLU(gate) * up backward fused into the down projection's
dgrad is checked against torch applying the reference's rounding points
(both sides round to bf16 there, so within two bf16 steps).
"""
import numpy as np
import pytest
import torch

from gpu_util import bf16_close, get_ops, ragged_counts, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).bfloat16()


def _ref_dgrad(go, w, counts):
    out = torch.empty((go.shape[0], w.shape[2]), dtype=torch.float32, device="cuda")
    s = 0
    for g, c in enumerate(counts.tolist()):
        out[s:s + c] = go[s:s + c].float() @ w[g].float()
        s += c
    return out


def _ref_wgrad(go, x, counts):
    G = counts.numel()
    out = torch.zeros((G, go.shape[1], x.shape[1]), dtype=torch.float32, device="cuda")
    s = 0
    for g, c in enumerate(counts.tolist()):
        if c:
            out[g] = go[s:s + c].float().T @ x[s:s + c].float()
        s += c
    return out


def _close(ours, ref, rel=2.0 ** -8):
    o, r = to_np(ours), to_np(ref)
    assert bf16_close(o, r, rel=rel), float(np.abs(o - r).max())
    assert O.max_rel(o, r) <= 1e-2


CASES = [
    # (M, N, K, G, zero groups, seed): N, K as in weight [G, N, K]
    (4000, 1536, 512, 64, 3, 1),     # down projection shapes (N = d, K = I)
    (3000, 1024, 1536, 64, 0, 2),    # gate_up shapes (N = 2I, K = d)
    (700, 40, 72, 5, 1, 3),          # sizes off the 64 / 128 / 256 tiles
    (257, 64, 1536, 1, 0, 4),        # one group (the router's shapes)
]


@pytest.mark.parametrize("M,N,K,G,zeros,seed", CASES)
def test_grouped_linear_backward_matches_fp32(M, N, K, G, zeros, seed):
    counts = torch.from_numpy(ragged_counts(M, G, seed, zeros)).to(torch.int32).cuda()
    x = _rand((M, K), seed)
    w = _rand((G, N, K), seed + 100, 0.05)
    go = _rand((M, N), seed + 200)
    gi, gw = get_ops().grouped_linear_backward(go, x, w, counts)
    torch.cuda.synchronize()
    _close(gi, _ref_dgrad(go, w, counts))
    _close(gw, _ref_wgrad(go, x, counts))


def test_wgrad_group_edges_and_empty_groups():
    """Groups of 0, 1, 63, 64, 65 and 129 rows: a group's last 64-row block
    runs into the next group's rows, which must add nothing; an empty group
    gets a zero gradient."""
    sizes = [0, 1, 63, 64, 65, 0, 129, 7]
    counts = torch.tensor(sizes, dtype=torch.int32, device="cuda")
    M, N, K = sum(sizes), 136, 200
    x = _rand((M, K), 7)
    go = _rand((M, N), 8)
    w = torch.zeros((len(sizes), N, K), dtype=torch.bfloat16, device="cuda")
    gi, gw = get_ops().grouped_linear_backward(go, x, w, counts)
    torch.cuda.synchronize()
    _close(gw, _ref_wgrad(go, x, counts))
    assert torch.equal(gw[0], torch.zeros_like(gw[0])) and torch.equal(gw[5], torch.zeros_like(gw[5]))
    assert torch.equal(gi, torch.zeros_like(gi))


def test_wgrad_ignores_non_finite_rows_of_the_next_group():
    """A group's last k-block reads the next group's first rows; those are
    zeroed in shared memory before the MMA, so a NaN there stays out."""
    sizes = [70, 50]
    counts = torch.tensor(sizes, dtype=torch.int32, device="cuda")
    M, N, K = 120, 64, 64
    x = _rand((M, K), 11)
    go = _rand((M, N), 12)
    x[70:] = float("nan")  # all of group 1
    go[70:] = float("nan")
    _, gw = get_ops().grouped_linear_backward(
        go, x, torch.empty((2, N, K), dtype=torch.bfloat16, device="cuda"), counts,
        need_input=False)
    torch.cuda.synchronize()
    assert torch.isfinite(gw[0]).all()
    _close(gw[0], (go[:70].float().T @ x[:70].float()))


def test_grouped_linear_autograd_matches_torch():
    ops = get_ops()
    M, N, K, G = 1000, 256, 384, 8
    counts = torch.from_numpy(ragged_counts(M, G, 5, 1)).to(torch.int32).cuda()
    x = _rand((M, K), 21).requires_grad_(True)
    w = _rand((G, N, K), 22, 0.05).requires_grad_(True)
    go = _rand((M, N), 23)
    y = ops.grouped_linear(x, w, counts)
    y.backward(go)
    _close(x.grad, _ref_dgrad(go, w.detach(), counts))
    _close(w.grad, _ref_wgrad(go, x.detach(), counts))


@pytest.mark.parametrize("M,d,I,G,seed", [(4000, 1536, 512, 64, 31), (333, 136, 72, 3, 32)])
def test_swiglu_backward_matches_reference_rounding(M, d, I, G, seed):
    counts = torch.from_numpy(ragged_counts(M, G, seed, 1)).to(torch.int32).cuda()
    go = _rand((M, d), seed)
    w_down = _rand((G, d, I), seed + 1, 0.05)
    gate_up = _rand((M, 2 * I), seed + 2, 2.0)
    dgu = get_ops().grouped_swiglu_backward(go, w_down, gate_up, counts)
    torch.cuda.synchronize()
    dh = _ref_dgrad(go, w_down, counts).bfloat16().float()
    g, u = gate_up[:, :I].float(), gate_up[:, I:].float()
    sg = torch.nn.functional.silu(g).bfloat16().float()
    d_up = (dh * sg).bfloat16()
    d_sg = (dh * u).bfloat16().float()
    s = torch.sigmoid(g)
    d_gate = (d_sg * s * (1 + g * (1 - s))).bfloat16()
    # the reference values are rounded bf16 as well: where the two fp32 sums
    # of dh (or the two exp implementations) straddle a rounding point the
    # results differ by a bf16 step or two (2^-6 relative)
    _close(dgu[:, I:], d_up, rel=2.0 ** -6)
    _close(dgu[:, :I], d_gate, rel=2.0 ** -6)
