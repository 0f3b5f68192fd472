"""Grouped GEMMs (tcgen05 bf16, CUDA-core fp32) vs a plain fp32 torch reference."""
import numpy as np
import pytest
import torch

from gpu_util import bf16_close, get_ops, ragged_counts, to_np
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _operands(M, N, K, G, dtype, seed, wrows=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    a = torch.randn((M, K), generator=g, device="cuda").to(dt)
    b = (torch.randn((G, wrows or N, K), generator=g, device="cuda") * 0.02).to(dt)
    return a, b


def _ref_grouped(a, b, counts):
    """fp32 per-group a @ b[g]^T (torch on the GPU: test reference only)."""
    out = torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float32, device="cuda")
    start = 0
    for gi, c in enumerate(counts.tolist()):
        if c:
            out[start:start + c] = a[start:start + c].float() @ b[gi].float().T
        start += c
    return out


GEMM_CASES = [
    # M, N, K, G, zeros
    (128, 256, 64, 1, 0),
    (1, 256, 64, 1, 0),
    (300, 512, 1536, 3, 1),
    (4096, 1536, 512, 64, 5),
    (2000, 1280, 448, 16, 0),
    (777, 64, 16, 7, 2),
    (16384, 1536, 512, 64, 0),
]


@pytest.mark.parametrize("M,N,K,G,zeros", GEMM_CASES)
def test_grouped_linear_bf16(M, N, K, G, zeros):
    counts = ragged_counts(M, G, seed=M + G, zeros=zeros)
    a, b = _operands(M, N, K, G, "bf16", seed=M)
    out = get_ops().grouped_linear(a, b, torch.from_numpy(counts).cuda())
    ref = _ref_grouped(a, b, counts)
    assert bf16_close(to_np(out), to_np(ref))


@pytest.mark.parametrize("M,N,K,G,zeros", GEMM_CASES[:6])
def test_grouped_swiglu_bf16(M, N, K, G, zeros):
    counts = ragged_counts(M, G, seed=M + 2 * G, zeros=zeros)
    a, b = _operands(M, N, K, G, "bf16", seed=M + 1, wrows=2 * N)
    out = to_np(get_ops().grouped_swiglu(a, b, torch.from_numpy(counts).cuda()))
    gu = O.round_to_bf16(to_np(_ref_grouped(a, b, counts)))
    gate, up = gu[:, :N], gu[:, N:]
    ref = O.round_to_bf16(O.round_to_bf16(O.silu_f32(gate)) * up)
    # gate_up is rounded to bf16 before the activation (as in the reference);
    # where the fp32 sums of the two sides straddle a bf16 rounding midpoint
    # the inputs differ by one ulp, which the three roundings can grow to a
    # few ulps of h.  Everything else must match bit for bit.
    diff = np.abs(out - ref)
    tol = 2.0 ** -6 * np.abs(ref) + 2.0 ** -10 * np.abs(ref).max()
    exact = np.mean(out == ref)
    assert (diff <= tol).all(), (diff.max(), (diff > tol).sum(), exact)
    assert exact > 0.97, exact


@pytest.mark.parametrize("M,N,K,G,zeros", [(300, 512, 128, 3, 1), (2000, 448, 1280, 64, 3),
                                            (65, 64, 16, 2, 0)])
def test_grouped_fp32(M, N, K, G, zeros):
    counts = ragged_counts(M, G, seed=M, zeros=zeros)
    a, b = _operands(M, N, K, G, "f32", seed=M + 3)
    out = get_ops().grouped_linear(a, b, torch.from_numpy(counts).cuda())
    ref = _ref_grouped(a, b, counts)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    b2 = torch.randn((G, 2 * N, K), device="cuda") * 0.02
    out2 = to_np(get_ops().grouped_swiglu(a, b2, torch.from_numpy(counts).cuda()))
    gu = to_np(_ref_grouped(a, b2, counts))
    ref2 = O.silu_f32(gu[:, :N]) * gu[:, N:]
    np.testing.assert_allclose(out2, ref2, rtol=1e-4, atol=1e-5)


def test_grouped_linear_errors():
    ops = get_ops()
    a = torch.zeros((4, 16), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.grouped_linear(a, torch.zeros((2, 8, 32), device="cuda", dtype=torch.bfloat16),
                           torch.tensor([2, 2], device="cuda"))
    with pytest.raises(TypeError):
        ops.grouped_linear(a.half(), torch.zeros((2, 8, 16), device="cuda", dtype=torch.half),
                           torch.tensor([2, 2], device="cuda"))
    empty = ops.grouped_linear(a[:0], torch.zeros((2, 8, 16), device="cuda", dtype=torch.bfloat16),
                               torch.tensor([0, 0], device="cuda"))
    assert tuple(empty.shape) == (0, 8)


def test_cta_pair_and_single_cta_kernels_agree(tmp_path):
    """The CTA-pair and single-CTA tcgen05 kernels give the same bits: each
    side runs in a child process that forces one kernel (HMOE_GEMM_KERNEL is
    read once per process), on every case of the worker."""
    import os
    import subprocess
    import sys

    import gemm_kernels_worker_gpu as W

    outs = {}
    for kern in ("pair", "single"):
        path = tmp_path / f"{kern}.pt"
        env = dict(os.environ, HMOE_GEMM_KERNEL=kern)
        subprocess.run([sys.executable, W.__file__, str(path)], env=env, check=True, timeout=600)
        outs[kern] = torch.load(path)
    assert outs["pair"].keys() == outs["single"].keys()
    for key in outs["pair"]:
        assert torch.equal(outs["pair"][key], outs["single"][key]), key
