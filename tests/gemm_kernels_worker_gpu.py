"""Grouped GEMM outputs for the kernel-agreement test (tests/test_gpu_03_gemm.py).

``compute()`` runs a fixed set of seeded bf16 grouped GEMMs (plain and
SwiGLU, ragged groups with empty and one-row groups) through the package and
returns their outputs on the host.  Run as a script it saves them with
torch.save to argv[1]; the test runs it in child processes whose environment
forces one tcgen05 kernel each (HMOE_GEMM_KERNEL is read once per process).
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

CASES = [
    # M, N, K, G, zeros
    (1, 256, 64, 1, 0),
    (512, 512, 1536, 64, 3),     # decode-sized: about 8 rows per group
    (2048, 1536, 512, 64, 0),    # about 32 rows per group
    (777, 64, 16, 7, 2),
    (3000, 1280, 448, 16, 3),
    (131072, 512, 1536, 64, 0),
    (131072, 1536, 512, 64, 4),
]


def compute():
    from gpu_util import get_ops, ragged_counts
    ops = get_ops()
    out = {}
    for (M, N, K, G, zeros) in CASES:
        counts = ragged_counts(M, G, seed=M + G, zeros=zeros)
        if G > 8:
            counts[1] += counts[2] - 1  # a one-row group
            counts[2] = 1
        g = torch.Generator(device="cuda").manual_seed(M + N)
        a = torch.randn((M, K), generator=g, device="cuda").bfloat16()
        b = (torch.randn((G, 2 * N, K), generator=g, device="cuda") * 0.02).bfloat16()
        c = torch.from_numpy(counts).cuda()
        out[f"linear_{M}x{N}x{K}"] = ops.grouped_linear(a, b[:, :N].contiguous(), c).cpu()
        out[f"swiglu_{M}x{N}x{K}"] = ops.grouped_swiglu(a, b, c).cpu()
    return out


if __name__ == "__main__":
    torch.save(compute(), sys.argv[1])
