"""Router outputs with every token on the exact-order fix-up pass
(tests/test_gpu_01_router.py::test_router_fixup_pass_is_exact_order).

Run as a script with HMOE_ROUTER_CERT_REL=1 in the environment (read once
per process): no token can then be certified by the tensor-core pass, so the
fix-up kernels route them all.  Saves (topk_idx, weights, logits) per case
with torch.save to argv[1]; ``cases()`` gives the seeded inputs to both sides.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def cases():
    """(name, x, w, bias, k, norm): bf16-exact float32 arrays."""
    from oracle import moe_oracle as O
    out = []
    for (T, d, E, k, seed, with_bias) in [(3000, 1536, 64, 8, 1, False),   # split fix-up
                                          (700, 1000, 64, 8, 2, True),     # partial last block
                                          (300, 40, 8, 3, 3, False),       # one partial block
                                          (257, 256, 64, 4, 4, True),      # quarters without blocks
                                          (513, 1536, 128, 8, 5, False),   # E = 128
                                          (10000, 1536, 64, 8, 6, False)]:  # T > 9472: single-pass kernel
        rng = np.random.default_rng(seed)
        x = O.round_to_bf16(rng.standard_normal((T, d), dtype=np.float32))
        w = O.round_to_bf16(rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02))
        bias = O.round_to_bf16(rng.standard_normal(E).astype(np.float32) * np.float32(0.1)) if with_bias else None
        out.append((f"T{T}_d{d}_E{E}_k{k}", x, w, bias, k, True))
    return out


def main(path):
    import torch
    from gpu_util import get_ops, to_dev
    ops = get_ops()
    res = {}
    for name, x, w, bias, k, norm in cases():
        idx, wt, logits = ops.router_topk(to_dev(x, "bf16"), to_dev(w, "bf16"), k, norm,
                                          None if bias is None else to_dev(bias, "bf16"),
                                          return_logits=True)
        res[name] = (idx.cpu(), wt.float().cpu(), logits.float().cpu())
    torch.save(res, path)


if __name__ == "__main__":
    main(sys.argv[1])
