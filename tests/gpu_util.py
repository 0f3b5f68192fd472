"""Helpers for the GPU parity tests (torch only for device memory)."""
from __future__ import annotations

import numpy as np
import torch

from _helpers import package

ops = None


def get_ops():
    global ops
    if ops is None:
        pkg = package()
        ops = pkg.ops
    return ops


def tdtype(dtype: str):
    return torch.bfloat16 if dtype == "bf16" else torch.float32


def to_dev(a: np.ndarray, dtype: str) -> torch.Tensor:
    """Lossless host->device copy (values are already exact in the dtype)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda").to(tdtype(dtype))


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.detach().cpu().numpy()


def bf16_close(ours: np.ndarray, ref: np.ndarray, rel: float = 2.0 ** -8,
               abs_frac: float = 2.0 ** -12) -> bool:
    """Element-wise: |o - r| <= rel*|r| + abs_frac*max|r| (bf16 output rounding)."""
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    return bool(np.all(np.abs(ours - ref) <= rel * np.abs(ref) + abs_frac * scale + 1e-30))


def random_topk(T: int, E: int, k: int, seed: int) -> np.ndarray:
    """[T, k] expert ids, each row k distinct experts."""
    rng = np.random.default_rng(seed)
    keys = rng.random((T, E))
    return np.argsort(keys, axis=1)[:, :k].astype(np.int32)


def ragged_counts(M: int, G: int, seed: int, zeros: int = 0) -> np.ndarray:
    """Random group sizes summing to M, ``zeros`` of them empty."""
    rng = np.random.default_rng(seed)
    w = rng.random(G) + 0.05
    if zeros:
        w[rng.choice(G, zeros, replace=False)] = 0.0
    c = np.floor(w / w.sum() * M).astype(np.int64)
    c[np.argmax(w)] += M - c.sum()
    return c
