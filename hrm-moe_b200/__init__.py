"""B200-native routed MoE-FFN forward for HRM-MoE.

Drop-in for the ``grouped_triton`` expert path of XiaoYee/HRM-MoE
(models/layers.py, models/moe_triton_grouped_gemm.py): hand-written sm_100a
kernels behind a C ABI (include/hrm_moe.h), with this package as the
Python host side.

    layers.SparseMoESwiGLU(..., implementation="grouped_b200")
    ops.ffn_forward / router_topk / dispatch / grouped_linear /
        grouped_swiglu / combine / experts_forward
    torch_ops: torch.ops.hrm_moe.ffn_forward / grouped_linear
    ep.PeerExpertParallel / ep.ep_forward (expert parallelism)
"""
from . import synthetic  # noqa: F401  (numpy only)

__all__ = ["layers", "ops", "torch_ops", "ep", "synthetic", "build", "load_library"]


def build(verbose: bool = False):
    """Compile the native library for sm_100a (see build.py)."""
    from .build import build as _build
    return _build(verbose=verbose)


def load_library():
    from . import _lib
    return _lib.load()


def __getattr__(name):
    if name in ("layers", "ops", "ep", "torch_ops"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
