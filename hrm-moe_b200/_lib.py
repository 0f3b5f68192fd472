"""ctypes binding of the native library (include/hrm_moe.h).

The library is loaded on first use.  There is no fallback: if
``libhrm_moe_b200.so`` is missing the call fails with an ImportError that
says how to build it.
"""
from __future__ import annotations

import ctypes
import errno
import pathlib
import re
import threading

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libhrm_moe_b200.so"
HEADER = HERE.parent / "include" / "hrm_moe.h"

HMOE_OK = 0
HMOE_EIO = errno.EIO
HMOE_EINVAL = errno.EINVAL
HMOE_ENOSPC = errno.ENOSPC
HMOE_ENOSYS = errno.ENOSYS
HMOE_ETIMEDOUT = errno.ETIMEDOUT
DTYPE_BF16 = 0
EP_HANDLE_BYTES = 80  # HMOE_EP_HANDLE_BYTES
DTYPE_F32 = 1

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t


class HmoeShape(ctypes.Structure):
    _fields_ = [
        ("tokens", c_int64),
        ("hidden", c_int32),
        ("experts", c_int32),
        ("intermediate", c_int32),
        ("top_k", c_int32),
        ("dtype", c_int32),
        ("norm_topk_prob", c_int32),
    ]


ShapeP = ctypes.POINTER(HmoeShape)

# name -> (restype, argtypes)
SIGNATURES = {
    "hmoe_version": (ctypes.c_char_p, []),
    "hmoe_last_error": (ctypes.c_char_p, []),
    "hmoe_ffn_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_ffn_forward": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    "hmoe_ffn_host_workspace_bytes": (c_size_t, [ShapeP, c_int64]),
    "hmoe_ffn_forward_host": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_int64, c_void_p, c_size_t, c_void_p]),
    "hmoe_ffn_forward_marked": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_int, c_void_p, c_size_t, c_void_p,
                                        ctypes.POINTER(c_void_p)]),
    "hmoe_router_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_router_topk": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_router_topk_sums": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_dispatch_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_dispatch": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_experts_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_experts_forward": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_grouped_linear_workspace_bytes": (c_size_t, [c_int32]),
    "hmoe_grouped_linear": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
                                    c_int32, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_grouped_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32,
                                    c_int32, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_grouped_linear_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                             c_int32, c_int32, c_int32, c_int32, c_void_p,
                                             c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_grouped_swiglu_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                             c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                             c_size_t, c_void_p]),
    "hmoe_ffn_train_saved_bytes": (c_size_t, [ShapeP]),
    "hmoe_ffn_train_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_ffn_forward_train": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_size_t,
                                       c_void_p, c_size_t, c_void_p]),
    "hmoe_ffn_backward": (c_int, [ShapeP, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                  c_void_p]),
    "hmoe_ffn_backward_marked": (c_int, [ShapeP, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_size_t, c_void_p, ctypes.POINTER(c_void_p)]),
    "hmoe_grouped_gemm_mapped": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
                                         c_int32, c_int32, c_int32, c_int32, c_int32, c_void_p,
                                         c_void_p, c_size_t, c_void_p]),
    "hmoe_combine_workspace_bytes": (c_size_t, [ShapeP]),
    "hmoe_combine": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_size_t, c_void_p]),
    "hmoe_workspace_status": (c_int, [c_void_p, c_void_p]),
    "hmoe_set_pdl_mask": (ctypes.c_uint, [ctypes.c_uint]),
    "hmoe_ep_symmetric_bytes": (c_size_t, [ShapeP, c_int64, c_int32]),
    "hmoe_ep_workspace_bytes": (c_size_t, [ShapeP, c_int64, c_int32]),
    "hmoe_ep_symmetric_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    "hmoe_ep_symmetric_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "hmoe_ep_symmetric_close": (c_int, [c_void_p]),
    "hmoe_ep_symmetric_free": (c_int, [c_void_p]),
    "hmoe_ep_forward": (c_int, [ShapeP, c_int64, c_int32, c_int32, ctypes.POINTER(c_void_p),
                                ctypes.c_uint32, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "hmoe_ep_forward_marked": (c_int, [ShapeP, c_int64, c_int32, c_int32,
                                       ctypes.POINTER(c_void_p), ctypes.c_uint32, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_size_t, c_void_p, ctypes.POINTER(c_void_p)]),
    "hmoe_dispatch_noalloc": (c_int, [ShapeP, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p]),
}

_lib = None
_lock = threading.Lock()


class HmoeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{errno.errorcode.get(code, code)}] {message}")
        self.code = code


def header_functions() -> list[str]:
    """Function names the public header declares."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(hmoe_\w+)\s*\(", text)


def load():
    """Load (once) and return the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"native library {LIB_PATH} is missing; build it with "
                    "`python hrm-moe_b200/build.py` (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().hmoe_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if rc == HMOE_OK:
        return
    msg = last_error()
    if rc == HMOE_EINVAL:
        raise ValueError(msg)
    raise HmoeError(rc, msg)
