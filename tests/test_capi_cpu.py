"""The C-ABI library loads without a GPU, exports every declared symbol and
rejects bad arguments before touching the device."""
import ctypes
import errno

import pytest

from _helpers import package


@pytest.fixture(scope="module")
def lib():
    pkg = package()
    pkg.build()
    from importlib import import_module
    return import_module("hrm-moe_b200._lib")


def test_every_header_function_is_exported(lib):
    names = lib.header_functions()
    assert len(names) >= 15
    so = ctypes.CDLL(str(lib.LIB_PATH))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing
    # and the binding table covers the header exactly
    assert set(names) == set(lib.SIGNATURES)


def test_version_and_errors_without_gpu(lib):
    so = lib.load()
    assert b"sm_100a" in so.hmoe_version()
    bad = lib.HmoeShape(16, 12, 8, 32, 2, 0, 1)  # hidden not a multiple of 8
    assert so.hmoe_ffn_workspace_bytes(ctypes.byref(bad)) == 0
    assert b"hidden" in so.hmoe_last_error()
    rc = so.hmoe_ffn_forward(ctypes.byref(bad), *([None] * 6), 0, *([None] * 5), 0, None)
    assert rc == errno.EINVAL
    for shape, word in [((4, 16, 0, 32, 1, 0, 1), b"experts"),
                        ((4, 16, 8, 32, 9, 0, 1), b"top_k"),
                        ((4, 16, 8, 32, 2, 7, 1), b"dtype"),
                        ((4, 16, 200, 32, 2, 0, 1), b"experts"),
                        ((-1, 16, 8, 32, 2, 0, 1), b"tokens")]:
        s = lib.HmoeShape(*shape)
        assert so.hmoe_ffn_workspace_bytes(ctypes.byref(s)) == 0
        assert word in so.hmoe_last_error()
    rc = so.hmoe_grouped_linear(None, None, None, 10, 12, 16, 2, 0, None, None, 0, None)
    assert rc == errno.EINVAL


def test_workspace_sizes(lib):
    so = lib.load()
    s = lib.HmoeShape(16384, 1536, 64, 512, 8, 0, 1)
    ffn = so.hmoe_ffn_workspace_bytes(ctypes.byref(s))
    exp = so.hmoe_experts_workspace_bytes(ctypes.byref(s))
    A = 16384 * 8
    # gathered rows [A, d] (reused for the down output) + activations [A, I]
    assert exp >= A * 1536 * 2 + A * 512 * 2
    assert ffn > exp
    assert ffn < exp + 4 * A * 4 + 64 * 1024  # + routing buffers only
    zero = lib.HmoeShape(0, 1536, 64, 512, 8, 0, 1)
    assert so.hmoe_ffn_workspace_bytes(ctypes.byref(zero)) > 0
