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
    # + routing buffers and the router's fix-up scratch (list, group counters
    # and the rounded logits of each fix slot) only
    assert ffn < exp + 4 * A * 4 + 16384 * (128 * 2 + 8) + 64 * 1024
    zero = lib.HmoeShape(0, 1536, 64, 512, 8, 0, 1)
    assert so.hmoe_ffn_workspace_bytes(ctypes.byref(zero)) > 0


def test_expert_parallel_arguments(lib):
    so = lib.load()
    import re
    text = lib.HEADER.read_text()
    assert int(re.search(r"#define HMOE_EP_HANDLE_BYTES (\d+)", text).group(1)) == lib.EP_HANDLE_BYTES
    s = lib.HmoeShape(4096, 1536, 64, 512, 8, 0, 1)
    T, d, k = 4096, 1536, 8
    for world in (2, 8):
        sym = so.hmoe_ep_symmetric_bytes(ctypes.byref(s), T, world)
        # every peer's rows can land here, and every own row can come back
        assert sym >= (world * T * k + T * k) * d * 2 + world * T * k * 4
        assert sym < (world * T * k + T * k) * d * 2 + world * T * k * 4 + (1 << 20)
        ws = so.hmoe_ep_workspace_bytes(ctypes.byref(s), T, world)
        # bf16: the activations of the local GEMMs only (the down GEMM stores
        # its rows straight back to their sources)
        assert world * T * k * 512 * 2 <= ws < world * T * k * (512 + d) * 2
        f = lib.HmoeShape(4096, 1536, 64, 512, 8, 1, 1)
        wsf = so.hmoe_ep_workspace_bytes(ctypes.byref(f), T, world)
        assert wsf >= world * T * k * (512 + d) * 4  # fp32: activations + outputs
    assert so.hmoe_ep_symmetric_bytes(ctypes.byref(s), T, 9) == 0
    assert so.hmoe_ep_workspace_bytes(ctypes.byref(s), T, 0) == 0
    bases = (ctypes.c_void_p * 2)(None, None)
    args = [None] * 6 + [None, 0, None]
    # rank outside the world, experts not divisible, too many tokens, NULL peer
    for rank, world, shape, max_tokens, word in [
            (2, 2, s, T, b"rank"),
            (0, 3, s, T, b"divisible"),
            (0, 2, s, T - 1, b"max_tokens"),
            (0, 2, s, T, b"NULL")]:
        rc = so.hmoe_ep_forward(ctypes.byref(shape), max_tokens, rank, world, bases, 1, *args)
        assert rc == errno.EINVAL, so.hmoe_last_error()
        assert word in so.hmoe_last_error()
    big = lib.HmoeShape(1 << 22, 1536, 64, 512, 8, 0, 1)
    rc = so.hmoe_ep_forward(ctypes.byref(big), 1 << 22, 0, 8, bases, 1, *args)
    assert rc == errno.EINVAL and b"2^28" in so.hmoe_last_error()
    assert so.hmoe_ep_symmetric_alloc(0, None, None) == errno.EINVAL
    assert so.hmoe_ep_symmetric_open(None, None) == errno.EINVAL


def test_pdl_mask_setter(lib):
    """hmoe_set_pdl_mask returns the previous mask and keeps only the four
    kernel-class bits; the default (HMOE_PDL unset) is every class but the
    combine.  Host state only: no GPU needed."""
    import os

    so = lib.load()
    start = so.hmoe_set_pdl_mask(7)
    try:
        if "HMOE_PDL" not in os.environ:
            assert start == 7
        assert so.hmoe_set_pdl_mask(0xFF) == 7
        assert so.hmoe_set_pdl_mask(0) == 15
        assert so.hmoe_set_pdl_mask(2) == 0
    finally:
        so.hmoe_set_pdl_mask(start)
