"""The integer round-to-nearest-even used for bf16 roundings on the host.

The synthetic inputs round with integer arithmetic in numpy
(synthetic.round_to_bf16).  That formula must equal an independent
conversion (torch's float -> bfloat16) for every non-NaN input: here every
high-half bit pattern with the low half at and around the tie point, at both
ends and at random.
"""
import numpy as np
import torch

from _helpers import package


def _formula(u):
    # round to nearest even on the bit pattern, restated on uint32 arrays
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    return np.where(nan, (u | np.uint32(0x00400000)) & np.uint32(0xFFFF0000), r)


def test_integer_rounding_matches_conversion():
    rng = np.random.default_rng(5)
    hi = np.arange(1 << 16, dtype=np.uint32) << np.uint32(16)
    lows = [0x0000, 0x0001, 0x7FFF, 0x8000, 0x8001, 0xFFFF]
    u = np.concatenate([hi | np.uint32(l) for l in lows] +
                       [hi | rng.integers(0, 1 << 16, hi.size, dtype=np.uint32)])
    f = u.view(np.float32)
    want = torch.from_numpy(f.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = (_formula(u) >> np.uint32(16)).astype(np.uint16)
    finite = ~np.isnan(f)
    assert np.array_equal(got[finite], want[finite])
    # NaN stays NaN
    back = (got[~finite].astype(np.uint32) << np.uint32(16)).view(np.float32)
    assert np.isnan(back).all()
    # the numpy helper the fixtures use agrees too
    syn = package().synthetic
    r = syn.round_to_bf16(f)
    assert np.array_equal(r.view(np.uint32)[finite] >> np.uint32(16), want[finite].astype(np.uint32))
