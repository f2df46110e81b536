"""ptq8_quantize_device_noalloc: the allocation-free device quantizer, called through the C ABI.

It must give exactly the codes of ptq8_quantize_device (int8 codes: the tolerance is zero) on consecutive
calls that share its fixed scratch, including a smaller call right after a full-size one.
"""
import ctypes

import numpy as np
import pytest

from oracle import ptq8_oracle as O
from ptq_int8_lab_b200 import engine as E

MAX_VALUES = 1 << 20     # PTQ8_NOALLOC_MAX_VALUES in include/ptq8.h


def _f(x):
    return x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _q(x):
    return x.ctypes.data_as(ctypes.POINTER(ctypes.c_int8))


def _noalloc(x, lo, hi, mode):
    out = np.full(x.size, 77, dtype=np.int8)
    err = ctypes.create_string_buffer(512)
    rc = E.lib().ptq8_quantize_device_noalloc(0, _f(x), x.size, lo, hi, mode, _q(out), err, len(err))
    assert rc == 0, (rc, err.value)
    assert err.value == b""
    return out


def _existing(x, lo, hi, mode):
    out = np.empty(x.size, dtype=np.int8)
    assert E.lib().ptq8_quantize_device(0, _f(x), x.size, lo, hi, mode, _q(out)) == 0
    return out


def test_rejects_size_beyond_scratch():
    x = np.zeros(MAX_VALUES + 1, dtype=np.float32)
    out = np.empty(x.size, dtype=np.int8)
    err = ctypes.create_string_buffer(512)
    rc = E.lib().ptq8_quantize_device_noalloc(0, _f(x), x.size, -1.0, 1.0, E.ACT_ABSMAX, _q(out), err, len(err))
    assert rc == 1  # PTQ8_ERR_INVALID
    assert b"exceeds the fixed scratch" in err.value


@pytest.mark.parametrize("lo,hi,mode,needle", [
    (2.0, 1.0, 1, b"lo > hi"),                     # MinMax with an inverted range
    (2.0, 1.0, 0, b"lo > hi"),
    (-np.inf, 1.0, 0, b"not finite"),
    (-1.0, np.inf, 1, b"not finite"),
    (np.nan, 1.0, 0, b"not finite"),
    (np.nan, np.nan, 1, b"not finite"),
    (-1.0, 1.0, 2, b"act mode 2"),
    (-1.0, 1.0, -1, b"act mode -1"),
])
def test_rejects_bad_range_or_mode_before_device_work(lo, hi, mode, needle):
    """Checked before any CUDA call (these run without a GPU): an infinite or NaN scale
    would otherwise leave the host-side multiplier search without an exit."""
    x = np.zeros(64, dtype=np.float32)
    out = np.empty(x.size, dtype=np.int8)
    err = ctypes.create_string_buffer(512)
    rc = E.lib().ptq8_quantize_device_noalloc(0, _f(x), x.size, lo, hi, mode, _q(out), err, len(err))
    assert rc == 1, err.value
    assert needle in err.value
    assert E.lib().ptq8_quantize_device(0, _f(x), x.size, lo, hi, mode, _q(out)) == 1


@pytest.mark.gpu
def test_matches_existing_entry_on_two_calls():
    rng = np.random.default_rng(11)
    lo1, hi1 = np.float32(-3.25), np.float32(5.5)
    x1 = rng.normal(0, 3, MAX_VALUES).astype(np.float32)               # fills the whole scratch
    lo2, hi2 = np.float32(-0.75), np.float32(0.6)
    s2 = O.act_scale_from_range(lo2, hi2, mode="minmax")
    ties = ((np.arange(-130, 130) + 0.5) * s2).astype(np.float32)      # rounding boundaries
    x2 = np.concatenate([ties, rng.normal(0, 1, 100_003).astype(np.float32)])   # ragged, smaller
    a1 = _noalloc(x1, lo1, hi1, E.ACT_ABSMAX)
    a2 = _noalloc(x2, lo2, hi2, E.ACT_MINMAX)
    b1 = _existing(x1, lo1, hi1, E.ACT_ABSMAX)
    b2 = _existing(x2, lo2, hi2, E.ACT_MINMAX)
    assert np.array_equal(a1, b1)
    assert np.array_equal(a2, b2)
    assert np.array_equal(a2, O.quantize_act(x2, s2))
