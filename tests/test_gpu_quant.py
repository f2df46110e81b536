"""Device quantizer (the epilogue's code path) vs the reference formula, incl. exact ties."""
from pathlib import Path

import numpy as np
import pytest

from oracle import ptq8_oracle as O

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


def test_golden_quant_sweeps():
    from ptq_int8_lab_b200 import engine as E
    kat = dict(np.load(G / "kat_ref_int8.npz"))
    for i in range(int(kat["n_quant_cases"])):
        lo, hi = kat[f"quant{i}_range"].tolist()
        x = kat[f"quant{i}_x"]
        got = E.quantize_device(x, lo, hi)
        assert np.array_equal(got, kat[f"quant{i}_codes"]), i


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_scales_dense_ties(seed):
    """All float32 neighbours of every rounding boundary k+0.5 for random scales."""
    from ptq_int8_lab_b200 import engine as E
    rng = np.random.default_rng(seed)
    for _ in range(4):
        lo, hi = float(-rng.uniform(0, 8)), float(rng.uniform(0, 8))
        lo32, hi32 = np.float32(lo), np.float32(hi)
        s = O.act_scale_from_range(lo32, hi32)
        ks = np.arange(-140, 140) + 0.5
        b = (ks * s).astype(np.float32)
        vals = [b]
        up, dn = b.copy(), b.copy()
        for _ in range(3):
            up = np.nextafter(up, np.float32(np.inf))
            dn = np.nextafter(dn, np.float32(-np.inf))
            vals += [up, dn]
        vals.append(rng.normal(0, 3 * hi + 1, 20000).astype(np.float32))
        x = np.concatenate(vals).astype(np.float32)
        got = E.quantize_device(x, lo32, hi32)
        assert np.array_equal(got, O.quantize_act(x, s))
