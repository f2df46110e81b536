"""Bit-exact parity at the batch sizes the benchmark runs.

The engine runs the whole batch; the oracle runs only a sample of its images (images are
independent: no state crosses images, BN is folded, scales are static), and every conv's
int8 input codes, the final fp32 map and the logits of the sampled images are compared.
The sample holds the first images, the two around the middle and the last eight (the last
M tile of every conv: layer4's tiles hold 8 images), so that a batch past 2^31 bytes of
fp32 map (config 4: layer1's map is 2.15 GB) and the persistent CTAs' last tiles are
covered.  A second forward of a random subset at a smaller batch must reproduce the full
batch's logits of those images bit for bit (a check of every position of the batch).
Reference: the composition of 06-gpu-int8/cpp/ref_e2e.py:208-256.
"""
import numpy as np
import pytest

from oracle import ptq8_oracle as O
from tests.parity import compare

pytestmark = pytest.mark.gpu


def _sample(batch: int):
    s = {0, 1, 2, batch // 2 - 1, batch // 2, batch - 1}
    s |= set(range(max(0, batch - 8), batch))
    return np.array(sorted(k for k in s if 0 <= k < batch))


def _check(eng, paths, batch, seed):
    x = np.random.default_rng(seed).standard_normal((batch, 3, 32, 32)).astype(np.float32)
    logits = eng.forward(x)
    idx = _sample(batch)
    om = O.read_model(paths["model"])
    from ptq_int8_lab_b200 import modelgen as mg
    orc = O.Oracle(om, O.read_ptqc(paths["calib"]), layer_bits=mg.read_layer_plan(paths["plan"]))
    tr = orc.forward(x[idx])
    compare(eng, tr, om, len(idx), logits[idx], images=idx)
    sub = np.random.default_rng(seed + 1).permutation(batch)[:min(batch, 256)]
    assert np.array_equal(eng.forward(x[sub]), logits[sub])


@pytest.mark.parametrize("cfg", [4, 0, 2, 3])
def test_config_at_bench_batch(make_model, cfg):
    from ptq_int8_lab_b200 import engine as E
    from ptq_int8_lab_b200 import modelgen as mg
    paths = make_model(cfg)
    batch = mg.CONFIGS[cfg]["batch"]
    eng = E.open_engine(paths["model"], paths["calib"], paths["plan"], max_batch=batch)
    _check(eng, paths, batch, seed=100 + cfg)


def test_config1_one_call_with_passes(make_model):
    """Config 1 through the one-call interface (ptq8_load with every graph pass) at batch
    1024.  On the CIFAR-stem graph the center-tap and 2x2 + DepthToSpace rewrites decline;
    the generalised positional pass runs the 8x8 / 4x4 convs as per-position sub-convs.
    Its codes must be config 0's, bit for bit."""
    from ptq_int8_lab_b200 import engine as E
    from ptq_int8_lab_b200 import modelgen as mg
    paths = make_model(1)
    batch = mg.CONFIGS[1]["batch"]
    eng = E.load_one_call(paths["model"], paths["calib"], paths["plan"], max_batch=batch, passes=E.PASS_ALL)
    log = [l for l in eng.passes_log().splitlines() if l]
    assert sum("positional" in l for l in log) == 8, log
    assert all(l.endswith("unchanged") for l in log if "positional" not in l)
    _check(eng, paths, batch, seed=101)
