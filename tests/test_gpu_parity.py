"""Bit-exact parity of the sm_100a engine with the CPU oracle (through the C ABI)."""
import numpy as np
import pytest

from oracle import ptq8_oracle as O
from tests.parity import compare

pytestmark = pytest.mark.gpu


def _run(paths, n, seed=7, passes=0, scale=1.0, max_ctas=0):
    from ptq_int8_lab_b200 import engine as E
    m = E.Model.load(paths["model"])
    ranges = E.load_ptqc(paths["calib"], m.n_conv)
    bits = E.load_layer_plan(paths["plan"], m.n_conv)
    eng = E.Int8Engine(0)
    eng.build(m, 8, 8, layer_bits=bits, passes=passes)
    eng.set_calib(ranges)
    eng.alloc_scratch(max(n, 8))
    if max_ctas:
        eng.set_max_ctas(max_ctas)
    x = (np.random.default_rng(seed).standard_normal((n, 3, 32, 32)) * scale).astype(np.float32)
    logits = eng.forward(x)
    om = O.read_model(paths["model"])
    orc = O.Oracle(om, O.read_ptqc(paths["calib"]), layer_bits=bits)
    tr = orc.forward(x)
    return eng, tr, om, logits


@pytest.mark.parametrize("cfg", [0, 2, 3])
def test_config_models(make_model, cfg):
    paths = make_model(cfg)
    eng, tr, om, logits = _run(paths, 6)
    compare(eng, tr, om, 6, logits)


@pytest.mark.parametrize("key,kw", [("resnet18", dict(seed=0, bn="data")),
                                    ("mobilenet_v2", dict(seed=1, bn="data")),
                                    ("mobilenet_v2", dict(seed=2, bn="data", mixed=True))])
def test_normalized_models(make_model, key, kw):
    paths = make_model(key, **kw)
    eng, tr, om, logits = _run(paths, 5, seed=11)
    compare(eng, tr, om, 5, logits)


def test_ragged_batch(make_model):
    """Batch not a multiple of the M-tile image count (layer3 packs 2 images, layer4 8)."""
    paths = make_model("resnet18", seed=0, bn="data")
    eng, tr, om, logits = _run(paths, 13, seed=3)
    compare(eng, tr, om, 13, logits)


@pytest.mark.parametrize("key,kw", [("resnet18", dict(seed=0, bn="data")),
                                    ("mobilenet_v2", dict(seed=2, bn="data", mixed=True))])
def test_many_tiles_per_cta(make_model, key, kw):
    """Three CTAs per conv: every CTA cycles through all accumulator buffers, barrier
    phases and pipeline stages many times (a full-size batch does the same on 148 SMs)."""
    paths = make_model(key, **kw)
    eng, tr, om, logits = _run(paths, 13, seed=5, max_ctas=3)
    compare(eng, tr, om, 13, logits)


def test_batch_512_full_grid(make_model):
    """Enough images that every CTA of the full persistent grid takes several tiles in the
    64- and 128-channel convs."""
    paths = make_model(0)
    eng, tr, om, logits = _run(paths, 512, seed=9)
    compare(eng, tr, om, 512, logits)


def test_w4_packed_config3(make_model):
    """Config 3 (MobileNetV2 W4/W8 mixed): the W4 convs hold their codes two per byte in
    device memory (unpacked into shared memory by the conv kernel, into registers by the
    depthwise kernel) and stay bit-exact."""
    paths = make_model(3)
    eng, tr, om, logits = _run(paths, 6, seed=19)
    compare(eng, tr, om, 6, logits)
    wb = eng.weight_bytes()
    assert wb["packed_w4_convs"] > 0, wb
    assert wb["device_bytes"] < wb["int8_bytes"], wb


def test_w4_resnet18_all_layers(make_model):
    """ResNet-18 at W4 on every conv (the reference's W4A8 run, ROOFLINE-int8.md:609-626):
    layers 1-2 keep resident weight slabs (packed; 64- and 128-byte swizzles), layers 3-4
    stream theirs (int8 storage)."""
    from ptq_int8_lab_b200 import engine as E
    paths = make_model("resnet18", seed=0, bn="data")
    m = E.Model.load(paths["model"])
    eng = E.Int8Engine(0)
    eng.build(m, 4, 8)
    eng.set_calib(E.load_ptqc(paths["calib"], m.n_conv))
    eng.alloc_scratch(8)
    x = np.random.default_rng(23).standard_normal((7, 3, 32, 32)).astype(np.float32)
    logits = eng.forward(x)
    om = O.read_model(paths["model"])
    tr = O.Oracle(om, O.read_ptqc(paths["calib"]), layer_bits=[4] * m.n_conv).forward(x)
    compare(eng, tr, om, 7, logits)
    assert eng.weight_bytes()["packed_w4_convs"] >= 8


RAGGED_MV2 = ((1, 16, 1, 1), (3, 40, 1, 2), (1, 40, 1, 1), (3, 24, 1, 2))


def test_ragged_depthwise_channels(make_model):
    """Depthwise convs of 32, 48, 40 and 120 channels at strides 1 and 2: the last group of 16
    channels is partly padding in two of them (8 of 16 channels valid)."""
    paths = make_model("mobilenet_v2", seed=4, bn="data", settings=RAGGED_MV2)
    eng, tr, om, logits = _run(paths, 9, seed=13)
    compare(eng, tr, om, 9, logits)


@pytest.mark.parametrize("key,kw", [("resnet18", dict(seed=0, bn="data")),
                                    ("mobilenet_v2", dict(seed=1, bn="data"))])
def test_batch_one(make_model, key, kw):
    """A single image: one partial M tile per conv, depthwise units holding fewer images
    than planned, a one-CTA head."""
    paths = make_model(key, **kw)
    eng, tr, om, logits = _run(paths, 1, seed=17)
    compare(eng, tr, om, 1, logits)
