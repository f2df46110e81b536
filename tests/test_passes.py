"""Graph passes (center tap, positional 2x2 + DepthToSpace, generalised positional
sub-convs) on the quantized layers.

CPU: which convs each pass rewrites or declines, for both ResNet-18 stems (the build step
needs no GPU).  GPU: the rewritten torchvision-stem network stays bit-exact with the
unrewritten oracle (tests/test_gpu_parity.py style)."""
import numpy as np
import pytest

from oracle import ptq8_oracle as O
from tests.parity import compare


def _log(paths, passes):
    from ptq_int8_lab_b200 import engine as E
    m = E.Model.load(paths["model"])
    eng = E.Int8Engine(0)
    eng.build(m, 8, 8, passes=passes)
    return eng.passes_log()


def test_cifar_stem_passes_decline(make_model):
    """Config 1: on the CIFAR-stem graph no precondition holds (layer4 is 4x4)."""
    log = _log(make_model(1), 3)
    lines = [l for l in log.splitlines() if l]
    assert lines and all(l.endswith("unchanged") for l in lines), log


def test_cifar_stem_positional(make_model):
    """Config 1 with the generalised positional pass: the 3x3 convs on 8x8 and 4x4 output maps
    run as per-position sub-convs (layer3.0.conv1 reads 16x16 with stride 2); 1x1 downsamples,
    the stem and the 32x32 / 16x16 layers stay as they are."""
    log = _log(make_model(1), 7)
    lines = [l for l in log.splitlines() if l]
    pos = [l for l in lines if "positional" in l]
    assert len(pos) == 8, log
    assert sum("positional 3x3 s1 on 4x4 -> 9 position classes (3x3)" in l for l in pos) == 3, log
    assert sum("positional 3x3 s2 on 8x8 -> 4 position classes (2x2)" in l for l in pos) == 1, log
    assert sum("positional 3x3 s1 on 8x8 -> 9 position classes (3x3)" in l for l in pos) == 3, log
    assert sum("positional 3x3 s2 on 16x16 -> 4 position classes (2x2)" in l for l in pos) == 1, log
    # 4x4 s1 3x3: 100 of 144 taps read inside the map
    l4 = next(l for l in pos if "s1 on 4x4" in l)
    before, after = (int(v) for v in l4.split("MACs ")[1].split(" per")[0].split(" -> "))
    assert after * 144 == before * 100, l4
    assert all(l.endswith("unchanged") for l in lines if "positional" not in l), log


def test_torchvision_stem_rewrites(make_model):
    p = make_model("resnet18", seed=3, stem="torchvision", bn="data", calib_n=64)
    log = _log(p, 3)
    rew = [l for l in log.splitlines() if "unchanged" not in l and l]
    # layer3: 4 stride-1 3x3 convs on 2x2 -> 2x2 conv, 4*256 outputs + D2S(2)
    assert sum("decompose 3x3 s1 on 2x2 -> 2x2 conv, 1024 outputs + DepthToSpace(2)" in l for l in rew) == 3, log
    # layer4.0.conv1: 3x3 s2 on 2x2 -> 2x2 slice conv, 1x1 output
    assert sum("decompose 3x3 s2 on 2x2 -> 2x2 conv, 512 outputs" in l for l in rew) == 1, log
    # layer4 stride-1 3x3 convs on 1x1 -> center tap
    assert sum("center-tap 3x3 -> 1x1" in l for l in rew) == 3, log


@pytest.mark.gpu
@pytest.mark.parametrize("n,max_ctas", [(130, 0), (9, 0), (300, 5)])
def test_cifar_stem_positional_bit_exact(make_model, n, max_ctas):
    """Per-position sub-convs skip the padding taps of layers 3-4: every int8 code, the
    final fp32 map and the logits stay those of the unrewritten oracle (a partial image
    block of the last M tiles; a capped grid with many tiles per CTA)."""
    from ptq_int8_lab_b200 import engine as E
    p = make_model(0)
    m = E.Model.load(p["model"])
    eng = E.Int8Engine(0)
    eng.build(m, 8, 8, passes=E.PASS_ALL)
    assert eng.passes_log().count("positional") == 8
    eng.set_calib(E.load_ptqc(p["calib"], m.n_conv))
    eng.alloc_scratch(n)
    if max_ctas:
        eng.set_max_ctas(max_ctas)
    x = np.random.default_rng(n).standard_normal((n, 3, 32, 32)).astype(np.float32)
    logits = eng.forward(x)
    om = O.read_model(p["model"])
    tr = O.Oracle(om, O.read_ptqc(p["calib"])).forward(x)
    compare(eng, tr, om, n, logits)


@pytest.mark.gpu
@pytest.mark.parametrize("passes", [0, 3, 7])
def test_torchvision_stem_bit_exact(make_model, passes):
    from ptq_int8_lab_b200 import engine as E
    p = make_model("resnet18", seed=3, stem="torchvision", bn="data", calib_n=64)
    m = E.Model.load(p["model"])
    eng = E.Int8Engine(0)
    eng.build(m, 8, 8, passes=passes)
    eng.set_calib(E.load_ptqc(p["calib"], m.n_conv))
    eng.alloc_scratch(16)
    x = np.random.default_rng(5).standard_normal((9, 3, 32, 32)).astype(np.float32)
    logits = eng.forward(x)
    om = O.read_model(p["model"])
    tr = O.Oracle(om, O.read_ptqc(p["calib"])).forward(x)
    compare(eng, tr, om, 9, logits)
