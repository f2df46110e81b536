"""The oracle against the reference's own outputs (fixtures made by tests/golden/make_golden.py)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import ptq8_oracle as O

G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def kat():
    return dict(np.load(G / "kat_ref_int8.npz"))


def test_literal_kats():
    """Known answers stated in 09-ptq-toolkit/tests/test_int8_ref.py:70-150."""
    s = O.act_scale_from_range(-2.0, 4.0)
    assert s == 4.0 / 127.0
    assert O.act_scale_from_range(-2.0, 4.0, mode="minmax") == 6.0 / 127.0
    assert O.quantize_act(np.array([-2.0, 0.0, 4.0], np.float32), s).tolist() == [-64, 0, 127]
    assert O.quantize_act(np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5]), 1.0).tolist() == [1, -1, 2, -2, 3, -3]
    assert O.quantize_act(np.array([1e9, -1e9]), 1.0).tolist() == [127, -128]
    s4 = O.act_scale_from_range(-4.0, 4.0)
    assert O.quantize_act(np.array([-4.0, 4.0]), s4).tolist() == [-127, 127]
    assert O.qmax_of(8) == 127 and O.qmax_of(4) == 7
    assert O.act_scale_from_range(0.0, 0.0) == 1e-8
    with pytest.raises(ValueError):
        O.act_scale_from_range(1.0, -1.0)


def test_padding_is_real_zero():
    """3x3 ones conv with p=1 on ones: output proportional to valid taps (test_int8_ref.py:230-247)."""
    x = np.ones((1, 1, 3, 3), np.float32)
    w = np.ones((1, 1, 3, 3), np.float32)
    s = O.act_scale_from_range(-1.0, 3.0)
    y, acc, codes = O.conv2d_int8(x, w, np.zeros(1, np.float32), s, padding=1)
    counts = np.array([[4, 6, 4], [6, 9, 6], [4, 6, 4]])
    assert np.array_equal(acc[0, 0], counts * int(codes[0, 0, 0, 0]) * 127)


def test_conv_cases(kat):
    for k in range(int(kat["n_conv_cases"])):
        groups, stride, pad, act, wb = kat[f"conv{k}_meta"].tolist()
        lo, hi = kat[f"conv{k}_range"].tolist()
        s = O.act_scale_from_range(lo, hi)
        y, acc, codes = O.conv2d_int8(kat[f"conv{k}_x"], kat[f"conv{k}_w"], kat[f"conv{k}_b"], s, w_bits=wb,
                                      stride=stride, padding=pad, groups=groups, activation=act)
        assert np.array_equal(codes, kat[f"conv{k}_codes"]), k
        assert np.array_equal(acc, kat[f"conv{k}_acc"]), k
        assert np.array_equal(y, kat[f"conv{k}_y"]), k


def test_gemm(kat):
    lo, hi = kat["gemm_range"].tolist()
    s = O.act_scale_from_range(lo, hi)
    for bits in (8, 4):
        y, acc = O.gemm_int8(kat["gemm_a"], kat["gemm_w"], kat["gemm_b"], s, w_bits=bits)
        assert np.array_equal(acc, kat[f"gemm_w{bits}_acc"])
        assert np.array_equal(y, kat[f"gemm_w{bits}_y"])


def test_quantize_ties_and_extremes(kat):
    for i in range(int(kat["n_quant_cases"])):
        lo, hi = kat[f"quant{i}_range"].tolist()
        s = O.act_scale_from_range(lo, hi)
        assert np.array_equal(O.quantize_act(kat[f"quant{i}_x"], s), kat[f"quant{i}_codes"]), i


def test_weight_quant(kat):
    for bits in (8, 4):
        c, s = O.quantize_weight_per_channel_sym(kat["wq_w"], bits)
        assert np.array_equal(c, kat[f"wq_w{bits}_codes"])
        assert np.array_equal(s, kat[f"wq_w{bits}_scale"])
        assert s[0] == np.float32(1e-8) and not c[0].any()


def _blocks_equal(tr, exp):
    n = len([k for k in exp if k.startswith("block")])
    assert n == len(tr.block_out)
    for i in range(n):
        assert np.array_equal(tr.block_out[i], exp[f"block{i}"]), f"block {i}"


def test_e2e_resnet18_torchvision_stem_ptqw():
    """ref_e2e.forward (06-gpu-int8/cpp/ref_e2e.py:208-256) on a PTQW model with stem maxpool."""
    d = G / "e2e_r18tv_tiny"
    exp = dict(np.load(d / "expected.npz"))
    m = O.read_model(d / "model.ptqw.bin")
    assert m.stem_pool == 1 and len(m.blocks) == 8
    ranges = O.read_ptqc(d / "calib.ptqc")
    tr = O.Oracle(m, ranges).forward(exp["x"])
    _blocks_equal(tr, exp)
    assert np.array_equal(tr.logits_f32, exp["logits"])
    ok, err = O.logits_close(tr.logits, exp["logits"].astype(np.float64), 1e-5)
    assert ok, err
    tr4 = O.Oracle(m, ranges, layer_bits=[4] * len(m.convs)).forward(exp["x"], trace=False)
    assert np.array_equal(tr4.logits_f32, exp["logits_w4"])


def test_e2e_mobilenet_v2_ptq2_mixed():
    """ref_int8.conv2d_int8 composed in topoblocks.replay_blocks order, mixed W4/W8 plan."""
    d = G / "e2e_mv2_tiny"
    exp = dict(np.load(d / "expected.npz"))
    m = O.read_model(d / "model.ptq2.bin")
    assert any(b.residual == 2 for b in m.blocks) and any(c.groups > 1 for c in m.convs)
    tr = O.Oracle(m, O.read_ptqc(d / "calib.ptqc"), layer_bits=exp["bits"].tolist()).forward(exp["x"])
    _blocks_equal(tr, exp)
    assert np.array_equal(tr.logits_f32, exp["logits"])


@pytest.mark.parametrize("cfg", ["0", "2"])
def test_modelgen_matches_reference_producer(tmp_path, cfg):
    """modelgen's PTQ2/PTQC bytes equal what the reference's producer code writes."""
    from ptq_int8_lab_b200 import modelgen as mg
    want = json.loads((G / "modelgen_sha.json").read_text())[cfg]
    r = mg.make_config(int(cfg), tmp_path)
    assert mg.sha256(r["model"]) == want["ptq2_sha256"]
    assert mg.sha256(r["calib"]) == want["ptqc_sha256"]


def test_u8_normalisation_matches_reference():
    """normalize_u8 mode 0 against ref_e2e.read_test_batch on raw CIFAR-10 records
    (tests/golden/u8_norm.npz): bit for bit."""
    d = np.load(G / "u8_norm.npz")
    rec = d["records"].reshape(-1, 3073)
    px = rec[:, 1:].reshape(-1, 3, 32, 32)
    got = O.normalize_u8(px, 0)
    assert got.dtype == np.float32 and np.array_equal(got.view(np.uint32), d["x"].view(np.uint32))


def test_u8_normalisation_mul_form():
    """Mode 1 restates main.cpp:245-261 step by step in float32; the two forms differ by at
    most a few ulps and agree on most values."""
    px = (np.arange(3 * 256) % 256).astype(np.uint8).reshape(1, 3, 16, 16)
    a, b = O.normalize_u8(px, 0), O.normalize_u8(px, 1)
    p = np.float32(px[0, 1, 3, 7])
    m = np.float32(0.4822) * np.float32(255.0)
    inv = np.float32(1.0) / (np.float32(0.2435) * np.float32(255.0))
    assert b[0, 1, 3, 7] == ((p / np.float32(255.0)) * np.float32(255.0) - m) * inv
    assert np.max(np.abs(a - b) / np.maximum(np.abs(a), 1e-3)) < 1e-6
