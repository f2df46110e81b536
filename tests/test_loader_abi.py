"""C-ABI library: exports, strict PTQ2/PTQW/PTQC loading, weight quantization (CPU only).

Cases mirror 06-gpu-int8/cpp/ptq2_reader_test.cpp:113-245 and
06-gpu-int8/cpp/ptq_model_test.cpp (format dispatch, EOF strictness, groups
semantics, PTQC strictness)."""
import ctypes
import json
import re
import struct
from pathlib import Path

import numpy as np
import pytest

from ptq_int8_lab_b200 import engine as E
from oracle import ptq8_oracle as O

ROOT = Path(__file__).resolve().parents[1]


def test_exports_match_header():
    hdr = (ROOT / "include" / "ptq8.h").read_text()
    declared = set(re.findall(r"\b(ptq8_[a-z0-9_]+)\s*\(", hdr))
    assert declared == set(E.EXPORTS), declared ^ set(E.EXPORTS)
    L = E.lib()
    for s in declared:
        assert hasattr(L, s), s
    assert L.ptq8_abi_version() == 1


def _conv(cout, cin, kh, kw, sh=1, sw=1, ph=0, pw=0, relu=0, groups=1, base=0.0):
    n = cout * cin * kh * kw
    w = (np.arange(n, dtype=np.float32) + base)
    b = -np.arange(cout, dtype=np.float32)
    return struct.pack("<10i", cout, cin, kh, kw, sh, sw, ph, pw, relu, groups) + w.tobytes() + b.tobytes()


def _load(tmp_path, blob, name="m.bin"):
    p = tmp_path / name
    p.write_bytes(blob)
    return E.Model.load(p)


def _valid_mv2_like(ncp=3):
    convs = [_conv(8, 3, 3, 3, 1, 1, 1, 1, relu=2), _conv(8, 1, 3, 3, 1, 1, 1, 1, relu=2, groups=8),
             _conv(8, 8, 1, 1), _conv(16, 8, 1, 1, relu=2), _conv(16, 1, 3, 3, 2, 2, 1, 1, relu=2, groups=16),
             _conv(16, 16, 1, 1)]
    blocks = [([1, 2], -1, 1, 2), ([3, 4, 5], -1, 2, 0)]
    blob = b"PTQ2" + struct.pack("<4i", len(convs), len(blocks), 0, ncp) + b"".join(convs)
    for cs, ds, st, res in blocks:
        cs = cs + [-1] * (ncp - len(cs))
        blob += struct.pack(f"<{ncp + 3}i", *cs, ds, st, res)
    blob += struct.pack("<2i", 16, 10) + np.full(160, 0.5, np.float32).tobytes() + np.arange(10, dtype=np.float32).tobytes()
    return blob


def test_ptq2_valid_model(tmp_path):
    m = _load(tmp_path, _valid_mv2_like())
    assert (m.n_conv, m.n_block, m.stem_pool, m.fc_in, m.fc_out) == (6, 2, 0, 16, 10)
    assert m.n_depthwise == 2 and m.n_grouped == 2 and m.n_relu6 == 4 and m.n_residual2 == 1
    assert m.conv(1)["groups"] == 8 and m.conv(1)["cin"] == 1
    assert m.block(0)["convs"] == [1, 2, -1] and m.block(1)["residual"] == 0
    w, b = m.weights(1)
    assert w.size == 8 * 9 and w[4] == 4.0 and b[3] == -3.0
    fw, fb = m.weights(-1)
    assert fw.size == 160 and fw[7] == 0.5 and fb[9] == 9.0
    om = O.read_model(tmp_path / "m.bin")
    assert [c.groups for c in om.convs] == [1, 8, 1, 1, 16, 1]


@pytest.mark.parametrize("mutate,needle", [
    (lambda b: b[: len(b) // 2], "truncated"),
    (lambda b: b[:18], "too short"),
    (lambda b: b + b"X", "trailing"),
    (lambda b: b"PTQX" + b[4:], "bad magic"),
    (lambda b: b[:4] + struct.pack("<i", -1) + b[8:], "negative"),
    (lambda b: b[:16] + struct.pack("<i", 0) + b[20:], "n_conv_per_block"),
])
def test_ptq2_rejects(tmp_path, mutate, needle):
    with pytest.raises(E.Ptq8Error, match=needle):
        _load(tmp_path, mutate(_valid_mv2_like()))


def _patch_conv_meta(blob, conv_idx, field, value):
    """Overwrite one meta int of conv `conv_idx` in a _valid_mv2_like blob."""
    off = 20
    sizes = [(8, 3, 3, 3), (8, 1, 3, 3), (8, 8, 1, 1), (16, 8, 1, 1), (16, 1, 3, 3), (16, 16, 1, 1)]
    for i in range(conv_idx):
        co, ci, kh, kw = sizes[i]
        off += 40 + 4 * (co * ci * kh * kw + co)
    off += 4 * field
    return blob[:off] + struct.pack("<i", value) + blob[off + 4:]


@pytest.mark.parametrize("field,value,needle", [(8, 3, "relu="), (9, 0, "groups="), (9, 3, "groups=")])
def test_ptq2_bad_meta(tmp_path, field, value, needle):
    with pytest.raises(E.Ptq8Error, match=needle):
        _load(tmp_path, _patch_conv_meta(_valid_mv2_like(), 1, field, value))


def test_missing_file(tmp_path):
    with pytest.raises(E.Ptq8Error, match="cannot open"):
        E.Model.load(tmp_path / "nope.bin")


def test_ptqw_and_golden_models():
    g = ROOT / "tests" / "golden"
    m = E.Model.load(g / "e2e_r18tv_tiny" / "model.ptqw.bin")
    assert m.format == "PTQW" and m.n_conv == 20 and m.n_block == 8 and m.stem_pool == 1
    assert m.block(2)["residual"] == 1 and m.block(2)["ds"] >= 0
    m2 = E.Model.load(g / "e2e_mv2_tiny" / "model.ptq2.bin")
    assert m2.format == "PTQ2" and m2.n_depthwise > 0 and m2.n_residual2 > 0
    om = O.read_model(g / "e2e_mv2_tiny" / "model.ptq2.bin")
    for i in range(m2.n_conv):
        w, b = m2.weights(i)
        assert np.array_equal(w, om.convs[i].weight.reshape(-1)) and np.array_equal(b, om.convs[i].bias)


def _ptqc(ranges, n=None, tail=b""):
    n = len(ranges) if n is None else n
    return b"PTQC" + struct.pack("<i", n) + b"".join(struct.pack("<2f", lo, hi) for lo, hi in ranges) + tail


def test_ptqc(tmp_path):
    p = tmp_path / "c.ptqc"
    p.write_bytes(_ptqc([(-1.9894737, 2.1264887), (0.0, 1.5)]))
    r = E.load_ptqc(p, 2)
    assert abs(r[0][0] + 1.9894737) < 1e-6 and r[1] == (0.0, 1.5)
    for blob, needle in [(_ptqc([(0, 1)], tail=b"x"), "length mismatch"), (_ptqc([(0, 1)], n=2), "length mismatch"),
                         (_ptqc([(0, 1), (0, 2)]), "layer count"), (_ptqc([(float("nan"), 1)]), "not finite"),
                         (_ptqc([(2.0, 1.0)]), "lo="), (b"PTQX" + struct.pack("<i", 0), "magic"), (b"PTQ", "too short"),
                         (b"PTQC" + struct.pack("<i", -1), "negative")]:
        p.write_bytes(blob)
        with pytest.raises(E.Ptq8Error, match=needle):
            E.load_ptqc(p, 1)


def test_act_scale_modes():
    """ptq_model_test.cpp: R18 layer-0 range, AbsMax vs MinMax ratio 1.9356."""
    lo, hi = -1.9894737, 2.1264887
    am = E.act_scale(lo, hi, 8, E.ACT_ABSMAX)
    mm = E.act_scale(lo, hi, 8, E.ACT_MINMAX)
    assert abs(mm / am - 1.935567) < 1e-4
    assert am == O.act_scale_from_range(np.float32(lo), np.float32(hi))
    assert E.act_scale(0.0, 0.0) == 1e-8


def test_weight_quant_matches_oracle():
    kat = dict(np.load(ROOT / "tests" / "golden" / "kat_ref_int8.npz"))
    for bits in (8, 4):
        c, s = E.quantize_weight(kat["wq_w"], bits)
        assert np.array_equal(c, kat[f"wq_w{bits}_codes"]) and np.array_equal(s, kat[f"wq_w{bits}_scale"])
    rng = np.random.default_rng(0)
    w = rng.normal(size=(64, 64, 3, 3)).astype(np.float32)
    for bits in (8, 4):
        c, s = E.quantize_weight(w, bits)
        c2, s2 = O.quantize_weight_per_channel_sym(w, bits)
        assert np.array_equal(c, c2) and np.array_equal(s, s2)


def test_layer_plan(tmp_path):
    import json
    p = tmp_path / "plan.json"
    p.write_text(json.dumps({"layers": [{"name": "a", "bits": 8, "scheme": "per_channel"},
                                        {"name": "b", "bits": 4, "scheme": "per_channel"}]}))
    assert E.load_layer_plan(p, 2) == [8, 4]
    with pytest.raises(E.Ptq8Error):
        E.load_layer_plan(p, 3)
    p.write_text(json.dumps({"layers": [{"name": "a", "bits": 4, "scheme": "per_group", "group_size": 32}]}))
    with pytest.raises(E.Ptq8Error, match="per_channel"):
        E.load_layer_plan(p, 1)


# ---- one-call interface: ptq8_load / ptq8_destroy (host side; no GPU work before a forward)

def _load_one(model, calib, plan=None, opts=None):
    import ctypes
    out = ctypes.c_void_p()
    err = ctypes.create_string_buffer(1024)
    rc = E.lib().ptq8_load(str(model).encode(), str(calib).encode(), str(plan).encode() if plan else None,
                           ctypes.byref(opts) if opts else None, ctypes.byref(out), err, len(err))
    return rc, out, err.value.decode()


def test_ptq8_load_good_and_destroy(make_model):
    p = make_model(0)
    opts = E.Opts(0, 8, 8, E.ACT_ABSMAX, 0, 0)
    rc, eng, msg = _load_one(p["model"], p["calib"], p["plan"], opts)
    assert rc == 0 and eng.value and msg == ""
    E.lib().ptq8_destroy(eng)


def test_ptq8_load_errors(make_model, tmp_path):
    p = make_model(0)
    rc, eng, msg = _load_one(tmp_path / "missing.bin", p["calib"])
    assert rc != 0 and not eng.value and msg
    bad = tmp_path / "plan.json"
    cases = {
        "{not json": "JSON",
        '{"layers": []}': "'layers' must list 20 convs",
        json.dumps({"layers": [{"bits": 6}] * 20}): "bits=6",
        json.dumps({"layers": [{"bits": 4, "scheme": "per_group"}] * 20}): "only per_channel",
        json.dumps({"layers": [{"bits": 8}] * 20}) + " x": "trailing data",
    }
    for text, want in cases.items():
        bad.write_text(text)
        rc, eng, msg = _load_one(p["model"], p["calib"], bad)
        assert rc == 2 and not eng.value and want in msg, (text[:30], msg)   # PTQ8_ERR_FORMAT


def test_ptq8_load_plan_matches_python_reader(make_model):
    p = make_model(3)   # mixed W4 / W8 MobileNetV2
    m = E.Model.load(p["model"])
    want = E.load_layer_plan(p["plan"], m.n_conv)
    assert 4 in want and 8 in want
    rc, eng, msg = _load_one(p["model"], p["calib"], p["plan"])
    assert rc == 0, msg
    E.lib().ptq8_destroy(eng)


def test_model_load_rejects_directory(tmp_path):
    with pytest.raises(E.Ptq8Error, match="not a regular file"):
        E.Model.load(tmp_path)


def test_u8_input_argument_checks(make_model):
    """8-bit input entry points reject bad arguments on the host (no GPU work needed)."""
    p = make_model(0)
    eng = E.Int8Engine(0)
    m = E.Model.load(p["model"])
    eng.build(m, 8, 8)
    L = E.lib()
    assert L.ptq8_engine_set_input_norm(eng._h, 2, None, None) == 1
    assert b"mode" in L.ptq8_engine_last_error(eng._h)
    mean = np.array([0.5, 0.5, 0.5], np.float32)
    bad = np.array([0.2, 0.0, 0.2], np.float32)
    assert L.ptq8_engine_set_input_norm(eng._h, 0, E._fptr(mean), E._fptr(bad)) == 1
    assert b"std" in L.ptq8_engine_last_error(eng._h)
    assert L.ptq8_engine_set_input_norm(eng._h, 0, E._fptr(mean), None) == 1
    assert L.ptq8_engine_forward_u8(eng._h, None, 4, 0, None) == 1
