"""The native PTQ8 package: W4 nibble packing, round trip through the C-ABI loader, strict
parsing, and (GPU) engine outputs identical to those built from the fp32 PTQ2 file.

The stored codes and scales must be the reference's per-channel quantization of the fp32
weights (09-ptq-toolkit/ptq_toolkit/ref_int8.py:146-160, pinned by tests/golden), so a
PTQ8 package is the same model as its PTQ2 source."""
import struct

import numpy as np
import pytest

from oracle import ptq8_oracle as O
from ptq_int8_lab_b200 import engine as E
from ptq_int8_lab_b200 import package as P


def test_w4_pack_round_trip():
    rng = np.random.default_rng(0)
    for k in (1, 2, 27, 64, 577):
        codes = rng.integers(-8, 8, size=(5, k)).astype(np.int8)
        codes[0, : min(k, 16)] = np.arange(-8, 8)[: min(k, 16)]
        packed = P.pack_w4(codes)
        assert packed.shape == (5, (k + 1) // 2)
        assert np.array_equal(P.unpack_w4(packed, k), codes)
    assert P.pack_w4(np.array([[-1, 7]], np.int8))[0, 0] == 0x7F   # code 0 low nibble, code 1 high
    with pytest.raises(ValueError):
        P.pack_w4(np.array([[8]], np.int8))


@pytest.mark.parametrize("cfg", [0, 3])
def test_native_package_round_trip(make_model, tmp_path, cfg):
    paths = make_model(cfg)
    bits = E.load_layer_plan(paths["plan"], E.Model.load(paths["model"]).n_conv)
    out = tmp_path / "m.ptq8.bin"
    r = P.write_native(paths["model"], out, layer_bits=bits)
    src = E.Model.load(paths["model"])
    m = E.Model.load(out)
    assert m.format == "PTQ8" and src.format == "PTQ2"
    assert (m.n_conv, m.n_block, m.stem_pool, m.fc_in, m.fc_out) == (src.n_conv, src.n_block, src.stem_pool,
                                                                     src.fc_in, src.fc_out)
    om = O.read_model(paths["model"])
    for i in range(m.n_conv):
        assert m.conv(i) == src.conv(i)
        codes, scale, b = m.codes(i)
        assert b == bits[i]
        want_codes, want_scale = O.quantize_weight_per_channel_sym(om.convs[i].weight, bits[i])
        assert np.array_equal(codes, want_codes.reshape(codes.shape)), i
        assert np.array_equal(scale, want_scale), i
        assert np.array_equal(m.weights(i)[1], src.weights(i)[1])
        assert m.weights(i)[0].size == 0
    for i in range(m.n_block):
        sb = src.block(i)
        assert m.block(i)["ds"] == sb["ds"] and m.block(i)["residual"] == sb["residual"]
    assert np.array_equal(m.weights(-1)[0], src.weights(-1)[0])
    if cfg == 3:   # W4 layers take half a byte per code
        assert r["code_bytes"] < r["code_bytes_int8"]
    else:
        assert r["code_bytes"] == r["code_bytes_int8"]


def _native_blob(tmp_path, make_model):
    paths = make_model(0)
    out = tmp_path / "m.ptq8.bin"
    P.write_native(paths["model"], out)
    return out.read_bytes()


def test_native_package_rejects(make_model, tmp_path):
    blob = _native_blob(tmp_path, make_model)
    first_conv = 4 + 4 * 5
    cases = [
        (blob[: len(blob) // 2], "truncated"),
        (blob + b"\0", "trailing"),
        (blob[:4] + struct.pack("<i", 2) + blob[8:], "version"),
        (blob[: first_conv + 40] + struct.pack("<i", 5) + blob[first_conv + 44:], "bits=5"),
        (blob[: first_conv + 44] + struct.pack("<f", -1.0) + blob[first_conv + 48:], "w_scale"),
        (blob[: first_conv + 44] + struct.pack("<f", float("nan")) + blob[first_conv + 48:], "w_scale"),
    ]
    for i, (b, needle) in enumerate(cases):
        p = tmp_path / f"bad{i}.bin"
        p.write_bytes(b)
        with pytest.raises(E.Ptq8Error, match=needle):
            E.Model.load(p)


def test_package_plan_must_agree(make_model, tmp_path):
    paths = make_model(0)
    out = tmp_path / "m.ptq8.bin"
    P.write_native(paths["model"], out)
    m = E.Model.load(out)
    eng = E.Int8Engine(0)
    eng.build(m, 8, 8)                       # the file's bits rule
    with pytest.raises(E.Ptq8Error, match="package stores W8"):
        E.Int8Engine(0).build(m, 8, 8, layer_bits=[4] * m.n_conv)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [0, 3])
def test_native_package_engine_identical(make_model, tmp_path, cfg):
    """The engine built from the PTQ8 package gives the same codes at every conv, the same
    final fp32 map and the same logits, bit for bit, as the engine built from the PTQ2
    file (and both match the oracle)."""
    from tests.parity import compare
    paths = make_model(cfg)
    m2 = E.Model.load(paths["model"])
    bits = E.load_layer_plan(paths["plan"], m2.n_conv)
    out = tmp_path / "m.ptq8.bin"
    P.write_native(paths["model"], out, layer_bits=bits)
    x = np.random.default_rng(29).standard_normal((10, 3, 32, 32)).astype(np.float32)
    a = E.open_engine(paths["model"], paths["calib"], paths["plan"], max_batch=16)
    b = E.open_engine(out, paths["calib"], None, max_batch=16)
    la, lb = a.forward(x), b.forward(x)
    assert np.array_equal(la, lb)
    for i in range(m2.n_conv):
        assert np.array_equal(a.dump_codes(i, 10), b.dump_codes(i, 10)), i
    assert np.array_equal(a.dump_final(10), b.dump_final(10))
    om = O.read_model(paths["model"])
    tr = O.Oracle(om, O.read_ptqc(paths["calib"]), layer_bits=bits).forward(x)
    compare(b, tr, om, 10, lb)
    assert b.weight_bytes() == a.weight_bytes()
