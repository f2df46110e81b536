# -*- coding: utf-8 -*-
"""The engine's native calibrated-model package (PTQ8) and its writer.

The reference's calibrated model is a PTQ2 (or PTQW) file of fp32 weights -- W4 layers
included, as fp32 QDQ values (09-ptq-toolkit/ptq_toolkit/pipeline.py:272-279) -- plus a
PTQC file of per-conv activation ranges and a layer-plan JSON; its engine re-quantizes
every weight at build time (06-gpu-int8/cpp/int8_engine.cuh:208).  PTQ8 carries what the
engine runs: each conv's per-channel weight codes (W4 two per byte), f32 scales, bias
and bits, in the PTQ2 topology layout, so the engine builds from it without quantizing.

    python -m ptq_int8_lab_b200.package model.ptq2.bin layer_plan.json out.ptq8.bin

Layout (little endian; the loader is csrc/ptq8_model.cpp):
    "PTQ8", i32 version = 1, i32 n_conv, n_block, stem_pool, ncp
    per conv: 10 x i32 (cout cin kh kw sh sw ph pw relu groups), i32 bits (8 | 4),
              f32 w_scale[cout], f32 bias[cout],
              codes: bits 8 -> int8 [cout][K]; bits 4 -> [cout][ceil(K/2)] bytes with code k
              of a row in the low nibble of byte k/2 for even k, the high nibble for odd k
    per block: (ncp + 3) x i32 (convs..., -1 padded, ds, stride, residual)
    i32 fc_in, fc_out, f32 fc_w[fc_out][fc_in], f32 fc_b[fc_out]

The activation ranges stay in the PTQC file: `write_percentile_ptqc` writes one from
percentile calibration (the reference's PTQC writer emits raw min/max only,
09-ptq-toolkit/ptq_toolkit/export/ptqc.py:175-191).
"""
from __future__ import annotations

import struct
import sys
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

from . import engine as E


def pack_w4(codes: np.ndarray) -> np.ndarray:
    """[cout, K] codes in [-8, 7] -> [cout, ceil(K/2)] bytes, code k in nibble k % 2 of byte k // 2."""
    codes = np.asarray(codes, dtype=np.int8)
    if codes.size and (codes.min() < -8 or codes.max() > 7):
        raise ValueError("W4 codes outside [-8, 7]")
    cout, k = codes.shape
    u = (codes.astype(np.int16) & 0xF).astype(np.uint8)
    if k % 2:
        u = np.concatenate([u, np.zeros((cout, 1), dtype=np.uint8)], axis=1)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_w4(packed: np.ndarray, k: int) -> np.ndarray:
    """Inverse of pack_w4: [cout, ceil(K/2)] bytes -> [cout, K] int8 codes."""
    p = np.asarray(packed, dtype=np.uint8)
    nib = np.stack([p & 0xF, p >> 4], axis=2).reshape(p.shape[0], -1)[:, :k].astype(np.int16)
    return np.where(nib >= 8, nib - 16, nib).astype(np.int8)


def write_native(model_path, out_path, layer_bits: Optional[Sequence[int]] = None, plan_path=None,
                 w_bits: int = 8) -> dict:
    """Write the PTQ8 package of a PTQ2 / PTQW model: the weights quantized per channel at
    each conv's bits (from `layer_bits`, a layer-plan JSON, or `w_bits` for all), with the
    engine's own quantizer (ptq8_quantize_weight, the algorithm of ptq_quant.h:72-110)."""
    m = E.Model.load(model_path)
    if m.format == "PTQ8":
        raise ValueError(f"{model_path} is already a PTQ8 package")
    if layer_bits is None:
        layer_bits = E.load_layer_plan(plan_path, m.n_conv) if plan_path else [w_bits] * m.n_conv
    layer_bits = [int(b) for b in layer_bits]
    if len(layer_bits) != m.n_conv or any(b not in (4, 8) for b in layer_bits):
        raise ValueError("layer bits must list 4 or 8 for every conv")
    blocks = [m.block(i) for i in range(m.n_block)]
    ncp = max([len(b["convs"]) for b in blocks] + [1])
    out = [b"PTQ8", struct.pack("<5i", 1, m.n_conv, m.n_block, m.stem_pool, ncp)]
    packed_bytes = int8_bytes = 0
    for i in range(m.n_conv):
        c = m.conv(i)
        w, bias = m.weights(i)
        codes, scale = E.quantize_weight(w.reshape(c["cout"], -1), layer_bits[i])
        codes = codes.reshape(c["cout"], -1)
        payload = pack_w4(codes) if layer_bits[i] == 4 else codes.view(np.uint8)
        packed_bytes += payload.size
        int8_bytes += codes.size
        out.append(struct.pack("<11i", c["cout"], c["cin"], c["kh"], c["kw"], c["sh"], c["sw"], c["ph"], c["pw"],
                               c["relu"], c["groups"], layer_bits[i]))
        out.append(np.ascontiguousarray(scale, dtype="<f4").tobytes())
        out.append(np.ascontiguousarray(bias, dtype="<f4").tobytes())
        out.append(np.ascontiguousarray(payload).tobytes())
    for b in blocks:
        cs = list(b["convs"]) + [-1] * (ncp - len(b["convs"]))
        out.append(struct.pack(f"<{ncp + 3}i", *cs, b["ds"], b["stride"], b["residual"]))
    fw, fb = m.weights(-1)
    out.append(struct.pack("<2i", m.fc_in, m.fc_out))
    out.append(np.ascontiguousarray(fw, dtype="<f4").tobytes())
    out.append(np.ascontiguousarray(fb, dtype="<f4").tobytes())
    Path(out_path).write_bytes(b"".join(out))
    return {"path": str(out_path), "n_conv": m.n_conv, "bits": layer_bits, "code_bytes": packed_bytes,
            "code_bytes_int8": int8_bytes}


def write_percentile_ptqc(model, images, path, percentile: Optional[float] = None) -> dict:
    """PTQC of per-conv activation ranges from percentile calibration of a torch model on
    `images` (the 03-ptq-lab calibration the synthetic configs use)."""
    from . import modelgen as mg
    ranges = mg.calibrate(model, images) if percentile is None else mg.calibrate(model, images, percentile=percentile)
    return mg.write_ptqc(path, ranges)


if __name__ == "__main__":
    if len(sys.argv) != 4:
        sys.exit("usage: python -m ptq_int8_lab_b200.package MODEL(PTQ2|PTQW) PLAN_JSON|- OUT.ptq8.bin")
    r = write_native(sys.argv[1], sys.argv[3], plan_path=None if sys.argv[2] == "-" else sys.argv[2])
    print(r)
