# -*- coding: utf-8 -*-
"""CPU oracle for the W8A8 / W4A8 quantized-conv forward (TEST INFRASTRUCTURE).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The shipped engine (``ptq_int8_lab_b200``) never calls into it.

It restates, in numpy, the reference's integer-simulated forward:

* ``round_half_away``      <- 09-ptq-toolkit/ptq_toolkit/quant/ptq.py:31-37
                              (== 06-gpu-int8/cpp/ref_e2e.py:111-113)
* ``qmax_of``              <- 09-ptq-toolkit/ptq_toolkit/quant/ptq.py:40-46
* ``act_scale_from_range`` <- 09-ptq-toolkit/ptq_toolkit/ref_int8.py:69-87
                              (== 06-gpu-int8/cpp/ref_e2e.py:116-127)
* ``quantize_act``         <- 09-ptq-toolkit/ptq_toolkit/ref_int8.py:89-91
* ``quantize_weight_per_channel_sym``
                           <- 09-ptq-toolkit/ptq_toolkit/ref_int8.py:146-160
* ``conv2d_int8``          <- 09-ptq-toolkit/ptq_toolkit/ref_int8.py:173-250
                              (im2col + int32 GEMM of 06-gpu-int8/cpp/ref_e2e.py:132-185)
* ``apply_activation``     <- 09-ptq-toolkit/ptq_toolkit/ref_int8.py:163-170
* ``forward``              <- topology order of
                              09-ptq-toolkit/ptq_toolkit/export/topoblocks.py:181-220 and
                              06-gpu-int8/cpp/ref_e2e.py:208-256
* ``maxpool3x3s2p1``       <- 06-gpu-int8/cpp/ref_e2e.py:192-203
* ``normalize_u8``         <- 06-gpu-int8/cpp/ref_e2e.py:261-276 (mode 0) and
                              06-gpu-int8/cpp/main.cpp:25-26,245-261 (mode 1)
* PTQ2 / PTQW / PTQC readers <- topoblocks.py:17-35,247-267, ref_e2e.py:42-87

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``ref_int8`` / ``ref_e2e`` code on seeded inputs and stores the results under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
them bit for bit (codes, int32 accumulators, fp32 outputs).

Integer arithmetic note: the reference accumulates in numpy int32.  Here the
same sums are formed with a float64 BLAS matmul of integer-valued matrices,
which is exact (every partial sum is an integer below 2**53) and then checked
to fit int32; the result is therefore identical to the int32 product.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

ACTIVATIONS = {0: None, 1: "relu", 2: "relu6"}


# --------------------------------------------------------------------------- quant semantics

def round_half_away(x: np.ndarray) -> np.ndarray:
    """Half-away-from-zero rounding (ptq.py:31-37)."""
    return np.where(x >= 0, np.floor(x + 0.5), np.ceil(x - 0.5))


def qmax_of(bits: int) -> int:
    """Symmetric code upper bound 2^(bits-1)-1 (ptq.py:40-46)."""
    return (1 << (bits - 1)) - 1


def act_scale_from_range(lo: float, hi: float, bits: int = 8,
                         mode: str = "absmax") -> float:
    """Per-tensor activation scale in float64 (ref_int8.py:69-87)."""
    if not (np.isfinite(lo) and np.isfinite(hi)) or lo > hi:
        raise ValueError(f"bad range lo={lo}, hi={hi}")
    qmax = qmax_of(bits)
    if mode == "absmax":
        s = max(abs(float(lo)), abs(float(hi))) / qmax
    elif mode == "minmax":
        s = (float(hi) - float(lo)) / qmax
    else:
        raise ValueError(f"unknown mode {mode!r}")
    return max(s, 1e-8)


def quantize_act(x: np.ndarray, scale: float, bits: int = 8) -> np.ndarray:
    """codes = clip(round_half_away(f64(x) / s), -(qmax+1), qmax) (ref_int8.py:89-91)."""
    qmax = qmax_of(bits)
    q = round_half_away(np.asarray(x, dtype=np.float64) / scale)
    return np.clip(q, -(qmax + 1), qmax).astype(np.int8)


def quantize_weight_per_channel_sym(weight: np.ndarray, bits: int = 8
                                    ) -> Tuple[np.ndarray, np.ndarray]:
    """Per-output-channel symmetric codes + f32 scales (ref_int8.py:146-160)."""
    w = np.asarray(weight, dtype=np.float64)
    qmax = qmax_of(bits)
    flat = w.reshape(w.shape[0], -1)
    amax = np.abs(flat).max(axis=1)
    scale = np.maximum(amax / qmax, 1e-8)
    code = round_half_away(flat / scale[:, None])
    code = np.clip(code, -(qmax + 1), qmax).astype(np.int8)
    return code.reshape(w.shape), scale.astype(np.float32)


def apply_activation(y: np.ndarray, act: int) -> np.ndarray:
    """0 none / 1 ReLU / 2 ReLU6 in fp32 (ref_int8.py:163-170)."""
    if act == 0:
        return y
    if act == 1:
        return np.maximum(y, np.float32(0.0))
    if act == 2:
        return np.clip(y, np.float32(0.0), np.float32(6.0))
    raise ValueError(f"unknown activation flag {act}")


# "blas": exact float64 BLAS product (fast, used by the parity tests);
# "int32": numpy int32 matmul exactly as 06-gpu-int8/cpp/ref_e2e.py:180 does it, with
# the weights as the reference lays them out (a row-major (Kpad, Cout) matrix, K padded
# to a multiple of 8, ref_e2e.py:213-218) -- numpy's integer matmul has no BLAS path, so
# its speed depends on that layout; single-threaded, used as the timed CPU baseline of
# the reference's algorithm.
MATMUL_MODE = {"mode": "blas"}


def int_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Exact int32 product of small-integer matrices."""
    if MATMUL_MODE["mode"] == "int32":
        k = a.shape[1]
        kpad = (k + 7) // 8 * 8
        a32 = np.asarray(a, dtype=np.int32)
        if kpad != k:   # the reference's im2col writes zero columns up to Kpad (ref_e2e.py:152-155)
            a32 = np.concatenate([a32, np.zeros((a32.shape[0], kpad - k), dtype=np.int32)], axis=1)
        bt = np.zeros((kpad, b.shape[1]), dtype=np.int8)
        bt[:k] = b
        return a32 @ bt.astype(np.int32)
    r = np.asarray(a, dtype=np.float64) @ np.asarray(b, dtype=np.float64)
    if r.size and (np.abs(r).max() >= 2 ** 31):
        raise OverflowError("int32 accumulator overflow")
    return r.astype(np.int32)


def conv_acc(codes: np.ndarray, wcode: np.ndarray, stride=(1, 1), pad=(0, 0),
             groups: int = 1) -> np.ndarray:
    """int32 accumulators of a conv over int8 codes, padding code 0.

    Same arithmetic as ref_int8.py:218-240 (pad with code 0 == zero point,
    per-position patch @ weight^T); the patch loop is replaced by an im2col
    view (ref_e2e.py:132-157).  K ordering does not affect an exact integer sum.
    """
    N, C, H, W = codes.shape
    Cout, Cin_g, kh, kw = wcode.shape
    sh, sw = stride
    ph, pw = pad
    OH = (H + 2 * ph - kh) // sh + 1
    OW = (W + 2 * pw - kw) // sw + 1
    xp = np.zeros((N, C, H + 2 * ph, W + 2 * pw), dtype=np.int8)
    xp[:, :, ph:ph + H, pw:pw + W] = codes
    cin_pg = C // groups
    cout_pg = Cout // groups
    acc = np.empty((N, Cout, OH, OW), dtype=np.int32)
    if groups == C and cin_pg == 1 and cout_pg == 1:
        # depthwise: 1 input channel per output channel -> tap loop
        a = np.zeros((N, C, OH, OW), dtype=np.int64)
        w64 = wcode.reshape(C, kh, kw).astype(np.int64)
        for i in range(kh):
            for j in range(kw):
                tap = xp[:, :, i:i + sh * (OH - 1) + 1:sh, j:j + sw * (OW - 1) + 1:sw]
                a += tap.astype(np.int64) * w64[None, :, i, j, None, None]
        return a.astype(np.int32)
    for g in range(groups):
        xg = np.ascontiguousarray(xp[:, g * cin_pg:(g + 1) * cin_pg])
        sg = xg.strides
        view = np.lib.stride_tricks.as_strided(
            xg, shape=(N, cin_pg, OH, OW, kh, kw),
            strides=(sg[0], sg[1], sg[2] * sh, sg[3] * sw, sg[2], sg[3]),
            writeable=False)
        col = view.transpose(0, 2, 3, 1, 4, 5).reshape(N * OH * OW, cin_pg * kh * kw)
        wg = wcode[g * cout_pg:(g + 1) * cout_pg].reshape(cout_pg, -1)
        r = int_matmul(col, wg.T)  # (N*OH*OW, cout_pg)
        acc[:, g * cout_pg:(g + 1) * cout_pg] = r.reshape(N, OH, OW, cout_pg).transpose(0, 3, 1, 2)
    return acc


def dequant(acc: np.ndarray, act_scale: float, w_scales: np.ndarray,
            bias: Optional[np.ndarray]) -> np.ndarray:
    """y = f32(acc) * f32(f32(s_a) * s_w[c]) then + bias: two roundings (ref_int8.py:242-246)."""
    factor = (np.float32(act_scale) * np.asarray(w_scales, dtype=np.float32))
    y = acc.astype(np.float32) * factor[None, :, None, None]
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)[None, :, None, None]
    return y


def conv2d_int8(x: np.ndarray, weight: np.ndarray, bias: Optional[np.ndarray],
                act_scale: float, w_bits: int = 8, stride=1, padding=0,
                groups: int = 1, activation: int = 0, a_bits: int = 8):
    """Restatement of ref_int8.conv2d_int8 for the symmetric path (ref_int8.py:173-250).

    Returns (y_fp32, acc_int32, codes_int8)."""
    stride = (stride, stride) if isinstance(stride, int) else tuple(stride)
    padding = (padding, padding) if isinstance(padding, int) else tuple(padding)
    codes = quantize_act(x, act_scale, a_bits)
    wcode, wscale = quantize_weight_per_channel_sym(weight, w_bits)
    acc = conv_acc(codes, wcode, stride, padding, groups)
    y = apply_activation(dequant(acc, act_scale, wscale, bias), activation)
    return y, acc, codes


def gemm_int8(a: np.ndarray, weight: np.ndarray, bias: Optional[np.ndarray], act_scale: float,
              w_bits: int = 8, activation: int = 0):
    """A[M,K] x W[N,K]^T for the symmetric path (ref_int8.py:253-289); returns (y, acc)."""
    codes = quantize_act(a, act_scale).astype(np.int32)
    wcode, wscale = quantize_weight_per_channel_sym(weight, w_bits)
    acc = int_matmul(codes, wcode.reshape(weight.shape[0], -1).T)
    factor = np.float32(act_scale) * wscale.astype(np.float32)
    y = acc.astype(np.float32) * factor[None, :]
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)[None, :]
    return apply_activation(y, activation), acc


def maxpool3x3s2p1(x: np.ndarray) -> np.ndarray:
    """Stem maxpool with -inf padding (ref_e2e.py:192-203)."""
    N, C, H, W = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (1, 1), (1, 1)), constant_values=-np.inf)
    OH = (H + 2 - 3) // 2 + 1
    OW = (W + 2 - 3) // 2 + 1
    s = xp.strides
    view = np.lib.stride_tricks.as_strided(
        xp, shape=(N, C, OH, OW, 3, 3),
        strides=(s[0], s[1], s[2] * 2, s[3] * 2, s[2], s[3]), writeable=False)
    return view.max(axis=(-1, -2)).astype(np.float32)


# --------------------------------------------------------------------------- 8-bit input

CIFAR_MEAN = (0.4914, 0.4822, 0.4465)   # main.cpp:25, ref_e2e.py:272
CIFAR_STD = (0.2470, 0.2435, 0.2616)    # main.cpp:26, ref_e2e.py:273


def normalize_u8(px: np.ndarray, mode: int = 0, mean=CIFAR_MEAN, std=CIFAR_STD) -> np.ndarray:
    """8-bit pixels [N][C][H][W] -> the fp32 network input, every step in float32.

    mode 0 (ref_e2e.py:271-275): x = (px - mean*255) / (std*255).
    mode 1 (main.cpp:245-261):   p = px / 255; x = (p*255 - mean*255) * (1 / (std*255)).
    """
    p = np.asarray(px).astype(np.float32)
    c = p.shape[1]
    m = (np.asarray(mean, dtype=np.float32) * np.float32(255.0)).reshape(1, c, 1, 1)
    sd = (np.asarray(std, dtype=np.float32) * np.float32(255.0)).reshape(1, c, 1, 1)
    if mode == 0:
        return ((p - m) / sd).astype(np.float32)
    inv = np.float32(1.0) / sd
    q = p / np.float32(255.0)
    return (((q * np.float32(255.0)) - m) * inv).astype(np.float32)


# --------------------------------------------------------------------------- model files

@dataclass
class Conv:
    cout: int
    cin: int          # per-group input channels (weight dim 1)
    kh: int
    kw: int
    sh: int
    sw: int
    ph: int
    pw: int
    relu: int         # 0 none / 1 ReLU / 2 ReLU6
    groups: int
    weight: np.ndarray
    bias: np.ndarray


@dataclass
class Block:
    convs: List[int]
    ds: int
    stride: int
    residual: int     # 0 none / 1 add+ReLU / 2 add only


@dataclass
class Model:
    convs: List[Conv]
    blocks: List[Block]
    stem_pool: int
    fc_w: np.ndarray  # (fc_out, fc_in)
    fc_b: np.ndarray
    stem: int = 0


def read_model(path) -> Model:
    """PTQ2 (topoblocks.py:17-35,247-267) or PTQW (ref_e2e.py:42-75), strict EOF."""
    d = open(path, "rb").read()
    magic = d[:4]
    off = 4
    if magic == b"PTQ2":
        n_conv, n_block, stem_pool, ncp = struct.unpack_from("<4i", d, off)
        off += 16
        nmeta = 10
    elif magic == b"PTQW":
        n_conv, n_block, stem_pool = struct.unpack_from("<3i", d, off)
        off += 12
        ncp = 2
        nmeta = 9
    else:
        raise ValueError(f"bad magic {magic!r}")
    convs = []
    for _ in range(n_conv):
        meta = struct.unpack_from(f"<{nmeta}i", d, off)
        off += 4 * nmeta
        cout, cin, kh, kw, sh, sw, ph, pw, relu = meta[:9]
        groups = meta[9] if nmeta == 10 else 1
        n = cout * cin * kh * kw
        w = np.frombuffer(d, dtype="<f4", count=n, offset=off).reshape(cout, cin, kh, kw).copy()
        off += 4 * n
        b = np.frombuffer(d, dtype="<f4", count=cout, offset=off).copy()
        off += 4 * cout
        convs.append(Conv(cout, cin, kh, kw, sh, sw, ph, pw, relu, groups, w, b))
    blocks = []
    for _ in range(n_block):
        if magic == b"PTQ2":
            v = struct.unpack_from(f"<{ncp + 3}i", d, off)
            off += 4 * (ncp + 3)
            cs = [c for c in v[:ncp] if c != -1]
            blocks.append(Block(cs, v[ncp], v[ncp + 1], v[ncp + 2]))
        else:
            c1, c2, ds, stride = struct.unpack_from("<4i", d, off)
            off += 16
            blocks.append(Block([c1, c2], ds, stride, 1))
    fc_in, fc_out = struct.unpack_from("<2i", d, off)
    off += 8
    fcw = np.frombuffer(d, dtype="<f4", count=fc_in * fc_out, offset=off).reshape(fc_out, fc_in).copy()
    off += 4 * fc_in * fc_out
    fcb = np.frombuffer(d, dtype="<f4", count=fc_out, offset=off).copy()
    off += 4 * fc_out
    if off != len(d):
        raise ValueError(f"{path}: {len(d) - off} trailing bytes")
    return Model(convs, blocks, stem_pool, fcw, fcb)


def read_ptqc(path) -> List[Tuple[float, float]]:
    """PTQC: 'PTQC', i32 n, n x (f32 lo, f32 hi); length exactly 8+8n (ptqc.py:87-111)."""
    d = open(path, "rb").read()
    if d[:4] != b"PTQC":
        raise ValueError("bad PTQC magic")
    n = struct.unpack_from("<i", d, 4)[0]
    if n < 0 or len(d) != 8 + 8 * n:
        raise ValueError("bad PTQC length")
    return [struct.unpack_from("<2f", d, 8 + 8 * i) for i in range(n)]


# --------------------------------------------------------------------------- network forward

@dataclass
class Trace:
    """Everything the forward produced, keyed by conv index."""
    codes: Dict[int, np.ndarray] = field(default_factory=dict)     # int8 NCHW conv-input codes
    acc: Dict[int, np.ndarray] = field(default_factory=dict)       # int32 NCHW accumulators
    conv_out: Dict[int, np.ndarray] = field(default_factory=dict)  # fp32 conv outputs (after act)
    block_out: List[np.ndarray] = field(default_factory=list)      # fp32 block outputs
    stem_out: Optional[np.ndarray] = None
    pooled: Optional[np.ndarray] = None                            # f64 GAP
    logits: Optional[np.ndarray] = None                            # f64 head
    logits_f32: Optional[np.ndarray] = None                        # f32 head as ref_e2e.py:255-256


class Oracle:
    """Integer-simulated forward over a PTQ2/PTQW topology.

    ``layer_bits[i]`` is the weight bit width of conv ``i`` (8 or 4; the
    reference's per-layer W4/W8 plan, quant/mixed.py:126-156).  Activations are
    int8 per-tensor symmetric with the scale from the PTQC range of the
    consuming conv.
    """

    def __init__(self, model: Model, ranges: Sequence[Tuple[float, float]],
                 layer_bits: Optional[Sequence[int]] = None, a_bits: int = 8,
                 act_mode: str = "absmax"):
        if len(ranges) != len(model.convs):
            raise ValueError("PTQC layer count != conv count")
        self.m = model
        self.a_bits = a_bits
        self.bits = list(layer_bits) if layer_bits is not None else [8] * len(model.convs)
        self.scales = [act_scale_from_range(lo, hi, a_bits, act_mode) for lo, hi in ranges]
        self.wq = [quantize_weight_per_channel_sym(c.weight, b)
                   for c, b in zip(model.convs, self.bits)]

    def conv(self, i: int, x: np.ndarray, tr: Optional[Trace]) -> np.ndarray:
        c = self.m.convs[i]
        codes = quantize_act(x, self.scales[i], self.a_bits)
        wcode, wscale = self.wq[i]
        acc = conv_acc(codes, wcode, (c.sh, c.sw), (c.ph, c.pw), c.groups)
        y = apply_activation(dequant(acc, self.scales[i], wscale, c.bias), c.relu)
        if tr is not None:
            tr.codes[i] = codes
            tr.acc[i] = acc
            tr.conv_out[i] = y
        return y

    def forward(self, x: np.ndarray, trace: bool = True) -> Trace:
        tr = Trace() if trace else None
        out = Trace()
        m = self.m
        y = self.conv(m.stem, np.asarray(x, dtype=np.float32), tr)
        if m.stem_pool:
            y = maxpool3x3s2p1(y)
        if tr is not None:
            tr.stem_out = y
        for blk in m.blocks:
            t = y
            for ci in blk.convs:
                t = self.conv(ci, t, tr)
            if blk.residual in (1, 2):
                ident = self.conv(blk.ds, y, tr) if blk.ds >= 0 else y
                s = (t + ident).astype(np.float32)
                y = np.maximum(s, np.float32(0.0)) if blk.residual == 1 else s
            else:
                y = t
            if tr is not None:
                tr.block_out.append(y)
        res = tr if tr is not None else out
        res.pooled = y.astype(np.float64).mean(axis=(2, 3))
        res.logits = res.pooled @ m.fc_w.astype(np.float64).T + m.fc_b.astype(np.float64)
        pooled32 = y.mean(axis=(2, 3))
        res.logits_f32 = (pooled32 @ m.fc_w.T + m.fc_b).astype(np.float32)
        return res


def logits_close(got: np.ndarray, want: np.ndarray, rtol: float = 1e-5) -> Tuple[bool, float]:
    """Logit tolerance: per image, max_j |got_j - want_j| <= rtol * max_j |want_j|.

    ``want`` is the float64 head; the relative error is measured against the
    image's logit scale so near-zero individual logits do not blow it up."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = np.maximum(np.abs(want).max(axis=1, keepdims=True), 1e-30)
    err = float((np.abs(got - want) / scale).max()) if want.size else 0.0
    return err <= rtol, err
