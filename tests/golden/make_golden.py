# -*- coding: utf-8 -*-
"""Generate the golden fixtures that pin the oracle to the reference's own code.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py /path/to/ptq-int8-lab

It imports the reference's Python (09-ptq-toolkit ref_int8 / quant / export,
03-ptq-lab calib / model, 06-gpu-int8/cpp/ref_e2e.py) and writes, next to this
script:

* ``kat_ref_int8.npz``  - conv / gemm / quantize / weight-quant cases computed
  by ``ptq_toolkit.ref_int8`` (codes, int32 accumulators, fp32 outputs).
* ``e2e_r18tv_tiny/``   - a narrow ResNet-18 topology with the torchvision stem
  (7x7/s2 + maxpool) exported by the reference's PTQW exporter, its PTQC, the
  inputs, and ``ref_e2e.forward`` outputs (logits + every block output).
* ``e2e_mv2_tiny/``     - a narrow MobileNetV2 exported by the reference's PTQ2
  exporter, its PTQC, and the forward composed from ``ref_int8.conv2d_int8``
  in ``topoblocks.replay_blocks`` order.
* ``u8_norm.npz``       - raw CIFAR-10-format records (every pixel value in every
  channel) and ``ref_e2e.read_test_batch``'s normalised fp32 input for them.
* ``modelgen_sha.json`` - SHA-256 of the PTQ2 / PTQC files the reference's
  own producer code (03 fold_all_bn + calib, 09 build_blocks/export) writes for
  benchmark configs 0 and 2, to pin ``ptq_int8_lab_b200.modelgen``.

Nothing here runs at test time; the tests read only the written fixtures.
"""
import hashlib
import json
import struct
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

OUT = Path(__file__).resolve().parent


def setup(ref_root: Path):
    for p in (ref_root / "09-ptq-toolkit", ref_root / "03-ptq-lab", ref_root / "03-ptq-lab" / "src",
              ref_root / "06-gpu-int8" / "cpp"):
        sys.path.insert(0, str(p))


# --------------------------------------------------------------------------- KATs

def make_kats():
    from ptq_toolkit.ref_int8 import SymActQuant, conv2d_int8, gemm_int8, quantize_weight_per_channel_sym
    d = {}
    cases = [  # (groups, stride, padding, activation, w_bits, seed)
        (1, 1, 1, None, 8, 11), (1, 2, 1, "relu", 8, 12), (2, 1, 1, "relu6", 8, 13), (4, 2, 1, None, 8, 14),
        (1, 1, 0, "relu", 4, 15), (1, 2, 0, None, 8, 16), (8, 1, 1, "relu6", 4, 17), (1, 1, 1, "relu", 8, 18),
    ]
    for k, (groups, stride, pad, act, wb, seed) in enumerate(cases):
        rng = np.random.default_rng(seed)
        n, cin, h, w = 2, 8, 7, 9
        cout = {1: 6, 2: 6, 4: 8, 8: 8}[groups]
        x = (rng.normal(size=(n, cin, h, w)).astype(np.float32) * 1.5 + 0.4)
        x[0, 0, 0, 0] = -3.0
        x[0, 1, 0, 0] = 5.0
        weight = rng.normal(size=(cout, cin // groups, 3, 3)).astype(np.float32)
        bias = rng.normal(size=cout).astype(np.float32)
        lo, hi = float(x.min()), float(x.max())
        aq = SymActQuant.from_range(lo, hi)
        # plant exact rounding ties x = (k + 0.5) * s (as float32) in the input
        x[1, 0, 0, :5] = (np.array([0.5, 1.5, -2.5, 10.5, -0.5]) * aq.scale).astype(np.float32)
        y, acc = conv2d_int8(x, weight, bias, act_quant=aq, w_bits=wb, stride=stride, padding=pad,
                             groups=groups, activation=act, return_acc=True)
        d[f"conv{k}_x"] = x
        d[f"conv{k}_w"] = weight
        d[f"conv{k}_b"] = bias
        d[f"conv{k}_meta"] = np.array([groups, stride, pad, {None: 0, "relu": 1, "relu6": 2}[act], wb])
        d[f"conv{k}_range"] = np.array([lo, hi], dtype=np.float64)
        d[f"conv{k}_codes"] = aq.quantize(x)
        d[f"conv{k}_acc"] = acc
        d[f"conv{k}_y"] = y
    d["n_conv_cases"] = np.array(len(cases))
    rng = np.random.default_rng(20261023)
    a = (rng.normal(size=(5, 13)).astype(np.float32) * 2.0 + 0.5)
    wt = rng.normal(size=(7, 13)).astype(np.float32)
    bt = rng.normal(size=7).astype(np.float32)
    aq = SymActQuant.from_range(float(a.min()), float(a.max()))
    for bits in (8, 4):
        y, acc = gemm_int8(a, wt, bt, act_quant=aq, w_bits=bits, return_acc=True)
        d[f"gemm_w{bits}_y"] = y
        d[f"gemm_w{bits}_acc"] = acc
    d["gemm_a"], d["gemm_w"], d["gemm_b"] = a, wt, bt
    d["gemm_range"] = np.array([float(a.min()), float(a.max())])
    # quantize sweep: dense grid + exact ties + extremes for several scales
    xs = []
    # ranges as PTQC stores them: float32 values
    for s_lohi in [(-2.0, 4.0), (0.0, 1.2268753), (-3.739, 3.6477), (0.0, 1e-9)]:
        s_lohi = (float(np.float32(s_lohi[0])), float(np.float32(s_lohi[1])))
        q = SymActQuant.from_range(*s_lohi)
        ks = np.arange(-130, 130) + 0.5
        ties = (ks * q.scale).astype(np.float32)
        v = np.concatenate([ties, np.nextafter(ties, np.float32(np.inf)), np.nextafter(ties, np.float32(-np.inf)),
                            np.linspace(-200 * q.scale, 200 * q.scale, 4001, dtype=np.float32),
                            np.array([0.0, -0.0, 1e30, -1e30, np.inf, -np.inf], dtype=np.float32)])
        xs.append((s_lohi, v, q.quantize(v)))
    for i, (lh, v, c) in enumerate(xs):
        d[f"quant{i}_range"] = np.array(lh, dtype=np.float64)
        d[f"quant{i}_x"] = v
        d[f"quant{i}_codes"] = c
    d["n_quant_cases"] = np.array(len(xs))
    w = np.random.default_rng(20261022).normal(size=(4, 3, 3, 3)).astype(np.float32)
    w[0] = 0.0
    w[1, 0, 0, 0] = -5.0
    d["wq_w"] = w
    for bits in (8, 4):
        c, s = quantize_weight_per_channel_sym(w, bits)
        d[f"wq_w{bits}_codes"], d[f"wq_w{bits}_scale"] = c, s
    np.savez_compressed(OUT / "kat_ref_int8.npz", **d)


# --------------------------------------------------------------------------- tiny models

class TinyResNet18TV(nn.Module):
    """ResNet-18 layer names/topology (torchvision stem) at widths 8/16/32/64."""

    def __init__(self, widths=(8, 16, 32, 64), num_classes=10):
        super().__init__()
        from torchvision.models.resnet import BasicBlock
        w0 = widths[0]
        self.conv1 = nn.Conv2d(3, w0, 7, 2, 3, bias=False)
        self.bn1 = nn.BatchNorm2d(w0)
        self.relu = nn.ReLU(inplace=True)
        self.maxpool = nn.MaxPool2d(3, 2, 1)
        cin = w0
        for li, wd in enumerate(widths):
            blocks = []
            for bi in range(2):
                stride = 2 if (bi == 0 and li > 0) else 1
                ds = None
                if stride != 1 or cin != wd:
                    ds = nn.Sequential(nn.Conv2d(cin, wd, 1, stride, bias=False), nn.BatchNorm2d(wd))
                blocks.append(BasicBlock(cin, wd, stride, ds))
                cin = wd
            setattr(self, f"layer{li + 1}", nn.Sequential(*blocks))
        self.avgpool = nn.AdaptiveAvgPool2d(1)
        self.fc = nn.Linear(cin, num_classes)

    def forward(self, x):
        x = self.maxpool(self.relu(self.bn1(self.conv1(x))))
        for i in range(1, 5):
            x = getattr(self, f"layer{i}")(x)
        return self.fc(torch.flatten(self.avgpool(x), 1))


def _data_bn(model, x, seed):
    g = torch.Generator().manual_seed(seed)
    for m in model.modules():
        if isinstance(m, nn.BatchNorm2d):
            m.reset_running_stats()
            m.momentum = None
            m.weight.data = 0.5 + torch.rand(m.num_features, generator=g)
            m.bias.data = 0.3 * torch.randn(m.num_features, generator=g)
    model.train()
    with torch.no_grad():
        model(x)
    model.eval()


def _ref_ranges(model, imgs):
    """Reference calibration: 03 collect_activations + the percentile rule of calib.py."""
    import calib
    torch.manual_seed(2026)
    loader = [(imgs[i:i + 32], None) for i in range(0, imgs.shape[0], 32)]
    store = calib.collect_activations(model, loader, device="cpu")
    out = []
    for name, m in model.named_modules():
        if isinstance(m, nn.Conv2d):
            x = store[name]
            out.append((calib._quantile(x, 1 - 0.9999), calib._quantile(x, 0.9999)))
    return out


def make_r18_tiny():
    import model as M03
    from ptq_toolkit.export import exporter, ptqc
    import ref_e2e
    d = OUT / "e2e_r18tv_tiny"
    d.mkdir(exist_ok=True)
    torch.manual_seed(5)
    m = TinyResNet18TV()
    imgs = torch.randn(128, 3, 32, 32, generator=torch.Generator().manual_seed(6))
    _data_bn(m, imgs[:64], 7)
    m = M03.fold_all_bn(m).eval()
    ranges = _ref_ranges(m, imgs)
    exporter.export_weights(m, d / "model.ptqw.bin", imgs[:2])
    ptqc.write_ptqc(d / "calib.ptqc", ranges)
    x = np.random.default_rng(8).standard_normal((3, 3, 32, 32)).astype(np.float32)
    convs, blocks, stem_pool, fcw, fcb = ref_e2e.read_model(str(d / "model.ptqw.bin"))
    rr = ref_e2e.read_calib(str(d / "calib.ptqc"))
    trace = []
    logits = ref_e2e.forward(x, convs, blocks, stem_pool, fcw, fcb, rr, 8, 8, trace=trace)
    logits4 = ref_e2e.forward(x, convs, blocks, stem_pool, fcw, fcb, rr, 4, 8)
    np.savez_compressed(d / "expected.npz", x=x, logits=logits, logits_w4=logits4,
                        **{f"block{i}": t for i, t in enumerate(trace)})


def make_mv2_tiny():
    import model as M03
    from ptq_toolkit.export import ptqc, topoblocks
    from ptq_toolkit.models import mobilenet_v2 as mv2
    from ptq_toolkit.ref_int8 import SymActQuant, add_residual, conv2d_int8
    d = OUT / "e2e_mv2_tiny"
    d.mkdir(exist_ok=True)
    saved = (mv2.MobileNetV2.SETTINGS, mv2.MobileNetV2.FIRST_CHANNEL, mv2.MobileNetV2.LAST_CHANNEL)
    mv2.MobileNetV2.SETTINGS = [(1, 8, 1, 1), (6, 8, 2, 1), (6, 16, 2, 2), (6, 24, 1, 1)]
    mv2.MobileNetV2.FIRST_CHANNEL = 16
    mv2.MobileNetV2.LAST_CHANNEL = 64
    try:
        torch.manual_seed(9)
        m = mv2.MobileNetV2(num_classes=10)
        imgs = torch.randn(128, 3, 32, 32, generator=torch.Generator().manual_seed(10))
        _data_bn(m, imgs[:64], 11)
        m = M03.fold_all_bn(m).eval()
        ranges = _ref_ranges(m, imgs)
        plan = mv2.topo_plan()
        topoblocks.export_blocks(m, d / "model.ptq2.bin", imgs[:2], plan)
        ptqc.write_ptqc(d / "calib.ptqc", ranges)
        act = next((p["_act"] for p in plan if "_act" in p), "relu")
        recs, blocks, stem_pool, stem_idx = topoblocks.build_blocks(m, plan, stem_pool=False, act=act)
    finally:
        mv2.MobileNetV2.SETTINGS, mv2.MobileNetV2.FIRST_CHANNEL, mv2.MobileNetV2.LAST_CHANNEL = saved
    acts = {0: None, 1: "relu", 2: "relu6"}
    bits = [8 if i % 3 else 4 for i in range(len(recs))]   # a mixed W4/W8 plan
    aqs = [SymActQuant.from_range(lo, hi) for lo, hi in ranges]

    def conv(i, t):
        r = recs[i]
        return conv2d_int8(t, r.weight, r.bias, act_quant=aqs[i], w_bits=bits[i], stride=(r.sh, r.sw),
                           padding=(r.ph, r.pw), groups=r.groups, activation=acts[r.relu])

    x = np.random.default_rng(12).standard_normal((3, 3, 32, 32)).astype(np.float32)
    y = conv(stem_idx, x)
    outs = []
    for blk in blocks:
        t = y
        for ci in blk.convs:
            t = conv(ci, t)
        if blk.residual in (1, 2):
            ident = conv(blk.ds, y) if blk.ds >= 0 else y
            y = add_residual(t, ident, "relu" if blk.residual == 1 else None)
        else:
            y = t
        outs.append(y)
    fc = [mm for _, mm in m.named_modules() if isinstance(mm, nn.Linear)][-1]
    logits = y.mean(axis=(2, 3)) @ fc.weight.detach().numpy().T + fc.bias.detach().numpy()
    np.savez_compressed(d / "expected.npz", x=x, logits=logits, bits=np.array(bits),
                        **{f"block{i}": t for i, t in enumerate(outs)})


# --------------------------------------------------------------------------- modelgen pin

def sha(p):
    return hashlib.sha256(Path(p).read_bytes()).hexdigest()


def make_modelgen_pin():
    """Reference producer code applied to the benchmark configs' seeded models."""
    import model as M03
    from ptq_toolkit.export import ptqc, topoblocks
    from ptq_toolkit.models import mobilenet_v2 as mv2
    from ptq_toolkit.models import resnet18_plan
    from ptq_toolkit.quant.ptq import quantize_per_channel_sym
    sys.path.insert(0, str(OUT.parents[1]))
    from ptq_int8_lab_b200 import modelgen as mg   # model construction + seeds only
    res = {}
    tmp = OUT / "_tmp"
    tmp.mkdir(exist_ok=True)
    for cfg in (0, 2):
        if cfg == 0:
            m = mg.build_resnet18(0, "cifar")
            plan = resnet18_plan.topo_plan()
        else:
            saved = mv2.MobileNetV2.SETTINGS
            mv2.MobileNetV2.SETTINGS = mg.MV2_SETTINGS_CIFAR
            try:
                torch.manual_seed(1)
                m = mv2.MobileNetV2(num_classes=10)
                for mod in m.modules():   # torchvision initialisation, as in modelgen.build_mobilenet_v2
                    if isinstance(mod, nn.Conv2d):
                        nn.init.kaiming_normal_(mod.weight, mode="fan_out")
                    elif isinstance(mod, nn.BatchNorm2d):
                        nn.init.ones_(mod.weight)
                        nn.init.zeros_(mod.bias)
                    elif isinstance(mod, nn.Linear):
                        nn.init.normal_(mod.weight, 0, 0.01)
                        nn.init.zeros_(mod.bias)
                m.eval()
                plan = mv2.topo_plan()
            finally:
                mv2.MobileNetV2.SETTINGS = saved
        m = M03.fold_all_bn(m).eval()
        imgs = mg.calib_images()
        import calib
        torch.manual_seed(mg.CALIB_SEED)
        store = calib.collect_activations(m, [(imgs[i:i + 64], None) for i in range(0, 512, 64)], device="cpu")
        ranges = []
        for name, mod in m.named_modules():
            if isinstance(mod, nn.Conv2d):
                ranges.append((calib._quantile(store[name], 1 - 0.9999), calib._quantile(store[name], 0.9999)))
        for name, mod in m.named_modules():
            if isinstance(mod, (nn.Conv2d, nn.Linear)):
                q = quantize_per_channel_sym(mod.weight.detach().numpy(), 8)
                mod.weight.data.copy_(torch.from_numpy(q.dequant()).reshape(mod.weight.shape))
        topoblocks.export_blocks(m, tmp / "m.bin", imgs[:2], plan)
        ptqc.write_ptqc(tmp / "c.ptqc", ranges)
        res[str(cfg)] = {"ptq2_sha256": sha(tmp / "m.bin"), "ptqc_sha256": sha(tmp / "c.ptqc")}
        (tmp / "m.bin").unlink()
        (tmp / "c.ptqc").unlink()
    tmp.rmdir()
    (OUT / "modelgen_sha.json").write_text(json.dumps(res, indent=2))


# --------------------------------------------------------------------------- 8-bit input

def make_u8_norm():
    """Raw CIFAR-10 records (1 label byte + 3072 pixel bytes) through the reference's
    decode + normalisation (ref_e2e.read_test_batch)."""
    import ref_e2e
    rng = np.random.default_rng(5)
    n = 3
    px = np.empty((n, 3, 32, 32), np.uint8)
    px[0] = (np.arange(3 * 1024) % 256).reshape(3, 32, 32)          # every value, every channel
    px[1] = (255 - np.arange(3 * 1024) % 256).reshape(3, 32, 32)
    px[2] = rng.integers(0, 256, size=(3, 32, 32), dtype=np.uint8)
    labels = np.array([3, 7, 9], np.uint8)
    rec = np.concatenate([labels[:, None], px.reshape(n, -1)], axis=1)
    tmp = OUT / "_u8.raw"
    tmp.write_bytes(rec.tobytes())
    try:
        x, lab = ref_e2e.read_test_batch(str(tmp), n)
    finally:
        tmp.unlink()
    assert lab.tolist() == labels.tolist()
    np.savez_compressed(OUT / "u8_norm.npz", records=rec.reshape(-1), x=np.asarray(x, np.float32))


STEPS = {"kats": make_kats, "r18": make_r18_tiny, "mv2": make_mv2_tiny, "modelgen": make_modelgen_pin,
         "u8": make_u8_norm}

if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/ptq-int8-lab [step ...]  "
                 f"(steps: {' '.join(STEPS)}; default all)")
    ref = Path(sys.argv[1])
    setup(ref)
    for name in sys.argv[2:] or list(STEPS):
        STEPS[name]()
    print("golden fixtures written to", OUT)
