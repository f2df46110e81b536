# -*- coding: utf-8 -*-
"""Synthetic calibrated-model producer: PTQ2 weights+topology, PTQC ranges, layer plan.

This is the upstream of the engine: it writes exactly the files the
reference's toolchain hands to its int8 engine, for the five benchmark
configurations, from seeded random weights (no trained checkpoint or dataset
is available).  Every step restates the reference's own producer:

* CIFAR ResNet-18: torchvision ``resnet18`` (as 03-ptq-lab/src/model.py:34-45
  builds it) with the stem replaced by a 3x3/s1/p1 conv and no maxpool; the
  replacement conv is Kaiming-normal (fan_out, relu) like torchvision's own
  init.  The torchvision-stem variant keeps the 7x7/s2 stem and maxpool.
* MobileNetV2: restatement of 09-ptq-toolkit/ptq_toolkit/models/mobilenet_v2.py:34-178
  (same module names, so the same conv order), with the stage table passed in
  so the CIFAR strides of the benchmark (stage (6,24,2,1)) can be used.
* BN fold: 03-ptq-lab/src/model.py:64-120 (``fold_bn_into_conv`` / ``fold_all_bn``).
* Calibration: 03-ptq-lab/src/calib.py:14-72 (forward hooks on every Conv2d
  input, 200k-value random subsample drawn from the CPU generator, kthvalue
  percentile) with the symmetric percentile rule of calib.py:105-107.
* Topology: 09-.../export/topoblocks.py:90-178 (``build_blocks``) with the
  plans of models/resnet18_plan.py:16-26 and models/mobilenet_v2.py:183-250.
* PTQ2 writer: topoblocks.py:247-267; PTQC writer: export/ptqc.py:51-84;
  layer plan: export/mixed_check.py:62-81 and quant/mixed.py:179-181.
* Weight QDQ before export: pipeline.py:363-372 / 774-781 (per-channel,
  bits from the layer plan).
"""
from __future__ import annotations

import hashlib
import json
import math
import struct
import time
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

# (t, c, n, s) stage tables.  The reference's table is torchvision's
# (mobilenet_v2.py:119-127); the benchmark's CIFAR table uses stride 1 on the
# 24-channel stage.
MV2_SETTINGS_REFERENCE = [(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2),
                          (6, 96, 3, 1), (6, 160, 3, 2), (6, 320, 1, 1)]
MV2_SETTINGS_CIFAR = [(1, 16, 1, 1), (6, 24, 2, 1), (6, 32, 3, 2), (6, 64, 4, 2),
                      (6, 96, 3, 1), (6, 160, 3, 2), (6, 320, 1, 1)]

CALIB_SEED = 2026          # 03-ptq-lab/config.py:130
CALIB_N = 512
CALIB_BATCH = 64
PERCENTILE = 0.9999
SAMPLES_PER_LAYER = 200000  # calib.py:23


# --------------------------------------------------------------------------- models

def _make_divisible(v: float, divisor: int = 8) -> int:
    if v < divisor:
        return int(v + 0.5)
    return int(v / divisor + 0.5) * divisor


class ConvBNReLU6(nn.Sequential):
    def __init__(self, inp, oup, kernel, stride, groups=1, act=True):
        padding = (kernel - 1) // 2
        layers = [nn.Conv2d(inp, oup, kernel, stride, padding, groups=groups, bias=False),
                  nn.BatchNorm2d(oup)]
        if act:
            layers.append(nn.ReLU6(inplace=True))
        super().__init__(*layers)


class InvertedResidual(nn.Module):
    def __init__(self, inp, oup, stride, expand_ratio):
        super().__init__()
        self.stride = stride
        self.use_res = (stride == 1 and inp == oup)
        hidden = int(round(inp * expand_ratio))
        layers: List[nn.Module] = []
        if expand_ratio != 1:
            layers.append(ConvBNReLU6(inp, hidden, kernel=1, stride=1))
        layers.extend([ConvBNReLU6(hidden, hidden, kernel=3, stride=stride, groups=hidden),
                       nn.Conv2d(hidden, oup, 1, 1, 0, bias=False),
                       nn.BatchNorm2d(oup)])
        self.conv = nn.Sequential(*layers)

    def forward(self, x):
        out = self.conv(x)
        return x + out if self.use_res else out


class MobileNetV2(nn.Module):
    """torchvision-structured MobileNetV2 with a 3x3/s1 stem (mobilenet_v2.py:111-173)."""

    def __init__(self, num_classes=10, settings=MV2_SETTINGS_CIFAR, first=32, last=1280):
        super().__init__()
        self.settings = list(settings)
        self.features = nn.Sequential()
        self.features.add_module("0", ConvBNReLU6(3, first, kernel=3, stride=1))
        cin = first
        idx = 1
        for t, c, n, s in self.settings:
            oup = _make_divisible(c)
            for i in range(n):
                self.features.add_module(str(idx), InvertedResidual(cin, oup, s if i == 0 else 1, t))
                cin = oup
                idx += 1
        self.proj_idx = idx
        self.features.add_module(str(idx), ConvBNReLU6(cin, last, kernel=1, stride=1))
        self.classifier = nn.Sequential(nn.Dropout(0.2), nn.Linear(last, num_classes))

    def forward(self, x):
        x = self.features(x)
        x = F.adaptive_avg_pool2d(x, 1).flatten(1)
        return self.classifier(x)


def build_resnet18(seed: int, stem: str = "cifar", num_classes: int = 10) -> nn.Module:
    """ResNet-18 from torchvision with either the CIFAR stem or the 7x7/s2+maxpool stem."""
    import torchvision
    torch.manual_seed(seed)
    m = torchvision.models.resnet18(num_classes=num_classes)
    if stem == "cifar":
        m.conv1 = nn.Conv2d(3, 64, kernel_size=3, stride=1, padding=1, bias=False)
        nn.init.kaiming_normal_(m.conv1.weight, mode="fan_out", nonlinearity="relu")
        m.maxpool = nn.Identity()
    elif stem != "torchvision":
        raise ValueError(f"unknown stem {stem!r}")
    return m.eval()


def build_mobilenet_v2(seed: int, settings=MV2_SETTINGS_CIFAR, num_classes: int = 10) -> nn.Module:
    """MobileNetV2 with torchvision's initialisation (Kaiming-normal fan_out convs)."""
    torch.manual_seed(seed)
    m = MobileNetV2(num_classes=num_classes, settings=settings)
    for mod in m.modules():
        if isinstance(mod, nn.Conv2d):
            nn.init.kaiming_normal_(mod.weight, mode="fan_out")
            if mod.bias is not None:
                nn.init.zeros_(mod.bias)
        elif isinstance(mod, nn.BatchNorm2d):
            nn.init.ones_(mod.weight)
            nn.init.zeros_(mod.bias)
        elif isinstance(mod, nn.Linear):
            nn.init.normal_(mod.weight, 0, 0.01)
            nn.init.zeros_(mod.bias)
    return m.eval()


@torch.no_grad()
def data_bn(model: nn.Module, x: torch.Tensor, seed: int) -> nn.Module:
    """BN statistics taken from a data batch plus random affine terms (test models).

    Randomly initialised deep nets shrink their activations layer by layer when
    BN keeps its default statistics; normalising every BN on real activations
    keeps all layers' codes non-trivial, which makes parity tests meaningful."""
    g = torch.Generator().manual_seed(seed)
    for mod in model.modules():
        if isinstance(mod, nn.BatchNorm2d):
            mod.reset_running_stats()
            mod.momentum = None
            mod.weight.data = 0.5 + torch.rand(mod.num_features, generator=g)
            mod.bias.data = 0.3 * torch.randn(mod.num_features, generator=g)
    model.train()
    model(x)
    model.eval()
    return model


def randomize_bn(model: nn.Module, seed: int) -> nn.Module:
    """Give every BN non-trivial statistics (test models: exercises the folded bias)."""
    g = torch.Generator().manual_seed(seed)
    for mod in model.modules():
        if isinstance(mod, nn.BatchNorm2d):
            c = mod.num_features
            mod.weight.data = 0.5 + torch.rand(c, generator=g)
            mod.bias.data = 0.2 * torch.randn(c, generator=g)
            mod.running_mean.data = 0.2 * torch.randn(c, generator=g)
            mod.running_var.data = 0.5 + torch.rand(c, generator=g)
    return model


# --------------------------------------------------------------------------- BN fold

def fold_bn_into_conv(conv: nn.Conv2d, bn: nn.BatchNorm2d) -> nn.Conv2d:
    """W' = W*A, b' = b*A + (beta - A*mean), A = gamma/sqrt(var+eps) (model.py:64-87)."""
    std = torch.sqrt(bn.running_var.data + bn.eps)
    A = bn.weight.data / std
    B = bn.bias.data - A * bn.running_mean.data
    w = conv.weight.data
    w.mul_(A.reshape(-1, 1, 1, 1))
    if conv.bias is None:
        conv.bias = nn.Parameter(torch.zeros(w.shape[0], dtype=w.dtype))
    conv.bias.data.mul_(A)
    conv.bias.data.add_(B)
    return conv


def fold_all_bn(model: nn.Module) -> nn.Module:
    """Fold every (Conv2d, BatchNorm2d) neighbour pair; BN becomes Identity (model.py:90-116)."""
    model.eval()
    children = list(model.named_children())
    for _, child in children:
        if len(list(child.children())) > 0:
            fold_all_bn(child)
    if isinstance(model, nn.Sequential):
        items = list(model)
        for i in range(len(items) - 1):
            if isinstance(items[i], nn.Conv2d) and isinstance(items[i + 1], nn.BatchNorm2d):
                fold_bn_into_conv(items[i], items[i + 1])
                model[i + 1] = nn.Identity()
        return model
    names = [n for n, _ in children]
    for i in range(len(names) - 1):
        a = getattr(model, names[i])
        b = getattr(model, names[i + 1])
        if isinstance(a, nn.Conv2d) and isinstance(b, nn.BatchNorm2d):
            fold_bn_into_conv(a, b)
            setattr(model, names[i + 1], nn.Identity())
    return model


# --------------------------------------------------------------------------- calibration

def calib_images(n: int = CALIB_N, seed: int = CALIB_SEED) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, 3, 32, 32, generator=g)


@torch.no_grad()
def collect_activations(model: nn.Module, batches, samples_per_layer: int = SAMPLES_PER_LAYER):
    """Per-conv input store with CPU-RNG subsampling (calib.py:23-72)."""
    store: Dict[str, torch.Tensor] = {}
    hooks = []
    for nm, mod in model.named_modules():
        if not isinstance(mod, nn.Conv2d):
            continue

        def mk(nm_):
            def hk(m, inp, out):
                f = inp[0].detach().reshape(-1)
                if f.numel() > samples_per_layer:
                    idx = torch.randint(0, f.numel(), (samples_per_layer,), device="cpu")
                    f = f[idx]
                f = f.float().cpu()
                cur = store.get(nm_)
                if cur is None:
                    store[nm_] = f
                else:
                    cat = torch.cat([cur, f])
                    if cat.numel() > samples_per_layer:
                        idx = torch.randperm(cat.numel())[:samples_per_layer]
                        cat = cat[idx]
                    store[nm_] = cat
            return hk

        hooks.append(mod.register_forward_hook(mk(nm)))
    model.eval()
    for x in batches:
        model(x)
    for h in hooks:
        h.remove()
    return store


def _quantile(x: torch.Tensor, q: float) -> float:
    """kthvalue percentile, k = clamp(round(n*q), 1, n) (calib.py:14-19)."""
    f = x.reshape(-1)
    n = f.numel()
    k = max(1, min(n, int(round(n * q))))
    return float(torch.kthvalue(f, k, keepdim=False)[0])


def percentile_ranges(model: nn.Module, store, percentile: float = PERCENTILE
                      ) -> List[Tuple[float, float]]:
    """(lo, hi) per conv in definition order (calib.py:105-107; ptqc.py:134-172)."""
    out = []
    for name, m in model.named_modules():
        if isinstance(m, nn.Conv2d):
            x = store[name]
            lo = _quantile(x, 1.0 - percentile)
            hi = _quantile(x, percentile)
            if not (math.isfinite(lo) and math.isfinite(hi)) or lo > hi:
                raise ValueError(f"bad range for {name}: {lo} {hi}")
            out.append((lo, hi))
    return out


def calibrate(model: nn.Module, images: torch.Tensor, batch: int = CALIB_BATCH,
              seed: int = CALIB_SEED, percentile: float = PERCENTILE):
    torch.manual_seed(seed)
    batches = [images[i:i + batch] for i in range(0, images.shape[0], batch)]
    store = collect_activations(model, batches)
    return percentile_ranges(model, store, percentile)


# --------------------------------------------------------------------------- topology

def resnet18_plan() -> List[dict]:
    """models/resnet18_plan.py:16-26."""
    plan = []
    for lname, ds_stage in (("layer1", False), ("layer2", True), ("layer3", True), ("layer4", True)):
        for bi in range(2):
            first = bi == 0 and ds_stage
            plan.append({"convs": [f"{lname}.{bi}.conv1", f"{lname}.{bi}.conv2"],
                         "downsample": f"{lname}.{bi}.downsample.0" if first else None,
                         "stride": 2 if first else 1})
    return plan


def mobilenet_v2_plan(settings=MV2_SETTINGS_CIFAR, first: int = 32) -> List[dict]:
    """models/mobilenet_v2.py:183-250, driven by the given stage table."""
    plan = []
    cin = first
    blk = 1
    for t, cout, n, stride in settings:
        for i in range(n):
            s = stride if i == 0 else 1
            use_res = (s == 1 and cin == cout)
            if t == 1:
                cs = [f"features.{blk}.conv.0.0", f"features.{blk}.conv.1"]
            else:
                cs = [f"features.{blk}.conv.0.0", f"features.{blk}.conv.1.0", f"features.{blk}.conv.2"]
            e = {"convs": cs, "downsample": None, "stride": s,
                 "_no_residual": not use_res, "_last_relu": False}
            if use_res:
                e["_post_relu"] = False
            plan.append(e)
            cin = cout
            blk += 1
    plan.append({"convs": [f"features.{blk}.0"], "downsample": None, "stride": 1, "_no_residual": True})
    plan[0]["_act"] = "relu6"
    return plan


def build_blocks(model: nn.Module, plan: List[dict], act: str = "relu"):
    """Conv records + blocks with the relu/residual flags of topoblocks.py:90-178."""
    act_val = {"relu": 1, "relu6": 2}[act]
    named = [(n, m) for n, m in model.named_modules() if isinstance(m, nn.Conv2d)]
    idx = {n: i for i, (n, _) in enumerate(named)}
    in_blocks = {n for p in plan for n in p["convs"]} | {p["downsample"] for p in plan if p.get("downsample")}
    outside = [n for n, _ in named if n not in in_blocks]
    if not outside:
        raise RuntimeError("no stem conv outside the blocks")
    stem_name = outside[0]
    if len(outside) > 1:
        raise RuntimeError(f"convs outside the plan: {outside[1:]}")
    recs = []
    for _, m in named:
        w = m.weight.detach().cpu().contiguous().numpy().astype(np.float32)
        b = (m.bias.detach().cpu().contiguous().numpy().astype(np.float32)
             if m.bias is not None else np.zeros(w.shape[0], np.float32))
        recs.append(dict(cout=w.shape[0], cin=w.shape[1], kh=w.shape[2], kw=w.shape[3],
                         sh=m.stride[0], sw=m.stride[1], ph=m.padding[0], pw=m.padding[1],
                         relu=act_val, groups=m.groups, weight=w, bias=b))
    blocks = []
    for p in plan:
        cs = [idx[n] for n in p["convs"]]
        ds = idx[p["downsample"]] if p.get("downsample") else -1
        res = 0 if p.get("_no_residual") else (1 if p.get("_post_relu", True) else 2)
        blocks.append(dict(convs=cs, ds=ds, stride=int(p.get("stride", 1)), residual=res))
    for p, blk in zip(plan, blocks):
        last_act = p["_last_relu"] if "_last_relu" in p else (blk["residual"] == 0)
        if not last_act:
            recs[blk["convs"][-1]]["relu"] = 0
        if blk["ds"] >= 0 and blk["residual"] in (1, 2):
            recs[blk["ds"]]["relu"] = 0
    recs[idx[stem_name]]["relu"] = act_val
    stem_pool = int(any(isinstance(m, nn.MaxPool2d) for m in model.modules()))
    return recs, blocks, stem_pool, idx[stem_name]


def replay_blocks(model: nn.Module, recs, blocks, stem_pool, x, stem_idx=0):
    """Torch replay of the exported topology (topoblocks.py:181-220)."""
    def conv(i, t):
        r = recs[i]
        y = F.conv2d(t, torch.from_numpy(r["weight"]), torch.from_numpy(r["bias"]),
                     stride=(r["sh"], r["sw"]), padding=(r["ph"], r["pw"]), groups=r["groups"])
        if r["relu"] == 1:
            return F.relu(y)
        if r["relu"] == 2:
            return F.hardtanh(y, 0.0, 6.0)
        return y
    y = conv(stem_idx, x)
    if stem_pool:
        y = F.max_pool2d(y, 3, 2, 1)
    for blk in blocks:
        t = y
        for ci in blk["convs"]:
            t = conv(ci, t)
        if blk["residual"] in (1, 2):
            ident = conv(blk["ds"], y) if blk["ds"] >= 0 else y
            s = t + ident
            y = F.relu(s) if blk["residual"] == 1 else s
        else:
            y = t
    fc = [m for _, m in model.named_modules() if isinstance(m, nn.Linear)][-1]
    return fc(y.mean(dim=(2, 3)).flatten(1))


def ptq2_bytes(model: nn.Module, recs, blocks, stem_pool) -> bytes:
    """PTQ2 blob (topoblocks.py:247-267)."""
    ncp = max(len(b["convs"]) for b in blocks)
    blob = bytearray(b"PTQ2")
    blob += struct.pack("<4i", len(recs), len(blocks), int(stem_pool), ncp)
    for r in recs:
        blob += struct.pack("<10i", r["cout"], r["cin"], r["kh"], r["kw"], r["sh"], r["sw"],
                            r["ph"], r["pw"], r["relu"], r["groups"])
        blob += np.ascontiguousarray(r["weight"], dtype="<f4").tobytes()
        blob += np.ascontiguousarray(r["bias"], dtype="<f4").tobytes()
    for b in blocks:
        cs = list(b["convs"]) + [-1] * (ncp - len(b["convs"]))
        blob += struct.pack(f"<{ncp + 3}i", *cs, b["ds"], b["stride"], b["residual"])
    fw = [m for _, m in model.named_modules() if isinstance(m, nn.Linear)][-1]
    W = fw.weight.detach().cpu().contiguous().numpy()
    B = fw.bias.detach().cpu().contiguous().numpy()
    blob += struct.pack("<2i", W.shape[1], W.shape[0])
    blob += np.ascontiguousarray(W, dtype="<f4").tobytes()
    blob += np.ascontiguousarray(B, dtype="<f4").tobytes()
    return bytes(blob)


def export_ptq2(model: nn.Module, path, plan: List[dict], x: torch.Tensor) -> dict:
    act = next((p["_act"] for p in plan if "_act" in p), "relu")
    recs, blocks, stem_pool, stem_idx = build_blocks(model, plan, act)
    with torch.no_grad():
        ref = model(x).float()
        got = replay_blocks(model, recs, blocks, stem_pool, x, stem_idx).float()
    d = float((got - ref).abs().max())
    if d > 1e-4:
        raise RuntimeError(f"PTQ2 topology self-check failed: max|diff|={d:.4g}")
    blob = ptq2_bytes(model, recs, blocks, stem_pool)
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_bytes(blob)
    return dict(path=str(p), n_conv=len(recs), n_block=len(blocks), stem_pool=stem_pool,
                bytes=len(blob), selfcheck_maxdiff=d)


def write_ptqc(path, ranges: Sequence[Tuple[float, float]]) -> dict:
    """PTQC writer with the checks of ptqc.py:51-84."""
    blob = bytearray(b"PTQC") + struct.pack("<i", len(ranges))
    for i, (lo, hi) in enumerate(ranges):
        lo, hi = float(lo), float(hi)
        if not (math.isfinite(lo) and math.isfinite(hi)) or lo > hi:
            raise ValueError(f"ranges[{i}] invalid: {lo} {hi}")
        blob += struct.pack("<2f", lo, hi)
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_bytes(bytes(blob))
    return dict(path=str(p), n=len(ranges), bytes=len(blob))


def write_layer_plan(path, model_key: str, plan_key: str, layers: List[dict]) -> dict:
    """layer_plan JSON in the schema of mixed_check.py:62-81."""
    counts: Dict[Tuple, int] = {}
    for e in layers:
        k = (e["bits"], e["scheme"], e.get("group_size", 0))
        counts[k] = counts.get(k, 0) + 1
    doc = {"schema": "ptq-layer-plan/v1", "model": model_key, "plan": plan_key,
           "created": time.strftime("%Y-%m-%dT%H:%M:%S%z"),
           "layer_order": "named_modules() Conv2d definition order",
           "counts": [{"bits": b, "scheme": s, "group_size": g, "layers": n}
                      for (b, s, g), n in sorted(counts.items())],
           "w8_layers": [e["name"] for e in layers if int(e["bits"]) == 8],
           "layers": layers}
    Path(path).write_text(json.dumps(doc, indent=2), encoding="utf-8")
    return doc


def mv2_w8_layers(model: nn.Module, n_w8: int = 24) -> List[str]:
    """The benchmark's W8 set for MobileNetV2 mixed precision.

    W8 = stem, head 1x1, the FC, and the first 1x1 conv of every stage; then
    depthwise convs are added in definition order until ``n_w8`` layers (the FC
    counts as one) are W8.  Returns conv names only (the FC is not a conv)."""
    named = [(n, m) for n, m in model.named_modules() if isinstance(m, nn.Conv2d)]
    settings = model.settings
    chosen = [named[0][0]]                                     # stem
    chosen.append(f"features.{model.proj_idx}.0")              # head 1x1
    blk = 1
    for t, c, n, s in settings:
        chosen.append(f"features.{blk}.conv.1" if t == 1 else f"features.{blk}.conv.0.0")
        blk += n
    n_fc = 1
    for name, m in named:
        if len(chosen) + n_fc >= n_w8:
            break
        if m.groups > 1 and m.groups == m.in_channels and name not in chosen:
            chosen.append(name)
    order = {n: i for i, (n, _) in enumerate(named)}
    return sorted(set(chosen), key=lambda n: order[n])


def qdq_weights(model: nn.Module, bits_by_name: Dict[str, int], fc_bits: Optional[int] = 8) -> None:
    """In-place per-channel QDQ of conv (and FC) weights (pipeline.py:363-372, 774-781)."""
    for name, m in model.named_modules():
        bits = None
        if isinstance(m, nn.Conv2d):
            bits = bits_by_name[name]
        elif isinstance(m, nn.Linear) and fc_bits:
            bits = fc_bits
        if bits is None:
            continue
        w = m.weight.detach().cpu().numpy().astype(np.float64)
        qmax = (1 << (bits - 1)) - 1
        flat = w.reshape(w.shape[0], -1)
        scale = np.maximum(np.abs(flat).max(axis=1) / qmax, 1e-8)
        v = flat / scale[:, None]
        code = np.clip(np.where(v >= 0, np.floor(v + 0.5), np.ceil(v - 0.5)), -(qmax + 1), qmax).astype(np.int8)
        deq = code.astype(np.float32) * scale.astype(np.float32)[:, None]   # int8 codes: no -0.0 weights
        m.weight.data.copy_(torch.from_numpy(deq.reshape(w.shape)))


# --------------------------------------------------------------------------- configs

CONFIGS = {
    0: dict(model="resnet18", stem="cifar", seed=0, batch=256, mixed=False),
    1: dict(model="resnet18", stem="cifar", seed=0, batch=1024, mixed=False, passes=True),
    2: dict(model="mobilenet_v2", seed=1, batch=1024, mixed=False),
    3: dict(model="mobilenet_v2", seed=2, batch=1024, mixed=True),
    4: dict(model="resnet18", stem="cifar", seed=0, batch=8192, mixed=False),
}


def build_calibrated(model_key: str, seed: int, stem: str = "cifar", mixed: bool = False,
                     out_dir=".", tag: Optional[str] = None, bn: str = "default",
                     calib_n: int = CALIB_N, settings: Optional[Sequence] = None) -> dict:
    """Build, fold, calibrate, QDQ and export one synthetic calibrated model.

    ``settings``: MobileNetV2 stage table (t, c, n, s) in place of the CIFAR one
    (e.g. expansion ratios whose depthwise channel counts are not multiples of 16)."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    if model_key == "resnet18":
        m = build_resnet18(seed, stem)
        plan = resnet18_plan()
    elif model_key == "mobilenet_v2":
        m = build_mobilenet_v2(seed, settings=settings if settings is not None else MV2_SETTINGS_CIFAR)
        plan = mobilenet_v2_plan(m.settings)
    else:
        raise ValueError(model_key)
    if bn == "random":
        randomize_bn(m, seed + 101)
    elif bn == "data":
        data_bn(m, calib_images(64, seed=CALIB_SEED + 1), seed + 101)
    m = fold_all_bn(m).eval()
    imgs = calib_images(calib_n)
    ranges = calibrate(m, imgs)
    names = [n for n, mm in m.named_modules() if isinstance(mm, nn.Conv2d)]
    if mixed:
        w8 = set(mv2_w8_layers(m))
        bits = {n: (8 if n in w8 else 4) for n in names}
    else:
        bits = {n: 8 for n in names}
    qdq_weights(m, bits, fc_bits=8)
    tag = tag or (f"{model_key}_{stem if model_key == 'resnet18' else 'cifar'}_s{seed}"
                  f"{'_mixed' if mixed else ''}{'' if bn == 'default' else '_bn' + bn}"
                  f"{'' if settings is None else '_st' + '_'.join('x'.join(map(str, r)) for r in settings)}")
    exp = export_ptq2(m, out / f"{tag}.ptq2.bin", plan, imgs[:2])
    pq = write_ptqc(out / f"calib_{tag}.ptqc", ranges)
    layers = [{"name": n, "bits": bits[n], "scheme": "per_channel"} for n in names]
    plan_path = out / f"layer_plan_{tag}.json"
    write_layer_plan(plan_path, model_key, "w4pc_w8x24" if mixed else "w8a8", layers)
    return dict(model=exp["path"], calib=pq["path"], plan=str(plan_path), tag=tag,
                n_conv=exp["n_conv"], names=names, bits=[bits[n] for n in names],
                selfcheck_maxdiff=exp["selfcheck_maxdiff"])


def make_config(cfg: int, out_dir=".", **kw) -> dict:
    c = CONFIGS[cfg]
    if c["model"] == "resnet18":
        return build_calibrated("resnet18", c["seed"], stem=c["stem"], out_dir=out_dir, **kw)
    return build_calibrated("mobilenet_v2", c["seed"], mixed=c["mixed"], out_dir=out_dir, **kw)


def read_layer_plan(path) -> List[int]:
    """Per-conv weight bits from a layer-plan JSON (``layers`` list in conv order)."""
    doc = json.loads(Path(path).read_text(encoding="utf-8"))
    layers = doc.get("layers")
    if not isinstance(layers, list) or not layers:
        raise ValueError(f"{path}: no 'layers' list")
    bits = []
    for i, e in enumerate(layers):
        b = int(e["bits"])
        if b not in (4, 8):
            raise ValueError(f"{path}: layer {i} bits={b} (only 4/8)")
        if e.get("scheme", "per_channel") != "per_channel":
            raise ValueError(f"{path}: layer {i} scheme {e.get('scheme')!r} not supported "
                             f"(the engine runs per-channel weights only)")
        bits.append(b)
    return bits


def sha256(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()
