# -*- coding: utf-8 -*-
"""Time the reference's own CPU integer forward beside the port bench.py times (TEST INFRASTRUCTURE).

    python oracle/time_vs_reference.py --reference <ptq-int8-lab checkout> [--images 8] [--out FILE]

bench.py's CPU baseline (its `cpu_baseline` leg and the `--impl reference` arm) runs the
restatement in oracle/ptq8_oracle.py with numpy int32 matmul, because the reference's
forward is Python that is not installed with the project (the checkout has no packaging
metadata) and is not present where the GPU runs.  This script runs, on the same host and
the same inputs, the reference's `06-gpu-int8/cpp/ref_e2e.py::forward` (imported from the
checkout given on the command line; its model reader needs PTQW, so the config-4 ResNet-18
is written as PTQW first) and the port, checks that their logits agree bit for bit, and
reports both times (median of 3 runs after a warm-up, the protocol of
09-ptq-toolkit/tools/stage0_bench.py).  Its output is a summary for profiles/.

Nothing in the product imports this file; it reads the reference checkout only when run
by hand in a container that has one.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import struct
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def write_ptqw(model, path) -> None:
    """A ResNet-18 PTQ2 model (oracle.Model) as PTQW (06-gpu-int8/cpp/export_weights.py:12-21):
    per conv 9 x i32 + weights + bias, per block (c1, c2, ds, stride), then the FC."""
    out = [b"PTQW", struct.pack("<3i", len(model.convs), len(model.blocks), model.stem_pool)]
    for c in model.convs:
        if c.groups != 1:
            raise ValueError("PTQW has no groups field")
        out.append(struct.pack("<9i", c.cout, c.cin, c.kh, c.kw, c.sh, c.sw, c.ph, c.pw, c.relu))
        out.append(np.ascontiguousarray(c.weight, dtype="<f4").tobytes())
        out.append(np.ascontiguousarray(c.bias, dtype="<f4").tobytes())
    for b in model.blocks:
        if len(b.convs) != 2 or b.residual != 1:
            raise ValueError("PTQW blocks are two convs with an add + ReLU residual")
        out.append(struct.pack("<4i", b.convs[0], b.convs[1], b.ds, b.stride))
    out.append(struct.pack("<2i", model.fc_w.shape[1], model.fc_w.shape[0]))
    out.append(np.ascontiguousarray(model.fc_w, dtype="<f4").tobytes())
    out.append(np.ascontiguousarray(model.fc_b, dtype="<f4").tobytes())
    Path(path).write_bytes(b"".join(out))


def median_time(fn, runs: int = 3):
    fn()   # warm-up
    ts = []
    for _ in range(runs):
        t0 = time.perf_counter()
        r = fn()
        ts.append(time.perf_counter() - t0)
    return sorted(ts)[len(ts) // 2], ts, r


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the PaperTigerL/ptq-int8-lab checkout")
    ap.add_argument("--images", type=int, default=8)
    ap.add_argument("--cache", default=os.path.join(tempfile.gettempdir(), "ptq8_models"))
    ap.add_argument("--out", default=None)
    a = ap.parse_args()

    from oracle import ptq8_oracle as O
    from ptq_int8_lab_b200 import modelgen as mg

    spec = importlib.util.spec_from_file_location("ref_e2e", Path(a.reference) / "06-gpu-int8" / "cpp" / "ref_e2e.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)

    paths = mg.make_config(4, a.cache)
    om = O.read_model(paths["model"])
    ptqw = Path(a.cache) / "resnet18_cifar_s0.ptqw.bin"
    write_ptqw(om, ptqw)
    convs, blocks, stem_pool, fcw, fcb = ref.read_model(str(ptqw))
    ranges = ref.read_calib(paths["calib"])
    x = np.random.default_rng(99).standard_normal((a.images, 3, 32, 32)).astype(np.float32)

    t_ref, ts_ref, l_ref = median_time(
        lambda: ref.forward(x, convs, blocks, stem_pool, fcw, fcb, ranges, 8, 8))
    O.MATMUL_MODE["mode"] = "int32"
    try:
        orc = O.Oracle(om, O.read_ptqc(paths["calib"]))
        t_port, ts_port, tr = median_time(lambda: orc.forward(x, trace=False))
    finally:
        O.MATMUL_MODE["mode"] = "blas"
    # the final fp32 map of both must be bit-identical (elementwise arithmetic); the logits
    # come from a float32 mean whose summation order follows each forward's memory layout,
    # so they agree within the logit tolerance, not bit for bit
    y_ref = ref.forward(x, convs, blocks, stem_pool, fcw, fcb, ranges, 8, 8, stop_after_block=len(blocks) - 1)
    y_port = O.Oracle(om, O.read_ptqc(paths["calib"])).forward(x).block_out[-1]
    same_map = bool(np.array_equal(np.asarray(y_ref, dtype=np.float32), y_port))
    ok_logits, lerr = O.logits_close(np.asarray(l_ref, dtype=np.float64), tr.logits, 1e-5)
    same = same_map and ok_logits
    try:
        cpu = next(l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name"))
    except (OSError, StopIteration):
        cpu = "unknown"
    lines = [
        "# CPU baseline: the reference's ref_e2e.forward beside the port bench.py times",
        "",
        "Command (in a container with the reference checkout; nothing here runs on the GPU box):",
        "",
        "```",
        f"python oracle/time_vs_reference.py --reference <checkout> --images {a.images}",
        "```",
        "",
        f"Workload: BASELINE config-4 ResNet-18 W8A8 (CIFAR stem, seed 0), {a.images} seeded N(0,1) images, "
        f"one process, numpy {np.__version__}, CPU `{cpu}`.",
        "",
        "| forward | median s | runs (s) | images/s |",
        "|---|---|---|---|",
        f"| reference `06-gpu-int8/cpp/ref_e2e.py::forward` (PTQW of the same model) | {t_ref:.3f} | "
        f"{', '.join(f'{t:.3f}' for t in ts_ref)} | {a.images / t_ref:.2f} |",
        f"| port `oracle/ptq8_oracle.py` (`MATMUL_MODE = int32`, as bench.py) | {t_port:.3f} | "
        f"{', '.join(f'{t:.3f}' for t in ts_port)} | {a.images / t_port:.2f} |",
        "",
        f"Final fp32 maps of the two forwards bit-identical: {same_map}; logits within 1e-5 of the "
        f"float64 head (max relative error {lerr:.2e}): {ok_logits}.  Port / reference time: {t_port / t_ref:.3f}.",
    ]
    text = "\n".join(lines) + "\n"
    print(text)
    if a.out:
        Path(a.out).write_text(text)
    if not same:
        sys.exit(1)


if __name__ == "__main__":
    main()
