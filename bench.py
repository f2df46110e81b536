# -*- coding: utf-8 -*-
"""Throughput benchmark: ResNet-18 W8A8 (CIFAR stem) images/sec on 1..N B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload: batch 8192 per GPU of seeded N(0,1) fp32
3x32x32 images, synthetic calibrated model (Kaiming-normal seed 0, BN folded,
99.99-percentile calibration on 512 seeded images).  Each rank runs an
independent replica on its batch shard (weak scaling); every step ends with an
NCCL all-gather of the fp32 logits when N > 1.

One JSON line on rank 0 (see the keys below).  `value` is device-timed with
inputs resident in HBM; `e2e` goes through the C-ABI host-buffer forward
(ptq8_engine_forward_async: H2D from pinned memory into one of two input slots,
graph, D2H, every step; step k+1's copy overlaps step k's forward), with the
synchronous ptq8_engine_forward (H2D, graph, D2H, sync) beside it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import datetime
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int8 images/sec ResNet-18 W8A8 32x32 at 1/2/4/8 B200; % of int8 TC/HBM roofline"
METRIC_MV2 = "int8 images/sec MobileNetV2 32x32 (BASELINE configs 2/3) on B200; % of int8 TC/HBM roofline"


def config_info(cfg: int) -> dict:
    """Model, metric, default batch and workload name of BASELINE config `cfg`."""
    from ptq_int8_lab_b200 import modelgen as mg
    c = mg.CONFIGS[cfg]
    mv2 = c["model"] == "mobilenet_v2"
    prec = "w4w8a8_mixed" if c.get("mixed") else "w8a8"
    return {"metric": METRIC_MV2 if mv2 else METRIC, "batch": c["batch"], "passes": 3 if c.get("passes") else 0,
            "name": f"{'mobilenet_v2' if mv2 else 'resnet18_' + c['stem']}_{prec}"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=4, choices=range(5),
                    help="BASELINE config (4: the headline ResNet-18 W8A8 at 8192 images per GPU)")
    ap.add_argument("--batch", type=int, default=None, help="images per GPU (default: the config's batch)")
    ap.add_argument("--model-cache", default=os.environ.get("PTQ8_MODEL_CACHE", "/tmp/ptq8_models"))
    ap.add_argument("--cpu-sample", type=int, default=12, help="images in the timed CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def model_files(cache: str, rank: int, world: int, barrier, cfg: int = 4):
    """Calibrated model files of BASELINE config `cfg` in `cache`: rank 0 writes them when
    missing (with a marker naming them), every rank returns after the barrier."""
    from ptq_int8_lab_b200 import modelgen as mg
    d = Path(cache)
    d.mkdir(parents=True, exist_ok=True)
    marker = d / f"config{cfg}.json"
    def ok():
        if not marker.exists():
            return False
        p = json.loads(marker.read_text())
        return all(Path(p[k]).exists() for k in ("model", "calib", "plan"))
    if rank == 0 and not ok():
        p = mg.make_config(cfg, d)
        marker.write_text(json.dumps({k: str(p[k]) for k in ("model", "calib", "plan")}))
    barrier()
    return json.loads(marker.read_text())


def max_over_ranks(x: float, device) -> float:
    """The largest x over all ranks of the process group (the whole job's time); x alone
    when there is no group or a single rank."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms.

    Started before the warm-up (NVML start-up takes a while); each sample carries
    a host timestamp, and only samples inside [t0, t1] of the timed region are
    summarised (the nearest sample on each side when none falls inside)."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self, wait_s: float = 5.0):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
            return
        t_end = time.time() + wait_s          # until the first sample has been written
        while time.time() < t_end and self.p.poll() is None:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

    @staticmethod
    def _ts(field: str):
        try:
            return datetime.strptime(field.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self, t0: float, t1: float) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 10 and self._ts(parts[0]) is not None:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = [r for r in rows if t0 <= self._ts(r[0]) <= t1]
        if not inside:
            before = [r for r in rows if self._ts(r[0]) < t0][-1:]
            after = [r for r in rows if self._ts(r[0]) > t1][:1]
            inside = before + after
        sm = [float(r[2]) for r in inside if r[2].replace(".", "", 1).isdigit()]
        mx = [float(r[3]) for r in inside if r[3].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in inside for k in range(4) if r[6 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def host_cpu() -> dict:
    """CPU model name and logical core count of this host."""
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count() or 1}


def cpu_baseline(paths, n_img: int, seed: int = 99, runs: int = 3) -> dict:
    """The reference's CPU integer forward (ref_e2e.py arithmetic: numpy int32 matmul,
    one core) on a bounded sample of the same workload, timed on this host with the
    reference's CPU protocol (09-ptq-toolkit/tools/stage0_bench.py: warm-up, then the
    median of `runs` timed runs)."""
    import numpy as np
    from oracle import ptq8_oracle as O
    from ptq_int8_lab_b200 import modelgen as mg
    O.MATMUL_MODE["mode"] = "int32"
    try:
        m = O.read_model(paths["model"])
        orc = O.Oracle(m, O.read_ptqc(paths["calib"]), layer_bits=mg.read_layer_plan(paths["plan"]))
        x = np.random.default_rng(seed).standard_normal((n_img, 3, 32, 32)).astype(np.float32)
        orc.forward(x[:1], trace=False)
        dts = []
        for _ in range(runs):
            t0 = time.perf_counter()
            orc.forward(x, trace=False)
            dts.append(time.perf_counter() - t0)
    finally:
        O.MATMUL_MODE["mode"] = "blas"
    dt = sorted(dts)[len(dts) // 2]
    return {"value": n_img / dt, "unit": "images/s", "cores": 1, "kind": "port",
            "sample": f"{n_img} images of the same workload, numpy int32 matmul (06-gpu-int8/cpp/ref_e2e.py:180), "
                      f"median of {runs} runs ({', '.join(f'{t:.2f}' for t in dts)} s) after a warm-up",
            **host_cpu()}


def _ref_worker(args):
    model, calib, plan, n_img, seed = args
    import numpy as np
    from oracle import ptq8_oracle as O
    from ptq_int8_lab_b200 import modelgen as mg
    O.MATMUL_MODE["mode"] = "int32"
    m = O.read_model(model)
    orc = O.Oracle(m, O.read_ptqc(calib), layer_bits=mg.read_layer_plan(plan))
    x = np.random.default_rng(seed).standard_normal((n_img, 3, 32, 32)).astype(np.float32)
    t0 = time.perf_counter()
    orc.forward(x, trace=False)
    return time.perf_counter() - t0


def run_reference(a):
    """Reference arm: the reference's CPU integer forward, all host cores, bounded sample per step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import multiprocessing as mp
    info = config_info(a.config)
    paths = model_files(a.model_cache, 0, 1, lambda: None, a.config)
    cores = os.cpu_count() or 1
    per = 2
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(max(a.warmup, 1) if a.warmup else 0):
            pool.map(_ref_worker, [(paths["model"], paths["calib"], paths["plan"], 1, 7 + i) for i in range(cores)])
        times = []
        for s in range(a.steps):
            t0 = time.perf_counter()
            pool.map(_ref_worker, [(paths["model"], paths["calib"], paths["plan"], per, 100 * s + i)
                                   for i in range(cores)])
            times.append(time.perf_counter() - t0)
    imgs = per * cores * a.steps
    tot = sum(times)
    v = imgs / tot
    line = {"impl": "reference", "metric": info["metric"], "value": v, "unit": "images/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tot / a.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{info['name']} (BASELINE configs[{a.config}] shapes)", "batch_per_step": per * cores,
                       "note": "bounded sample per step on host cores"},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"{per} images per process x {cores} spawn processes per step, "
                                       f"numpy int32 matmul as ref_e2e.py:180", **host_cpu()},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return
    import numpy as np
    import torch
    import torch.distributed as dist
    from ptq_int8_lab_b200 import engine as E

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        barrier = lambda: dist.barrier()
    else:
        barrier = lambda: None
    info = config_info(a.config)
    paths = model_files(a.model_cache, rank, world, barrier, a.config)
    B = a.batch or info["batch"]
    eng = E.open_engine(paths["model"], paths["calib"], paths["plan"], max_batch=B, device=local,
                        passes=info["passes"])
    # a real (non-legacy) stream shared by the engine, torch events and NCCL
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)

    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    x = torch.randn(B, 3, 32, 32, device="cuda", generator=g, dtype=torch.float32)
    logits = torch.empty(B, 10, device="cuda", dtype=torch.float32)
    gathered = torch.empty(world * B, 10, device="cuda", dtype=torch.float32) if world > 1 else None
    eng.forward_device(x.data_ptr(), B, logits.data_ptr())   # stage the input in the engine buffer

    def step():
        eng.run(B)
        if world > 1:
            eng.copy_logits(B, logits.data_ptr())          # same stream as the collective
            dist.all_gather_into_tensor(gathered, logits)

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    eng.sync()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    for _ in range(a.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop(t_wall0, time.time())
    ms = ev0.elapsed_time(ev1)
    eng.sync()
    ms = max_over_ranks(ms, "cuda")
    ms_per_step = ms / a.steps
    value = world * B * a.steps / (ms / 1e3)

    # ---- per-launch profile (device events per step) -> roofline of the dense convs
    prof = eng.profile(B, iters=3)
    if os.environ.get("PTQ8_BENCH_LAYERS"):
        kinds = {0: "stem", 1: "conv_tc", 2: "dw", 3: "maxpool", 4: "head"}
        for p in prof:
            t = p["ms"] / 1e3
            print(f"[layer] step {p['step']:2d} {kinds[p['kind']]:8s} {p['ms']:8.3f} ms  "
                  f"{2 * p['macs'] / t / 1e12 if t else 0:8.1f} TOPS  {p['bytes'] / t / 1e9 if t else 0:8.1f} GB/s",
                  file=sys.stderr)
    tc = [p for p in prof if p["kind"] in (0, 1)]
    tc_ms = sum(p["ms"] for p in tc)
    tc_ops = sum(2.0 * p["macs"] for p in tc)
    hbm, bf16, src = measured_peaks()
    int8_peak = 2.0 * bf16   # dense int8 tensor rate is twice the dense bf16 rate on B200
    achieved = tc_ops / (tc_ms / 1e3) / 1e12
    # DRAM bytes of all dense-conv launches of one forward, from the committed ncu summary
    # (captured at batch 2048 and scaled by 4; see the file); per forward like `achieved`
    traffic = None
    tp = ROOT / "profiles" / "conv_tc_traffic_resnet18_b8192.txt"
    if tp.exists() and a.config == 4 and B == 8192:
        for line in tp.read_text().splitlines():
            if line.startswith("traffic_bytes_per_forward_b8192 ="):
                traffic = int(line.split("=")[1].strip())
    roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                "frac": achieved / int8_peak, "traffic": traffic,
                "kernel": "conv_tc_kernel (all dense convs of one forward)",
                "peak_source": f"2 x bf16_tflops of {src} MEASURED_PEAKS.json",
                "dense_conv_ms": tc_ms, "forward_ms_sum_of_launches": sum(p["ms"] for p in prof)}

    # ---- end to end through the C-ABI host-buffer forwards (H2D + graph + D2H every step).
    # Headline: ptq8_engine_forward_async, the pipelined call (step k+1's H2D overlaps step
    # k's forward, two input slots); also the synchronous ptq8_engine_forward (the
    # reference's Int8Engine::forward semantics: copy, run, copy back, wait).
    xh = torch.empty(B, 3, 32, 32, dtype=torch.float32, pin_memory=True)
    xh.copy_(x.cpu())
    lh = torch.empty(B, 10, dtype=torch.float32, pin_memory=True)

    def host_loop(pipelined: bool) -> float:
        for _ in range(2):
            eng.forward_host_ptr(xh.data_ptr(), B, 3, 32, 32, lh.data_ptr())
            eng.forward_async(xh.data_ptr(), B, lh.data_ptr())
        eng.sync()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for _ in range(a.steps):
            if pipelined:
                eng.forward_async(xh.data_ptr(), B, lh.data_ptr())
            else:
                eng.forward_host_ptr(xh.data_ptr(), B, 3, 32, 32, lh.data_ptr())
        eng.sync()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1), "cuda")

    ems = host_loop(True)
    ems_sync = host_loop(False)
    e2e = {"value": world * B * a.steps / (ems / 1e3), "unit": "images/s",
           "h2d_bytes_per_step": B * 3 * 32 * 32 * 4, "d2h_bytes_per_step": B * 10 * 4,
           "call": "ptq8_engine_forward_async (pinned host buffers; step k+1's H2D overlaps step k's forward)",
           "sync_call_value": world * B * a.steps / (ems_sync / 1e3)}

    if rank == 0:
        line = {"metric": info["metric"], "value": value, "unit": "images/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic",
                "config": {"workload": f"{info['name']}_b{B} (BASELINE configs[{a.config}])", "batch_per_gpu": B,
                           "parallelism": f"dp{world}", "l2": "inputs and activations larger than L2 (>10 GB/step)",
                           "logits_gather": "nccl all_gather per step" if world > 1 else "none"},
                "roofline": roofline, "e2e": e2e, "clocks": clk,
                "gpu_launches": a.steps * eng.n_launches()}
        if not a.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(paths, a.cpu_sample)
        print(json.dumps(line), flush=True)
    del eng
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
