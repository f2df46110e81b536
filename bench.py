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
    return {"metric": METRIC_MV2 if mv2 else METRIC, "batch": c["batch"], "passes": 7 if c.get("passes") else 0,
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
    ap.add_argument("--cpu-sample", type=int, default=6,
                    help="images in the timed CPU-baseline sample (about 8 s per run at the reference's rate)")
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


def gather_logits(gathered, local):
    """The multi-GPU step's one collective: every rank's fp32 logits [B, 10], concatenated
    in rank order into `gathered` [world * B, 10] on every rank."""
    import torch.distributed as dist
    dist.all_gather_into_tensor(gathered, local)


def all_ranks(x: float, device) -> list:
    """x of every rank, in rank order ([x] without a process group)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [x]
    t = torch.tensor([x], dtype=torch.float64, device=device)
    out = torch.empty(dist.get_world_size(), dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t)
    return [float(v) for v in out.cpu()]


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

    def stop(self, windows) -> dict:
        """Summary of the samples taken inside the timed windows [(t0, t1), ...]."""
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
        inside = [r for r in rows if any(t0 <= self._ts(r[0]) <= t1 for t0, t1 in windows)]
        if not inside:
            t0, t1 = windows[0]
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
            "sample": f"{n_img} images of the same workload, numpy int32 matmul with the reference's weight layout "
                      f"(06-gpu-int8/cpp/ref_e2e.py:180,213-218; times within 1% of ref_e2e.forward, "
                      f"profiles/cpu_baseline_port_vs_ref_e2e.md), median of {runs} runs "
                      f"({', '.join(f'{t:.2f}' for t in dts)} s) after a warm-up",
            **host_cpu()}


_REF_ORACLE = None


def _ref_init(model, calib, plan):
    """Pool initializer: each worker process loads the model and quantizes its weights once
    (the reference's forward does this before its timed loop, ref_e2e.py:210-219)."""
    global _REF_ORACLE
    from oracle import ptq8_oracle as O
    from ptq_int8_lab_b200 import modelgen as mg
    O.MATMUL_MODE["mode"] = "int32"
    _REF_ORACLE = O.Oracle(O.read_model(model), O.read_ptqc(calib), layer_bits=mg.read_layer_plan(plan))


def _ref_worker(args):
    n_img, seed = args
    import numpy as np
    x = np.random.default_rng(seed).standard_normal((n_img, 3, 32, 32)).astype(np.float32)
    t0 = time.perf_counter()
    _REF_ORACLE.forward(x, trace=False)
    return time.perf_counter() - t0


def run_reference(a):
    """Reference arm: the reference's CPU integer forward (the bit-pinned port, with the
    reference's GEMM layout and speed) on all host cores, a bounded sample per step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import multiprocessing as mp
    info = config_info(a.config)
    paths = model_files(a.model_cache, 0, 1, lambda: None, a.config)
    cores = os.cpu_count() or 1
    per = 1
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores, initializer=_ref_init, initargs=(paths["model"], paths["calib"], paths["plan"])) as pool:
        for w in range(max(a.warmup, 1)):
            pool.map(_ref_worker, [(1, 7 + 1000 * w + i) for i in range(cores)])
        times = []
        for s in range(a.steps):
            t0 = time.perf_counter()
            pool.map(_ref_worker, [(per, 100 * s + i) for i in range(cores)])
            times.append(time.perf_counter() - t0)
    imgs = per * cores * a.steps
    tot = sum(times)
    v = imgs / tot
    line = {"impl": "reference", "metric": info["metric"], "value": v, "unit": "images/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tot / a.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{info['name']} (BASELINE configs[{a.config}] shapes)", "batch_per_step": per * cores,
                       "note": "bounded sample per step on host cores; the CPU arm cannot run the GPU batch"},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"{per} image per process x {cores} spawn processes per step, model loaded "
                                       f"once per process; numpy int32 matmul with the reference's weight layout "
                                       f"(ref_e2e.py:180,213-218), timed within 1% of ref_e2e.forward "
                                       f"(profiles/cpu_baseline_port_vs_ref_e2e.md)", **host_cpu()},
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
    eng.forward_device(x.data_ptr(), B, logits.data_ptr())   # stage the input in the engine buffer

    # N > 1: step k's logits go to buffer k % 2 on the engine stream; the all-gather runs on a
    # side stream once they are there, so the next forward does not wait for the collective.
    # The engine stream only waits for the gather two steps back (it read the same buffer).
    comm = torch.cuda.Stream() if world > 1 else None
    lbuf = [torch.empty(B, 10, device="cuda", dtype=torch.float32) for _ in range(2)]
    gbuf = [torch.empty(world * B, 10, device="cuda", dtype=torch.float32) for _ in range(2)] if world > 1 else None
    ev_ready = [torch.cuda.Event() for _ in range(2)]
    ev_read = [torch.cuda.Event() for _ in range(2)]

    def step(k: int):
        eng.run(B)
        if world > 1:
            i = k & 1
            stream.wait_event(ev_read[i])
            eng.copy_logits(B, lbuf[i].data_ptr())
            ev_ready[i].record(stream)
            with torch.cuda.stream(comm):
                comm.wait_event(ev_ready[i])
                gather_logits(gbuf[i], lbuf[i])
                ev_read[i].record(comm)

    clocks = ClockSampler(local)
    clocks.start()
    for k in range(a.warmup):
        step(k)
    torch.cuda.synchronize()
    eng.sync()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev_fwd = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    for k in range(a.steps):
        step(k)
    ev_fwd.record(stream)          # this rank's forwards (and logits copies) are done
    if comm is not None:
        stream.wait_stream(comm)   # ... and every gather
    ev1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms_local = ev0.elapsed_time(ev1)
    fwd_ms_by_rank = [v / a.steps for v in all_ranks(ev0.elapsed_time(ev_fwd), "cuda")]
    eng.sync()
    ms = max_over_ranks(ms_local, "cuda")
    ms_per_step = ms / a.steps
    value = world * B * a.steps / (ms / 1e3)
    multi = None
    if world > 1:
        # the gather's own device time (comm stream, after the timed region), max over ranks
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        g0.record(comm)
        for _ in range(10):
            with torch.cuda.stream(comm):
                gather_logits(gbuf[0], lbuf[0])
        g1.record(comm)
        torch.cuda.synchronize()
        multi = {"gather_ms": max_over_ranks(g0.elapsed_time(g1) / 10, "cuda"),
                 "gather_bytes_per_rank": B * 10 * 4,
                 "forward_ms_per_step_by_rank": fwd_ms_by_rank,
                 "rank_spread_ms_per_step": max(fwd_ms_by_rank) - min(fwd_ms_by_rank),
                 "gather": "NCCL all_gather of fp32 logits on a side stream, double-buffered; "
                           "the timed region ends after the last gather"}

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
    # Second denominator: the kind::i8 MMA issue rate measured on this pool (N >= 128 shapes:
    # 8192 MAC per clock per SM) at the median SM clock of the timed region.
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                "frac": achieved / int8_peak, "traffic": traffic,
                "kernel": "conv_tc_kernel (all dense convs of one forward)",
                "peak_source": f"2 x bf16_tflops of {src} MEASURED_PEAKS.json",
                "dense_conv_ms": tc_ms, "forward_ms_sum_of_launches": sum(p["ms"] for p in prof),
                "per_launch": [{"step": p["step"], "kind": "stem" if p["kind"] == 0 else "conv",
                                "ms": p["ms"], "tops": 2.0 * p["macs"] / (p["ms"] / 1e3) / 1e12,
                                "frac": 2.0 * p["macs"] / (p["ms"] / 1e3) / 1e12 / int8_peak}
                               for p in tc if p["ms"] > 0]}
    # memory-bound launches (depthwise convs, maxpool, pooling head): algorithmic bytes (codes
    # read once, codes / fp32 written once, weights once) over their device time, against the
    # measured HBM copy bandwidth
    memk = [p for p in prof if p["kind"] in (2, 3, 4) and p["ms"] > 0]
    roofline_hbm = None
    if memk:
        m_ms = sum(p["ms"] for p in memk)
        m_gbs = sum(p["bytes"] for p in memk) / (m_ms / 1e3) / 1e9
        names = {2: "depthwise", 3: "maxpool", 4: "head"}
        roofline_hbm = {"bound": "hbm", "achieved": m_gbs, "peak": hbm, "unit": "GB/s", "frac": m_gbs / hbm,
                        "kernel": "dw3x3_kernel / dw_conv_kernel (depthwise), maxpool_kernel, head_kernel",
                        "peak_source": f"hbm_gbs of {src} MEASURED_PEAKS.json", "ms": m_ms,
                        "per_launch": [{"step": p["step"], "kind": names[p["kind"]], "ms": p["ms"],
                                        "gbs": p["bytes"] / (p["ms"] / 1e3) / 1e9,
                                        "frac": p["bytes"] / (p["ms"] / 1e3) / 1e9 / hbm} for p in memk]}
    wb = eng.weight_bytes()

    # ---- end to end through the C-ABI host-buffer forwards (H2D + graph + D2H every step).
    # Headline: ptq8_engine_forward_async, the pipelined call (step k+1's H2D overlaps step
    # k's forward, two input slots); also the synchronous ptq8_engine_forward (the
    # reference's Int8Engine::forward semantics: copy, run, copy back, wait).
    xh = torch.empty(B, 3, 32, 32, dtype=torch.float32, pin_memory=True)
    xh.copy_(x.cpu())
    lh = torch.empty(B, 10, dtype=torch.float32, pin_memory=True)

    windows = [(t_wall0, t_wall1)]   # host-time windows of the timed regions (clock samples)

    # 8-bit pixels (CIFAR-10 record format without the label byte): decode + normalise +
    # quantize run in the stem kernel, 1 byte per input value over PCIe instead of 4
    ph = torch.from_numpy(np.random.default_rng(1234 + rank).integers(0, 256, size=(B, 3, 32, 32),
                                                                        dtype=np.uint8)).pin_memory()

    def call(mode: str):
        if mode == "async":
            eng.forward_async(xh.data_ptr(), B, lh.data_ptr())
        elif mode == "u8":
            eng.forward_u8_async(ph.data_ptr(), B, 0, lh.data_ptr())
        else:
            eng.forward_host_ptr(xh.data_ptr(), B, 3, 32, 32, lh.data_ptr())

    def host_loop(mode: str) -> float:
        # warm-up: the pipelined calls alternate between two input slots, each with its own
        # CUDA graph, so both graphs are captured here and not inside the timed loop
        for _ in range(4):
            call(mode)
        eng.sync()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        w0 = time.time()
        e0.record(stream)
        for _ in range(a.steps):
            call(mode)
        eng.sync()
        e1.record(stream)
        torch.cuda.synchronize()
        windows.append((w0, time.time()))
        return max_over_ranks(e0.elapsed_time(e1), "cuda")

    ems = host_loop("async")
    ems_sync = host_loop("sync")
    ems_u8 = host_loop("u8")
    clk = clocks.stop(windows)
    clk["windows"] = "the device-timed loop and the three e2e loops"
    roofline["peak_i8_issue_rate"] = (8192 * sms * clk["sm_mhz"] * 1e6 * 2 / 1e12) if clk.get("sm_mhz") else None
    if roofline["peak_i8_issue_rate"]:
        roofline["frac_of_i8_issue_rate"] = achieved / roofline["peak_i8_issue_rate"]
    e2e = {"value": world * B * a.steps / (ems / 1e3), "unit": "images/s",
           "h2d_bytes_per_step": B * 3 * 32 * 32 * 4, "d2h_bytes_per_step": B * 10 * 4,
           "call": "ptq8_engine_forward_async (pinned host buffers; step k+1's H2D overlaps step k's forward)",
           "sync_call_value": world * B * a.steps / (ems_sync / 1e3),
           "u8_input": {"value": world * B * a.steps / (ems_u8 / 1e3), "h2d_bytes_per_step": B * 3 * 32 * 32,
                        "call": "ptq8_engine_forward_u8_async (8-bit CIFAR-10 pixels; normalisation and "
                                "quantization in the stem kernel)"}}

    if rank == 0:
        line = {"metric": info["metric"], "value": value, "unit": "images/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic",
                "config": {"workload": f"{info['name']}_b{B} (BASELINE configs[{a.config}])", "batch_per_gpu": B,
                           "parallelism": f"dp{world}", "l2": "inputs and activations larger than L2 (>10 GB/step)",
                           "logits_gather": "nccl all_gather per step (side stream)" if world > 1 else "none"},
                "roofline": roofline, "roofline_hbm": roofline_hbm, "e2e": e2e, "clocks": clk, "weights": wb,
                "gpu_launches": a.steps * eng.n_launches()}
        if multi is not None:
            line["multi_gpu"] = multi
        if not a.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(paths, a.cpu_sample)
        print(json.dumps(line), flush=True)
    del eng
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
