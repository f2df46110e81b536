"""Host-side logic of bench.py that needs no GPU: the workload of each BASELINE config,
the host CPU record, and the CPU-baseline record (the reference's integer forward on
the host cores, timed with the reference's protocol: warm-up, then the median of 3 runs)."""
import bench
from ptq_int8_lab_b200 import modelgen as mg


def test_config_info_matches_configs():
    for cfg, c in mg.CONFIGS.items():
        info = bench.config_info(cfg)
        assert info["batch"] == c["batch"]
        if c["model"] == "mobilenet_v2":
            assert info["metric"] == bench.METRIC_MV2 and info["name"].startswith("mobilenet_v2")
        else:
            assert info["metric"] == bench.METRIC and info["name"].startswith("resnet18_" + c["stem"])
        assert ("mixed" in info["name"]) == bool(c.get("mixed"))
        assert info["passes"] == (7 if c.get("passes") else 0)
    assert bench.config_info(4)["batch"] == 8192   # the headline workload


def test_host_cpu_record():
    h = bench.host_cpu()
    assert set(h) == {"cpu_model", "nproc"}
    assert isinstance(h["cpu_model"], str) and h["cpu_model"]
    assert h["nproc"] >= 1


def test_cpu_baseline_record(make_model):
    r = bench.cpu_baseline(make_model(0), 1, runs=3)
    assert r["value"] > 0 and r["unit"] == "images/s"
    assert r["cores"] == 1 and r["kind"] == "port"
    assert "median of 3 runs" in r["sample"]
    assert r["nproc"] >= 1 and r["cpu_model"]
