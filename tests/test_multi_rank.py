"""bench.py's multi-process host logic, world_size 2 on the gloo backend (CPU).

The GPU bench runs one process per GPU (torchrun): rank 0 writes the calibrated model
files while the other ranks wait at a barrier, every rank then opens the same files,
and the timed figures are the maximum over ranks.  This checks that orchestration
without a GPU.
"""
import json
import os
import socket
from datetime import timedelta

import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, cache: str, out: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    import bench
    r, w, local = bench.dist_env()
    paths = bench.model_files(cache, r, w, dist.barrier, cfg=0)
    import torch
    B = 5
    local_logits = torch.arange(B * 10, dtype=torch.float32).reshape(B, 10) + 1000.0 * r
    gathered = torch.empty(w * B, 10, dtype=torch.float32)
    bench.gather_logits(gathered, local_logits)
    res = {"env": [r, w, local], "paths": paths, "sizes": {k: os.path.getsize(v) for k, v in paths.items()},
           "max_ms": bench.max_over_ranks(10.0 * (r + 1), "cpu"),
           "all_ms": bench.all_ranks(1.5 + r, "cpu"),
           "gathered": gathered.tolist()}
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def test_two_ranks_share_model_files_and_max_time(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path / "cache"), str(tmp_path)), nprocs=world, join=True)
    r = [json.loads((tmp_path / f"rank{i}.json").read_text()) for i in range(world)]
    assert [x["env"] for x in r] == [[0, 2, 0], [1, 2, 1]]
    assert r[0]["paths"] == r[1]["paths"]
    assert all(v > 0 for v in r[0]["sizes"].values()) and r[0]["sizes"] == r[1]["sizes"]
    assert r[0]["max_ms"] == r[1]["max_ms"] == 20.0
    assert r[0]["all_ms"] == r[1]["all_ms"] == [1.5, 2.5]
    # every rank holds every rank's logits, in rank order
    import numpy as np
    want = np.concatenate([np.arange(50, dtype=np.float32).reshape(5, 10) + 1000.0 * k for k in range(world)])
    for x in r:
        assert np.array_equal(np.asarray(x["gathered"], dtype=np.float32), want)


def test_single_process_max_is_identity():
    import bench
    assert bench.max_over_ranks(3.5, "cpu") == 3.5
