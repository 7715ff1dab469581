"""CPU, world_size 2 over gloo: the data-parallel plumbing of bench.py.

Sequences are independent, so N GPUs decode disjoint shards with no
collective on the data path; the only communication is the barrier around
the timed region and the MAX of per-rank times.  Covered here without a GPU:
  * each rank's shard is disjoint and equals the single-process definition
    of those global sequence indices;
  * the timing reduction takes the slowest rank;
  * a rank that dies between steps makes the survivor's next collective fail
    (short process-group timeout) instead of hanging.
"""
import datetime
import json
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, outdir, scenario):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    res = {"rank": rank}
    try:
        if scenario == "shard":
            prompts, rng = bench.workload_prompts(rank * bench.WL["batch"], bench.WL["batch"])
            res["prompts"] = prompts.tolist()
            res["rng"] = rng
            t = bench.max_over_ranks(dist, [10.0 + rank, 3.0 - rank], "cpu")
            res["max"] = t
            res["rate"] = bench.whole_job_rate(world, 1024, t[0] / 1e3)
            dist.barrier()
        elif scenario == "dead_rank":
            dist.barrier()                      # both ranks finish step 1
            if rank == 1:
                os._exit(0)                     # leaves between steps, nothing in flight
            try:
                dist.barrier()
                res["error"] = None
            except Exception as e:              # noqa: BLE001
                res["error"] = type(e).__name__
    finally:
        with open(os.path.join(outdir, f"r{rank}.json"), "w") as fh:
            json.dump(res, fh)
    if scenario != "dead_rank":
        dist.destroy_process_group()


def _run(world, scenario, tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), scenario))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("worker hung")
    out = {}
    for r in range(world):
        path = tmp_path / f"r{r}.json"
        if path.exists():
            out[r] = json.loads(path.read_text())
    return out


def test_shards_are_disjoint_and_timing_takes_the_slowest_rank(tmp_path):
    import bench
    out = _run(2, "shard", tmp_path)
    assert set(out) == {0, 1}
    p0, p1 = np.array(out[0]["prompts"]), np.array(out[1]["prompts"])
    assert p0.shape == p1.shape == (bench.WL["batch"], bench.WL["prompt"])
    assert not any((p0[i] == p1[j]).all() for i in range(len(p0)) for j in range(len(p1)))
    assert out[0]["rng"] == [1, 2, 3, 4] and out[1]["rng"] == [5, 6, 7, 8]
    # global sequence g = rank * B + b uses prompt seed 1000 + g, as a single process would
    for rank, p in ((0, p0), (1, p1)):
        for b in range(len(p)):
            g = rank * bench.WL["batch"] + b
            assert (bench.prompt_ids(bench.WL["prompt"], bench.WL["vocab"], 1000 + g) == p[b]).all()
    assert out[0]["max"] == out[1]["max"] == [11.0, 3.0]
    assert out[0]["rate"] == pytest.approx(2 * 1024 / 0.011)


def test_dead_rank_fails_the_next_collective(tmp_path):
    out = _run(2, "dead_rank", tmp_path)
    assert out[0]["error"] is not None
