"""CPU: the parts of bench.py that need no GPU.

* algorithmic_bytes, the numerator of the roofline, against its closed
  form: per token step t in [t0, T) the layer weights (and RMSNorm scales),
  the tied lm_head on steps that produce logits (t >= P - 1), and per
  sequence the K and V rows 0..t of every layer plus one embedding row.
  The bench workload's figure (prefill of 127 positions, then 256 steps) is
  pinned to the number the B200 runs report.
* whole_job_rate: tokens of every rank over the slowest rank's time.
* the reference arm's JSON line (the reference's own generate() on the host
  cores) carries the keys and units of the native arm's line, and a rank
  other than 0 exits 0 without work.
"""
import json
import os
import subprocess
import sys

import pytest

import bench
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def closed_form_bytes(P, nnew, B, t0):
    V, D, L, H, F = (bench.WL[k] for k in ("vocab", "dim", "n_layers", "n_heads", "ffn_dim"))
    K = O.kv_head_count(H)
    kvd = K * (D // H)
    Q = D + 2 * kvd
    T = P + nnew - 1
    steps = T - t0
    w_layers = L * (Q * D + D * D + 3 * F * D) * 4 + 2 * L * D * 4
    w_head = V * D * 4 + D * 4
    heads = max(0, T - max(t0, P - 1))
    # sum over t of (t + 1) for t0 <= t < T
    pos_sum = (T * (T + 1) - t0 * (t0 + 1)) // 2
    return steps * w_layers + heads * w_head + B * (L * 2 * kvd * 4 * pos_sum + steps * D * 4)


@pytest.mark.parametrize("P,nnew,B,t0", [(128, 256, 4, 127), (128, 256, 4, 0), (5, 3, 2, 0),
                                         (10, 1, 1, 4), (64, 64, 8, 63)])
def test_algorithmic_bytes_closed_form(P, nnew, B, t0):
    assert bench.algorithmic_bytes(P, nnew, B, t0=t0) == closed_form_bytes(P, nnew, B, t0)


def test_algorithmic_bytes_of_the_bench_workload():
    # 256 token steps of the default 5.8M model for 4 sequences after a
    # 127-position prefill: 7.87 MB of layer weights and 15.36 MB of lm_head
    # per step plus 1.07 GB of K/V rows over the launch
    assert bench.algorithmic_bytes(128, 256, 4, t0=127) == 7_019_823_104


def test_whole_job_rate_is_all_ranks_over_the_slowest():
    assert bench.whole_job_rate(4, 1024, 0.5) == pytest.approx(8192.0)
    assert bench.whole_job_rate(1, 1024, 0.5) == pytest.approx(2048.0)


def _run_reference_arm(env_extra):
    env = dict(os.environ)
    env.update(env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=300)


@pytest.mark.skipif(not (O.ref_available() or os.path.exists(O.ORC_LIB)),
                    reason="neither oracle/_ref nor the oracle library is built here")
def test_reference_arm_json_line():
    r = _run_reference_arm({})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["higher_is_better"] is True and d["scaling"] == "weak" and d["vs_baseline"] is None
    assert d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"] == bench.workload_config(1)
    cb = d["cpu_baseline"]
    assert cb["kind"] == ("reference" if O.ref_available() else "port")
    assert cb["cores"] >= 1 and cb["value"] == d["value"] and cb["unit"] == bench.UNIT
    assert d["e2e"] == {"value": d["value"], "unit": bench.UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_no_work():
    r = _run_reference_arm({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


_MAPS_PROBE = r"""
import argparse, sys
sys.path.insert(0, sys.argv[1])
import bench
bench.reference_arm(argparse.Namespace(gpus=1, steps=1, warmup=0))
with open("/proc/self/maps") as fh:
    libs = sorted({l.split()[-1] for l in fh if ".so" in l})
print("LIBS", " ".join(libs))
"""


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")
def test_reference_arm_loads_only_oracle_libraries():
    """The reference arm's process maps the reference build (oracle/_ref) and
    none of this repository's product libraries, so every function the
    reference calls is its own."""
    r = subprocess.run([sys.executable, "-c", _MAPS_PROBE, ROOT], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    libs = [l for l in r.stdout.splitlines() if l.startswith("LIBS ")][0].split()[1:]
    ours = [l for l in libs if l.startswith(ROOT)]
    assert any(l.endswith("oracle/_ref/libminima_ref.so") for l in ours)
    assert not [l for l in ours if "/minima_b200/" in l], ours
