"""bench.py's reference arm (`--impl reference`) on the CPU: the JSON line the driver reads, on the same
`config` and metric as the GPU arm, with the cpu_baseline and e2e objects; non-zero ranks print nothing;
the 48-layer model workloads say why they are not sampled."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _run(*extra, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--cpu-budget", "0.5", *extra], cwd=ROOT, env=e, capture_output=True,
                       text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    return [json.loads(l) for l in lines]


@pytest.mark.parametrize("workload,metric", [("decode8", "MoE-layer tok/s (decode8)"),
                                             ("layer_decode1", "decoder-layer tok/s (layer_decode1)")])
def test_reference_arm_line(workload, metric):
    import bench
    (out,) = _run("--workload", workload)
    assert out["impl"] == "reference" and out["metric"] == metric and out["unit"] == "tok/s"
    assert out["value"] > 0 and out["higher_is_better"] is True and out["vs_baseline"] is None
    assert out["n_gpus"] == 1 and out["steps"] == 1 and out["warmup"] == 0 and out["scaling"] == "weak"
    assert out["config"] == bench.workload_config(workload)   # the GPU arm reports this same object
    T = bench.WORKLOADS[workload][0]
    assert out["ms_per_step"] == pytest.approx(T / out["value"] * 1e3)
    cb = out["cpu_baseline"]
    assert cb["value"] == out["value"] and cb["unit"] == "tok/s" and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference") and cb["sample"]
    assert out["e2e"] == {"value": out["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert _run(env={"RANK": "1", "WORLD_SIZE": "2"}) == []


def test_reference_arm_model_workload_is_declared_unavailable():
    (out,) = _run("--workload", "model48_decode8")
    assert out["impl"] == "reference" and "unavailable" in out
