"""The reference arm of bench.py (`--impl reference`) on CPU: one JSON line with the
contract's keys, the same metric, unit and config as the CUDA arm, and an e2e object
without host-device traffic (it runs the oracle port on the host cores). Each timed step
is one pair over the full parameter set, so the timed region is steps x ms_per_step."""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_reference_arm_prints_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["unit"] == "ZO steps/s" and line["value"] > 0
    assert line["config"]["params"] == 1235814400 and line["config"]["tensors"] == 146
    assert line["config"]["seeds_per_step"] == 64
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"] == bench.workload_config(1, 64, 1235814400, 146)    # the CUDA arm's config
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert abs(line["timed_region_s"] - line["steps"] * line["ms_per_step"] / 1000) < 0.5 * line["timed_region_s"]
    assert line["full_step_s"] > 64 * line["ms_per_step"] / 1000
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
