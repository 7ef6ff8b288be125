"""CPU check of bench.py's reference arm: the line a driver reads.

`bench.py --impl reference` times the reference's CPU path (the oracle's
restatement of predict_mask, read_neurons + dequantisation and sparse_ffn,
engine.py:173-209, splitter.py:354-403) on the host cores; its JSON line must
carry the same metric, unit and workload as the GPU arm, say what a step was
(one token through the sampled layers) and declare no host-device copies.
"""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    import bench
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["config"]["workload"] == bench.WORKLOAD
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 0
    # a step is one token through the sampled layers; tokens/s scales its per-layer time to all layers
    per_layer_s = line["ms_per_step"] / 1e3 / line["config"]["timed_layers_per_step"]
    assert abs(line["value"] - 1.0 / (per_layer_s * bench.LAYERS)) <= 1e-6 * line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
