"""The benchmark's reference arm (the CPU oracle port, runnable without a GPU)
prints one JSON line with the fields the driver contract requires, on the
same metric as the native arm."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(*args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_json_line():
    j = _run("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "3")
    assert j["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in j, key
    assert j["metric"].startswith("causal bf16 FlashAttn fwd+bwd TFLOP/s")
    assert j["unit"].startswith("TFLOP/s") and j["higher_is_better"] is True
    assert j["value"] > 0 and j["n_gpus"] == 1 and j["steps"] == 1 and j["warmup"] >= 3
    assert j["config"]["workload"].startswith("c1:")
    cb = j["cpu_baseline"]
    assert cb["value"] == j["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["sample"]
    e2e = j["e2e"]
    assert e2e["value"] == j["value"] and e2e["unit"] == j["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_both_arms_share_the_config_object():
    """The reference arm prints the same `config` object as the GPU arm for the
    same workload and split (bench.arm_config builds both)."""
    sys.path.insert(0, str(ROOT))
    import bench
    j = _run("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "3")
    assert j["config"] == bench.arm_config("c1", 1, "weak")
    assert j["unit"] == bench.UNIT
    strong = bench.arm_config("c4", 8, "strong")
    assert strong["parallelism"].startswith("(batch x head) shards, 16 on rank 0 of 128")
    assert strong["global_batch"] == 4
