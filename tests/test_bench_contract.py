"""CPU check of bench.py's JSON line for its host-only workload (the GPU
workloads are exercised on a B200)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "e2e"}


def run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_tokenizer_bench_line(built_lib):
    d = run("--workload", "tokenizer", "--steps", "3", "--warmup", "3")
    assert KEYS <= set(d), KEYS - set(d)
    assert d["metric"] == "tokenizer_encode_mb_per_sec" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] > 0
    assert d["e2e"]["value"] > 0 and d["gpu_launches"] == 0
    r = run("--workload", "tokenizer", "--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r["impl"] == "reference" and r["metric"] == d["metric"] and r["unit"] == d["unit"]
    assert r["e2e"]["h2d_bytes_per_step"] == 0
