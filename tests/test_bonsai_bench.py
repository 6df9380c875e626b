"""The drop-in bench entry point (nnzap_b200/bonsai_bench.py) against the
reference's bench protocol and schema (nnmetal/examples/bonsai_bench.zig) and
the way labrat reads it (labrat/src/toolbox.zig:580-720)."""
import datetime
import json

import pytest

from nnzap_b200 import bonsai_bench as B

REF_KEYS = ["timestamp_utc", "model", "prompt_tokens", "warmup_tokens", "measured_tokens", "load_ms",
            "prefill_tok_per_sec", "decode_tok_per_sec", "decode_p50_us", "decode_p99_us", "power_source"]


def test_compute_results_protocol():
    # 8 warm-up timings (huge: must be skipped) + 64 measured ones of 1000..1063 us
    t = [10**9] * 8 + [(1000 + i) * 1000 for i in range(64)]
    r = B.compute_results(2_000_000, 4_000_000, 20, t, 8, 64)
    assert r["decode_p50_us"] == 1032 and r["decode_p99_us"] == 1063     # sorted[n/2], sorted[n*99/100]
    assert r["decode_tok_per_sec"] == pytest.approx(64 / (sum(range(1000, 1064)) * 1e-6))
    assert r["prefill_tok_per_sec"] == pytest.approx(20 / 4e-3)
    assert r["load_ms"] == pytest.approx(2.0) and r["measured_tokens"] == 64


def test_schema_and_labrat_extraction():
    r = B.compute_results(1_500_000_000, 7_000_000, 512, [800_000] * 72, 8, 64)
    text = B.format_json(r, 512, 8, when=datetime.datetime(2026, 1, 2, 3, 4, 5, tzinfo=datetime.timezone.utc))
    d = json.loads(text)
    assert list(d) == REF_KEYS
    assert d["timestamp_utc"] == "2026-01-02T03:04:05Z" and d["model"] == "Bonsai-1.7B"
    assert d["power_source"] in ("ac", "battery", "unknown")
    # labrat's scanner finds the three keys it consumes
    assert B.extract_json_float(text, "decode_tok_per_sec") == pytest.approx(1250.0)
    assert B.extract_json_float(text, "prefill_tok_per_sec") == pytest.approx(512 / 7e-3, rel=1e-4)
    assert B.extract_json_float(text, "decode_p99_us") == 800.0
    assert B.extract_json_float(text, "missing_key") is None
    # ... and in bench.py's one-line form too
    line = json.dumps({"metric": "decode_tok_per_sec", "decode_tok_per_sec": 1234.5, "decode_p99_us": 810.0})
    assert B.extract_json_float(line, "decode_tok_per_sec") == 1234.5


@pytest.mark.gpu
def test_bench_entry_point_runs(cuda, built_lib):
    """One run of the entry point on a small random-init Q1 model."""
    from nnzap_b200 import synth
    d = synth.ModelDims(vocab=1000, hidden=256, inter=768, layers=2, n_q=4, n_kv=2, head_dim=128, gs=128,
                        quant="q1")
    text = B.run(None, 24, dims=d)
    out = json.loads(text)
    assert list(out) == REF_KEYS
    assert out["measured_tokens"] == 64 and out["warmup_tokens"] == 8 and out["prompt_tokens"] == 24
    for k in ("decode_tok_per_sec", "prefill_tok_per_sec", "decode_p99_us"):
        assert B.extract_json_float(text, k) > 0
