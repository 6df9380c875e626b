"""Drop-in for the reference's Bonsai benchmark binary
(nnmetal/examples/bonsai_bench.zig): same protocol, same JSON keys, so the
labrat agent loop (labrat/src/toolbox.zig:580-720, which reads
``decode_tok_per_sec``, ``prefill_tok_per_sec`` and ``decode_p99_us`` from it)
can run this engine unchanged.

Protocol (bonsai_bench.zig:27-29, 255-320): one generate() call of
8 warm-up + 64 measured greedy tokens after the prompt's prefill; the first 8
per-token timings are skipped; decode tok/s = 64 / (sum of the measured
per-token times); p50 = sorted[n / 2], p99 = sorted[n * 99 / 100], in whole
microseconds; prefill tok/s = prompt tokens / prefill time; load_ms = the
weight load.

    python -m nnzap_b200.bonsai_bench [--model-dir DIR] [--prompt-tokens N]

With ``--model-dir`` (safetensors shards + tokenizer.json of an MLX Q1
Bonsai-1.7B checkpoint) the prompt is the reference's bench prompt through
the Qwen3 chat template, as in the reference.  Without it the model is the
Bonsai-1.7B architecture with seeded random 1-bit weights and the prompt is
``--prompt-tokens`` seeded random ids (no checkpoint or tokenizer exists on
this machine).
"""
from __future__ import annotations

import argparse
import datetime
import json
import sys
import time
from pathlib import Path

import numpy as np

BENCH_PROMPT = "Explain the theory of general relativity in detail."
WARMUP_TOKENS = 8
MEASURE_TOKENS = 64


def compute_results(load_ns: int, prefill_ns: int, prompt_len: int, timings_ns, warmup: int, measure: int) -> dict:
    """computeResults (bonsai_bench.zig:255-320)."""
    assert prompt_len > 0 and measure > 0 and warmup + measure <= len(timings_ns)
    load_ms = load_ns / 1e6
    prefill_ms = prefill_ns / 1e6
    prefill_tps = prompt_len / (prefill_ms / 1000.0) if prefill_ms > 0 else 0.0
    meas = sorted(int(t) for t in timings_ns[warmup:warmup + measure])
    decode_ms = sum(meas) / 1e6
    decode_tps = measure / (decode_ms / 1000.0) if decode_ms > 0 else 0.0
    return {"load_ms": load_ms, "prefill_tok_per_sec": prefill_tps, "decode_tok_per_sec": decode_tps,
            "decode_p50_us": meas[measure // 2] // 1000, "decode_p99_us": meas[(measure * 99) // 100] // 1000,
            "measured_tokens": measure}


def format_json(r: dict, prompt_len: int, warmup: int, when: datetime.datetime | None = None,
                power_source: str = "unknown") -> str:
    """The reference's JSON block (bonsai_bench.zig:370-392), key for key.
    power_source: the reference asks macOS pmset (AC / battery) and reports
    "unknown" when that fails, as it does on this Linux host."""
    when = when or datetime.datetime.now(datetime.timezone.utc)
    ts = when.strftime("%Y-%m-%dT%H:%M:%SZ")
    return ("{\n"
            f'  "timestamp_utc": "{ts}",\n'
            '  "model": "Bonsai-1.7B",\n'
            f'  "prompt_tokens": {prompt_len},\n'
            f'  "warmup_tokens": {warmup},\n'
            f'  "measured_tokens": {r["measured_tokens"]},\n'
            f'  "load_ms": {r["load_ms"]:.1f},\n'
            f'  "prefill_tok_per_sec": {r["prefill_tok_per_sec"]:.1f},\n'
            f'  "decode_tok_per_sec": {r["decode_tok_per_sec"]:.1f},\n'
            f'  "decode_p50_us": {r["decode_p50_us"]},\n'
            f'  "decode_p99_us": {r["decode_p99_us"]},\n'
            f'  "power_source": "{power_source}"\n'
            "}\n")


def extract_json_float(text: str, key: str):
    """labrat's extractJsonFloat (labrat/src/toolbox.zig:580-630): the number
    after '"key":' scanned without a JSON parser, or None."""
    i = 0
    while i + len(key) + 3 < len(text):
        if text[i] != '"':
            i += 1
            continue
        ks, ke = i + 1, i + 1 + len(key)
        if ke >= len(text):
            break
        if text[ks:ke] != key or text[ke] != '"':
            i += 1
            continue
        c = ke + 1
        while c < len(text) and text[c] == " ":
            c += 1
        if c >= len(text) or text[c] != ":":
            i += 1
            continue
        c += 1
        while c < len(text) and text[c] in " \t":
            c += 1
        if c >= len(text):
            return None
        s = c
        while c < len(text) and (text[c].isdigit() or text[c] in ".-eE+"):
            c += 1
        try:
            return float(text[s:c])
        except ValueError:
            return None
    return None


def run(model_dir: str | None, prompt_tokens: int, seed: int = 0, dims=None, max_context: int | None = None) -> str:
    from . import GenerateOpts, Model, config_from_dims, generate, synth
    d = dims or synth.BONSAI_1_7B_Q1
    t0 = time.perf_counter_ns()
    if model_dir:
        from .tokenizer import Tokenizer
        shards = sorted(Path(model_dir).glob("*.safetensors"))
        if not shards:
            raise SystemExit(f"no .safetensors shards in {model_dir}")
        tok = Tokenizer.from_file(Path(model_dir) / "tokenizer.json")
        prompt = tok.apply_chat_template(BENCH_PROMPT)
        ctx = max_context or max(1024, len(prompt) + WARMUP_TOKENS + MEASURE_TOKENS + 1)
        cfg = config_from_dims(d, max_context_length=ctx, max_batch=1).replace(q1_scales_are_mlx=True)
        model = Model(cfg)
        model.load_safetensors([str(p) for p in shards])
    else:
        prompt = np.random.default_rng(seed).integers(0, d.vocab, prompt_tokens).tolist()
        ctx = max_context or len(prompt) + WARMUP_TOKENS + MEASURE_TOKENS + 8
        W = synth.make_model(d, seed=seed)
        model = Model(config_from_dims(d, max_context_length=ctx, max_batch=1))
        model.load_weights(synth.iter_named_tensors(W))
        del W
    load_ns = time.perf_counter_ns() - t0
    res = generate(model, GenerateOpts(prompt_ids=prompt, max_new=WARMUP_TOKENS + MEASURE_TOKENS))
    n = res.tokens_generated
    warm = min(WARMUP_TOKENS, n)
    meas = min(MEASURE_TOKENS, n - warm)
    if meas <= 0:
        raise SystemExit(f"error: not enough tokens generated ({n})")
    r = compute_results(load_ns, res.prefill_ns, len(prompt), res.per_token_ns, warm, meas)
    model.free()
    return format_json(r, len(prompt), WARMUP_TOKENS)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model-dir", default=None, help="MLX Q1 Bonsai-1.7B checkpoint (safetensors + tokenizer.json)")
    ap.add_argument("--prompt-tokens", type=int, default=512, help="synthetic prompt length (no --model-dir)")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    sys.stdout.write(run(a.model_dir, a.prompt_tokens, a.seed))
    sys.stdout.flush()


if __name__ == "__main__":
    main()
