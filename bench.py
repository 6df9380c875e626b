#!/usr/bin/env python
"""Benchmark: Bonsai-1.7B-shaped 1-bit (Q1 g128) greedy decode at batch 1.

Workload (benchmark configuration 3, the full model): random-init 28-layer Qwen3-1.7B architecture
with packed 1-bit weights and a tied 1-bit embedding, a 512-token prompt
(ids uniform from seed 0, tokenizer bypassed) prefilled, then 256 greedy
tokens.  One "step" = one generate() call = prefill 512 + decode 256.

Prints ONE JSON line (rank 0).  ``value`` is decode tok/s measured on the
device (CUDA events around every graph replay, max over ranks); ``e2e`` is
the same job timed on the host around the public generate() call (prompt
host->device, tokens device->host, prefill included).  Multi-GPU runs are
independent replicas (batch-1 decode does not shard), so ``value`` sums the
ranks' tokens over the slowest rank's time.

The line also carries the reference bench's own keys (decode_tok_per_sec,
prefill_tok_per_sec, decode_p50_us, decode_p99_us; see
nnzap_b200/bonsai_bench.py for the drop-in entry point), a parity check of
the benchmarked run itself (every generated token against the CPU oracle's
teacher-forced logits), and ``tp_config4``: benchmark configuration 4
(batch 64, KV 4096) decoded tensor-parallel over the job's N GPUs, with a
TP-N vs TP-1 logits check at N > 1 and the 4-bit variant at N = 1.

``--impl reference`` times the CPU oracle's token-at-a-time decode on a
bounded sample (the reference engine itself needs Apple Metal + Zig).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT, GEN = 512, 256
# ncu (dram__bytes_read.sum + dram__bytes_write.sum) of one decode launch of
# the config-3 model at context TRAFFIC_CTX, captured with
# `python -m nnzap_b200.microbench decode1 --ctx 512 --steps 4` under
# `ncu --clock-control none -k regex:d1_kernel -s 2 -c 1`
TRAFFIC_BYTES, TRAFFIC_CTX = 310.53e6, 515
METRIC = "decode_tok_per_sec"
UNIT = "tok/s"


def rank_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid, self.proc, self.lines = uuid, None, []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.uuid:
            cmd[1:1] = ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def algorithmic_bytes_per_token(d, ctx):
    """Weights streamed per decode token (1 bit + fp16 scale per group) plus
    the K/V history read at context length ctx."""
    qd, kvd = d.n_q * d.head_dim, d.n_kv * d.head_dim
    layer_params = d.hidden * (qd + 2 * kvd) + qd * d.hidden + 3 * d.hidden * d.inter
    per_param = 1 / 8 + 2 / d.gs
    weights = d.layers * layer_params * per_param + d.vocab * d.hidden * per_param
    kv = d.layers * 2 * d.n_kv * ctx * d.head_dim * 2
    return weights + kv


def launches_per_step(d, prompt, gen, chunk=512):
    """Our kernels launched per generate(): GEMM prefill per 512-row chunk
    (embed, 9 per layer: norm, QKV GEMM, K/V write, attention + split
    combine, O GEMM, norm, gate/up GEMM, down GEMM; LM head on the last
    chunk) plus the decode: one single-row kernel launch for all greedy
    tokens (NNZ_DECODE_PATH=mega: one persistent kernel per token; =graph:
    embed + 7 per layer + LM head per token)."""
    chunks = -(-prompt // chunk)
    path = os.environ.get("NNZ_DECODE_PATH")
    decode = gen * (1 + d.layers * 7 + 1) if path == "graph" else gen if path == "mega" else 1
    return chunks * (1 + d.layers * 9) + 1 + decode


def oracle_cfg(d):
    from oracle import qwen3_ref as R
    return R.Cfg(vocab=d.vocab, hidden=d.hidden, inter=d.inter, layers=d.layers, n_q=d.n_q,
                 n_kv=d.n_kv, head_dim=d.head_dim, gs=d.gs, quant=d.quant)


def cpu_decode_sample(d, W, n_prompt=8, n_decode=16):
    """Token-at-a-time CPU decode with the oracle (all host cores via BLAS),
    every weight matrix dequantized once and kept (the first prompt token
    pays for that)."""
    from oracle import qwen3_ref as R
    R.set_dequant_cache(True)
    cfg = oracle_cfg(d)
    prompt = np.random.default_rng(0).integers(0, d.vocab, n_prompt)
    kv = []
    t0 = time.perf_counter()
    for p, tok in enumerate(prompt):
        lg = R.decode_one(cfg, W, kv, int(tok), p)
    t1 = time.perf_counter()
    tok = int(np.argmax(lg))
    times = []
    for i in range(n_decode):
        a = time.perf_counter()
        lg = R.decode_one(cfg, W, kv, tok, n_prompt + i)
        tok = int(np.argmax(lg))
        times.append(time.perf_counter() - a)
    R.set_dequant_cache(False)
    return {"decode_tok_per_sec": n_decode / sum(times), "prefill_tok_per_sec": n_prompt / (t1 - t0),
            "decode_s": sum(times), "prefill_s": t1 - t0, "n_prompt": n_prompt, "n_decode": n_decode}


def run_reference(args):
    rank, world, _ = rank_env()
    if rank != 0:
        return
    from nnzap_b200 import synth
    from oracle import qwen3_ref as R
    d = synth.BONSAI_1_7B_Q1
    W = synth.make_model(d, seed=0)
    cfg = oracle_cfg(d)
    R.set_dequant_cache(True)     # dequantize once, like a real CPU engine keeps its weights
    n_prompt = 8
    kv = []
    for p, tok in enumerate(np.random.default_rng(0).integers(0, d.vocab, n_prompt)):
        lg = R.decode_one(cfg, W, kv, int(tok), p)
    tok, pos = int(np.argmax(lg)), n_prompt
    for _ in range(args.warmup):
        lg = R.decode_one(cfg, W, kv, tok, pos)
        tok, pos = int(np.argmax(lg)), pos + 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lg = R.decode_one(cfg, W, kv, tok, pos)
        tok, pos = int(np.argmax(lg)), pos + 1
    dt = time.perf_counter() - t0
    v = args.steps / dt
    cores = os.cpu_count()
    sample = (f"oracle token-at-a-time decode of {args.steps} tokens (after an {n_prompt}-token "
              f"prompt and {args.warmup} warm-up tokens) on the full config-3 model, numpy/BLAS, "
              "weights dequantized once to f32")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config 3: Bonsai-1.7B-shaped Q1 g128, b=1 greedy decode (bounded CPU sample)",
                   "model": "Qwen3-1.7B arch, random-init 1-bit", "global_batch": 1,
                   "seq_len": PROMPT + GEN, "parallelism": "none (CPU)"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference engine needs Apple Metal + Zig (absent); this arm times the CPU "
                "restatement of its decode (oracle/qwen3_ref.py)"}), flush=True)


def qmv_config0(torch, replays=20):
    """Standalone benchmark configuration 0: one QMV (Q4 6144x2048 g64, fp16
    in/out) over 48 rotating weight copies (340 MB > L2).  The 48 calls are
    captured once in a CUDA graph and replayed, so the per-call time is the
    kernel's, not the Python call's; `host_call_us` is the same call made
    from Python one at a time."""
    from nnzap_b200 import synth
    from nnzap_b200._capi import check, lib, ptr
    M, K, gs = 6144, 2048, 64
    L = lib()
    t = synth.rand_q4(np.random.default_rng(0), M, K, gs)
    nb = L.nnz_packed_bytes(1, M, K, gs, 1)
    packed = np.zeros(nb, dtype=np.uint8)
    check(L.nnz_pack_weights(1, ptr(t["weight"]), ptr(t["scales"]), ptr(t["biases"]), M, K, gs, 1, 0,
                             ptr(packed)))
    copies = 48                                     # 48 x 7.1 MB = 340 MB > L2
    dev = torch.from_numpy(packed).cuda().repeat(copies)
    x = torch.randn(K, device="cuda").half()
    y = torch.empty(M, device="cuda", dtype=torch.float16)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        stream = side.cuda_stream
        for i in range(copies):   # warm-up (first use sets up the workspace)
            check(L.nnz_qmv(1, 0, 0, dev.data_ptr() + i * nb, M, K, gs, ptr(x), K, 1, ptr(y), M, 0, stream))
        side.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(side)
        for i in range(4 * copies):
            c = i % copies
            check(L.nnz_qmv(1, 0, 0, dev.data_ptr() + c * nb, M, K, gs, ptr(x), K, 1, ptr(y), M, 0, stream))
        b.record(side)
        side.synchronize()
        host_us = a.elapsed_time(b) * 1000 / (4 * copies)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(copies):
                check(L.nnz_qmv(1, 0, 0, dev.data_ptr() + i * nb, M, K, gs, ptr(x), K, 1, ptr(y), M, 0,
                                torch.cuda.current_stream().cuda_stream))
        g.replay()
        side.synchronize()
        a.record(side)
        for _ in range(replays):
            g.replay()
        b.record(side)
        side.synchronize()
    us = a.elapsed_time(b) * 1000 / (replays * copies)
    alg = M * K / 2 + 2 * 2 * (M * K // gs) + K * 2 + M * 2
    return us, alg / (us * 1e-6) / 1e9, alg, host_us


C4_BATCH, C4_CTX = 64, 4096


def _barrier(torch, world):
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize()


def _gpu_uuid(torch, local):
    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


def tp_parity(torch, model, d, W, rank, world, local, rows=C4_BATCH, pos=16):
    """TP-N logits vs a TP-1 model of the same weights on the same inputs
    (fresh caches, one decode step of `rows` rows at position `pos`): the
    vocabulary shards are gathered on rank 0, which builds the TP-1 model.
    Returns {"max_abs": ..., "argmax_equal": ..., "near_ties": ...} on rank 0."""
    from nnzap_b200 import Model, config_from_dims
    tok = np.random.default_rng(1).integers(0, d.vocab, rows).astype(np.uint32)
    _, lg = model.forward_decode(tok, np.full(rows, pos, np.uint32), want_logits=True)
    shard = torch.from_numpy(np.ascontiguousarray(lg)).cuda()
    parts = [torch.empty_like(shard) for _ in range(world)]
    torch.distributed.all_gather(parts, shard)
    if rank != 0:
        _barrier(torch, world)
        return None
    full = torch.cat(parts, dim=1).cpu().numpy()
    ref = Model(config_from_dims(d, max_context_length=pos + 8, max_batch=rows), device=local)
    ref.load_weights(__import__("nnzap_b200").synth.iter_named_tensors(W))
    _, want = ref.forward_decode(tok, np.full(rows, pos, np.uint32), want_logits=True)
    ref.free()
    _barrier(torch, world)
    am_n, am_1 = full.argmax(1), want.argmax(1)
    top2 = np.sort(want, axis=1)[:, -2:]
    near = (top2[:, 1] - top2[:, 0]) < 2e-2
    return {"rows": rows, "position": pos, "max_abs": float(np.abs(full - want).max()),
            "argmax_equal": int((am_n == am_1).sum()), "near_ties": int(near.sum()),
            "ok": bool(np.abs(full - want).max() <= 2e-2 and ((am_n == am_1) | near).all())}


def config4_measure(torch, rank, world, local, quant, steps, warmup, parity=False):
    """Benchmark configuration 4: 64 sequences decoded together with a
    4096-position KV cache, tensor-parallel over the job's GPUs (tp = N:
    heads, gate/up rows and vocabulary split, all-reduce after o/down inside
    the decode graph).  A step = one decode step of all 64 rows; positions
    start at 4096 - steps - warmup so the last step attends over 4095
    positions.  Collective over the job's ranks; returns the result dict on
    rank 0 (None elsewhere)."""
    from nnzap_b200 import Model, config_from_dims, synth, tp_unique_id
    d = synth.BONSAI_1_7B_Q1 if quant == "q1" else synth.BONSAI_1_7B_Q4
    t0 = time.perf_counter()
    W = synth.make_model(d, seed=0)
    uid = None
    if world > 1:
        box = [tp_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(box, src=0)
        uid = box[0]
    cfg = config_from_dims(d, max_context_length=C4_CTX, max_batch=C4_BATCH).replace(
        tp_rank=rank, tp_size=world)
    model = Model(cfg, device=local, tp_unique_id=uid)
    model.load_weights(synth.iter_named_tensors(W))
    load_ms = (time.perf_counter() - t0) * 1000
    par = tp_parity(torch, model, d, W, rank, world, local) if (parity and world > 1) else None
    del W
    tok = np.random.default_rng(0).integers(0, d.vocab, C4_BATCH).astype(np.uint32)
    p0 = C4_CTX - steps - warmup - 1
    model.decode_steps(tok, np.full(C4_BATCH, p0, np.uint32), warmup)
    clocks = ClockSampler(_gpu_uuid(torch, local))
    clocks.start()
    _barrier(torch, world)
    w0 = time.perf_counter()
    out, ns = model.decode_steps(tok, np.full(C4_BATCH, p0 + warmup, np.uint32), steps, timings=True)
    wall = time.perf_counter() - w0
    _barrier(torch, world)
    clk = clocks.stop()
    model.free()
    stats = torch.tensor([float(ns.sum()) / 1e9, wall], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
    dev_s, wall_s = stats.tolist()
    if rank != 0:
        return None
    hbm, peak_kind = measured_peaks()
    mean_ctx = p0 + warmup + (steps + 1) / 2
    per_param = (1 / 8 + 2 / d.gs) if d.quant == "q1" else (1 / 2 + 4 / d.gs)
    qd, kvd = d.n_q * d.head_dim, d.n_kv * d.head_dim
    wbytes = (d.layers * (d.hidden * (qd + 2 * kvd) + qd * d.hidden + 3 * d.hidden * d.inter)
              + d.vocab * d.hidden) * per_param
    kvbytes = C4_BATCH * d.layers * 2 * kvd * mean_ctx * 2
    step_bytes_gpu = (wbytes + kvbytes) / world
    achieved = step_bytes_gpu / (dev_s / steps) / 1e9
    per_step_launches = 1 + d.layers * 9 + 4 + (4 * d.layers + 1 if world > 1 else 0)
    return {"quant": d.quant, "tp": world, "batch": C4_BATCH, "kv": C4_CTX, "steps": steps, "warmup": warmup,
            "value": C4_BATCH * steps / dev_s, "unit": "tok/s", "ms_per_step": dev_s / steps * 1000,
            "load_ms": load_ms, "wall_s": wall_s, "mean_ctx": mean_ctx,
            "roofline": {"bound": "hbm", "kernel": "decode step (CUDA graph: attn_tc_kernel dominant)",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_step_per_gpu": step_bytes_gpu},
            "gpu_launches": per_step_launches * steps, "clocks": clk, "parity_vs_tp1": par,
            "sample_tokens": out[-1][:8].tolist()}


def run_config4(args):
    """`--workload config4`: the configuration-4 measurement as the line itself."""
    import torch
    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    r = config4_measure(torch, rank, world, local, args.quant, args.steps, args.warmup, parity=True)
    if rank != 0:
        if world > 1:
            torch.distributed.barrier()
        return
    print(json.dumps({
        "metric": "decode_tok_per_sec", "value": r["value"], "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": f"{r['quant']} weights; fp16 KV, f32 accumulate", "data": "synthetic",
        "config": {"workload": f"config 4: batch {C4_BATCH}, KV {C4_CTX}, Bonsai-1.7B-shaped {r['quant']} "
                               "random-init, greedy decode steps",
                   "model": "Qwen3-1.7B architecture (28 layers, vocab 151936)", "global_batch": C4_BATCH,
                   "seq_len": C4_CTX, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2: 30 GB of KV cache read per step",
                   "kv_contents": "zero-initialised cache (attention time does not depend on values)"},
        "load_ms": r["load_ms"], "roofline": r["roofline"], "cpu_baseline": None,
        "e2e": {"value": C4_BATCH * args.steps / r["wall_s"], "unit": "tok/s (nnz_decode_steps wall time)",
                "h2d_bytes_per_step": C4_BATCH * 8 / args.steps, "d2h_bytes_per_step": C4_BATCH * 4},
        "gpu_launches": r["gpu_launches"], "clocks": r["clocks"], "parity_vs_tp1": r["parity_vs_tp1"],
        "sample_tokens": r["sample_tokens"]}), flush=True)
    if world > 1:
        torch.distributed.barrier()


def tokenizer_text(seed: int, nbytes: int) -> bytes:
    """Seeded synthetic prompt text: syllable words, numbers, punctuation,
    contractions, accented / CJK / emoji runs, tabs, newlines and the chat
    special tokens (the reference's bench prompt text is replaced by this)."""
    import random
    rng = random.Random(seed)
    syl = [a + b for a in "bcdfghjklmnprstvwz" for b in "aeiou"]
    words = ["".join(rng.choice(syl) for _ in range(rng.randint(1, 4))) for _ in range(2000)]
    extra = ["é", "日本", "中文", "😀", "—", "…", "don't", "it's", "(x)", "!?", "\n", "\t",
             "<|im_start|>", "<|im_end|>", "  "]
    out, n = [], 0
    while n < nbytes:
        r = rng.random()
        w = rng.choice(words) if r < 0.8 else str(rng.randint(0, 99999)) if r < 0.88 else rng.choice(extra)
        piece = (" " + w).encode()
        out.append(piece)
        n += len(piece)
    return b"".join(out)[:nbytes]


def run_tokenizer(args):
    """Host workload: BPE encode throughput of the library's C++ tokenizer
    (value) and through the Python mirror (e2e) on ~1 MiB of text, with the
    oracle (the literal restatement of the reference's tokenizer) timed on a
    bounded sample beside it."""
    rank, world, _ = rank_env()
    if rank != 0:
        return
    from oracle import tokenizer_ref as R
    js = (ROOT / "tests" / "golden" / "tokenizer_synth.json").read_bytes()
    text = tokenizer_text(0, 1 << 20)
    mb = len(text) / 1e6
    sample = text[: 64 << 10]

    def time_ref():
        ref = R.Tokenizer(js)
        t0 = time.perf_counter()
        ref.encode(sample)
        return len(sample) / 1e6 / (time.perf_counter() - t0)

    cfg = {"workload": "BPE encode (tokenizer.zig encode): 1 MiB of seeded synthetic text incl. "
                       "UTF-8 and chat special tokens", "tokenizer": "synthetic byte-level BPE, "
                       "3000 entries, 2740 merges (tests/golden/tokenizer_synth.json)",
           "global_batch": 1, "parallelism": "host, 1 thread"}
    ref_note = (f"oracle/tokenizer_ref.py (pure Python, the reference's algorithm and data "
                f"structures) encoding the first {len(sample)} bytes")
    if args.impl == "reference":
        for _ in range(args.warmup):
            time_ref()
        vals = [time_ref() for _ in range(args.steps)]
        v = statistics.median(vals)
        print(json.dumps({
            "impl": "reference", "metric": "tokenizer_encode_mb_per_sec", "value": v, "unit": "MB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": len(sample) / 1e6 / v * 1000, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": v, "unit": "MB/s", "cores": 1, "kind": "port", "sample": ref_note},
            "e2e": {"value": v, "unit": "MB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    import ctypes as C
    from nnzap_b200 import _capi
    from nnzap_b200.tokenizer import Tokenizer
    tok = Tokenizer.from_json(js)
    L = _capi.lib()
    out = np.empty(len(text) + 1, np.uint32)
    n = C.c_uint32()

    def step_lib():
        t0 = time.perf_counter()
        _capi.check(L.nnz_tokenizer_encode(tok._h, text, len(text), out.ctypes.data, len(out), C.byref(n)))
        return time.perf_counter() - t0

    def step_py():
        t0 = time.perf_counter()
        tok.encode(text)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step_lib()
        step_py()
    lib_t = [step_lib() for _ in range(args.steps)]
    py_t = [step_py() for _ in range(args.steps)]
    assert out[: n.value].tolist() == tok.encode(text)   # same ids through both entry points
    ms = statistics.median(lib_t) * 1000
    cpu = None if args.no_cpu_baseline else {
        "value": time_ref(), "unit": "MB/s", "cores": 1, "kind": "port", "sample": ref_note}
    print(json.dumps({
        "metric": "tokenizer_encode_mb_per_sec", "value": mb / (ms / 1000), "unit": "MB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": cfg, "tokens_per_step": int(n.value),
        "cpu_baseline": cpu,
        "e2e": {"value": mb / statistics.median(py_t), "unit": "MB/s (Tokenizer.encode -> list)",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0, "note": "host-only row: the tokenizer runs on the CPU in the reference "
                                   "and here (C++ in libnnz_b200.so)"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config3", choices=["config3", "config4", "tokenizer"],
                    help="config3: b=1 generate (default, replicas for N>1); config4: batch-64 "
                         "decode at KV 4096, tensor-parallel over the N GPUs; tokenizer: host BPE "
                         "encode throughput")
    ap.add_argument("--quant", default="q1", choices=["q1", "q4"], help="config4 weights")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the benchmarked tokens")
    ap.add_argument("--no-tp", action="store_true", help="skip the appended tensor-parallel config-4 run")
    args = ap.parse_args()
    if args.workload == "tokenizer":
        run_tokenizer(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "config4":
        run_config4(args)
        return

    import torch
    rank, world, local = rank_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from nnzap_b200 import GenerateOpts, Model, config_from_dims, generate, synth

    d = synth.BONSAI_1_7B_Q1
    t0 = time.perf_counter()
    W = synth.make_model(d, seed=0)
    cfg = config_from_dims(d, max_context_length=PROMPT + GEN + 8, max_batch=1)
    model = Model(cfg, device=local)
    model.load_weights(synth.iter_named_tensors(W))
    load_ms = (time.perf_counter() - t0) * 1000
    prompt = np.random.default_rng(0).integers(0, d.vocab, PROMPT).tolist()
    opts = GenerateOpts(prompt_ids=prompt, max_new=GEN)

    for _ in range(args.warmup):
        generate(model, opts)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
            torch.cuda.synchronize()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    barrier()
    per_token, prefill_ns, decode_ns, walls, tokens = [], 0, 0, [], None
    for _ in range(args.steps):
        w0 = time.perf_counter()
        res = generate(model, opts)          # host prompt in, host tokens out
        walls.append(time.perf_counter() - w0)
        prefill_ns += res.prefill_ns
        decode_ns += res.decode_ns
        per_token += res.per_token_ns
        tokens = res.tokens
    barrier()
    clk = clocks.stop()

    # configuration 4 tensor parallel over the same GPUs (collective: every rank)
    tp4 = None
    if not args.no_tp:
        tp4 = config4_measure(torch, rank, world, local, "q1", 8, 3, parity=True)
        if world == 1:
            q4 = config4_measure(torch, rank, world, local, "q4", 8, 3)
            tp4 = {"q1": tp4, "q4_g64": q4}
        else:
            tp4 = {"q1": tp4} if rank == 0 else None
    stats = torch.tensor([decode_ns / 1e9, prefill_ns / 1e9, sum(walls)], dtype=torch.float64,
                         device="cuda")
    if world > 1:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
    dec_s, pre_s, wall_s = stats.tolist()
    value = GEN * args.steps * world / dec_s
    prefill_tps = PROMPT * args.steps * world / pre_s
    pt = sorted(per_token)
    p50 = pt[len(pt) // 2] / 1000
    p99 = pt[(len(pt) * 99) // 100] / 1000

    if rank != 0:
        if world > 1:
            torch.distributed.barrier()
        return
    hbm, peak_kind = measured_peaks()
    mean_ctx = PROMPT + (GEN + 1) / 2
    bytes_tok = algorithmic_bytes_per_token(d, mean_ctx)
    us_tok = dec_s / (GEN * args.steps) * 1e6
    achieved = bytes_tok / (us_tok * 1e-6) / 1e9
    q0_us, q0_gbs, q0_bytes, q0_host = qmv_config0(torch)
    parity = None
    if not args.no_parity:
        # the benchmarked run itself: every generated token against the oracle's
        # teacher-forced logits over prompt + generated (ids identical unless the
        # oracle has a near tie; the reference's own check is exact ids,
        # nnmetal/examples/bonsai_golden.zig:304-357)
        from oracle import qwen3_ref as R
        R.set_dequant_cache(True)
        t_par = time.perf_counter()
        exact, worst, _ = R.greedy_check(oracle_cfg(d), W, prompt, tokens)
        R.set_dequant_cache(False)
        parity = {"checked_tokens": len(tokens), "exact": exact, "worst_gap": worst,
                  "tolerance": 2e-2, "ok": worst <= 2e-2, "oracle_s": time.perf_counter() - t_par}
    cpu = None
    if not args.no_cpu_baseline:
        c = cpu_decode_sample(d, W)
        cpu = {"value": c["decode_tok_per_sec"], "unit": UNIT, "cores": os.cpu_count(),
               "kind": "port",
               "sample": (f"oracle token-at-a-time decode: {c['n_prompt']}-token prompt "
                          f"({c['prefill_s']:.1f} s) then {c['n_decode']} greedy tokens "
                          f"({c['decode_s']:.1f} s), full config-3 model, numpy/BLAS on "
                          f"{os.cpu_count()} host threads")}
    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": wall_s / args.steps * 1000,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q1 weights, int8 tensor-core MMA, f32 accumulate", "data": "synthetic",
        "config": {"workload": "config 3: Bonsai-1.7B-shaped 1-bit (Q1 g128) random-init, "
                               "512-token prompt prefill + 256 greedy tokens, batch 1",
                   "model": "Qwen3-1.7B architecture (28 layers, vocab 151936)", "global_batch": world,
                   "seq_len": PROMPT + GEN, "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: 242 MB of weights streamed per token"},
        "decode_tok_per_sec": GEN * args.steps / dec_s, "prefill_tok_per_sec": prefill_tps,
        "decode_p50_us": p50, "decode_p99_us": p99,
        "load_ms": load_ms, "prompt_tokens": PROMPT, "measured_tokens": GEN * args.steps,
        "roofline": {"bound": "hbm",
                     "kernel": ("decode step: CUDA graph" if os.environ.get("NNZ_DECODE_PATH") == "graph"
                                else "decode step: single-row cooperative kernel d1_kernel"),
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind,
                     # DRAM bytes (read + write) of one single-token decode launch
                     # measured by ncu at context TRAFFIC_CTX, moved to the mean
                     # context by the K/V bytes a position adds
                     "traffic": TRAFFIC_BYTES + d.layers * 2 * d.n_kv * (mean_ctx - TRAFFIC_CTX) * d.head_dim * 2,
                     "algorithmic_bytes_per_token": bytes_tok},
        "qmv_config0": {"us": q0_us, "achieved_gbs": q0_gbs, "frac": q0_gbs / hbm,
                        "algorithmic_bytes": q0_bytes, "host_call_us": q0_host,
                        "timing": "48 calls on rotating weight copies captured in a CUDA graph, replayed"},
        "cpu_baseline": cpu,
        "e2e": {"value": GEN * args.steps * world / wall_s, "unit": "tok/s (generate() wall time, "
                "512-token prefill included)", "h2d_bytes_per_step": PROMPT * 4,
                "d2h_bytes_per_step": GEN * 4},
        "gpu_launches": launches_per_step(d, PROMPT, GEN) * args.steps,
        "clocks": clk,
        "sample_tokens": tokens[:8],
        "parity": parity,
        "tp_config4": tp4,
    }
    print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
