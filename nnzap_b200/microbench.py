"""Kernel-level timing drivers: each runs one kernel family on a small,
seeded case and prints one line of CUDA-event timings (small enough to
capture a single launch under a profiler).

  python -m nnzap_b200.microbench attn --rows 16 --ctx 4032
      tensor-core decode attention (nnz_attn_decode) over a random fp16 KV
      cache: Bonsai head layout (16 query / 8 kv heads, head_dim 128)
  python -m nnzap_b200.microbench gemm --M 512 --K 2048 --N 4096
      tcgen05 GEMM on a random 1-bit weight matrix (nnz_prefill_gemm)
  python -m nnzap_b200.microbench prefill --tokens 512
      full Bonsai-1.7B-shaped Q1 model: prompt prefill through nnz_prefill
  python -m nnzap_b200.microbench decode --batch 64 --ctx 256 --steps 2
      full model: batched greedy decode steps (nnz_decode_steps)
"""
from __future__ import annotations

import argparse

import numpy as np


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def attn(args):
    import torch
    from ._capi import check, lib
    n_q, n_kv, hd, max_ctx = 16, 8, 128, 4096
    rows, ctx = args.rows, args.ctx
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = torch.randn(rows, n_kv, max_ctx, hd, device="cuda", generator=g).half()
    vc = torch.randn(rows, n_kv, max_ctx, hd, device="cuda", generator=g).half()
    qkv = torch.randn(rows, (n_q + 2 * n_kv) * hd, device="cuda", generator=g).half()
    qn = torch.ones(hd, device="cuda")
    kn = torch.ones(hd, device="cuda")
    pos = torch.full((rows,), ctx - 1, dtype=torch.int32, device="cuda")
    out = torch.empty(rows, n_q * hd, device="cuda").half()
    st = torch.cuda.current_stream().cuda_stream

    def run():
        check(L.nnz_attn_decode(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                max_ctx, pos.data_ptr(), rows, n_q, n_kv, hd, 1e-6, 1e6, 0, 0,
                                out.data_ptr(), st))
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    a, b = _events(torch)
    a.record()
    for _ in range(args.iters):
        run()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1000 / args.iters
    byts = rows * n_kv * ctx * hd * 2 * 2
    print(f"attn rows {rows} ctx {ctx}: {us:.1f} us per call, {byts / us / 1e3:.0f} GB/s of K/V")


def gemm(args):
    import torch
    from . import synth
    from ._capi import check, lib
    L = lib()
    M, K, N, gs = args.M, args.K, args.N, 128
    t = synth.rand_q1(np.random.default_rng(0), N, K, gs)
    w = torch.from_numpy(t["weight"]).cuda()
    s = torch.from_numpy(t["scales"]).cuda()
    x = torch.randn(M, K, device="cuda").half()
    y = torch.empty(M, N, device="cuda").half()

    def run():
        check(L.nnz_prefill_gemm(0, 0, w.data_ptr(), s.data_ptr(), None, M, K, N, gs, x.data_ptr(),
                                 y.data_ptr(), 0, None))
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    a, b = _events(torch)
    a.record()
    for _ in range(args.iters):
        run()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1000 / args.iters
    print(f"gemm M{M} K{K} N{N} (Q1 g128): {us:.1f} us per call, {2 * M * N * K / us / 1e6:.0f} TFLOP/s")


def _model(batch, ctx):
    from . import Model, config_from_dims, synth
    d = synth.BONSAI_1_7B_Q1
    W = synth.make_model(d, seed=0)
    m = Model(config_from_dims(d, max_context_length=ctx, max_batch=batch))
    m.load_weights(synth.iter_named_tensors(W))
    return d, m


def prefill(args):
    import time
    d, m = _model(1, max(1024, args.tokens + 8))
    prompt = np.random.default_rng(0).integers(0, d.vocab, args.tokens)
    m.prefill(prompt)
    t0 = time.perf_counter()
    for _ in range(args.iters):
        nxt, _ = m.prefill(prompt)
    dt = (time.perf_counter() - t0) / args.iters
    print(f"prefill {args.tokens} tokens: {dt * 1e3:.2f} ms per call (host wall), next token {nxt}")


def decode(args):
    d, m = _model(args.batch, args.ctx)
    tok = np.random.default_rng(0).integers(0, d.vocab, args.batch).astype(np.uint32)
    pos = np.full(args.batch, args.ctx - args.steps - 1, np.uint32)
    out, ns = m.decode_steps(tok, pos, args.steps, timings=True)
    print(f"decode batch {args.batch} ctx {args.ctx}: per-step ms {np.round(ns / 1e6, 3).tolist()}")


def main():
    ap = argparse.ArgumentParser(prog="python -m nnzap_b200.microbench")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("attn")
    p.add_argument("--rows", type=int, default=16)
    p.add_argument("--ctx", type=int, default=4032)
    p.add_argument("--iters", type=int, default=20)
    p = sub.add_parser("gemm")
    p.add_argument("--M", type=int, default=512)
    p.add_argument("--K", type=int, default=2048)
    p.add_argument("--N", type=int, default=4096)
    p.add_argument("--iters", type=int, default=20)
    p = sub.add_parser("prefill")
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--iters", type=int, default=2)
    p = sub.add_parser("decode")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=256)
    p.add_argument("--steps", type=int, default=2)
    args = ap.parse_args()
    {"attn": attn, "gemm": gemm, "prefill": prefill, "decode": decode}[args.cmd](args)


if __name__ == "__main__":
    main()
