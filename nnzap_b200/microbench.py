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
  python -m nnzap_b200.microbench decode1 --ctx 512 --steps 4
      full model: single-row decode launches (one token each) after a prefill
  python -m nnzap_b200.microbench qmv
      BASELINE configuration 0 (Q4 6144x2048 g64 matvec, fp16 in/out)
  python -m nnzap_b200.microbench attn --hd 64 --heads 8 --kv-heads 2
      CUDA-core decode attention (head_dim 64)
  python -m nnzap_b200.microbench sample --rows 4
      top-k / top-p sampling over the full vocabulary
"""
from __future__ import annotations

import argparse

import numpy as np


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def attn(args):
    import torch
    from ._capi import check, lib
    n_q, n_kv, hd, max_ctx = args.heads, args.kv_heads, args.hd, 4096
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


def decode1(args):
    d, m = _model(1, args.ctx + args.steps + 8)
    prompt = np.random.default_rng(0).integers(0, d.vocab, args.ctx)
    nxt, _ = m.prefill(prompt)
    import time
    ts = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        am, _ = m.forward_decode([nxt], [args.ctx + i])
        ts.append(time.perf_counter() - t0)
        nxt = int(am[0])
    print(f"single-row decode at ctx {args.ctx}: host ms per token {np.round(np.array(ts) * 1e3, 3).tolist()}")


def qmv(args):
    import torch
    from . import synth
    from ._capi import check, lib, ptr
    M, K, gs = 6144, 2048, 64
    L = lib()
    t = synth.rand_q4(np.random.default_rng(0), M, K, gs)
    packed = np.zeros(L.nnz_packed_bytes(1, M, K, gs, 1), dtype=np.uint8)
    check(L.nnz_pack_weights(1, ptr(t["weight"]), ptr(t["scales"]), ptr(t["biases"]), M, K, gs, 1, 0,
                             ptr(packed)))
    w = torch.from_numpy(packed).cuda()
    x = torch.randn(K, device="cuda").half()
    y = torch.empty(M, device="cuda", dtype=torch.float16)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(args.iters):
        check(L.nnz_qmv(1, 0, 0, w.data_ptr(), M, K, gs, ptr(x), K, 1, ptr(y), M, 0, st))
    torch.cuda.synchronize()
    print(f"qmv config 0: {args.iters} calls done")


def sample(args):
    import torch
    from ._capi import check, lib
    V = 151936
    g = torch.Generator(device="cuda").manual_seed(0)
    lg = torch.randn(args.rows, V, device="cuda", generator=g) * 3
    u = torch.rand(args.rows, device="cuda", generator=g)
    out = torch.empty(args.rows, dtype=torch.int32, device="cuda")
    for _ in range(args.iters):
        check(lib().nnz_sample(lg.data_ptr(), args.rows, V, V, 0.8, 40, 0.9, u.data_ptr(), out.data_ptr(),
                               torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    print(f"sample rows {args.rows}: tokens {out.tolist()}")


def main():
    ap = argparse.ArgumentParser(prog="python -m nnzap_b200.microbench")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("attn")
    p.add_argument("--rows", type=int, default=16)
    p.add_argument("--hd", type=int, default=128)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--kv-heads", type=int, default=8)
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
    p = sub.add_parser("decode1")
    p.add_argument("--ctx", type=int, default=512)
    p.add_argument("--steps", type=int, default=4)
    p = sub.add_parser("qmv")
    p.add_argument("--iters", type=int, default=20)
    p = sub.add_parser("sample")
    p.add_argument("--rows", type=int, default=4)
    p.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    {"attn": attn, "gemm": gemm, "prefill": prefill, "decode": decode, "decode1": decode1, "qmv": qmv,
     "sample": sample}[args.cmd](args)


if __name__ == "__main__":
    main()
