"""Tensor-parallel host logic on CPU.

* nnz_shard_weights (the loader's slicing) against numpy slicing of the
  dequantized matrix, rows and columns, Q1 and Q4, bit-exact.
* Two gloo ranks run the row-/column-split projection algebra the decode
  path uses (column-split q/gate rows, row-split o/down inputs with a sum
  all-reduce, vocabulary-split LM head with a (value, index) max) on
  shards cut by the C ABI, and must reproduce the unsharded oracle result.
"""
import os
import socket

import numpy as np
import pytest

from nnzap_b200 import shard_weights, synth
from oracle import qwen3_ref as R


def _cfg(fmt, gs, K):
    return R.Cfg(vocab=8, hidden=K, inter=K, layers=1, n_q=1, n_kv=1, head_dim=128, gs=gs,
                 quant="q1" if fmt == "q1_0" else "q4")


def _rand(fmt, rng, M, K, gs):
    return synth.rand_q1(rng, M, K, gs) if fmt == "q1_0" else synth.rand_q4(rng, M, K, gs)


def _deq(fmt, t, M, K, gs):
    return R.dequant_tensor(_cfg(fmt, gs, K), t, M, K)


@pytest.mark.parametrize("fmt,gs", [("q1_0", 128), ("q4_mlx", 64)])
@pytest.mark.parametrize("axis", [0, 1])
def test_shard_matches_slicing(built_lib, fmt, gs, axis):
    rng = np.random.default_rng(3)
    M, K, T = 256, 1024, 4
    t = _rand(fmt, rng, M, K, gs)
    full = _deq(fmt, t, M, K, gs)
    n = (M if axis == 0 else K) // T
    for r in range(T):
        w, s, b = shard_weights(fmt, axis, t["weight"], t["scales"], t.get("biases"), M, K, gs,
                                r * n, (r + 1) * n)
        part = {"weight": w if fmt == "q1_0" else w.view(np.uint32), "scales": s}
        if b is not None:
            part["biases"] = b
        Mo, Ko = (n, K) if axis == 0 else (M, n)
        got = _deq(fmt, part, Mo, Ko, gs)
        want = full[r * n:(r + 1) * n] if axis == 0 else full[:, r * n:(r + 1) * n]
        np.testing.assert_array_equal(got, want)


def test_shard_rejects_unaligned_columns(built_lib):
    from nnzap_b200._capi import NnzError
    t = synth.rand_q1(np.random.default_rng(0), 8, 256, 128)
    with pytest.raises(NnzError):
        shard_weights("q1_0", 1, t["weight"], t["scales"], None, 8, 256, 128, 64, 192)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fmt, gs, H, I, V = "q1_0", 128, 256, 512, 96
        rng = np.random.default_rng(7)          # every rank builds the same full model
        gate = synth.rand_q1(rng, I, H, gs)
        down = synth.rand_q1(rng, H, I, gs)
        lm = synth.rand_q1(rng, V, H, gs)
        x = rng.standard_normal(H).astype(np.float32)
        # column-split gate rows -> this rank's slice of the intermediate
        n = I // world
        w, s, _ = shard_weights(fmt, 0, gate["weight"], gate["scales"], None, I, H, gs, rank * n,
                                (rank + 1) * n)
        h = _deq(fmt, {"weight": w, "scales": s}, n, H, gs) @ x
        # row-split down: partial over this rank's intermediate columns, sum-reduced
        w, s, _ = shard_weights(fmt, 1, down["weight"], down["scales"], None, H, I, gs, rank * n,
                                (rank + 1) * n)
        part = torch.from_numpy(_deq(fmt, {"weight": w, "scales": s}, H, n, gs) @ h)
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        # vocabulary-split LM head: local argmax -> (value, global index) max
        per = V // world
        w, s, _ = shard_weights(fmt, 0, lm["weight"], lm["scales"], None, V, H, gs, rank * per,
                                (rank + 1) * per)
        logits = _deq(fmt, {"weight": w, "scales": s}, per, H, gs) @ part.numpy()
        loc = int(np.argmax(logits))
        cand = [None] * world
        dist.all_gather_object(cand, (float(logits[loc]), rank * per + loc))
        best = max(cand, key=lambda c: (c[0], -c[1]))
        if rank == 0:
            full_h = _deq(fmt, gate, I, H, gs) @ x
            full_y = _deq(fmt, down, H, I, gs) @ full_h
            full_l = _deq(fmt, lm, V, H, gs) @ full_y
            q.put((np.abs(part.numpy() - full_y).max(), best[1], int(np.argmax(full_l))))
    finally:
        dist.destroy_process_group()


def test_tp_algebra_two_gloo_ranks(built_lib):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    err, tok, want = q.get(timeout=5)
    assert err < 1e-3
    assert tok == want


def _init_rank_main(rank, world, port, nccl_lib, q):
    """One gloo rank of the tensor-parallel set-up handshake: rank 0 asks the
    library for the NCCL unique id and broadcasts it (or its failure) over
    the host channel; every rank reports what it saw."""
    import torch.distributed as dist
    if nccl_lib is not None:
        os.environ["NNZ_NCCL_LIB"] = nccl_lib
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nnzap_b200 import tp_unique_id
        from nnzap_b200._capi import NnzError
        msg = [None]
        if rank == 0:
            try:
                msg[0] = ("ok", tp_unique_id())
            except NnzError as e:
                msg[0] = ("err", (e.code, str(e)))
        dist.broadcast_object_list(msg, src=0)
        q.put((rank, msg[0]))
    finally:
        dist.destroy_process_group()


def _run_init(nccl_lib):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_init_rank_main, args=(r, 2, port, nccl_lib, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    return dict(q.get(timeout=5) for _ in procs)


def test_tp_init_nccl_missing_two_gloo_ranks(built_lib):
    """Host-injected failure: the NCCL library the deployment pins is absent.
    Rank 0's unique-id request fails with NNZ_ENCCL (no device touched, no
    hang) and every rank learns it over the host channel before any model
    or collective exists."""
    from nnzap_b200._capi import NNZ_ENCCL
    seen = _run_init("/nonexistent/libnccl.so.2")
    for rank in (0, 1):
        kind, (code, text) = seen[rank]
        assert kind == "err" and code == NNZ_ENCCL and "NNZ_NCCL_LIB" in text


def test_tp_init_unique_id_two_gloo_ranks(built_lib):
    """The same handshake with the real library: every rank receives the same
    128-byte id (ncclGetUniqueId needs no GPU)."""
    seen = _run_init(None)
    assert seen[0] == seen[1] and seen[0][0] == "ok" and len(seen[0][1]) == 128
