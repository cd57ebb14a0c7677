"""Tensor-parallel host logic on world_size-2 gloo ranks (CPU): row shards, column shards with
an all-reduce of fp32 partials, and the vocab-sharded greedy key reduction.  The per-rank compute
here is the oracle (this is a test of the sharding and the collectives, which the CUDA path
shares through edgexpu-llm_b200/tp.py)."""

import os
import socket

import numpy as np
import pytest

from _oracle import TYPE_Q4_K, TYPE_Q8_0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_q):
    import sys

    sys.path.insert(0, os.path.dirname(__file__))
    import torch
    import torch.distributed as dist

    import _oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = _oracle.load_pkg()
        from edgexpu_llm_b200 import synth, tp

        port_ = _oracle.Port()
        rng = np.random.default_rng(42)  # same full tensors on every rank
        errs = []

        # Row-sharded projection (q/k/v/gate/up): local rows, no exchange.
        w = synth.q4_k_weight(rng, 96, 1024)
        x = synth.activations(rng, 2, 1024)
        full = port_.linear(x, w, TYPE_Q4_K, 96)
        r0, per = tp.row_range(96, world, rank)
        local = port_.linear(x, tp.shard_rows(w, world, rank), TYPE_Q4_K, per)
        gathered = [torch.empty((2, per)) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(local))
        if not np.array_equal(torch.cat(gathered, dim=1).numpy(), full):
            errs.append("row shards differ from the unsharded product")

        # Column-sharded projection (o/down): partials + SUM all-reduce.
        for wtype, n_out, n_in in ((TYPE_Q4_K, 64, 2048), (TYPE_Q8_0, 40, 576 * 2)):
            w = synth.weight(rng, wtype, n_out, n_in)
            x = synth.activations(rng, 3, n_in)
            c0, cn = tp.col_range(n_in, wtype, world, rank)
            xs = np.ascontiguousarray(x[:, c0:c0 + cn])
            q_full = port_.quantize(x, wtype)
            q_part = port_.quantize(xs, wtype)
            bb = q_part.shape[1]
            if not np.array_equal(q_full[:, rank * bb:(rank + 1) * bb], q_part):
                errs.append(f"type {wtype}: activation blocks straddle ranks")
            part = torch.from_numpy(port_.linear(xs, tp.shard_cols(w, n_in, wtype, world, rank), wtype, n_out))
            tp.allreduce_partial_(part)
            want = port_.linear(x, w, wtype, n_out)
            bound = port_.linear_bound(x, w, wtype, n_out)
            if not np.all(np.abs(part.numpy().astype(np.float64) - want) <= 1e-5 * bound):
                errs.append(f"type {wtype}: column-shard sum out of tolerance")

        # Vocab-sharded greedy token.
        for wtype, n_embd in ((TYPE_Q8_0, 64), (TYPE_Q4_K, 256)):
            vocab = 512
            w = synth.weight(rng, wtype, vocab, n_embd)
            h = synth.activations(rng, 1, n_embd)[0]
            w[vocab - 1] = w[3]  # equal best candidates on different ranks resolve to the lower id
            tok_full, _, scores = port_.logits(w, wtype, h, vocab)
            v0, nv = tp.row_range(vocab, world, rank)
            tok, sc, _ = port_.logits(tp.shard_rows(w, world, rank), wtype, h, nv)
            key = torch.tensor([tp.key_as_int64(tp.make_key(sc, v0 + tok))], dtype=torch.int64)
            tp.allreduce_argmax_(key)
            if tp.key_id(int(key.item())) != tok_full:
                errs.append(f"type {wtype}: sharded greedy {tp.key_id(int(key.item()))} != {tok_full}")
        result_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_gloo_world2():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: [], 1: []}, results


def test_key_packing_orders_like_scores():
    import _oracle

    _oracle.load_pkg()
    from edgexpu_llm_b200 import tp

    vals = [-3.5, -0.0, 0.0, 1e-30, 2.0, 2.0, 7.25]
    keys = [tp.make_key(v, i) for i, v in enumerate(vals)]
    assert keys[4] > keys[5]  # equal scores: lower id wins
    assert keys[6] == max(keys) and keys[0] == min(keys)
    assert tp.make_key(float("nan"), 1) == 0 and tp.make_key(float("-inf"), 1) == 0
    assert tp.key_id(keys[6]) == 6
    signed = np.array([tp.key_as_int64(k) for k in keys], np.int64)
    order = np.argsort(tp.to_signed_key(signed), kind="stable")
    assert list(order) == sorted(range(len(keys)), key=lambda i: keys[i])
