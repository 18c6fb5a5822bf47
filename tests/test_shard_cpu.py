"""(batch x head) sharding across ranks, on CPU with the gloo backend.

World size 2: each rank computes its slices (with the oracle, on CPU), the
outputs are all-gathered, and the reference's per-call decision is rebuilt
from per-rank partial statistics with one all-reduce. Both must equal the
single-process result.
"""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from adaattn_b200.shard import gather_slices, global_decision, local_slices, shard_range
from adaattn_b200.workloads import WORKLOADS, make_qkv


def test_shard_ranges_cover_everything():
    for n in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 8):
            ranges = [shard_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(2)
        w = WORKLOADS["adaptive_mix"].scaled(batch=2, heads=3, seq=96)
        q, k, v = make_qkv(w, seed=0)
        scale = 1.0 / math.sqrt(w.head_dim)
        lq, lk, lv = (local_slices(x.contiguous(), rank, world) for x in (q, k, v))
        out_local = O.dense_attention(lq, lk, lv, O.FP32, scale, False)
        full = gather_slices(out_local, w.batch, w.heads)
        sums, stats, s = O.head_entropy_sums(lq, lk, scale, 1e-6)
        dec = global_decision(sums.flatten(), stats, s, min(q.shape[2], k.shape[2]), q.dtype)
        if rank == 0:
            result_q.put((full, dec))
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_and_global_decision():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    import queue
    import time
    deadline = time.time() + 240
    while True:
        try:
            full, dec = q_out.get(timeout=2)
            break
        except queue.Empty:
            failed = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if failed or time.time() > deadline:
                for p in procs:
                    if p.is_alive():
                        p.kill()
                raise AssertionError(f"rank process failed: exit codes {failed}")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = WORKLOADS["adaptive_mix"].scaled(batch=2, heads=3, seq=96)
    q, k, v = make_qkv(w, seed=0)
    scale = 1.0 / math.sqrt(w.head_dim)
    want = O.dense_attention(q, k, v, O.FP32, scale, False)
    torch.testing.assert_close(full, want, rtol=0, atol=0)
    ref = O.analyze(q, k, O.OracleConfig(), scale)
    assert dec["low_rank"] == ref["low_rank"]
    assert dec["precision"] == ref["precision"]
    assert dec["ne"] == pytest.approx(ref["ne"], abs=1e-6)
    assert dec["max_score"] == pytest.approx(ref["max_score"], rel=1e-6)
    assert dec["max_prob"] == pytest.approx(ref["max_prob"], rel=1e-6)
