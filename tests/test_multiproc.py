"""The N > 1 host path on CPU: two gloo ranks shard utterances, run the
oracle's greedy sampling on their shards, take the max-over-ranks time and
gather the tokens on rank 0 — the replica scheme bench.py uses over NCCL."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
N_UTT, V = 11, 1025


def _logits(u):
    rng = np.random.default_rng(1000 + u)
    return rng.standard_normal(V).astype(np.float32), rng.integers(0, V - 1, size=8).astype(np.int32)


def _sample_all(ora, utts):
    out = []
    for u in utts:
        lg, hist = _logits(u)
        tok, _ = ora.t2s_greedy_sample(lg.copy(), hist, True)
        out.append(int(tok))
    return out


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, ROOT)
    import __graft_entry__
    import oracle

    rep = __graft_entry__.package().replicas
    rep.init("gloo", rank, world, timeout_s=60)
    try:
        utts = list(rep.shard(N_UTT, rank, world))
        toks = _sample_all(oracle, utts)
        t = rep.max_over_ranks(0.5 + rank, world)
        rep.barrier(world)
        got = rep.gather_to_rank0((utts, toks, t), rank, world)
        if rank == 0:
            q.put(got)
    finally:
        rep.close(world)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_partitions_exactly():
    sys.path.insert(0, ROOT)
    import __graft_entry__

    rep = __graft_entry__.package().replicas
    for n in (0, 1, 7, 64, 500):
        for world in (1, 2, 3, 8):
            owned = [i for r in range(world) for i in rep.shard(n, r, world)]
            assert owned == list(range(n))
            sizes = [len(rep.shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= (1 if n else 0)
    with pytest.raises(ValueError):
        rep.shard(4, 2, 2)


def test_two_gloo_ranks_match_one_process(ora):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    utts = [u for part in got for u in part[0]]
    toks = [t for part in got for t in part[1]]
    assert utts == list(range(N_UTT))  # every utterance exactly once, in rank order
    assert toks == _sample_all(ora, range(N_UTT))  # same tokens as one process
    assert all(part[2] == 1.5 for part in got)  # the max over ranks, seen by every rank
