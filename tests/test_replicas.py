"""Multi-replica host logic on CPU: the reference's device split and dynamic batching, and a
world_size-2 gloo run in which each rank embeds its own share of a request (CPU oracle as the
stand-in compute) and rank 0 reassembles the result in request order."""
import dataclasses
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import replicas
import synth


def test_dynamic_batches_matches_reference_test():
    # internal/embeddings/dynamic_batch_test.go:13-60: [100,100,2000,100], max 4 seqs / 1000 tokens
    assert replicas.dynamic_batches([100, 100, 2000, 100], 4, 1000) == [(0, 2), (2, 3), (3, 4)]
    assert replicas.dynamic_batches([5] * 10, 4, 1000) == [(0, 4), (4, 8), (8, 10)]
    assert replicas.dynamic_batches([], 4, 1000) == []


def test_split_by_weight():
    lens = [10] * 10
    assert replicas.split_by_weight(lens, [1, 1]) == [(0, 5), (5, 10)]
    assert replicas.split_by_weight(lens, [3, 1]) == [(0, 8), (8, 10)]
    assert replicas.split_by_weight(lens, [0, 0]) == [(0, 5), (5, 10)]  # no metrics yet: equal
    assert replicas.split_by_weight([7], [1, 1, 1]) == [(0, 1)]  # fewer sequences than devices
    r = replicas.split_by_weight(list(range(1, 40)), [1, 1, 1, 1])
    assert r[0][0] == 0 and r[-1][1] == 39 and all(a[1] == b[0] for a, b in zip(r, r[1:]))


def test_pack():
    ids, lens = replicas.pack([[5, 6], [7]])
    assert ids.tolist() == [101, 5, 6, 102, 101, 7, 102] and lens.tolist() == [4, 3]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1)
    blob = synth.make_weights(cfg, 0)
    lens = synth.make_lengths(9, 8, 64, 3)
    ids = synth.make_ids(lens, cfg.vocab_size, 3)
    ranges = replicas.split_by_weight(lens, [1.0] * world)
    rows = replicas.shard_rows(lens, ranges)
    import torch
    vec, off = torch.zeros((0, cfg.hidden)), 0
    if rank < len(ranges):
        (a, b), (t0, t1) = ranges[rank], rows[rank]
        vec, off = torch.from_numpy(oracle.forward(cfg, blob, ids[t0:t1], lens[a:b], threads=1)["mean"]), a
    out = replicas.gather_pooled(vec, off, len(lens)).numpy()  # unequal row counts per rank
    if rank == 0:
        full = oracle.forward(cfg, blob, ids, lens, threads=1)["mean"]
        q.put(float(np.abs(out - full).max()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_replicas():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) <= 1e-6
