"""CPU tests of the native host runtime (csrc/runtime.cu) with its fake replicas (no GPU): the
reference's split and batching rules (embeddings.go:436-501, 704-731) against their Python
restatement, the embedder's request order, and the server's in-flight sequence cap
(server.go:101), round-robin dispatch, latency bookkeeping, batches that grow with the load, and
failed batches."""
import concurrent.futures as cf
import ctypes
import time

import numpy as np
import pytest

import embedder
import fletcher
import replicas


def _requests(n, seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        k = int(rng.integers(1, 17))
        lens = rng.integers(8, 64, size=k).astype(np.int32)
        ids = np.arange(int(lens.sum()), dtype=np.int32) + 2000 * i
        out.append((ids, lens))
    return out


def _check_vectors(vecs, ids, lens):
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    np.testing.assert_array_equal(vecs[:, 0], ids[starts])
    np.testing.assert_array_equal(vecs[:, 1], lens)


def test_split_and_batches_match_the_restatement():
    L = fletcher.lib()
    rng = np.random.default_rng(0)
    for case in range(300):
        n = int(rng.integers(0, 60))
        lens = rng.integers(1, 600, size=n).astype(np.int32)
        nd = int(rng.integers(1, 9))
        w = rng.uniform(0, 5, size=nd) if case % 3 else np.zeros(nd)
        if case % 7 == 0:
            w[0] = 0.0
        ranges = np.zeros(2 * nd, np.int32)
        k = L.Cuda_Runtime_SplitByWeight(fletcher._i32p(lens), n, w.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                                         nd, fletcher._i32p(ranges))
        assert [tuple(ranges[2 * i:2 * i + 2]) for i in range(k)] == replicas.split_by_weight(lens, list(w))
        mb, mt = int(rng.integers(1, 40)), int(rng.integers(1, 3000))
        cap = max(n, 1)
        br = np.zeros(2 * cap, np.int32)
        k = L.Cuda_Runtime_DynamicBatches(fletcher._i32p(lens), n, mb, mt, fletcher._i32p(br), cap)
        assert [tuple(br[2 * i:2 * i + 2]) for i in range(k)] == replicas.dynamic_batches(lens, mb, mt)


def test_embed_keeps_request_order_across_uneven_replicas():
    emb = embedder.Embedder.fake(3, hidden=4, delay_us=200, max_batch=5, max_tokens=300)
    try:
        emb.set_throughput([3.0, 1.0, 0.5])
        ids, lens = _requests(1, seed=4)[0]
        lens = np.random.default_rng(4).integers(8, 120, size=61).astype(np.int32)
        ids = np.arange(int(lens.sum()), dtype=np.int32)
        out = emb.embed(ids, lens)
        _check_vectors(out, ids, lens)
        ranges = replicas.split_by_weight(lens, [3.0, 1.0, 0.5])
        want = np.concatenate([np.full(b - a, d) for d, (a, b) in enumerate(ranges)])
        np.testing.assert_array_equal(out[:, 2], want)  # each share went to its replica
        jobs, seqs = emb.counts()
        assert list(seqs) == [b - a for a, b in ranges]
        assert all(t > 0 and t != 1.0 for t in emb.throughput())  # measured after a batch
    finally:
        emb.close()


def test_server_returns_each_request_its_vectors():
    emb = embedder.Embedder.fake(2, delay_us=5000)
    srv = embedder.Server(emb, max_in_flight=64)
    reqs = _requests(200)
    futs = [srv.submit(*r) for r in reqs]
    for (ids, lens), f in zip(reqs, futs):
        vecs, lat = f.result(timeout=30)
        assert lat > 0
        _check_vectors(vecs, ids, lens)
    srv.close()
    jobs, _ = emb.counts()
    assert all(j > 0 for j in jobs)  # both replicas served batches
    emb.close()


def test_in_flight_cap_and_growing_batches():
    emb = embedder.Embedder.fake(1, delay_us=50000)
    srv = embedder.Server(emb, max_in_flight=100, jobs_per_replica=1)
    reqs = _requests(120, seed=1)
    futs = [srv.submit(*r) for r in reqs]
    for f in futs:
        f.result(timeout=60)
    st = srv.stats()
    srv.close()
    emb.close()
    assert st["max_busy"] <= 100
    assert st["completed"] == st["requests"] == 120
    # One replica taking one batch at a time: requests that arrive meanwhile join the next batch,
    # so the backlog goes out in a few large batches rather than one batch per request.
    assert st["batches"] < len(reqs) / 4


def test_arrival_time_counts_in_latency():
    emb = embedder.Embedder.fake(1)
    srv = embedder.Server(emb)
    ids, lens = _requests(1)[0]
    t0 = time.perf_counter() - 0.5  # scheduled half a second ago
    _, lat = srv.submit(ids, lens, arrival=t0).result(timeout=10)
    assert 0.5 <= lat < 5
    srv.close()
    emb.close()


def test_budget_is_shared_by_the_replicas():
    """Under a saturating load every replica holds work at once: no batch of two or more
    requests takes more than its share of the in-flight budget."""
    emb = embedder.Embedder.fake(4, delay_us=20000)
    srv = embedder.Server(emb, max_in_flight=64, jobs_per_replica=2)
    reqs = _requests(300, seed=2)
    futs = [srv.submit(*r) for r in reqs]
    for f in futs:
        f.result(timeout=60)
    st = srv.stats()
    srv.close()
    jobs, _ = emb.counts()
    emb.close()
    assert st["max_batch_seqs"] <= 64 // 8
    assert st["max_busy"] <= 64 or st["max_request_seqs"] > 64
    assert all(j > 0 for j in jobs)


def test_packed_submission_and_latencies():
    """Many requests in one call (the open-loop load path): vectors land at their rows of one
    output array, every ticket gets a latency, and drain() waits for all of them."""
    emb = embedder.Embedder.fake(3, delay_us=1000)
    srv = embedder.Server(emb, max_in_flight=128)
    reqs = _requests(500, seed=3)
    ids = np.concatenate([r[0] for r in reqs])
    lens = np.concatenate([r[1] for r in reqs])
    seq_off = np.concatenate([[0], np.cumsum([len(r[1]) for r in reqs])]).astype(np.int64)
    out = np.zeros((int(seq_off[-1]), 4), np.float32)
    now = srv.clock_ns()
    arrival = now + np.arange(len(reqs), dtype=np.int64) * 1000
    first = srv.submit_packed(ids, lens, seq_off, out, arrival)
    srv.drain()
    lat = srv.latencies(first, len(reqs))
    assert np.all(np.isfinite(lat)) and np.all(lat > 0)
    _check_vectors(out, ids, lens)
    srv.close()
    emb.close()


def test_failed_batch_fails_its_requests_only():
    """A batch that fails (here a negative id, as an out-of-range id fails a model's batch) fails
    every request in it with the replica's message; later requests still complete."""
    emb = embedder.Embedder.fake(1, delay_us=0)
    srv = embedder.Server(emb, jobs_per_replica=1)
    bad = srv.submit(np.array([-5, 1, 2], np.int32), np.array([3], np.int32))
    with pytest.raises(fletcher.FletcherError, match="negative id"):
        bad.result(timeout=10)
    ids, lens = _requests(1, seed=9)[0]
    vecs, _ = srv.submit(ids, lens).result(timeout=10)
    _check_vectors(vecs, ids, lens)
    srv.close()
    emb.close()


def test_concurrent_submitters():
    emb = embedder.Embedder.fake(2, delay_us=2000)
    srv = embedder.Server(emb, max_in_flight=256)
    reqs = _requests(400, seed=5)
    with cf.ThreadPoolExecutor(8) as ex:
        futs = list(ex.map(lambda r: srv.submit(*r), reqs))
    srv.close()  # completes everything; the tickets keep their outcome
    for (ids, lens), f in zip(reqs, futs):
        vecs, lat = f.result(timeout=60)
        assert lat > 0
        _check_vectors(vecs, ids, lens)
    emb.close()
