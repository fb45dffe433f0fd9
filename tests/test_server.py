"""CPU tests of the request batcher (embedder.Server) with fake replicas: the in-flight sequence
cap (the reference server's semaphore, server.go:101), round-robin dispatch, request order and
latency bookkeeping, and batches that grow with the load while the replicas are busy."""
import concurrent.futures as cf
import threading
import time

import numpy as np

import embedder


class FakeReplica:
    def __init__(self, hidden, delay, log, lock):
        self.hidden, self.delay, self.log, self.lock = hidden, delay, log, lock

    def run(self, ids, lengths, max_batch, max_tokens):
        fut = cf.Future()
        with self.lock:
            self.log.append((self, len(lengths)))

        def done():
            time.sleep(self.delay)
            # vector i carries (its first id, its length) so the caller can check the order
            out = np.zeros((len(lengths), self.hidden), np.float32)
            off = 0
            for i, l in enumerate(lengths):
                out[i, 0], out[i, 1] = ids[off], l
                off += l
            fut.set_result(out)
        threading.Thread(target=done, daemon=True).start()
        return fut


class FakeEmbedder:
    def __init__(self, n, delay):
        self.log, self.lock = [], threading.Lock()
        self.replicas = [FakeReplica(4, delay, self.log, self.lock) for _ in range(n)]
        self.max_batch, self.max_tokens = 512, 65536


def _requests(n, seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        k = int(rng.integers(1, 17))
        lens = rng.integers(8, 64, size=k).astype(np.int32)
        ids = np.arange(int(lens.sum()), dtype=np.int32) + 2000 * i
        out.append((ids, lens))
    return out


def test_server_returns_each_request_its_vectors():
    emb = FakeEmbedder(2, 0.005)
    srv = embedder.Server(emb, max_in_flight=64)
    reqs = _requests(200)
    futs = [srv.submit(*r) for r in reqs]
    for (ids, lens), f in zip(reqs, futs):
        vecs, lat = f.result(timeout=30)
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        assert lat > 0
        np.testing.assert_array_equal(vecs[:, 0], ids[starts])
        np.testing.assert_array_equal(vecs[:, 1], lens)
    srv.close()
    used = {id(r) for r, _ in emb.log}
    assert used == {id(r) for r in emb.replicas}  # both replicas served batches


def test_in_flight_cap_and_growing_batches():
    emb = FakeEmbedder(1, 0.05)
    srv = embedder.Server(emb, max_in_flight=100, jobs_per_replica=1)
    reqs = _requests(120, seed=1)
    futs = [srv.submit(*r) for r in reqs]
    for f in futs:
        f.result(timeout=60)
    srv.close()
    sizes = [n for _, n in emb.log]
    assert max(sizes) <= 100 or all(n <= 16 for n in sizes)  # a single request may exceed it alone
    # One replica taking one batch at a time: requests that arrive meanwhile join the next batch,
    # so the backlog goes out in a few large batches rather than one batch per request.
    assert len(sizes) < len(reqs) / 4


def test_arrival_time_counts_in_latency():
    emb = FakeEmbedder(1, 0.0)
    srv = embedder.Server(emb)
    ids, lens = _requests(1)[0]
    t0 = time.perf_counter() - 0.5  # scheduled half a second ago
    _, lat = srv.submit(ids, lens, arrival=t0).result(timeout=10)
    assert lat >= 0.5
    srv.close()


def test_budget_is_shared_by_the_replicas():
    """Under a saturating load every replica holds work at once: no single batch takes more than
    its share of the in-flight budget."""
    emb = FakeEmbedder(4, 0.02)
    srv = embedder.Server(emb, max_in_flight=64, jobs_per_replica=2)
    reqs = _requests(300, seed=2)
    futs = [srv.submit(*r) for r in reqs]
    for f in futs:
        f.result(timeout=60)
    srv.close()
    assert max(n for _, n in emb.log) <= max(64 // 8, 16)  # one request may exceed the share alone
    assert {id(r) for r, _ in emb.log} == {id(r) for r in emb.replicas}
