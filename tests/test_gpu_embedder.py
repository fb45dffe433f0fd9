"""GPU tests of the native multi-replica embedder and request server (csrc/runtime.cu through
embedder.py).  Two replicas share GPU 0 here; the split, batching and reassembly logic is the same
as across GPUs."""
import concurrent.futures as cf
import dataclasses

import numpy as np
import pytest

import synth
from helpers import assert_close_16

pytestmark = pytest.mark.gpu

CFG = dataclasses.replace(synth.NOMIC, num_layers=2)


@pytest.fixture(scope="module")
def emb():
    import build
    build.build()
    import embedder
    e = embedder.Embedder(CFG, synth.make_weights(CFG, 1), devices=[0, 0], dtype="bf16", max_batch=7,
                          max_tokens=900)
    yield e
    e.close()


def _direct(e, ids, lens):  # called while the replicas are idle
    return e.replicas[0].model.forward_batch(ids, lens, 1)


def test_embed_matches_single_replica(emb):
    lens = synth.make_lengths(40, 8, 300, 5, "loguniform")
    ids = synth.make_ids(lens, CFG.vocab_size, 5)
    want = _direct(emb, ids, lens)
    emb.set_throughput([3.0, 1.0])  # uneven split
    got = emb.embed(ids, lens)
    # Packing- and batching-invariant up to the fp32 summation order of small batches' split-K
    # GEMMs (their number of partial sums depends on the batch's token count).
    assert_close_16(got, want, "replicas vs one replica", cos_min=0.99999)


def test_server_requests(emb):
    import embedder
    srv = embedder.Server(emb, max_in_flight=64)
    rng = np.random.default_rng(3)
    reqs = []
    for i in range(60):
        lens = synth.make_lengths(int(rng.integers(1, 17)), 8, 200, 100 + i, "loguniform")
        reqs.append((synth.make_ids(lens, CFG.vocab_size, 100 + i), lens))
    with cf.ThreadPoolExecutor(8) as ex:
        futs = list(ex.map(lambda r: srv.submit(*r), reqs))
    srv.close()
    for (ids, lens), f in zip(reqs, futs):
        vecs, lat = f.result(timeout=60)
        assert lat > 0 and vecs.shape == (len(lens), CFG.hidden)
        assert_close_16(vecs, _direct(emb, ids, lens), "served vs direct", cos_min=0.99999)


def test_server_packed_open_loop(emb):
    """The bench's path: many requests per submission with scheduled arrivals; vectors land in
    their rows and every request has a latency."""
    import embedder
    srv = embedder.Server(emb, max_in_flight=128)
    rng = np.random.default_rng(8)
    reqs = []
    for i in range(40):
        lens = synth.make_lengths(int(rng.integers(1, 17)), 8, 200, 300 + i, "loguniform")
        reqs.append((synth.make_ids(lens, CFG.vocab_size, 300 + i), lens))
    ids = np.concatenate([r[0] for r in reqs])
    lens = np.concatenate([r[1] for r in reqs]).astype(np.int32)
    seq_off = np.concatenate([[0], np.cumsum([len(r[1]) for r in reqs])]).astype(np.int64)
    out = np.zeros((int(seq_off[-1]), CFG.hidden), np.float32)
    arrival = srv.clock_ns() + np.arange(len(reqs), dtype=np.int64) * 100000
    first = srv.submit_packed(ids, lens, seq_off, out, arrival)
    srv.drain()
    lat = srv.latencies(first, len(reqs))
    srv.close()
    assert np.all(np.isfinite(lat))
    for r, (i_, l_) in enumerate(reqs):
        assert_close_16(out[seq_off[r]:seq_off[r + 1]], _direct(emb, i_, l_), "packed vs direct", cos_min=0.99999)


def test_bad_id_fails_the_request(emb):
    import embedder
    import fletcher
    srv = embedder.Server(emb)
    t = srv.submit(np.array([101, CFG.vocab_size + 5, 102], np.int32), np.array([3], np.int32))
    with pytest.raises(fletcher.FletcherError, match="out of bounds"):
        t.result(timeout=60)
    lens = np.array([5, 9], np.int32)
    ids = synth.make_ids(lens, CFG.vocab_size, 77)
    vecs, _ = srv.submit(ids, lens).result(timeout=60)
    srv.close()
    assert_close_16(vecs, _direct(emb, ids, lens), "after a failed request", cos_min=0.99999)
