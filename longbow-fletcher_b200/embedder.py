"""Multi-GPU embedder and request batcher on top of the C ABI (the reference's Embedder,
internal/embeddings/embeddings.go).

Embedder.embed: one model replica per GPU, each driven by its own host thread (ctypes releases
the GIL during library calls, so the replicas run concurrently).  A request is split across
replicas by token count weighted by each replica's measured throughput (embeddings.go:436-501),
each replica cuts its share into dynamic batches of at most `max_batch` sequences /
`max_tokens` tokens (embeddings.go:704-731), and the vectors come back in request order.
Sequences are independent, so no collective is involved.

Server: a request queue in front of the replicas — the batcher drains pending requests into a
batch capped at `max_in_flight` sequences (server.go's sequence semaphore, 16384 by default) and
hands batches to the replicas round-robin; every request gets its vectors and its latency.
"""
from __future__ import annotations

import concurrent.futures as cf
import queue
import threading
import time

import numpy as np

import fletcher
import replicas
import synth


class Replica:
    """One GPU: its own context, model and worker thread."""

    def __init__(self, device, cfg, blob, dtype, pooling):
        self.pool = cf.ThreadPoolExecutor(max_workers=1)
        self.device = device
        self.pooling = pooling
        self.throughput = 0.0  # sequences/s, exponential moving average (embeddings.go GPUMetrics)

        def init():
            self.be = fletcher.Backend(device, dtype)
            self.model = fletcher.BertModel(self.be, cfg, dtype)
            self.model.load_raw(blob)

        self.pool.submit(init).result()

    def run(self, ids, lengths, max_batch, max_tokens):
        """Embeds packed (ids, lengths) in dynamic batches; returns [B, H] float32."""
        def work():
            t0 = time.perf_counter()
            out = []
            cu = np.concatenate([[0], np.cumsum(lengths)])
            for a, b in replicas.dynamic_batches(lengths, max_batch, max_tokens):
                out.append(self.model.forward_batch(ids[cu[a]:cu[b]], lengths[a:b], self.pooling))
            dt = time.perf_counter() - t0
            if dt > 0 and len(lengths):
                r = len(lengths) / dt
                self.throughput = r if self.throughput == 0 else 0.8 * self.throughput + 0.2 * r
            return np.concatenate(out) if out else np.zeros((0, self.model.cfg.hidden), np.float32)
        return self.pool.submit(work)

    def close(self):
        def fin():
            self.model.close()
            self.be.close()
        self.pool.submit(fin).result()
        self.pool.shutdown()


class Embedder:
    def __init__(self, cfg: synth.BertConfig, blob, devices=None, dtype="bf16", pooling=fletcher.POOL_MEAN_L2,
                 max_batch=512, max_tokens=None):
        n = fletcher.lib().Cuda_GetDeviceCount()
        devices = list(range(n)) if devices is None else list(devices)
        if not devices:
            raise fletcher.FletcherError(-1, "no CUDA device")
        self.cfg = cfg
        self.replicas = [Replica(d, cfg, blob, dtype, pooling) for d in devices]
        if max_tokens is None:
            # The reference's Linux GPU default is 16384 tokens per device batch, "VRAM dependent"
            # (embeddings.go:177-190).  On devices with 64 GB or more (a B200 has 180 GB) the
            # budget is 65536 tokens: about 1 GB of workspace, and batches that keep the GEMMs
            # efficient.
            total = min(r.be.vram_usage()[1] for r in self.replicas)
            max_tokens = 65536 if total >= 64 << 30 else 16384
        self.max_batch, self.max_tokens = max_batch, max_tokens

    def embed(self, ids, lengths):
        """Packed ids ([CLS] ... [SEP] per sequence) and lengths -> [B, H] in request order."""
        lengths = np.ascontiguousarray(lengths, np.int32)
        ids = np.ascontiguousarray(ids, np.int32)
        ranges = replicas.split_by_weight(lengths, [r.throughput for r in self.replicas])
        rows = replicas.shard_rows(lengths, ranges)
        futs = [r.run(ids[t0:t1], lengths[a:b], self.max_batch, self.max_tokens)
                for r, (a, b), (t0, t1) in zip(self.replicas, ranges, rows)]
        parts = [f.result() for f in futs]
        return np.concatenate(parts) if parts else np.zeros((0, self.cfg.hidden), np.float32)

    def close(self):
        for r in self.replicas:
            r.close()


class Server:
    """Request queue + dynamic batcher + round-robin dispatch to the replicas."""

    def __init__(self, embedder: Embedder, max_in_flight=16384):
        self.emb = embedder
        self.max_in_flight = max_in_flight
        self.q = queue.Queue()
        self.rr = 0
        self.stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, ids, lengths):
        """Returns a Future resolving to (vectors [n, H], latency seconds)."""
        fut = cf.Future()
        self.q.put((time.perf_counter(), np.asarray(ids, np.int32), np.asarray(lengths, np.int32), fut))
        return fut

    def _loop(self):
        inflight = []  # (replica future, [requests])
        while not self.stop or not self.q.empty():
            reqs, nseq = [], 0
            try:
                reqs.append(self.q.get(timeout=0.01))
                nseq = len(reqs[0][2])
            except queue.Empty:
                pass
            while reqs and nseq < self.max_in_flight:
                try:
                    r = self.q.get_nowait()
                except queue.Empty:
                    break
                reqs.append(r)
                nseq += len(r[2])
            if reqs:
                rep = self.emb.replicas[self.rr % len(self.emb.replicas)]
                self.rr += 1
                ids = np.concatenate([r[1] for r in reqs])
                lens = np.concatenate([r[2] for r in reqs])
                inflight.append((rep.run(ids, lens, self.emb.max_batch, self.emb.max_tokens), reqs))
            done = [x for x in inflight if x[0].done()]
            inflight = [x for x in inflight if not x[0].done()]
            for f, rq in done:
                self._finish(f, rq)
        for f, rq in inflight:
            self._finish(f, rq)

    @staticmethod
    def _finish(f, reqs):
        now = time.perf_counter()
        try:
            vecs = f.result()
        except Exception as e:  # the reference fails the whole batch (embeddings.go:757-764)
            for r in reqs:
                r[3].set_exception(e)
            return
        off = 0
        for t0, _, lens, fut in reqs:
            fut.set_result((vecs[off:off + len(lens)], now - t0))
            off += len(lens)

    def close(self):
        self.stop = True
        self.thread.join()
