"""Multi-GPU embedder and request batcher on top of the C ABI (the reference's Embedder,
internal/embeddings/embeddings.go).

Embedder.embed: one model replica per GPU, each driven by its own host thread (ctypes releases
the GIL during library calls, so the replicas run concurrently).  Each replica keeps two device
batches in flight (Cuda_Model_ForwardBatchAsync with pinned buffers), so host work overlaps the
device.  A request is split across
replicas by token count weighted by each replica's measured throughput (embeddings.go:436-501),
each replica cuts its share into dynamic batches of at most `max_batch` sequences /
`max_tokens` tokens (embeddings.go:704-731), and the vectors come back in request order.
Sequences are independent, so no collective is involved.

Server: a request queue in front of the replicas — the batcher drains pending requests into a
batch capped at `max_in_flight` sequences (server.go's sequence semaphore, 16384 by default) and
hands batches to the replicas round-robin; every request gets its vectors and its latency.
"""
from __future__ import annotations

import collections
import concurrent.futures as cf
import queue
import threading
import time

import numpy as np

import fletcher
import replicas
import synth


class _Job:
    """One run() call: its device batches, output rows and future."""

    def __init__(self, ids, lengths, max_batch, max_tokens, hidden):
        self.ids, self.lengths = ids, lengths
        self.cu = np.concatenate([[0], np.cumsum(lengths)])
        self.todo = collections.deque(replicas.dynamic_batches(lengths, max_batch, max_tokens))
        self.pending = len(self.todo)  # device batches not yet collected
        self.out = np.zeros((len(lengths), hidden), np.float32)
        self.error = None
        self.future = cf.Future()
        self.t0 = time.perf_counter()


class Replica:
    """One GPU: its own context, model and worker thread.

    The worker keeps two device batches in flight (Cuda_Model_ForwardBatchAsync with pinned
    ids and vectors): while the device runs batch k+1, the host stages the next batch and
    collects batch k, across run() calls as well as within one.  run() returns a future."""

    def __init__(self, device, cfg, blob, dtype, pooling):
        self.device = device
        self.pooling = pooling
        self.throughput = 0.0  # sequences/s, exponential moving average (embeddings.go GPUMetrics)
        self.slots = [(None, None), (None, None)]  # pinned ids / vectors of the two in-flight batches
        self.jobs = queue.Queue()
        ready = cf.Future()
        self.thread = threading.Thread(target=self._loop, args=(cfg, blob, dtype, ready), daemon=True)
        self.thread.start()
        ready.result()

    def _slot(self, k, n_ids, n_seq):
        """Pinned staging buffers of in-flight slot k (grown when a batch does not fit)."""
        ids_buf, out_buf = self.slots[k]
        if ids_buf is None or ids_buf.array.size < n_ids:
            if ids_buf is not None:
                ids_buf.close()
            ids_buf = fletcher.PinnedArray(self.be, (max(n_ids, 1 << 14),), np.int32)
        if out_buf is None or out_buf.array.shape[0] < n_seq:
            if out_buf is not None:
                out_buf.close()
            out_buf = fletcher.PinnedArray(self.be, (max(n_seq, 64), self.model.cfg.hidden), np.float32)
        self.slots[k] = (ids_buf, out_buf)
        return ids_buf, out_buf

    def _finish(self, job):
        if job.error is not None:
            job.future.set_exception(job.error)
            return
        dt = time.perf_counter() - job.t0
        if dt > 0 and len(job.lengths):
            r = len(job.lengths) / dt
            self.throughput = r if self.throughput == 0 else 0.8 * self.throughput + 0.2 * r
        job.future.set_result(job.out)

    def _loop(self, cfg, blob, dtype, ready):
        try:
            self.be = fletcher.Backend(self.device, dtype)
            self.model = fletcher.BertModel(self.be, cfg, dtype)
            self.model.load_raw(blob)
        except Exception as e:  # noqa: BLE001 - reported to the constructor
            ready.set_exception(e)
            return
        ready.set_result(None)
        todo = collections.deque()      # jobs with device batches left to enqueue
        inflight = collections.deque()  # (ticket, slot, job, a, b)
        nslot = 0
        stop = False
        while not stop or todo or inflight:
            if not stop:
                try:
                    job = self.jobs.get(block=not (todo or inflight))
                    if job is None:
                        stop = True
                    else:
                        todo.append(job)
                    continue
                except queue.Empty:
                    pass
            if todo and len(inflight) < len(self.slots):
                job = todo[0]
                a, b = job.todo.popleft()
                if not job.todo:
                    todo.popleft()
                k = nslot % len(self.slots)  # FIFO collection frees slots in this order
                nslot += 1
                ticket = None
                if job.error is None:
                    try:
                        ids_buf, out_buf = self._slot(k, int(job.cu[b] - job.cu[a]), b - a)
                        ids_buf.array[:job.cu[b] - job.cu[a]] = job.ids[job.cu[a]:job.cu[b]]
                        ticket = self.model.forward_batch_async(ids_buf.ptr, job.lengths[a:b], self.pooling,
                                                                out_buf.ptr)
                    except Exception as e:  # noqa: BLE001 - the reference fails the whole request
                        job.error = e
                inflight.append((ticket, k, job, a, b))
            elif inflight:
                ticket, k, job, a, b = inflight.popleft()
                if ticket is not None:
                    try:
                        self.model.wait(ticket)
                        if job.error is None:
                            job.out[a:b] = self.slots[k][1].array[:b - a]
                    except Exception as e:  # noqa: BLE001
                        job.error = e
                job.pending -= 1
                if job.pending == 0:
                    self._finish(job)
        for bufs in self.slots:
            for buf in bufs:
                if buf is not None:
                    buf.close()
        self.model.close()
        self.be.close()

    def run(self, ids, lengths, max_batch, max_tokens):
        """Embeds packed (ids, lengths) in dynamic batches; a future of [B, H] float32."""
        job = _Job(ids, np.asarray(lengths), max_batch, max_tokens, self.model.cfg.hidden)
        if job.pending == 0:
            job.future.set_result(job.out)
        else:
            self.jobs.put(job)
        return job.future

    def close(self):
        self.jobs.put(None)
        self.thread.join()


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

    def __init__(self, embedder: Embedder, max_in_flight=16384, jobs_per_replica=2):
        self.emb = embedder
        self.max_in_flight = max_in_flight
        # A replica takes a new batch only while it holds fewer than this many: requests that
        # arrive meanwhile wait and join one larger batch, so batches grow with the load instead
        # of fragmenting into many small device batches.
        self.jobs_per_replica = jobs_per_replica
        self.q = queue.Queue()
        self.rr = 0
        self.stop = False
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, ids, lengths, arrival=None):
        """Returns a Future resolving to (vectors [n, H], latency seconds).  Latency runs from
        `arrival` (a time.perf_counter() value, e.g. a request's scheduled arrival in an
        open-loop load) or from this call."""
        fut = cf.Future()
        t0 = time.perf_counter() if arrival is None else arrival
        self.q.put((t0, np.asarray(ids, np.int32), np.asarray(lengths, np.int32), fut))
        return fut

    def _loop(self):
        """Drains the queue into batches of at most the free in-flight budget (sequences handed to
        the replicas and not yet returned stay below max_in_flight, as the reference's server
        semaphore caps them, server.go:101) and dispatches them round-robin."""
        inflight = []  # (replica future, [requests], sequences, replica index)
        held = collections.deque()  # requests taken off the queue, not yet dispatched
        busy = 0
        nrep = len(self.emb.replicas)
        jobs = [0] * nrep
        # One batch takes at most its replica's share of the in-flight budget, so that every
        # replica can hold work at once under the cap.
        share = max(1, self.max_in_flight // (nrep * self.jobs_per_replica))
        while not self.stop or not self.q.empty() or held:
            if not held:
                try:
                    held.append(self.q.get(timeout=0.002 if inflight else 0.01))
                except queue.Empty:
                    pass
            while True:  # everything queued now, so that one batch takes it all
                try:
                    held.append(self.q.get_nowait())
                except queue.Empty:
                    break
            # The next replica in round-robin order with room for another batch.
            rep = None
            for k in range(nrep):
                i = (self.rr + k) % nrep
                if jobs[i] < self.jobs_per_replica:
                    rep = i
                    break
            reqs, nseq = [], 0

            def fits(n):
                if not reqs:  # a batch's first request: within the budget, or alone when nothing runs
                    return busy + n <= self.max_in_flight or busy == 0
                return busy + nseq + n <= self.max_in_flight and nseq + n <= share

            while rep is not None and held and fits(len(held[0][2])):
                r = held.popleft()
                reqs.append(r)
                nseq += len(r[2])
            if reqs:
                self.rr = rep + 1
                ids = np.concatenate([r[1] for r in reqs])
                lens = np.concatenate([r[2] for r in reqs])
                fut = self.emb.replicas[rep].run(ids, lens, self.emb.max_batch, self.emb.max_tokens)
                inflight.append((fut, reqs, nseq, rep))
                busy += nseq
                jobs[rep] += 1
            done = [x for x in inflight if x[0].done()]
            if done:
                inflight = [x for x in inflight if not x[0].done()]
                for f, rq, n, i in done:
                    busy -= n
                    jobs[i] -= 1
                    self._finish(f, rq)
            elif inflight and held and not reqs:
                cf.wait([x[0] for x in inflight], timeout=0.01, return_when=cf.FIRST_COMPLETED)
        for f, rq, _, _ in inflight:
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
