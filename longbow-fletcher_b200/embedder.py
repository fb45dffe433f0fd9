"""Multi-GPU embedder and request server: Python handles on the library's native host runtime
(Cuda_Embedder_* / Cuda_Server_*, csrc/runtime.cu), the restatement of the reference's Embedder
(internal/embeddings/embeddings.go) and of its server's in-flight cap (server.go:101).

Embedder: one model replica per GPU.  The runtime gives each replica a host thread that keeps
two device batches in flight (Cuda_Model_ForwardBatchAsync into pinned buffers), splits a
request across replicas by token count weighted by each replica's measured throughput
(embeddings.go:436-501) and cuts each share into dynamic batches of at most `max_batch`
sequences / `max_tokens` tokens (embeddings.go:704-731).  Sequences are independent, so no
collective is involved.

Server: a request queue in front of the replicas.  The native batcher joins queued requests into
batches under the in-flight budget (16384 sequences by default) and hands them round-robin to
replicas holding fewer than `jobs_per_replica` batches; every request gets its vectors and its
latency.  No Python runs per request inside the runtime.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np

import fletcher
import synth

_i64p = ctypes.POINTER(ctypes.c_int64)
_f64p = ctypes.POINTER(ctypes.c_double)


class ServerStats(ctypes.Structure):
    _fields_ = [("requests", ctypes.c_int64), ("completed", ctypes.c_int64), ("batches", ctypes.c_int64),
                ("max_batch_seqs", ctypes.c_int64), ("max_request_seqs", ctypes.c_int64),
                ("max_busy", ctypes.c_int64)]


class Replica:
    """One GPU's backend and model (the runtime drives it; direct calls only while it is idle)."""

    def __init__(self, device, cfg, blob, dtype):
        self.device = device
        self.be = fletcher.Backend(device, dtype)
        self.model = fletcher.BertModel(self.be, cfg, dtype)
        self.model.load_raw(blob)

    def close(self):
        self.model.close()
        self.be.close()


class Embedder:
    def __init__(self, cfg: synth.BertConfig, blob, devices=None, dtype="bf16", pooling=fletcher.POOL_MEAN_L2,
                 max_batch=512, max_tokens=None, _fake=None):
        L = fletcher.lib()
        h = ctypes.c_void_p()
        self.cfg = cfg
        if _fake is not None:  # CPU test double: (replicas, hidden, delay_us)
            n, hidden, delay_us = _fake
            self.replicas = []
            self._check(L.Cuda_Embedder_CreateFake(n, hidden, delay_us, max_batch, max_tokens or 0, ctypes.byref(h)))
            self.n = n
        else:
            n = L.Cuda_GetDeviceCount()
            devices = list(range(n)) if devices is None else list(devices)
            if not devices:
                raise fletcher.FletcherError(-1, "no CUDA device")
            self.replicas = [Replica(d, cfg, blob, dtype) for d in devices]
            self.n = len(self.replicas)
            models = (ctypes.c_void_p * self.n)(*[r.model.h.value for r in self.replicas])
            # max_tokens None: the reference's VRAM-dependent budget (65536 tokens per batch on
            # devices with >= 64 GB, else 16384; embeddings.go:177-190), chosen by the runtime.
            self._check(L.Cuda_Embedder_Create(models, self.n, pooling, max_batch, max_tokens or 0, ctypes.byref(h)))
        self.h = h
        mb, mt = ctypes.c_int32(), ctypes.c_int64()
        L.Cuda_Embedder_MaxBatch(self.h, ctypes.byref(mb), ctypes.byref(mt))
        self.max_batch, self.max_tokens = mb.value, mt.value
        self.hidden = L.Cuda_Embedder_Hidden(self.h)

    @classmethod
    def fake(cls, n, hidden=4, delay_us=0, max_batch=512, max_tokens=65536):
        """Replicas with no GPU: sequence i of a batch gets (first id, length, replica, 0, ...)."""
        return cls(None, None, max_batch=max_batch, max_tokens=max_tokens, _fake=(n, hidden, delay_us))

    def _check(self, rc):
        if rc != 0:
            raise fletcher.FletcherError(rc, self.last_error() if getattr(self, "h", None) else "embedder")

    def last_error(self):
        buf = ctypes.create_string_buffer(1024)
        fletcher.lib().Cuda_Embedder_LastError(self.h, buf, len(buf))
        return buf.value.decode(errors="replace")

    def embed(self, ids, lengths):
        """Packed ids ([CLS] ... [SEP] per sequence) and lengths -> [B, H] in request order."""
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((lens.size, self.hidden), np.float32)
        self._check(fletcher.lib().Cuda_Embedder_Embed(self.h, fletcher._i32p(ids), fletcher._i32p(lens), lens.size,
                                                       fletcher._f32p(out)))
        return out

    def throughput(self):
        t = np.zeros(self.n, np.float64)
        self._check(fletcher.lib().Cuda_Embedder_Throughput(self.h, t.ctypes.data_as(_f64p), self.n, 0))
        return t

    def set_throughput(self, values):
        t = np.ascontiguousarray(values, np.float64)
        self._check(fletcher.lib().Cuda_Embedder_Throughput(self.h, t.ctypes.data_as(_f64p), self.n, 1))

    def counts(self):
        """(batches handed to each replica, their sequences)."""
        jobs, seqs = np.zeros(self.n, np.int64), np.zeros(self.n, np.int64)
        self._check(fletcher.lib().Cuda_Embedder_Counts(self.h, jobs.ctypes.data_as(_i64p), seqs.ctypes.data_as(_i64p),
                                                        self.n))
        return jobs, seqs

    def close(self):
        if self.h:
            fletcher.lib().Cuda_Embedder_Destroy(self.h)
            self.h = None
        for r in self.replicas:
            r.close()
        self.replicas = []


class Ticket:
    """A submitted request: result() -> (vectors [n, H] float32, latency in seconds)."""

    def __init__(self, srv, ticket, out):
        self.srv, self.ticket, self.out = srv, ticket, out

    def result(self, timeout=None):
        if self.srv.h is None:  # the server was closed: every request completed before that
            lat_s = self.srv._final.get(self.ticket)
            if lat_s is None:
                raise fletcher.FletcherError(-1, self.srv._final_err or f"request {self.ticket}: result unavailable")
            return self.out, lat_s
        lat = ctypes.c_int64()
        rc = fletcher.lib().Cuda_Server_Wait(self.srv.h, self.ticket, -1.0 if timeout is None else float(timeout),
                                             ctypes.byref(lat))
        if rc == -1:
            raise TimeoutError(f"request {self.ticket} not complete after {timeout} s")
        self.srv._keep.pop(self.ticket, None)
        if rc != 0:
            raise fletcher.FletcherError(rc, self.srv.emb.last_error())
        return self.out, lat.value * 1e-9


class Server:
    """Request queue + dynamic batcher + round-robin dispatch to the replicas (native)."""

    def __init__(self, embedder: Embedder, max_in_flight=16384, jobs_per_replica=2):
        self.emb = embedder
        h = ctypes.c_void_p()
        rc = fletcher.lib().Cuda_Server_Create(embedder.h, max_in_flight, jobs_per_replica, ctypes.byref(h))
        if rc:
            raise fletcher.FletcherError(rc, "Cuda_Server_Create")
        self.h = h
        self._keep = {}  # output arrays of requests whose result() was not read yet
        self._final, self._final_err = {}, ""  # outcomes kept at close()
        # The runtime's clock against time.perf_counter, for arrival times given as perf_counter values.
        self._off = fletcher.lib().Cuda_Server_Clock() - time.perf_counter_ns()

    def clock_ns(self):
        return fletcher.lib().Cuda_Server_Clock()

    def submit(self, ids, lengths, arrival=None):
        """One request; latency runs from `arrival` (a time.perf_counter() value, e.g. a request's
        scheduled arrival in an open-loop load) or from this call.  Returns a Ticket."""
        lens = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((lens.size, self.emb.hidden), np.float32)
        arr = None if arrival is None else np.array([int(arrival * 1e9) + self._off], np.int64)
        first = self.submit_packed(ids, lens, np.array([0, lens.size], np.int64), out, arr)
        self._keep[first] = out  # the runtime writes into it until the request completes
        return Ticket(self, first, out)

    def submit_packed(self, ids, lengths, seq_off, out, arrival_ns=None):
        """n = len(seq_off) - 1 requests at once: request r holds sequences seq_off[r] ..
        seq_off[r+1]-1 (ids packed in order) and its vectors go to out[seq_off[r]:seq_off[r+1]].
        `out` must stay alive until the requests complete.  arrival_ns: per-request arrival on the
        runtime's clock (clock_ns()).  Returns the first ticket (the rest follow consecutively)."""
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lengths, np.int32)
        so = np.ascontiguousarray(seq_off, np.int64)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.shape[0] >= so[-1]
        arr = None if arrival_ns is None else np.ascontiguousarray(arrival_ns, np.int64)
        first = ctypes.c_int64()
        rc = fletcher.lib().Cuda_Server_Submit(self.h, so.size - 1, fletcher._i32p(ids), fletcher._i32p(lens),
                                               so.ctypes.data_as(_i64p),
                                               None if arr is None else arr.ctypes.data_as(_i64p),
                                               fletcher._f32p(out), ctypes.byref(first))
        if rc:
            raise fletcher.FletcherError(rc, "Cuda_Server_Submit")
        return first.value

    def latencies(self, first, n):
        """Seconds per ticket first .. first+n-1 (nan: not complete or failed)."""
        lat = np.zeros(n, np.int64)
        fletcher.lib().Cuda_Server_Latencies(self.h, first, n, lat.ctypes.data_as(_i64p))
        out = lat.astype(np.float64) * 1e-9
        out[lat < 0] = np.nan
        return out

    def drain(self):
        fletcher.lib().Cuda_Server_Drain(self.h)

    def stats(self):
        st = ServerStats()
        fletcher.lib().Cuda_Server_Stats(self.h, ctypes.byref(st))
        return {k: getattr(st, k) for k, _ in ServerStats._fields_}

    def close(self):
        """Completes every submitted request, then stops the batcher.  Tickets whose result() was
        not read yet keep their outcome."""
        if self.h:
            self.drain()
            for t in self._keep:
                lat = self.latencies(t, 1)[0]
                self._final[t] = None if np.isnan(lat) else float(lat)
            if any(v is None for v in self._final.values()):
                self._final_err = self.emb.last_error()
            fletcher.lib().Cuda_Server_Destroy(self.h)
            self.h = None
        self._keep.clear()
