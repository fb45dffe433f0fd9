"""Python host binding of libcuda_fletcher.so (ctypes), mirroring the reference's Go device
interface for the embedding forward pass.

    Backend  ~ device.Backend  (internal/device/device.go:137-162)
    Tensor   ~ device.Tensor   (internal/device/device.go:5-117), the methods the hot path uses
    BertModel~ model.BertModel (internal/embeddings/model/bert.go:77-169) on the device

Every method calls the C ABI declared in include/fletcher_cuda.h; there is no CPU fallback:
if the library or a GPU is missing, construction raises.  Errors from the library raise
FletcherError carrying the library's message, the way the reference's Go wrapper panics
(cuda_linux.go:28-30).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

import synth

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcuda_fletcher.so")

F32, F16, BF16 = 0, 1, 2
ACT_IDENTITY, ACT_GELU, ACT_TANH, ACT_SOFTMAX, ACT_SWIGLU = 0, 1, 2, 3, 4
POOL_CLS_TANH, POOL_MEAN_L2 = 0, 1
HALF_REFERENCE, HALF_RNE = 0, 1
DTYPES = {"f32": F32, "f16": F16, "bf16": BF16}
_NP = {F32: np.float32, F16: np.float16}

_lib = None


class FletcherError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def _sig(L):
    vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
    i32p, i64p = ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)
    f32p = ctypes.POINTER(ctypes.c_float)
    sigs = {
        "Cuda_Init": (vp, []),
        "Cuda_GetDeviceCount": (i32, []),
        "Cuda_SetDevice": (i32, [vp, i32]),
        "Cuda_FreeContext": (None, [vp]),
        "Cuda_GetLastError": (i32, [vp, ctypes.c_char_p, i32]),
        "Cuda_Synchronize": (i32, [vp]),
        "Cuda_GetStream": (vp, [vp]),
        "Cuda_MemGetInfo": (i32, [vp, i64p, i64p]),
        "Cuda_Alloc": (vp, [vp, i64]),
        "Cuda_AllocTensor": (vp, [vp, i64, i64, i32]),
        "Cuda_FreeBuffer": (i32, [vp, vp]),
        "Cuda_CopyToDevice": (i32, [vp, i64, vp, i64]),
        "Cuda_CopyToHost": (i32, [vp, i64, vp, i64]),
        "Cuda_GetBufferContents": (vp, [vp]),
        "Cuda_BufferInfo": (i32, [vp, i64p, i64p, i32p]),
        "Cuda_CopyFromFloat32": (i32, [vp, f32p, i64]),
        "Cuda_ToHostFloat32": (i32, [vp, f32p, i64]),
        "Cuda_Linear_Fused": (i32, [vp, vp, i64, i64, vp, i64, vp, vp, i32]),
        "Cuda_LayerNorm": (i32, [vp, vp, vp, vp, vp, i64, i64, f32]),
        "Cuda_AddLayerNorm": (i32, [vp, vp, vp, vp, vp, i64, i64, f32]),
        "Cuda_Softmax": (i32, [vp, vp, vp, i64, i64]),
        "Cuda_Gather": (i32, [vp, vp, i32p, vp, i64, i64]),
        "Cuda_Add": (i32, [vp, vp, vp, i64]),
        "Cuda_Scale": (i32, [vp, vp, f32, i64]),
        "Cuda_AddScalar": (i32, [vp, vp, f32, i64]),
        "Cuda_AddBias": (i32, [vp, vp, vp, i64, i64]),
        "Cuda_Activation": (i32, [vp, vp, i64, i64, i32]),
        "Cuda_Cast": (i32, [vp, vp, vp, i64]),
        "Cuda_HasNaN": (i32, [vp, vp, i64, i32p]),
        "Cuda_Attention_Fused": (i32, [vp, vp, vp, vp, vp, i64, i64, i64, i32, f32]),
        "Cuda_Attention_VarLen": (i32, [vp, vp, vp, vp, vp, i32p, i32, i64, i32, f32]),
        "Cuda_Attention_VarLen_NoAlloc": (i32, [vp, vp, vp, vp, vp, i32p, i32, i64, i32, f32]),
        "Cuda_ApplyRoPE": (i32, [vp, vp, i64, i64, i32, i32]),
        "Cuda_ApplyRoPE_VarLen": (i32, [vp, vp, i32p, i32, i32, i32, f32]),
        "Cuda_MeanPoolL2": (i32, [vp, vp, i32p, i32, i64, vp]),
        "Cuda_Model_Create": (i32, [vp, vp, i32, ctypes.POINTER(vp)]),
        "Cuda_Model_LoadRaw": (i32, [vp, f32p, i64]),
        "Cuda_Model_WeightCount": (i64, [vp]),
        "Cuda_Model_ForwardBatch": (i32, [vp, i32p, i32p, i32, i32, f32p]),
        "Cuda_Model_ForwardBatchDevice": (i32, [vp, vp, i32p, i32, i32, vp]),
        "Cuda_Model_ForwardBatchEx": (i32, [vp, i32p, i32p, i32, i32, i32, vp]),
        "Cuda_Model_ForwardBatchAsync": (i32, [vp, vp, i32p, i32, i32, i32, vp, i64p]),
        "Cuda_Model_Wait": (i32, [vp, i64]),
        "Cuda_HostAlloc": (vp, [vp, i64]),
        "Cuda_HostFree": (None, [vp, vp]),
        "Cuda_Model_LastHidden": (i32, [vp, f32p, i64]),
        "Cuda_Model_SetStageTiming": (i32, [vp, i32]),
        "Cuda_Model_SetGraphs": (i32, [vp, i32]),
        "Cuda_Model_StageTimes": (i32, [vp, f32p, i64p, i32]),
        "Cuda_GetLaunchCount": (i64, [vp]),
        "Cuda_Debug_WaitTimeoutProbe": (i32, [vp, i64, i32]),
        "Cuda_Model_Free": (i32, [vp]),
        "Cuda_SetHalfConversion": (i32, [vp, i32]),
        "Cuda_Model_LoadTensor": (i32, [vp, ctypes.c_char_p, i32, vp, i64, i64, i32]),
        "Cuda_Model_TensorCount": (i32, [vp]),
        "Cuda_Model_TensorName": (i32, [vp, i32, ctypes.c_char_p, i32]),
        "Cuda_Model_IsLoaded": (i32, [vp]),
        "Cuda_Model_SetKeepHidden": (i32, [vp, i32]),
        "Cuda_At": (i32, [vp, i64, i64, f32p]),
        "Cuda_Set": (i32, [vp, i64, i64, f32]),
        "Cuda_Copy": (i32, [vp, vp, i64, vp, i64, i64]),
        "Cuda_Slice": (i32, [vp, vp, i64, i64, i64, i64, vp]),
        "Cuda_Mul": (i32, [vp, vp, i32, vp, i32, vp, i64, i64, i64]),
        "Cuda_Embedder_Create": (i32, [ctypes.POINTER(vp), i32, i32, i32, i64, ctypes.POINTER(vp)]),
        "Cuda_Embedder_CreateFake": (i32, [i32, i32, i64, i32, i64, ctypes.POINTER(vp)]),
        "Cuda_Embedder_Embed": (i32, [vp, i32p, i32p, i32, f32p]),
        "Cuda_Embedder_Throughput": (i32, [vp, ctypes.POINTER(ctypes.c_double), i32, i32]),
        "Cuda_Embedder_Counts": (i32, [vp, i64p, i64p, i32]),
        "Cuda_Embedder_Hidden": (i32, [vp]),
        "Cuda_Embedder_MaxBatch": (i32, [vp, i32p, i64p]),
        "Cuda_Embedder_LastError": (i32, [vp, ctypes.c_char_p, i32]),
        "Cuda_Embedder_Destroy": (None, [vp]),
        "Cuda_Server_Create": (i32, [vp, i32, i32, ctypes.POINTER(vp)]),
        "Cuda_Server_Submit": (i32, [vp, i32, i32p, i32p, i64p, i64p, f32p, i64p]),
        "Cuda_Server_Clock": (i64, []),
        "Cuda_Server_Wait": (i32, [vp, i64, ctypes.c_double, i64p]),
        "Cuda_Server_Latencies": (i32, [vp, i64, i64, i64p]),
        "Cuda_Server_Drain": (i32, [vp]),
        "Cuda_Server_Stats": (i32, [vp, vp]),
        "Cuda_Server_Destroy": (None, [vp]),
        "Cuda_Runtime_SplitByWeight": (i32, [i32p, i32, ctypes.POINTER(ctypes.c_double), i32, i32p]),
        "Cuda_Runtime_DynamicBatches": (i32, [i32p, i32, i32, i64, i32p, i32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def lib():
    """Loads the in-tree library (built by longbow-fletcher_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FletcherError(-1, f"{LIB_PATH} is missing; run longbow-fletcher_b200/build.py")
        _lib = _sig(ctypes.CDLL(LIB_PATH))
    return _lib


def _i32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def _f32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class PinnedArray:
    """Page-locked host array (Cuda_HostAlloc) viewed as numpy; freed with close()."""

    def __init__(self, be, shape, dtype):
        self.be = be
        self.dtype = np.dtype(dtype)
        n = int(np.prod(shape)) * self.dtype.itemsize
        self.ptr = lib().Cuda_HostAlloc(be.ctx, max(n, 1))
        if not self.ptr:
            be.check(3)  # FLETCHER_ERR_OOM
        buf = (ctypes.c_uint8 * max(n, 1)).from_address(self.ptr)
        self.array = np.frombuffer(buf, dtype=self.dtype, count=int(np.prod(shape))).reshape(shape)

    def close(self):
        if self.ptr:
            self.array = None
            lib().Cuda_HostFree(self.be.ctx, self.ptr)
            self.ptr = None


class Backend:
    """device.Backend on one GPU (NewCudaBackend / SetDevice, embeddings.go:105-135)."""

    def __init__(self, device: int = 0, dtype: str = "f32"):
        L = lib()
        n = L.Cuda_GetDeviceCount()
        if n <= 0:
            raise FletcherError(-1, "no CUDA device")
        self.ctx = L.Cuda_Init()
        if not self.ctx:
            raise FletcherError(-1, "Cuda_Init failed")
        self.dtype = DTYPES[dtype] if isinstance(dtype, str) else dtype
        if device:
            self.check(L.Cuda_SetDevice(self.ctx, device))
        self.device = device

    def name(self):
        return "CUDA-B200"

    def check(self, rc):
        if rc != 0:
            buf = ctypes.create_string_buffer(1024)
            lib().Cuda_GetLastError(self.ctx, buf, 1024)
            raise FletcherError(rc, buf.value.decode())
        return rc

    def new_tensor(self, r, c, data=None, dtype=None):
        return Tensor(self, r, c, self.dtype if dtype is None else dtype, data)

    def synchronize(self):
        self.check(lib().Cuda_Synchronize(self.ctx))

    def device_count(self):
        return lib().Cuda_GetDeviceCount()

    def set_half_conversion(self, mode):
        """FLETCHER_HALF_REFERENCE (the reference's utils.go bytes, default) or FLETCHER_HALF_RNE."""
        self.check(lib().Cuda_SetHalfConversion(self.ctx, mode))

    def vram_usage(self):
        a, t = ctypes.c_int64(), ctypes.c_int64()
        self.check(lib().Cuda_MemGetInfo(self.ctx, ctypes.byref(a), ctypes.byref(t)))
        return a.value, t.value

    def stream(self):
        return lib().Cuda_GetStream(self.ctx)

    def launch_count(self):
        return lib().Cuda_GetLaunchCount(self.ctx)

    def close(self):
        if self.ctx:
            lib().Cuda_FreeContext(self.ctx)
            self.ctx = None


class Tensor:
    """device.Tensor: a dtype-tagged device buffer of (rows, cols).  T() returns a transposed
    view sharing the buffer (cpu_backend.go:306-314); only Mul reads the flag, as in the
    reference, where every other op sees the stored layout."""

    def __init__(self, be: Backend, r, c, dtype, data=None):
        self.be, self.rows, self.cols, self.dtype = be, int(r), int(c), dtype
        self.trans = False
        self._owner = None
        self.buf = lib().Cuda_AllocTensor(be.ctx, self.rows, self.cols, dtype)
        if not self.buf:
            be.check(3)
        if data is not None:
            self.copy_from_float32(data)

    def __del__(self):
        try:
            if self._owner is None and self.buf and self.be.ctx:
                lib().Cuda_FreeBuffer(self.be.ctx, self.buf)
        except Exception:
            pass

    def dims(self):
        return (self.cols, self.rows) if self.trans else (self.rows, self.cols)

    def T(self):
        v = Tensor.__new__(Tensor)
        v.be, v.rows, v.cols, v.dtype, v.buf = self.be, self.rows, self.cols, self.dtype, self.buf
        v.trans = not self.trans
        v._owner = self._owner or self  # keeps the buffer alive; the view never frees it
        return v

    def at(self, i, j):
        r = ctypes.c_float()
        self.be.check(lib().Cuda_At(self.buf, i, j, ctypes.byref(r)))
        return r.value

    def set(self, i, j, v):
        self.be.check(lib().Cuda_Set(self.buf, i, j, float(v)))

    def copy(self, other: "Tensor"):
        """device.Tensor.Copy: same dims, element-wise (cpu_backend.go:259-286)."""
        if self.dims() != other.dims():
            raise FletcherError(1, f"Copy: dimension mismatch {self.dims()} <- {other.dims()}")
        self.be.check(lib().Cuda_Copy(self.be.ctx, self.buf, 0, other.buf, 0, self.rows * self.cols))

    def slice(self, i, k, j, l):
        """device.Tensor.Slice: a new tensor holding a copy of [i:k, j:l] (cpu_backend.go:288-303)."""
        if k - i <= 0 or l - j <= 0:
            raise FletcherError(1, "Slice: invalid dimensions")
        out = Tensor(self.be, k - i, l - j, self.dtype)
        self.be.check(lib().Cuda_Slice(self.be.ctx, self.buf, i, k, j, l, out.buf))
        return out

    def mul(self, a: "Tensor", b: "Tensor"):
        """device.Tensor.Mul: self = a . b, honouring T() views (cpu_backend.go:316-372)."""
        ar, ac = a.dims()
        br, bc = b.dims()
        if ac != br:
            raise FletcherError(1, f"Mul: dimension mismatch a_cols={ac} b_rows={br}")
        if self.dims() != (ar, bc):
            raise FletcherError(1, f"Mul: result tensor dimension mismatch. Expected {ar}x{bc}, got {self.dims()}")
        self.be.check(lib().Cuda_Mul(self.be.ctx, a.buf, int(a.trans), b.buf, int(b.trans), self.buf, ar, bc, ac))

    def ptr(self):
        return lib().Cuda_GetBufferContents(self.buf)

    def copy_from_float32(self, data):
        a = np.ascontiguousarray(data, np.float32).reshape(-1)
        assert a.size == self.rows * self.cols
        self.be.check(lib().Cuda_CopyFromFloat32(self.buf, _f32p(a), a.size))

    def to_host(self):
        out = np.empty(self.rows * self.cols, np.float32)
        self.be.check(lib().Cuda_ToHostFloat32(self.buf, _f32p(out), out.size))
        return out.reshape(self.rows, self.cols)

    def raw_bytes(self):
        es = 4 if self.dtype == F32 else 2
        out = np.empty(self.rows * self.cols * es, np.uint8)
        self.be.check(lib().Cuda_CopyToHost(self.buf, 0, out.ctypes.data, out.size))
        return out

    # ---- ops (device.go:42-116)
    def linear(self, x: "Tensor", w: "Tensor", b: "Tensor | None", act=ACT_IDENTITY):
        n_out = w.cols // 2 if act == ACT_SWIGLU else w.cols
        y = Tensor(self.be, x.rows, n_out, x.dtype)
        self.be.check(lib().Cuda_Linear_Fused(self.be.ctx, x.buf, x.rows, x.cols, w.buf, w.cols,
                                              b.buf if b is not None else None, y.buf, act))
        return y

    def layer_norm(self, g, b, eps):
        self.be.check(lib().Cuda_LayerNorm(self.be.ctx, self.buf, g.buf, b.buf, self.buf, self.rows, self.cols, eps))

    def add_layer_norm(self, residual, g, b, eps):
        self.be.check(lib().Cuda_AddLayerNorm(self.be.ctx, self.buf, residual.buf, g.buf, b.buf,
                                              self.rows, self.cols, eps))

    def softmax(self):
        self.be.check(lib().Cuda_Softmax(self.be.ctx, self.buf, self.buf, self.rows, self.cols))

    def gather(self, indices):
        idx = np.ascontiguousarray(indices, np.int32)
        out = Tensor(self.be, idx.size, self.cols, self.dtype)
        self.be.check(lib().Cuda_Gather(self.be.ctx, self.buf, _i32p(idx), out.buf, idx.size, self.cols))
        return out

    def add(self, other):
        self.be.check(lib().Cuda_Add(self.be.ctx, self.buf, other.buf, self.rows * self.cols))

    def scale(self, v):
        self.be.check(lib().Cuda_Scale(self.be.ctx, self.buf, v, self.rows * self.cols))

    def add_scalar(self, v):
        self.be.check(lib().Cuda_AddScalar(self.be.ctx, self.buf, v, self.rows * self.cols))

    def add_bias(self, bias):
        self.be.check(lib().Cuda_AddBias(self.be.ctx, self.buf, bias.buf, self.rows, self.cols))

    def activation(self, act):
        self.be.check(lib().Cuda_Activation(self.be.ctx, self.buf, self.rows, self.cols, act))

    def cast(self, dtype):
        out = Tensor(self.be, self.rows, self.cols, dtype)
        self.be.check(lib().Cuda_Cast(self.be.ctx, self.buf, out.buf, self.rows * self.cols))
        return out

    def has_nan(self):
        r = ctypes.c_int32()
        self.be.check(lib().Cuda_HasNaN(self.be.ctx, self.buf, self.rows * self.cols, ctypes.byref(r)))
        return bool(r.value)

    def attention(self, q, k, v, batch, seq, heads, scale):
        out = Tensor(self.be, q.rows, q.cols, q.dtype)
        self.be.check(lib().Cuda_Attention_Fused(self.be.ctx, q.buf, k.buf, v.buf, out.buf, batch, seq, q.cols,
                                                 heads, scale))
        return out

    def attention_varlen(self, q, k, v, lengths, heads, scale):
        lens = np.ascontiguousarray(lengths, np.int32)
        out = Tensor(self.be, q.rows, q.cols, q.dtype)
        self.be.check(lib().Cuda_Attention_VarLen(self.be.ctx, q.buf, k.buf, v.buf, out.buf, _i32p(lens), lens.size,
                                                  q.cols, heads, scale))
        return out

    def apply_rope(self, batch, seq, heads, head_dim):
        self.be.check(lib().Cuda_ApplyRoPE(self.be.ctx, self.buf, batch, seq, heads, head_dim))

    def apply_rope_varlen(self, lengths, heads, head_dim, base):
        lens = np.ascontiguousarray(lengths, np.int32)
        self.be.check(lib().Cuda_ApplyRoPE_VarLen(self.be.ctx, self.buf, _i32p(lens), lens.size, heads, head_dim,
                                                  base))

    def mean_pool_l2(self, lengths):
        lens = np.ascontiguousarray(lengths, np.int32)
        out = Tensor(self.be, lens.size, self.cols, F32)
        self.be.check(lib().Cuda_MeanPoolL2(self.be.ctx, self.buf, _i32p(lens), lens.size, self.cols, out.buf))
        return out


class BertModel:
    """model.BertModel on the device (Cuda_Model_*): ForwardBatch(ids, lengths) -> [B, H]."""

    def __init__(self, be: Backend, cfg: synth.BertConfig, dtype=None):
        self.be, self.cfg = be, cfg
        self.dtype = be.dtype if dtype is None else (DTYPES[dtype] if isinstance(dtype, str) else dtype)
        self._c = synth.to_c(cfg)
        h = ctypes.c_void_p()
        be.check(lib().Cuda_Model_Create(be.ctx, ctypes.byref(self._c), self.dtype, ctypes.byref(h)))
        self.h = h

    def weight_count(self):
        return lib().Cuda_Model_WeightCount(ctypes.byref(self._c))

    def load_raw(self, blob):
        b = np.ascontiguousarray(blob, np.float32)
        self.be.check(lib().Cuda_Model_LoadRaw(self.h, _f32p(b), b.size))

    def load_tensor(self, name, array, dtype, transposed=False):
        """One checkpoint tensor by its reference name; `array` holds the raw values of `dtype`
        (float32, float16, or bfloat16 bit patterns as uint16), 1-D or 2-D."""
        a = np.ascontiguousarray(array)
        rows, cols = (1, a.size) if a.ndim <= 1 else (a.shape[0], int(np.prod(a.shape[1:])))
        self.be.check(lib().Cuda_Model_LoadTensor(self.h, name.encode(), dtype, a.ctypes.data, rows, cols,
                                                  int(transposed)))

    def is_loaded(self):
        return bool(lib().Cuda_Model_IsLoaded(self.h))

    def forward_batch(self, ids, lengths, pooling=POOL_MEAN_L2):
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((lens.size, self.cfg.hidden), np.float32)
        self.be.check(lib().Cuda_Model_ForwardBatch(self.h, _i32p(ids), _i32p(lens), lens.size, pooling, _f32p(out)))
        return out

    def forward_batch_16(self, ids, lengths, pooling=POOL_MEAN_L2, out_dtype=F16):
        """Vectors as float16 (or bfloat16 bit patterns in uint16) — the fp16 transport."""
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(lengths, np.int32)
        out = np.empty((lens.size, self.cfg.hidden), np.float16 if out_dtype == F16 else np.uint16)
        self.be.check(lib().Cuda_Model_ForwardBatchEx(self.h, _i32p(ids), _i32p(lens), lens.size, pooling, out_dtype,
                                                      out.ctypes.data))
        return out

    def forward_batch_async(self, ids_ptr, lengths, pooling, out_ptr, out_dtype=F32):
        """Enqueues a batch (ids and out: host pointers that stay valid until wait(ticket));
        returns its ticket.  The double-buffering half of the batcher loop."""
        lens = np.ascontiguousarray(lengths, np.int32)
        t = ctypes.c_int64()
        self.be.check(lib().Cuda_Model_ForwardBatchAsync(self.h, ctypes.c_void_p(ids_ptr), _i32p(lens), lens.size,
                                                         pooling, out_dtype, ctypes.c_void_p(out_ptr),
                                                         ctypes.byref(t)))
        return t.value

    def wait(self, ticket):
        self.be.check(lib().Cuda_Model_Wait(self.h, ticket))

    def forward_batch_device(self, d_ids_ptr, lengths, pooling, d_out_ptr):
        lens = np.ascontiguousarray(lengths, np.int32)
        self.be.check(lib().Cuda_Model_ForwardBatchDevice(self.h, ctypes.c_void_p(d_ids_ptr), _i32p(lens), lens.size,
                                                          pooling, ctypes.c_void_p(d_out_ptr)))

    STAGES = ["embed", "gemm_qkv", "rope", "attention", "gemm_o", "layernorm", "gemm_up", "activation",
              "gemm_down", "pool"]

    def set_keep_hidden(self, on: bool):
        self.be.check(lib().Cuda_Model_SetKeepHidden(self.h, int(on)))

    def set_graphs(self, on: bool):
        self.be.check(lib().Cuda_Model_SetGraphs(self.h, int(on)))

    def set_stage_timing(self, on: bool):
        self.be.check(lib().Cuda_Model_SetStageTiming(self.h, int(on)))

    def stage_times(self):
        """{stage: (milliseconds, timed calls)} since the last read."""
        n = len(self.STAGES)
        ms = np.zeros(n, np.float32)
        cnt = np.zeros(n, np.int64)
        self.be.check(lib().Cuda_Model_StageTimes(self.h, _f32p(ms), cnt.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), n))
        return {s: (float(ms[i]), int(cnt[i])) for i, s in enumerate(self.STAGES)}

    def last_hidden(self, T):
        out = np.empty((T, self.cfg.hidden), np.float32)
        self.be.check(lib().Cuda_Model_LastHidden(self.h, _f32p(out), out.size))
        return out

    def close(self):
        if self.h:
            lib().Cuda_Model_Free(self.h)
            self.h = None
