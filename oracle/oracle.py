"""TEST INFRASTRUCTURE ONLY — ctypes binding of the CPU oracle (oracle/ref_cpu.cpp).

Only tests/, __graft_entry__.smoke() (as a checker) and bench.py's CPU-baseline leg use
this module.  The product path (the CUDA library) never calls it.
"""
from __future__ import annotations

import ctypes
import glob
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libfletcher_oracle.so")
MODE_LITERAL, MODE_SPEC = 0, 1

_lib = None


def openblas_path() -> str:
    """The OpenBLAS that numpy bundles (ILP64, `scipy_` prefixed symbols)."""
    import numpy
    d = os.path.join(os.path.dirname(os.path.dirname(numpy.__file__)), "numpy.libs")
    hits = sorted(glob.glob(os.path.join(d, "libscipy_openblas64_*.so")))
    if not hits:
        raise RuntimeError(f"no bundled OpenBLAS under {d}")
    return hits[0]


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(
            os.path.join(HERE, "ref_cpu.cpp")):
        subprocess.check_call(["make", "-s", "-C", HERE, "-B" if force else "all"])
    return LIB


def lib(threads: int | None = None):
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        f32p = ctypes.POINTER(ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        L.ref_init.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.ref_weight_count.restype = ctypes.c_int64
        L.ref_weight_count.argtypes = [ctypes.c_void_p]
        for n in ("ref_exp_fast", "ref_tanh_fast", "ref_gelu_fast"):
            getattr(L, n).restype = ctypes.c_float
            getattr(L, n).argtypes = [ctypes.c_float]
        L.ref_softmax_fast.argtypes = [f32p, ctypes.c_int64]
        L.ref_layer_norm.argtypes = [f32p, ctypes.c_int64, ctypes.c_int64, f32p, f32p, ctypes.c_float]
        L.ref_sgemm.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int64, ctypes.c_float, f32p, ctypes.c_int64, f32p,
                                ctypes.c_int64, f32p, ctypes.c_int64]
        L.ref_rope.argtypes = [f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, i32p, ctypes.c_double]
        L.ref_linear_activation.argtypes = [f32p, ctypes.c_int64, ctypes.c_int64, f32p, ctypes.c_int64, f32p,
                                            ctypes.c_int, f32p]
        L.ref_attention.argtypes = [f32p, f32p, f32p, f32p, ctypes.c_int64, ctypes.c_int, i32p, ctypes.c_int,
                                    ctypes.c_float]
        L.ref_forward.argtypes = [ctypes.c_void_p, f32p, ctypes.c_int64, i32p, i32p, ctypes.c_int32,
                                  ctypes.c_int32, f32p, f32p, f32p]
        _lib = L
    n = threads if threads is not None else (os.cpu_count() or 1)
    rc = _lib.ref_init(openblas_path().encode(), int(n))
    if rc != 0:
        raise RuntimeError(f"ref_init failed: {rc}")
    return _lib


def fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def ip(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def forward(cfg, blob, ids, lengths, mode=MODE_SPEC, threads=None, want_hidden=False):
    """Returns dict(cls=[B,H], mean=[B,H], hidden=[T,H] or None)."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "longbow-fletcher_b200"))
    import synth
    L = lib(threads)
    ids = np.ascontiguousarray(ids, np.int32)
    lengths = np.ascontiguousarray(lengths, np.int32)
    blob = np.ascontiguousarray(blob, np.float32)
    B, H, T = len(lengths), cfg.hidden, int(lengths.sum())
    cls = np.zeros((B, H), np.float32)
    mean = np.zeros((B, H), np.float32)
    hid = np.zeros((T, H), np.float32) if want_hidden else None
    c = synth.to_c(cfg)
    rc = L.ref_forward(ctypes.byref(c), fp(blob), blob.size, ip(ids), ip(lengths), B, mode,
                       fp(cls), fp(mean), fp(hid) if hid is not None else None)
    if rc != 0:
        raise RuntimeError(f"ref_forward failed: {rc}")
    return {"cls": cls, "mean": mean, "hidden": hid}
