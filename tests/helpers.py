"""Shared helpers for the tests: golden fixtures and vector comparisons."""
import dataclasses
import os

import numpy as np

import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances stated by the spec: fp32 per-vector cosine >= 0.99999 and max-abs <= 1e-4;
# fp16/bf16 per-vector cosine >= 0.999.
COS_F32, MAXABS_F32, COS_16 = 0.99999, 1e-4, 0.999


def golden_cfg(name):
    tiny = synth.BERT_TINY
    nomic2 = dataclasses.replace(synth.NOMIC, num_layers=2)
    return {
        "tiny_ragged_spec": tiny,
        "tiny_ragged_literal": dataclasses.replace(tiny, layer_norm_eps=1e-7),
        "tiny_uniform_literal": dataclasses.replace(tiny, layer_norm_eps=1e-7),
        "nomic2_ragged_spec": nomic2,
        "nomic2_uniform_literal": dataclasses.replace(nomic2, layer_norm_eps=1e-7, rope_base=10000.0),
    }[name]


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    cfg = golden_cfg(name)
    return cfg, {k: z[k] for k in z.files}


def cosines(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    na = np.linalg.norm(a, axis=1)
    nb = np.linalg.norm(b, axis=1)
    return (a * b).sum(1) / np.maximum(na * nb, 1e-300)


def assert_close_f32(got, want, what=""):
    cos = cosines(got, want)
    mx = float(np.abs(np.asarray(got, np.float64) - want).max())
    assert cos.min() >= COS_F32 and mx <= MAXABS_F32, f"{what}: min cos {cos.min():.8f}, max abs {mx:.3e}"


def assert_close_16(got, want, what="", cos_min=COS_16):
    cos = cosines(got, want)
    assert cos.min() >= cos_min, f"{what}: min cos {cos.min():.6f} (mean {cos.mean():.6f})"


def exp_fast_np(x):
    """ExpFast (internal/simd/simd.go:7-46) vectorised in float32 numpy."""
    x = np.asarray(x, np.float32)
    t = (x * np.float32(1.442695)).astype(np.float32)
    k = np.trunc(t).astype(np.int64)
    k = np.where(t < 0, k - 1, k)
    f = (t - k.astype(np.float32)).astype(np.float32)
    p = np.float32(1) + f * (np.float32(0.6931472) + f * (np.float32(0.2402265) + f * np.float32(0.0555041)))
    kk = np.clip(k, -149, 127)
    out = (p * np.ldexp(np.float32(1), kk).astype(np.float32)).astype(np.float32)
    out = np.where(x > 88, np.float32(1e38), out)
    return np.where(x < -88, np.float32(0), out).astype(np.float32)


def attention_np(q, k, v, lengths, heads, scale, fast=True):
    """Per-sequence multi-head attention (cpu_backend.go:662-758) in numpy."""
    T, H = q.shape
    dh = H // heads
    out = np.zeros((T, H), np.float32)
    off = 0
    for L in lengths:
        for h in range(heads):
            sl = slice(h * dh, (h + 1) * dh)
            s = (q[off:off + L, sl].astype(np.float32) @ k[off:off + L, sl].astype(np.float32).T) * np.float32(scale)
            s = s - s.max(axis=1, keepdims=True)
            e = exp_fast_np(s) if fast else np.exp(s)
            p = e / e.sum(axis=1, keepdims=True)
            out[off:off + L, sl] = p @ v[off:off + L, sl].astype(np.float32)
        off += L
    return out


def bf16_round(x):
    """Rounds float32 to bfloat16 precision (round to nearest even), returned as float32."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def f32_to_f16_ref(x):
    """Float32ToFloat16 (internal/device/utils.go:13-72) vectorised: uint16 bit patterns.
    NaN -> 0x7E00; +-Inf -> 0x7C00/0xFC00; clamp to +-65504; 0 < |x| < 2^-14 -> signed zero;
    else sign | (exp-127+15) << 10 | mantissa >> 13 (truncated), 0x7BFF on exponent overflow,
    signed zero on underflow."""
    x = np.ascontiguousarray(x, np.float32).copy()
    nan, pinf, ninf = np.isnan(x), np.isposinf(x), np.isneginf(x)
    fin = ~(nan | pinf | ninf)
    x[fin] = np.clip(x[fin], np.float32(-65504.0), np.float32(65504.0))
    a = np.abs(x)
    tiny = fin & (a < np.float32(6.103515625e-05)) & (a > 0)
    bits = x.view(np.uint32)
    sign = ((bits >> 16) & 0x8000).astype(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 127 + 15
    frac = ((bits >> 13) & 0x3FF).astype(np.uint32)
    out = (sign | (np.clip(e, 0, 31).astype(np.uint32) << 10) | frac).astype(np.uint32)
    out = np.where(e >= 0x1F, sign | 0x7BFF, out)
    out = np.where(e <= 0, sign, out)
    out = np.where(tiny, np.where(x < 0, 0x8000, 0), out)
    out = np.where(nan, 0x7E00, out)
    out = np.where(pinf, 0x7C00, out)
    out = np.where(ninf, 0xFC00, out)
    return out.astype(np.uint16)


def f16_to_f32_ref(h):
    """Float16ToFloat32 (internal/device/utils.go:75-91): zero and subnormals -> +0.0; exponent
    31 keeps the payload (Inf/NaN); normals widen exactly."""
    h = np.ascontiguousarray(h, np.uint16).astype(np.uint32)
    sign, e, frac = (h >> 15) & 1, (h >> 10) & 0x1F, h & 0x3FF
    normal = (sign << 31) | ((e + (127 - 15)) << 23) | (frac << 13)
    special = (sign << 31) | (0xFF << 23) | (frac << 13)
    bits = np.where(e == 31, special, normal)
    bits = np.where(e == 0, 0, bits).astype(np.uint32)
    return bits.view(np.float32)


def half_conversion_probe(n=1_000_000, seed=7):
    """Inputs for the fp16 byte tests: random floats over the whole fp16 range and beyond, plus
    NaN, +-Inf, +-65504, +-65520, +-1e6, the subnormal band, +-0 and values whose truncation
    and round-to-nearest-even differ."""
    rng = np.random.default_rng(seed)
    mags = np.exp2(rng.uniform(-30, 20, n)).astype(np.float32)
    x = (mags * rng.choice(np.array([-1, 1], np.float32), n)).astype(np.float32)
    special = np.array([np.nan, np.inf, -np.inf, 65504, -65504, 65520, -65520, 65519.99, 1e6, -1e6, 0.0, -0.0,
                        6.1e-5, -6.1e-5, 6.103515625e-05, -6.103515625e-05, 6.1035156e-05, 5.96e-8, 1e-7, -3e-6,
                        1.0, -2.0, 1.0009765625, 1.00048828125, 1.0014648, 2049.0, 0.1, -0.3333333], np.float32)
    return np.concatenate([special, x]).astype(np.float32)


def f16_round_ref(x):
    """float32 -> the value an fp16 tensor holds after CopyFromFloat32 under the reference's
    conversion (truncation, flush, saturation), as float32."""
    return f16_to_f32_ref(f32_to_f16_ref(x))
