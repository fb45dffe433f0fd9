"""CPU tests of the oracle (oracle/ref_cpu.cpp): the reference's own known-answer tests for
this path, the golden fixtures, and the relations between its literal and spec modes."""
import ctypes
import dataclasses
import math

import numpy as np
import pytest

import synth
from helpers import golden_cfg, load_golden


def fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def test_layernorm_known_answer(oracle_mod):
    # internal/device/device_test.go:69-96
    L = oracle_mod.lib()
    x = np.array([1, 2, 3, 4], np.float32)
    g = np.ones(4, np.float32)
    b = np.zeros(4, np.float32)
    L.ref_layer_norm(fp(x), 1, 4, fp(g), fp(b), 1e-6)
    np.testing.assert_allclose(x, [-1.3416407, -0.4472136, 0.4472136, 1.3416407], atol=1e-4)


def test_mul_known_answer(oracle_mod):
    # internal/device/device_test.go:27-54 (Mul -> sgemm)
    L = oracle_mod.lib()
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    c = np.zeros((2, 2), np.float32)
    L.ref_sgemm(0, 0, 2, 2, 3, 1.0, fp(a), 3, fp(b), 2, fp(c), 2)
    np.testing.assert_allclose(c.ravel(), [58, 64, 139, 154], atol=1e-6)


@pytest.mark.parametrize("name,std", [("ref_exp_fast", math.exp), ("ref_tanh_fast", math.tanh)])
def test_fast_math_bounds(oracle_mod, name, std):
    # internal/simd/simd_test.go:72-104: within 5% relative (or 1e-3 absolute)
    fn = getattr(oracle_mod.lib(), name)
    for x in [-10, -5, -2, -1, -0.5, 0, 0.5, 1, 2, 5, 10]:
        got, want = fn(x), std(x)
        diff = abs(got - want)
        rel = diff / (abs(want) if want != 0 else 1.0)
        assert diff <= 1e-3 or rel <= 0.05, (name, x, got, want)


def test_exp_fast_formula(oracle_mod):
    # simd.go:7-46 restated in numpy float32, bit for bit.
    L = oracle_mod.lib()
    xs = np.linspace(-90, 90, 20001, dtype=np.float32)
    for x in xs[::37]:
        x = np.float32(x)
        if x > 88:
            want = np.float32(1e38)
        elif x < -88:
            want = np.float32(0)
        else:
            t = np.float32(x * np.float32(1.442695))
            k = int(t)
            if t < 0:
                k -= 1
            f = np.float32(t - np.float32(k))
            p = np.float32(1) + f * (np.float32(0.6931472) + f * (np.float32(0.2402265) + f * np.float32(0.0555041)))
            want = np.float32(p * np.float32(2.0 ** k))
        assert np.float32(L.ref_exp_fast(float(x))) == want, x


def test_gelu_fast_formula(oracle_mod):
    # simd.go:49-75: Pade tanh, clamped at |x|>4.
    L = oracle_mod.lib()
    for x in np.linspace(-8, 8, 161, dtype=np.float32):
        u = np.float32(0.7978846) * (x + np.float32(0.044715) * x * x * x)
        th = np.float32(1) if u > 4 else np.float32(-1) if u < -4 else u * (np.float32(27) + u * u) / (np.float32(27) + np.float32(9) * u * u)
        want = np.float32(0.5) * x * (np.float32(1) + th)
        assert abs(np.float32(L.ref_gelu_fast(float(x))) - want) <= 1e-6 * max(1.0, abs(float(want))), x


def test_rope_formula(oracle_mod):
    # cpu_backend.go:760-805 / rope_test.go: rotate-half with float64 trig, base 10000.
    L = oracle_mod.lib()
    rng = np.random.default_rng(1337)
    B, S, nh, dh = 2, 16, 4, 64
    x = rng.standard_normal((B * S, nh * dh)).astype(np.float32)
    pos = (np.arange(B * S) % S).astype(np.int32)
    got = x.copy()
    L.ref_rope(fp(got), B * S, nh, dh, pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 10000.0)
    want = x.copy().reshape(B * S, nh, dh)
    i = np.arange(dh // 2)
    theta = pos[:, None].astype(np.float64) * np.power(10000.0, -2.0 * i / dh)[None, :]
    c = np.cos(theta).astype(np.float32)[:, None, :]
    s = np.sin(theta).astype(np.float32)[:, None, :]
    x1, x2 = want[..., : dh // 2].copy(), want[..., dh // 2:].copy()
    want[..., : dh // 2] = x1 * c - x2 * s
    want[..., dh // 2:] = x1 * s + x2 * c
    np.testing.assert_allclose(got, want.reshape(B * S, -1), rtol=0, atol=1e-6)


@pytest.mark.parametrize("name", ["tiny_ragged_spec", "tiny_ragged_literal", "tiny_uniform_literal",
                                  "nomic2_ragged_spec", "nomic2_uniform_literal"])
def test_oracle_reproduces_golden(oracle_mod, name):
    cfg, g = load_golden(name)
    blob = synth.make_weights(cfg, int(g["weight_seed"]))
    r = oracle_mod.forward(cfg, blob, g["ids"], g["lengths"], mode=int(g["mode"]), threads=2)
    np.testing.assert_allclose(r["mean"], g["mean"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(r["cls"], g["cls"], rtol=0, atol=1e-6)


def test_literal_equals_spec_on_uniform_batches(oracle_mod):
    cfg = dataclasses.replace(synth.BERT_TINY, layer_norm_eps=1e-7)
    blob = synth.make_weights(cfg, 0)
    lens = np.full(5, 24, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 11)
    a = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_LITERAL, want_hidden=True)
    b = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_SPEC, want_hidden=True)
    assert np.array_equal(a["hidden"], b["hidden"])
    nomic = dataclasses.replace(synth.NOMIC, num_layers=1, layer_norm_eps=1e-7, rope_base=10000.0)
    blob = synth.make_weights(nomic, 1)
    ids = synth.make_ids(lens, nomic.vocab_size, 12)
    a = oracle_mod.forward(nomic, blob, ids, lens, mode=oracle_mod.MODE_LITERAL, want_hidden=True)
    b = oracle_mod.forward(nomic, blob, ids, lens, mode=oracle_mod.MODE_SPEC, want_hidden=True)
    assert np.array_equal(a["hidden"], b["hidden"])


def test_literal_ragged_batches_have_no_attention_mixing(oracle_mod):
    """With unequal lengths the reference's CPU fallback loses its attention output
    (bert.go:699-708 copies into a Slice, which is a copy: cpu_backend.go:288-303), so every
    row depends only on its own token and position.  Changing one token must leave every other
    row of the last hidden state bit-identical."""
    cfg = dataclasses.replace(synth.BERT_TINY, layer_norm_eps=1e-7)
    blob = synth.make_weights(cfg, 0)
    lens = np.array([10, 20, 7], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 3)
    a = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_LITERAL, want_hidden=True)["hidden"]
    ids2 = ids.copy()
    ids2[15] = 4242
    b = oracle_mod.forward(cfg, blob, ids2, lens, mode=oracle_mod.MODE_LITERAL, want_hidden=True)["hidden"]
    diff = np.abs(a - b).max(axis=1)
    assert diff[15] > 0 and np.all(np.delete(diff, 15) == 0)
    # whereas spec mode mixes within the sequence (rows 10..29) and nowhere else
    a = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_SPEC, want_hidden=True)["hidden"]
    b = oracle_mod.forward(cfg, blob, ids2, lens, mode=oracle_mod.MODE_SPEC, want_hidden=True)["hidden"]
    diff = np.abs(a - b).max(axis=1)
    assert np.all(diff[10:30] > 0) and np.all(diff[:10] == 0) and np.all(diff[30:] == 0)


def test_weight_count_matches_layout(oracle_mod):
    for cfg in (synth.BERT_TINY, synth.NOMIC):
        c = synth.to_c(cfg)
        assert oracle_mod.lib().ref_weight_count(ctypes.byref(c)) == synth.weight_count(cfg)


# ---- the reference's fp16 host conversion (internal/device/utils.go:13-91), restated in numpy
# (tests/helpers.py) and pinned here against the reference's own byte KAT and hand-derived values.

def test_half_conversion_restatement_known_answers():
    from helpers import f16_to_f32_ref, f32_to_f16_ref
    # internal/device/cast_test.go:11-47: 1.0 -> 0x3c00, -2.0 -> 0xc000
    assert list(f32_to_f16_ref([1.0, -2.0])) == [0x3C00, 0xC000]
    cases = [
        (float("nan"), 0x7E00), (float("inf"), 0x7C00), (float("-inf"), 0xFC00),  # utils.go:15-23
        (65504.0, 0x7BFF), (70000.0, 0x7BFF), (-1e6, 0xFBFF),  # clamped to +-65504 (utils.go:31-36)
        (65520.0, 0x7BFF),  # IEEE would round this to Inf
        (5e-5, 0x0000), (-5e-5, 0x8000), (6.103515625e-05, 0x0400),  # flush below 2^-14 (utils.go:39-48)
        (0.0, 0x0000), (-0.0, 0x8000),
        (1.0009765625, 0x3C01), (1.00146484375, 0x3C01),  # truncation: IEEE RNE gives 0x3C02 for the second
        (0.1, 0x2E66),  # IEEE RNE gives 0x2E66 too (0.1 rounds down)
        (-0.3333333, 0xB555),
    ]
    for x, want in cases:
        got = int(f32_to_f16_ref(np.array([x], np.float32))[0])
        assert got == want, (x, hex(got), hex(want))
    # Float16ToFloat32: subnormals and -0 read as +0; Inf/NaN keep their bits.
    got = f16_to_f32_ref(np.array([0x0001, 0x83FF, 0x8000, 0x3C00, 0xC000, 0x7C00, 0xFC00, 0x7E00, 0x7BFF], np.uint16))
    assert list(got.view(np.uint32)[:3]) == [0, 0, 0]
    assert got[3] == 1.0 and got[4] == -2.0 and np.isposinf(got[5]) and np.isneginf(got[6]) and np.isnan(got[7])
    assert got[8] == 65504.0
    # Every normal fp16 survives the round trip bit for bit.
    h = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    e = (h >> 10) & 0x1F
    normal = (e > 0) & (e < 31)
    assert np.array_equal(f32_to_f16_ref(f16_to_f32_ref(h[normal])), h[normal])


# ---- SwiGLU and naive attention known-answer tests of the reference, restated on the oracle.

def _swiglu_kat_expected(data, n, inter):
    # internal/device/swiglu_test.go:68-77: silu(first half) * second half, float64 exp
    ref = np.zeros((n, inter), np.float32)
    for i in range(n):
        for j in range(inter):
            x = data[i * 2 * inter + j]
            y = data[i * 2 * inter + j + inter]
            sw = np.float32(x / (np.float32(1.0) + np.float32(math.exp(-float(x)))))
            ref[i, j] = np.float32(sw * y)
    return ref


def test_swiglu_known_answer(oracle_mod):
    # swiglu_test.go:10-120: X = I(10), W = data (10 x 256), bias 0 -> LinearActivation(SwiGLU).
    n, inter = 10, 128
    data = (np.arange(n * inter * 2) % 100).astype(np.float32) / np.float32(10.0)
    want = _swiglu_kat_expected(data, n, inter)
    L = oracle_mod.lib()
    x = np.eye(n, dtype=np.float32)
    out = np.zeros((n, inter), np.float32)
    L.ref_linear_activation(fp(x), n, n, fp(data), 2 * inter, None, 4, fp(out))
    assert np.abs(out - want).max() <= 1e-6  # the reference test allows 0.1 (for its fp16 kernel)


def simple_attention_cpu(q, k, v, batch, seq, head_dim, heads, scale):
    """simpleAttentionCPU (internal/device/attention_test.go:13-68), float32 loops with a float64
    exp, as the reference writes it."""
    H = head_dim * heads
    out = np.zeros(batch * seq * H, np.float32)
    for b in range(batch):
        for h in range(heads):
            sc = np.zeros(seq * seq, np.float32)
            for i in range(seq):
                for j in range(seq):
                    s = np.float32(0)
                    for d in range(head_dim):
                        s = np.float32(s + np.float32(q[b * seq * H + i * H + h * head_dim + d] *
                                                      k[b * seq * H + j * H + h * head_dim + d]))
                    sc[i * seq + j] = np.float32(s * np.float32(scale))
            for i in range(seq):
                mx = np.float32(-np.finfo(np.float32).max)
                for j in range(seq):
                    mx = max(mx, sc[i * seq + j])
                tot = np.float32(0)
                for j in range(seq):
                    e = np.float32(math.exp(float(np.float32(sc[i * seq + j] - mx))))
                    sc[i * seq + j] = e
                    tot = np.float32(tot + e)
                for j in range(seq):
                    sc[i * seq + j] = np.float32(sc[i * seq + j] / tot)
            for i in range(seq):
                for d in range(head_dim):
                    s = np.float32(0)
                    for j in range(seq):
                        s = np.float32(s + np.float32(sc[i * seq + j] * v[b * seq * H + j * H + h * head_dim + d]))
                    out[b * seq * H + i * H + h * head_dim + d] = s
    return out


def attention_kat_inputs():
    # attention_test.go:71-93: batch 1, seq 4, 2 heads of 4, q = i*0.1, k = (n-i)*0.1, v = (i%3)*0.5
    batch, seq, heads, hd = 1, 4, 2, 4
    n = batch * seq * heads * hd
    i = np.arange(n)
    q = (i.astype(np.float32) * np.float32(0.1)).astype(np.float32)
    k = ((n - i).astype(np.float32) * np.float32(0.1)).astype(np.float32)
    v = ((i % 3).astype(np.float32) * np.float32(0.5)).astype(np.float32)
    return q, k, v, batch, seq, heads, hd, np.float32(1.0 / math.sqrt(hd))


def test_attention_known_answer(oracle_mod):
    q, k, v, batch, seq, heads, hd, scale = attention_kat_inputs()
    want = simple_attention_cpu(q, k, v, batch, seq, hd, heads, scale)
    L = oracle_mod.lib()
    out = np.zeros_like(q)
    lens = np.array([seq] * batch, np.int32)
    L.ref_attention(fp(q), fp(k), fp(v), fp(out), heads * hd, heads, lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                    batch, float(scale))
    mse = float(((out.astype(np.float64) - want) ** 2).mean())
    assert mse <= 1e-3  # the reference's bound (attention_test.go:121-124)
    # The oracle uses ExpFast where the KAT uses float64 exp: well inside ExpFast's error.
    assert np.abs(out - want).max() <= 5e-3
