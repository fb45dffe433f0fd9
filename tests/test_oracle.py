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
