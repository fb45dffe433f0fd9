"""GPU tests of the tensor-op entry points against numpy restatements of the reference ops."""
import ctypes

import numpy as np
import pytest

from helpers import attention_np, bf16_round, exp_fast_np, f16_round_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fl():
    import build
    build.build()
    import fletcher
    return fletcher


@pytest.fixture(scope="module")
def be(fl):
    return fl.Backend(0)


def test_mul_known_answer(fl, be):
    # internal/device/device_test.go:27-54
    a = be.new_tensor(2, 3, [1, 2, 3, 4, 5, 6])
    b = be.new_tensor(3, 2, [7, 8, 9, 10, 11, 12])
    np.testing.assert_allclose(a.linear(a, b, None).to_host().ravel(), [58, 64, 139, 154], atol=1e-6)


def test_layernorm_known_answer(fl, be):
    # internal/device/device_test.go:69-96
    a = be.new_tensor(1, 4, [1, 2, 3, 4])
    g = be.new_tensor(1, 4, [1, 1, 1, 1], dtype=fl.F32)
    b = be.new_tensor(1, 4, [0, 0, 0, 0], dtype=fl.F32)
    a.layer_norm(g, b, 1e-6)
    np.testing.assert_allclose(a.to_host().ravel(), [-1.3416407, -0.4472136, 0.4472136, 1.3416407], atol=1e-4)


def test_cast_bytes(fl, be):
    # internal/device/cast_test.go:11-47: 1.0 -> 0x3c00, -2.0 -> 0xc000
    t = be.new_tensor(1, 2, [1.0, -2.0])
    h = t.cast(fl.F16)
    assert list(h.raw_bytes().view(np.uint16)) == [0x3C00, 0xC000]


@pytest.mark.parametrize("rows,cols", [(7, 128), (300, 768), (5, 100), (3, 1536)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_add_layernorm(fl, be, rows, cols, dtype):
    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    r = rng.standard_normal((rows, cols)).astype(np.float32)
    g = rng.standard_normal(cols).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    dt = fl.DTYPES[dtype]
    tx, tr = be.new_tensor(rows, cols, x, dt), be.new_tensor(rows, cols, r, dt)
    tx.add_layer_norm(tr, be.new_tensor(1, cols, g, fl.F32), be.new_tensor(1, cols, b, fl.F32), 1e-12)
    if dtype == "bf16":
        x, r = bf16_round(x), bf16_round(r)
    s = x + r
    want = (s - s.mean(1, keepdims=True)) / np.sqrt(s.var(1, keepdims=True) + 1e-12) * g + b
    tol = 1e-4 if dtype == "f32" else 3e-2
    np.testing.assert_allclose(tx.to_host(), want, atol=tol * max(1, np.abs(want).max()))


@pytest.mark.parametrize("M,K,N,act", [(1, 64, 128, 0), (127, 128, 384, 0), (128, 768, 2304, 0), (300, 768, 768, 1),
                                       (513, 512, 128, 1), (200, 768, 6144, 4), (64, 128, 1024, 4), (1000, 3072, 768, 0)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_linear_tensor_core(fl, be, M, K, N, act, dtype):
    """16-bit Linear runs on the tcgen05 GEMM; compare with fp32 numpy on the same rounded inputs."""
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    dt = fl.DTYPES[dtype]
    tx, tw, tb = be.new_tensor(M, K, x, dt), be.new_tensor(K, N, w, dt), be.new_tensor(1, N, b, dt)
    got = tx.linear(tx, tw, tb, act).to_host()
    q = bf16_round if dtype == "bf16" else f16_round_ref
    y = q(x).astype(np.float64) @ q(w).astype(np.float64) + q(b)
    if act == 1:
        u = 0.7978846 * (y + 0.044715 * y ** 3)
        th = np.clip(u * (27 + u * u) / (27 + 9 * u * u), -np.inf, np.inf)
        th = np.where(u > 4, 1, np.where(u < -4, -1, th))
        y = 0.5 * y * (1 + th)
    elif act == 4:
        a, c = y[:, : N // 2], y[:, N // 2:]
        y = a / (1 + np.exp(-a)) * c
    err = np.abs(got - y).max() / max(1e-3, np.abs(y).max())
    assert err < (1e-2 if dtype == "bf16" else 2e-3), err


@pytest.mark.parametrize("M,K,N,act", [(64, 768, 3072, 1), (200, 3072, 768, 0), (1, 768, 6144, 4), (300, 768, 2304, 0)])
def test_linear_split_k(fl, be, M, K, N, act):
    """Small-M 16-bit GEMMs split K across CTAs (fp32 partial sums + a finishing epilogue kernel)
    once a model has lent its split-K workspace to the context; same check as above."""
    import dataclasses
    import synth
    cfg = dataclasses.replace(synth.NOMIC, num_layers=1)
    m = fl.BertModel(be, cfg, "bf16")
    m.load_raw(synth.make_weights(cfg, 1))
    lens = np.array([1024], np.int32)  # sizes the workspace for batches of up to 1024 tokens
    m.forward_batch(synth.make_ids(lens, cfg.vocab_size, 1), lens, 1)
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    dt = fl.DTYPES["bf16"]
    tx, tw, tb = be.new_tensor(M, K, x, dt), be.new_tensor(K, N, w, dt), be.new_tensor(1, N, b, dt)
    got = tx.linear(tx, tw, tb, act).to_host()
    y = bf16_round(x).astype(np.float64) @ bf16_round(w).astype(np.float64) + bf16_round(b)
    if act == 1:
        u = 0.7978846 * (y + 0.044715 * y ** 3)
        th = np.where(u > 4, 1, np.where(u < -4, -1, u * (27 + u * u) / (27 + 9 * u * u)))
        y = 0.5 * y * (1 + th)
    elif act == 4:
        a, c = y[:, : N // 2], y[:, N // 2:]
        y = a / (1 + np.exp(-a)) * c
    err = np.abs(got - y).max() / max(1e-3, np.abs(y).max())
    assert err < 1e-2, err
    del m


@pytest.mark.parametrize("act", [0, 1, 2, 4])
def test_linear_f32(fl, be, act):
    rng = np.random.default_rng(act)
    M, K, N = 37, 96, 160
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.1).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    tx = be.new_tensor(M, K, x)
    got = tx.linear(tx, be.new_tensor(K, N, w), be.new_tensor(1, N, b), act).to_host()
    y = x @ w + b
    if act == 1:
        u = np.float32(0.7978846) * (y + np.float32(0.044715) * y * y * y)
        th = np.where(u > 4, 1, np.where(u < -4, -1, u * (27 + u * u) / (27 + 9 * u * u)))
        y = 0.5 * y * (1 + th)
    elif act == 2:
        y = np.where(y > 4, 1, np.where(y < -4, -1, y * (27 + y * y) / (27 + 9 * y * y)))
    elif act == 4:
        a, c = y[:, : N // 2], y[:, N // 2:]
        y = a / (1 + np.exp(-a.astype(np.float64))) * c
    np.testing.assert_allclose(got, y, atol=2e-4, rtol=1e-4)


@pytest.mark.parametrize("lengths", [[1], [5, 64, 65], [128, 1, 200], [63, 127, 129]])
def test_attention_varlen_f32(fl, be, lengths):
    rng = np.random.default_rng(sum(lengths))
    H, nh = 128, 2
    T = sum(lengths)
    q, k, v = (rng.standard_normal((T, H)).astype(np.float32) for _ in range(3))
    tq, tk, tv = (be.new_tensor(T, H, a) for a in (q, k, v))
    got = tq.attention_varlen(tq, tk, tv, lengths, nh, 1 / 8).to_host()
    np.testing.assert_allclose(got, attention_np(q, k, v, lengths, nh, 1 / 8), atol=1e-5)


@pytest.mark.parametrize("lengths", [[1], [5, 64, 65], [128, 1, 200], [63, 127, 129, 700]])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_flash_attention_varlen(fl, be, lengths, dtype):
    rng = np.random.default_rng(sum(lengths))
    H, nh = 768, 12
    T = sum(lengths)
    q, k, v = (rng.standard_normal((T, H)).astype(np.float32) for _ in range(3))
    dt = fl.DTYPES[dtype]
    tq, tk, tv = (be.new_tensor(T, H, a, dt) for a in (q, k, v))
    got = tq.attention_varlen(tq, tk, tv, lengths, nh, 0.125).to_host()
    qq = bf16_round if dtype == "bf16" else f16_round_ref
    want = attention_np(qq(q), qq(k), qq(v), lengths, nh, 0.125, fast=False)
    assert np.abs(got - want).max() < (3e-2 if dtype == "bf16" else 5e-3)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_flash_attention_moving_max(fl, be, dtype):
    """Scores spread over hundreds of units: row maxima jump between 64-key blocks by more than
    the P range (2^64 for bf16, 2^15 for fp16), so the kernel's reference-max update and O
    rescale run, including on rows whose first key is far below the row max."""
    rng = np.random.default_rng(11)
    lengths = [700, 130, 64, 1, 257]
    H, nh = 768, 12
    T = sum(lengths)
    q = (rng.standard_normal((T, H)) * 6).astype(np.float32)
    k = (rng.standard_normal((T, H)) * 6).astype(np.float32)
    v = rng.standard_normal((T, H)).astype(np.float32)
    k[650] *= 4  # a late key with much larger scores in the first sequence
    dt = fl.DTYPES[dtype]
    tq, tk, tv = (be.new_tensor(T, H, a, dt) for a in (q, k, v))
    got = tq.attention_varlen(tq, tk, tv, lengths, nh, 0.125).to_host()
    qq = bf16_round if dtype == "bf16" else f16_round_ref
    want = attention_np(qq(q), qq(k), qq(v), lengths, nh, 0.125, fast=False)
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() < (6e-2 if dtype == "bf16" else 2e-2)


def test_attention_uniform_matches_varlen(fl, be):
    rng = np.random.default_rng(0)
    B, S, H, nh = 3, 40, 128, 2
    q, k, v = (rng.standard_normal((B * S, H)).astype(np.float32) for _ in range(3))
    tq, tk, tv = (be.new_tensor(B * S, H, a) for a in (q, k, v))
    a = tq.attention(tq, tk, tv, B, S, nh, 0.125).to_host()
    b = tq.attention_varlen(tq, tk, tv, [S] * B, nh, 0.125).to_host()
    assert np.array_equal(a, b)


def test_rope_matches_oracle(fl, be, oracle_mod):
    rng = np.random.default_rng(1337)
    B, S, nh, dh = 2, 128, 4, 64  # rope_test.go:11-75 shapes
    x = rng.standard_normal((B * S, nh * dh)).astype(np.float32)
    t = be.new_tensor(B * S, nh * dh, x)
    t.apply_rope(B, S, nh, dh)
    want = x.copy()
    pos = (np.arange(B * S) % S).astype(np.int32)
    oracle_mod.lib().ref_rope(want.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), B * S, nh, dh,
                              pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 10000.0)
    np.testing.assert_allclose(t.to_host(), want, atol=2e-6)


def test_softmax_matches_expfast(fl, be):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((9, 300)) * 4).astype(np.float32)
    t = be.new_tensor(9, 300, x)
    t.softmax()
    e = exp_fast_np(x - x.max(1, keepdims=True))
    np.testing.assert_allclose(t.to_host(), e / e.sum(1, keepdims=True), atol=1e-6)


@pytest.mark.parametrize("H", [128, 768, 100])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_mean_pool_l2(fl, be, H, dtype):
    rng = np.random.default_rng(H)
    lengths = [1, 7, 300, 64]
    x = rng.standard_normal((sum(lengths), H)).astype(np.float32)
    t = be.new_tensor(sum(lengths), H, x, fl.DTYPES[dtype])
    got = t.mean_pool_l2(lengths).to_host()
    xs = bf16_round(x) if dtype == "bf16" else x
    off, want = 0, []
    for L in lengths:
        m = xs[off:off + L].astype(np.float64).mean(0)
        want.append(m / np.linalg.norm(m))
        off += L
    np.testing.assert_allclose(got, np.array(want), atol=1e-5)


def test_has_nan_and_gather(fl, be):
    t = be.new_tensor(4, 3, np.arange(12, dtype=np.float32))
    assert not t.has_nan()
    g = t.gather([3, 0, 3])
    np.testing.assert_array_equal(g.to_host(), np.arange(12, dtype=np.float32).reshape(4, 3)[[3, 0, 3]])
    t2 = be.new_tensor(2, 2, [1, np.nan, 3, 4])
    assert t2.has_nan()
    t3 = be.new_tensor(1, 2, [np.inf, 0], fl.BF16)
    assert t3.has_nan()
    with pytest.raises(fl.FletcherError):
        t.gather([4])


def test_vram_usage_and_elementwise(fl, be):
    alloc, total = be.vram_usage()
    assert total > 100e9 and alloc > 0
    t = be.new_tensor(2, 2, [1, 2, 3, 4])
    t.scale(2.0)
    t.add_scalar(1.0)
    t.add(be.new_tensor(2, 2, [1, 1, 1, 1]))
    t.add_bias(be.new_tensor(1, 2, [10, 20]))
    np.testing.assert_allclose(t.to_host().ravel(), [14, 26, 18, 30])
