"""The op-level boundary as a drop-in: bert.go's ForwardBatch (bert.go:149-488, 610-820) replayed
op by op through the tensor ABI (longbow-fletcher_b200/bert_ops.py) against the oracle's literal
mode, which is the reference as written.  fp32: per-vector cosine >= 0.99999 and max-abs <= 1e-4;
bf16: cosine >= 0.999.  Plus the ops that route needs (Slice, Mul with T() views, Copy) against
numpy, and the cached weight packing of Linear."""
import dataclasses

import numpy as np
import pytest

import synth
from helpers import assert_close_16, assert_close_f32, bf16_round, f16_round_ref

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


TINY = synth.BERT_TINY
NOMIC2 = dataclasses.replace(synth.NOMIC, num_layers=2)
CASES = [
    ("tiny_uniform", TINY, [37, 37, 37, 37]),
    ("tiny_ragged", TINY, [12, 128, 1, 77, 40]),
    ("nomic2_uniform", NOMIC2, [96, 96, 96]),
    ("nomic2_ragged", NOMIC2, [20, 150, 64, 33]),  # lengths[0] smallest: literal RoPE stays in bounds
]


@pytest.mark.parametrize("name,cfg,lengths", CASES, ids=[c[0] for c in CASES])
def test_bert_go_replay_matches_oracle_literal_f32(fl, be, oracle_mod, name, cfg, lengths):
    import bert_ops
    lens = np.array(lengths, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 17)
    blob = synth.make_weights(cfg, 5)
    m = bert_ops.OpsBertModel(be, cfg, blob, fl.F32)
    want = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_LITERAL)
    assert_close_f32(m.forward_batch(ids, lens, fl.POOL_CLS_TANH), want["cls"], f"{name} cls")
    assert_close_f32(m.forward_batch(ids, lens, fl.POOL_MEAN_L2), want["mean"], f"{name} mean")


def test_bert_go_replay_literal_rope_out_of_bounds(fl, be, oracle_mod):
    """lengths[0] longest with RoPE: the reference rotates batch*lengths[0] rows, past the packed
    rows (its goroutines index out of the slice and the Go runtime panics).  Both sides refuse."""
    import bert_ops
    lens = np.array([150, 20, 64], np.int32)
    ids = synth.make_ids(lens, NOMIC2.vocab_size, 3)
    blob = synth.make_weights(NOMIC2, 5)
    with pytest.raises(RuntimeError):
        oracle_mod.forward(NOMIC2, blob, ids, lens, mode=oracle_mod.MODE_LITERAL)
    m = bert_ops.OpsBertModel(be, NOMIC2, blob, fl.F32)
    with pytest.raises(fl.FletcherError):
        m.forward_batch(ids, lens)


@pytest.mark.parametrize("name,cfg,lengths", [CASES[0], CASES[2]], ids=["tiny_uniform", "nomic2_uniform"])
def test_bert_go_replay_bf16(fl, be, oracle_mod, name, cfg, lengths):
    import bert_ops
    lens = np.array(lengths, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 17)
    blob = synth.make_weights(cfg, 5)
    m = bert_ops.OpsBertModel(be, cfg, blob, fl.BF16)
    want = oracle_mod.forward(cfg, blob, ids, lens, mode=oracle_mod.MODE_LITERAL)
    assert_close_16(m.forward_batch(ids, lens, fl.POOL_MEAN_L2), want["mean"], f"{name} bf16 mean")


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(5, 7, 3), (128, 192, 256), (300, 64, 128)])
def test_mul_transposed_views(fl, be, dtype, ta, tb, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    dt = fl.DTYPES[dtype]
    q = (lambda a: a) if dtype == "f32" else bf16_round if dtype == "bf16" else f16_round_ref
    A = q(rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32))
    B = q(rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32))
    ta_, tb_ = be.new_tensor(*A.shape, A, dt), be.new_tensor(*B.shape, B, dt)
    c = be.new_tensor(m, n, None, dt)
    c.mul(ta_.T() if ta else ta_, tb_.T() if tb else tb_)
    want = (A.T if ta else A).astype(np.float64) @ (B.T if tb else B).astype(np.float64)
    got = c.to_host()
    tol = 1e-4 if dtype == "f32" else 2e-2 * np.sqrt(k) / 8
    assert np.abs(got - want).max() <= tol * max(1.0, np.abs(want).max())


def test_mul_known_answer_and_shape_errors(fl, be):
    # device_test.go:27-54 through Mul
    a = be.new_tensor(2, 3, [1, 2, 3, 4, 5, 6])
    b = be.new_tensor(3, 2, [7, 8, 9, 10, 11, 12])
    c = be.new_tensor(2, 2)
    c.mul(a, b)
    np.testing.assert_allclose(c.to_host().ravel(), [58, 64, 139, 154], atol=1e-6)
    with pytest.raises(fl.FletcherError):
        c.mul(a, a)  # 2x3 . 2x3
    d = be.new_tensor(3, 3)
    d.mul(a.T(), a)  # 3x2 . 2x3
    A = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    np.testing.assert_allclose(d.to_host(), A.T @ A, atol=1e-5)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_slice_is_a_copy_and_copy_with_offsets(fl, be, dtype):
    dt = fl.DTYPES[dtype]
    x = np.arange(12 * 10, dtype=np.float32).reshape(12, 10)
    t = be.new_tensor(12, 10, x, dt)
    s = t.slice(3, 7, 2, 9)
    np.testing.assert_array_equal(s.to_host(), x[3:7, 2:9])
    s.scale(0.0)  # writing the slice leaves the source alone (cpu_backend.go:288-303)
    np.testing.assert_array_equal(t.to_host(), x)
    with pytest.raises(fl.FletcherError):
        t.slice(5, 5, 0, 1)
    with pytest.raises(fl.FletcherError):
        t.slice(0, 13, 0, 1)
    u = be.new_tensor(1, 30, None, dt)
    be.check(fl.lib().Cuda_Copy(be.ctx, u.buf, 10, t.buf, 50, 20))
    want = np.zeros(30, np.float32)
    want[10:30] = x.ravel()[50:70]
    np.testing.assert_array_equal(u.to_host().ravel(), want)


def test_linear_caches_the_packed_weight(fl, be):
    """Repeated Linear calls on one 16-bit weight pack it once; writing the weight invalidates it."""
    rng = np.random.default_rng(0)
    x = bf16_round(rng.standard_normal((256, 256)).astype(np.float32))
    w1 = bf16_round(rng.standard_normal((256, 512)).astype(np.float32) * 0.05)
    w2 = bf16_round(rng.standard_normal((256, 512)).astype(np.float32) * 0.05)
    tx, tw = be.new_tensor(256, 256, x, fl.BF16), be.new_tensor(256, 512, w1, fl.BF16)
    y = tx.linear(tx, tw, None)
    n0 = be.launch_count()
    alloc0 = be.vram_usage()[0]
    for _ in range(3):
        y = tx.linear(tx, tw, None)
    assert be.launch_count() - n0 == 3  # one GEMM per call, no repacking
    be.synchronize()
    del y
    assert be.vram_usage()[0] <= alloc0
    np.testing.assert_allclose(tx.linear(tx, tw, None).to_host(), x @ w1, atol=5e-2)
    tw.copy_from_float32(w2)
    np.testing.assert_allclose(tx.linear(tx, tw, None).to_host(), x @ w2, atol=5e-2)
