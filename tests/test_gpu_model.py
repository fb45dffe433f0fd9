"""GPU parity of the whole forward pass (Cuda_Model_*) against the CPU oracle and its golden
fixtures.  fp32: per-vector cosine >= 0.99999 and max-abs <= 1e-4; bf16/fp16: cosine >= 0.999."""
import dataclasses

import numpy as np
import pytest

import synth
from helpers import assert_close_16, assert_close_f32, load_golden

pytestmark = pytest.mark.gpu

GOLDEN = ["tiny_ragged_spec", "tiny_uniform_literal", "nomic2_ragged_spec", "nomic2_uniform_literal"]


@pytest.fixture(scope="module")
def be():
    import build
    build.build()
    import fletcher
    b = fletcher.Backend(0)
    yield b


_models = {}


def model(be, cfg, dtype, seed):
    import fletcher
    key = (cfg, dtype, seed)
    if key not in _models:
        m = fletcher.BertModel(be, cfg, dtype)
        m.load_raw(synth.make_weights(cfg, seed))
        _models[key] = m
    return _models[key]


@pytest.mark.parametrize("name", GOLDEN)
@pytest.mark.parametrize("pooling", [0, 1])
def test_f32_matches_golden(be, name, pooling):
    cfg, g = load_golden(name)
    m = model(be, cfg, "f32", int(g["weight_seed"]))
    got = m.forward_batch(g["ids"], g["lengths"], pooling)
    assert_close_f32(got, g["mean" if pooling == 1 else "cls"], f"{name} pooling={pooling}")


@pytest.mark.parametrize("name", GOLDEN)
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_16bit_matches_golden(be, name, dtype):
    cfg, g = load_golden(name)
    m = model(be, cfg, dtype, int(g["weight_seed"]))
    for pooling, key in ((1, "mean"), (0, "cls")):
        got = m.forward_batch(g["ids"], g["lengths"], pooling)
        assert_close_16(got, g[key], f"{name} {dtype} {key}")


def test_cfg1_full_batch_f32(be, oracle_mod):
    w = synth.WORKLOADS["cfg1"]
    lens = w.lengths()
    ids = synth.make_ids(lens, w.cfg.vocab_size, w.seed)
    blob = synth.make_weights(w.cfg, w.seed)
    want = oracle_mod.forward(w.cfg, blob, ids, lens)
    m = model(be, w.cfg, "f32", w.seed)
    assert_close_f32(m.forward_batch(ids, lens, 1), want["mean"], "cfg1 mean")
    assert_close_f32(m.forward_batch(ids, lens, 0), want["cls"], "cfg1 cls")


@pytest.mark.parametrize("lengths", [[1], [2, 1, 3], [63, 64, 65], [127, 128, 129, 1], [300, 17],
                                     [700, 601],  # single-SM tiles, no split-K (1024 < T < 2048)
                                     [2048, 700, 64]])  # cfg4 long context; 2-SM tiles
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_edge_lengths_nomic(be, oracle_mod, lengths, dtype):
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    lens = np.array(lengths, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 21)
    blob = synth.make_weights(cfg, 1)
    want = oracle_mod.forward(cfg, blob, ids, lens)
    got = model(be, cfg, dtype, 1).forward_batch(ids, lens, 1)
    (assert_close_f32 if dtype == "f32" else assert_close_16)(got, want["mean"], f"{dtype} {lengths}")


def test_packing_invariance_bitexact(be):
    """A sequence's embedding does not depend on the other sequences packed with it: bit-exact
    while the batch and the single sequence both run unsplit GEMMs (more than 1024 tokens),
    within 16-bit tolerance when the shorter batches' GEMMs split K into a different number of
    fp32 partial sums."""
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    m = model(be, cfg, "bf16", 1)
    for lengths, exact in (([1100, 1030, 1500], True), ([200, 5, 64, 129, 31], False)):
        lens = np.array(lengths, np.int32)
        ids = synth.make_ids(lens, cfg.vocab_size, 9)
        full = m.forward_batch(ids, lens, 1)
        off = 0
        for i, L in enumerate(lens):
            single = m.forward_batch(ids[off:off + L], lens[i:i + 1], 1)
            if exact:
                assert np.array_equal(single[0], full[i]), (lengths, i)
            else:
                assert_close_16(single, full[i:i + 1], f"packed vs single {lengths} {i}")
            off += L


def _oracle_subset(oracle_mod, cfg, blob, ids, lens, pick):
    """Spec-mode oracle vectors of the sequences `pick` of a packed batch, in one packed call."""
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    sub_ids = np.concatenate([ids[starts[i]:starts[i] + lens[i]] for i in pick]).astype(np.int32)
    return oracle_mod.forward(cfg, blob, sub_ids, lens[pick])["mean"]


def test_cfg3_full_size_bf16(be, oracle_mod):
    """BASELINE cfg3 at full size (12 layers, B=256, l in [32,512], seed 1): finite unit vectors,
    and 64 sequences spread over the length range (every 4th by length, the shortest and the
    longest included) against the oracle."""
    w = synth.WORKLOADS["cfg3"]
    lens = w.lengths()
    ids = synth.make_ids(lens, w.cfg.vocab_size, w.seed)
    blob = synth.make_weights(w.cfg, w.seed)
    m = model(be, w.cfg, "bf16", w.seed)
    got = m.forward_batch(ids, lens, 1)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-4)
    order = np.argsort(lens, kind="stable")
    pick = np.unique(np.concatenate([order[::4], order[-1:]]))
    assert len(pick) >= 64
    assert_close_16(got[pick], _oracle_subset(oracle_mod, w.cfg, blob, ids, lens, pick), "cfg3 sample")


def test_cfg4_full_depth_long_context_bf16(be, oracle_mod):
    """BASELINE cfg4 at full depth and size: 12 layers, B=32, l log-uniform in [64, 2048], seed 1,
    packed varlen.  Every sequence, the longest included, against the oracle."""
    w = synth.WORKLOADS["cfg4"]
    lens = w.lengths()
    assert lens.max() > 1024
    ids = synth.make_ids(lens, w.cfg.vocab_size, w.seed)
    blob = synth.make_weights(w.cfg, w.seed)
    m = model(be, w.cfg, "bf16", w.seed)
    got = m.forward_batch(ids, lens, 1)
    assert np.isfinite(got).all()
    pick = np.arange(len(lens))
    assert_close_16(got, _oracle_subset(oracle_mod, w.cfg, blob, ids, lens, pick), "cfg4 all 32")


def test_cfg2_full_batch_bf16(be, oracle_mod):
    """BASELINE cfg2: bert-tiny bf16, B=1024, l in [8,128]: every sequence against the oracle, both
    pooling heads."""
    w = synth.WORKLOADS["cfg2"]
    lens = w.lengths()
    ids = synth.make_ids(lens, w.cfg.vocab_size, w.seed)
    blob = synth.make_weights(w.cfg, w.seed)
    want = oracle_mod.forward(w.cfg, blob, ids, lens)
    m = model(be, w.cfg, "bf16", w.seed)
    assert_close_16(m.forward_batch(ids, lens, 1), want["mean"], "cfg2 mean")
    assert_close_16(m.forward_batch(ids, lens, 0), want["cls"], "cfg2 cls")


def test_errors_are_reported(be):
    import fletcher
    cfg = synth.BERT_TINY
    m = fletcher.BertModel(be, cfg, "f32")
    with pytest.raises(fletcher.FletcherError):
        m.load_raw(np.zeros(10, np.float32))
    m.load_raw(synth.make_weights(cfg, 0))
    with pytest.raises(fletcher.FletcherError) as e:
        m.forward_batch(np.array([101, 99999, 102], np.int32), np.array([3], np.int32))
    assert "out of bounds" in str(e.value)
    m.close()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_graph_replay_matches_eager(be, dtype):
    """Repeated shapes are captured into a CUDA graph and replayed: results stay bit-identical
    to eager execution, also when other shapes are interleaved."""
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    m = model(be, cfg, dtype, 1)
    batches = []
    for seed, lens in ((31, [40, 7, 130]), (32, [64]), (33, [5, 200])):
        lens = np.array(lens, np.int32)
        batches.append((synth.make_ids(lens, cfg.vocab_size, seed), lens))
    m.set_graphs(False)
    eager = [m.forward_batch(i, l, 1) for i, l in batches]
    m.set_graphs(True)
    for rep in range(4):  # first call eager, second captures, then replays
        for (i, l), want in zip(batches, eager):
            assert np.array_equal(m.forward_batch(i, l, 1), want), rep


@pytest.mark.parametrize("out", ["f16", "bf16"])
def test_16bit_output_transport(be, out):
    """ForwardBatchEx returns the vectors converted to 16 bits on the device: fp16 bit-identical
    to the reference's Float32ToFloat16 (utils.go:13-72) of the float32 result (or to IEEE
    rounding under FLETCHER_HALF_RNE), bf16 to round-to-nearest-even."""
    import fletcher
    from helpers import bf16_round, f32_to_f16_ref
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    m = model(be, cfg, "bf16", 1)
    lens = np.array([50, 3, 129], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 41)
    f32 = m.forward_batch(ids, lens, 1)
    if out == "f16":
        got = m.forward_batch_16(ids, lens, 1, fletcher.F16)
        assert np.array_equal(got.view(np.uint16), f32_to_f16_ref(f32))
        be.set_half_conversion(fletcher.HALF_RNE)
        try:
            assert np.array_equal(m.forward_batch_16(ids, lens, 1, fletcher.F16), f32.astype(np.float16))
        finally:
            be.set_half_conversion(fletcher.HALF_REFERENCE)
    else:
        got = m.forward_batch_16(ids, lens, 1, fletcher.BF16)
        assert np.array_equal((got.astype(np.uint32) << 16).view(np.float32), bf16_round(f32))


def test_safetensors_checkpoint_end_to_end(be, tmp_path, oracle_mod):
    """A BF16 SafeTensors checkpoint (HF names, (out, in) Linear weights) loads through the
    ingest path and embeds like the oracle on the same (bf16-rounded) weights."""
    import fletcher
    import weights
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    blob = synth.make_weights(cfg, 1)
    p = tmp_path / "nomic2.safetensors"
    weights.write_safetensors(str(p), weights.safetensors_from_blob(blob, cfg), "BF16")
    loaded = weights.blob_from_safetensors(str(p), cfg)
    m = fletcher.BertModel(be, cfg, "bf16")
    m.load_raw(loaded)
    lens = np.array([77, 20], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 13)
    want = oracle_mod.forward(cfg, loaded, ids, lens)["mean"]
    assert_close_16(m.forward_batch(ids, lens, 1), want, "safetensors bf16")
    m.close()


def test_async_batches_match_sync(be):
    """Cuda_Model_ForwardBatchAsync / Cuda_Model_Wait: several batches in flight (more than the
    eight slots), pinned buffers, waits in any order; the vectors equal the synchronous call's."""
    import fletcher
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    m = model(be, cfg, "bf16", 1)
    batches = []
    for i, lengths in enumerate([[40, 7, 300], [129, 64], [512], [5, 5, 5, 5]] * 3):
        lens = np.array(lengths, np.int32)
        batches.append((synth.make_ids(lens, cfg.vocab_size, 40 + i), lens))
    want = [m.forward_batch(ids, lens, 1) for ids, lens in batches]
    bufs = [(fletcher.PinnedArray(be, (ids.size,), np.int32), fletcher.PinnedArray(be, (lens.size, cfg.hidden), np.float32))
            for ids, lens in batches]
    tickets = []
    for (ids, lens), (bi, bo) in zip(batches, bufs):
        bi.array[:] = ids
        tickets.append(m.forward_batch_async(bi.ptr, lens, 1, bo.ptr))
    for t in reversed(tickets):
        m.wait(t)
    for w, (bi, bo) in zip(want, bufs):
        assert np.array_equal(bo.array, w)
        bi.close()
        bo.close()



@pytest.mark.parametrize("lengths", [[700, 601], [2048, 700, 64]])
def test_fp16_tiled_paths_nomic(be, oracle_mod, lengths):
    """fp16 through the non-split GEMMs (single-SM and 2-SM tiles, both residual epilogues)."""
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    lens = np.array(lengths, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 23)
    blob = synth.make_weights(cfg, 1)
    want = oracle_mod.forward(cfg, blob, ids, lens)
    got = model(be, cfg, "f16", 1).forward_batch(ids, lens, 1)
    assert_close_16(got, want["mean"], f"f16 {lengths}")


# BERT-base shape (GELU, absolute positions, biases) from bert-tiny's architecture.
BERT_BASE_2L = dataclasses.replace(synth.BERT_TINY, hidden=768, num_heads=12, intermediate=3072, num_layers=2)


@pytest.mark.parametrize("cfg_name,lengths", [
    ("base", [512, 512, 500, 400, 300, 512, 200]),  # 2,936 tokens: 2-SM tiles
    ("base", [512, 500, 301]),                      # 1,313 tokens: single-SM tiles, no split-K
    ("tiny", [128] * 20 + [77] * 30 + [5] * 9),      # 4,915 tokens: tiled, 128-wide tiles
])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_gelu_absolute_tiled_paths(be, oracle_mod, cfg_name, lengths, dtype):
    """The GELU epilogue, absolute positions and both poolers through the non-split GEMMs."""
    cfg = BERT_BASE_2L if cfg_name == "base" else synth.BERT_TINY
    lens = np.array(lengths, np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 31)
    blob = synth.make_weights(cfg, 3)
    want = oracle_mod.forward(cfg, blob, ids, lens)
    m = model(be, cfg, dtype, 3)
    assert_close_16(m.forward_batch(ids, lens, 1), want["mean"], f"{cfg_name} {dtype} mean")
    assert_close_16(m.forward_batch(ids, lens, 0), want["cls"], f"{cfg_name} {dtype} cls")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_absolute_positions_clamp_past_max(be, oracle_mod, dtype):
    """Rows at or past max_positions (512 for bert-tiny) use the last position row (bert.go's
    clamp to max - 1)."""
    cfg = synth.BERT_TINY
    lens = np.array([600, 30, 513], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 41)
    blob = synth.make_weights(cfg, 3)
    want = oracle_mod.forward(cfg, blob, ids, lens)
    got = model(be, cfg, dtype, 3).forward_batch(ids, lens, 1)
    (assert_close_f32 if dtype == "f32" else assert_close_16)(got, want["mean"], f"{dtype} clamp")


@pytest.mark.parametrize("file_dtype,model_dtype", [("BF16", "bf16"), ("F32", "bf16"), ("F16", "f16"), ("F32", "f32")])
def test_direct_16bit_checkpoint_ingest(be, tmp_path, file_dtype, model_dtype):
    """Cuda_Model_LoadTensor takes each SafeTensors tensor in its stored dtype, (out, in) Linear
    weights included, with no host fp32 blob: the model it builds is bit-identical (same
    outputs) to LoadRaw of the host-widened blob.  fp16 is compared under IEEE conversion,
    because the reference's fp16 conversion of the widened blob would flush the file's
    subnormals that a direct fp16 copy keeps."""
    import fletcher
    import weights
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2, has_bias=True)
    blob = synth.make_weights(cfg, 21)
    path = str(tmp_path / f"ckpt_{file_dtype}.safetensors")
    weights.write_safetensors(path, weights.safetensors_from_blob(blob, cfg), file_dtype)
    lens = np.array([77, 3, 200], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 8)
    if file_dtype == "F16":
        be.set_half_conversion(fletcher.HALF_RNE)
    try:
        direct = fletcher.BertModel(be, cfg, model_dtype)
        weights.load_safetensors_direct(direct, path)
        viaraw = fletcher.BertModel(be, cfg, model_dtype)
        viaraw.load_raw(weights.blob_from_safetensors(path, cfg))
        for pooling in (0, 1):
            a = direct.forward_batch(ids, lens, pooling)
            b = viaraw.forward_batch(ids, lens, pooling)
            assert np.array_equal(a, b), (pooling, np.abs(a - b).max())
        direct.close()
        viaraw.close()
    finally:
        be.set_half_conversion(fletcher.HALF_REFERENCE)


def test_load_tensor_errors(be):
    import fletcher
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1)
    m = fletcher.BertModel(be, cfg, "bf16")
    with pytest.raises(fletcher.FletcherError, match="not part of this model"):
        m.load_tensor("encoder.layer.1.attention.self.query.weight", np.zeros((128, 128), np.float32), fletcher.F32)
    with pytest.raises(fletcher.FletcherError, match="size mismatch"):
        m.load_tensor("embeddings.LayerNorm.weight", np.zeros(127, np.float32), fletcher.F32)
    with pytest.raises(fletcher.FletcherError, match="shape mismatch"):
        m.load_tensor("encoder.layer.0.intermediate.dense.weight", np.zeros((128, 512), np.float32), fletcher.F32,
                      transposed=True)
    with pytest.raises(fletcher.FletcherError, match="only Linear weights"):
        m.load_tensor("embeddings.word_embeddings.weight", np.zeros((128, 30522), np.float32), fletcher.F32,
                      transposed=True)
    assert not m.is_loaded()
    with pytest.raises(fletcher.FletcherError, match="not loaded"):
        m.forward_batch(np.array([101, 102], np.int32), np.array([2], np.int32))
    m.close()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_final_layernorm_fused_into_pool(be, dtype):
    """A mean-pooled 16-bit forward normalises its final rows inside the pooling kernels: the
    vectors equal those of the unfused path (separate LayerNorm pass + pool) up to fp32 summation
    order, the final hidden state is not stored, and keeping it restores LastHidden."""
    import fletcher
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    m = fletcher.BertModel(be, cfg, dtype)
    m.load_raw(synth.make_weights(cfg, 4))
    lens = np.array([1, 64, 65, 200, 513, 7, 130], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 12)
    fused = m.forward_batch(ids, lens, fletcher.POOL_MEAN_L2)
    with pytest.raises(fletcher.FletcherError, match="SetKeepHidden"):
        m.last_hidden(int(lens.sum()))
    m.set_keep_hidden(True)
    plain = m.forward_batch(ids, lens, fletcher.POOL_MEAN_L2)
    hid = m.last_hidden(int(lens.sum()))
    assert np.abs(fused - plain).max() <= 2e-6
    # The unfused path's pool of the stored hidden state, restated in numpy.
    starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
    mean = np.stack([hid[a:a + l].astype(np.float64).mean(0) for a, l in zip(starts, lens)])
    mean /= np.linalg.norm(mean, axis=1, keepdims=True)
    assert np.abs(fused - mean).max() <= 2e-6
    m.close()
