"""Weight ingestion on CPU: SafeTensors (F32 / F16 / BF16) and raw files map onto the raw blob
with the reference's names and transpose rule (loader.go:155-296)."""
import dataclasses

import numpy as np
import pytest

import synth
import weights


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_safetensors_round_trip(tmp_path, dtype):
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1, vocab_size=300, max_positions=64)
    blob = synth.make_weights(cfg, 3)
    p = tmp_path / "m.safetensors"
    weights.write_safetensors(str(p), weights.safetensors_from_blob(blob, cfg), dtype)
    got = weights.blob_from_safetensors(str(p), cfg)
    if dtype == "F32":
        assert np.array_equal(got, blob)
    else:
        tol = 1e-3 if dtype == "F16" else 8e-3
        np.testing.assert_allclose(got, blob, rtol=tol, atol=1e-6)


def test_linear_weights_are_transposed(tmp_path):
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1, vocab_size=300, max_positions=64)
    blob = synth.make_weights(cfg, 4)
    t = weights.safetensors_from_blob(blob, cfg)
    wq = synth.weight_views(cfg, blob)["layer0.wq"]  # (in, out)
    assert np.array_equal(t["encoder.layer.0.attention.self.query.weight"], wq.T)  # HF (out, in)
    assert t["embeddings.word_embeddings.weight"].shape == (300, 128)  # not transposed


def test_missing_and_mismatched_tensors(tmp_path):
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1, vocab_size=300, max_positions=64)
    t = weights.safetensors_from_blob(synth.make_weights(cfg, 5), cfg)
    p = tmp_path / "m.safetensors"
    bad = dict(t)
    del bad["pooler.dense.bias"]
    weights.write_safetensors(str(p), bad)
    with pytest.raises(KeyError):
        weights.blob_from_safetensors(str(p), cfg)
    bad = dict(t)
    bad["encoder.layer.0.output.dense.weight"] = np.zeros((10, 10), np.float32)
    weights.write_safetensors(str(p), bad)
    with pytest.raises(ValueError):
        weights.blob_from_safetensors(str(p), cfg)


def test_raw_file(tmp_path):
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1, vocab_size=300, max_positions=64)
    blob = synth.make_weights(cfg, 6)
    p = tmp_path / "m.bin"
    blob.astype("<f4").tofile(p)
    assert np.array_equal(weights.read_raw(str(p), cfg), blob)
    blob[:-1].tofile(p)
    with pytest.raises(ValueError):
        weights.read_raw(str(p), cfg)


@pytest.mark.parametrize("dtype,npdt", [("F32", np.float32), ("F16", np.float16), ("BF16", np.uint16)])
def test_raw_reader_keeps_stored_bytes(tmp_path, dtype, npdt):
    """The direct loader's reader hands each tensor over in its stored dtype (no widening)."""
    cfg = dataclasses.replace(synth.BERT_TINY, num_layers=1, vocab_size=300, max_positions=64)
    t = weights.safetensors_from_blob(synth.make_weights(cfg, 7), cfg)
    p = tmp_path / "m.safetensors"
    weights.write_safetensors(str(p), t, dtype)
    raw = weights.read_safetensors_raw(str(p))
    arr, tag = raw["encoder.layer.0.intermediate.dense.weight"]
    assert tag == dtype and arr.dtype == npdt and arr.shape == (512, 128)  # (out, in) as stored
    widened = weights.read_safetensors(str(p))["encoder.layer.0.intermediate.dense.weight"]
    back = (arr.astype(np.uint32) << 16).view(np.float32) if dtype == "BF16" else arr.astype(np.float32)
    assert np.array_equal(back, widened)


def test_checkpoint_tensor_names_match_the_library(tmp_path):
    """The names the direct loader sends are the ones Cuda_Model_TensorName enumerates."""
    import ctypes

    import build
    build.build()
    import fletcher
    cfg = dataclasses.replace(synth.NOMIC, num_layers=2)
    c = synth.to_c(cfg)
    L = fletcher.lib()
    n = L.Cuda_Model_TensorCount(ctypes.byref(c))
    names = []
    for i in range(n):
        buf = ctypes.create_string_buffer(128)
        assert L.Cuda_Model_TensorName(ctypes.byref(c), i, buf, 128) == 0
        names.append(buf.value.decode())
    assert names == [hf for hf, _ in weights.hf_names(cfg)]
