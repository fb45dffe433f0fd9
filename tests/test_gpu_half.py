"""fp16 bytes on the device against the reference's host conversion (internal/device/utils.go:13-91),
which its fp16 CUDA backend applies in CopyFromFloat32, Set and ToHost (cuda_linux.go:128,148,163).
Byte-level work: the bar is bit-exact, against the numpy restatement in tests/helpers.py."""
import numpy as np
import pytest

from helpers import f16_to_f32_ref, f32_to_f16_ref, half_conversion_probe

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


def _bits_equal(got, want):
    got, want = np.asarray(got, np.uint16), np.asarray(want, np.uint16)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: got {got[bad[:5]]}, want {want[bad[:5]]}"


def test_copy_from_float32_bytes(fl, be):
    x = half_conversion_probe()
    t = be.new_tensor(1, x.size, x, fl.F16)
    _bits_equal(t.raw_bytes().view(np.uint16), f32_to_f16_ref(x))


def test_to_host_float32_every_pattern(fl, be):
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    t = be.new_tensor(1, h.size, None, fl.F16)
    be.check(fl.lib().Cuda_CopyToDevice(t.buf, 0, h.ctypes.data, h.nbytes))
    got = t.to_host().ravel()
    want = f16_to_f32_ref(h)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_cast_and_copy_bytes(fl, be):
    x = half_conversion_probe(200_000, seed=11)
    src = be.new_tensor(1, x.size, x, fl.F32)
    _bits_equal(src.cast(fl.F16).raw_bytes().view(np.uint16), f32_to_f16_ref(x))
    dst = be.new_tensor(1, x.size, None, fl.F16)
    dst.copy(src)  # Copy across dtypes converts like Cast
    _bits_equal(dst.raw_bytes().view(np.uint16), f32_to_f16_ref(x))


def test_at_set(fl, be):
    vals = np.array([1.0, -2.0, 65520.0, 5e-5, np.nan, 1.00146484375, -1e6], np.float32)
    t = be.new_tensor(1, vals.size, None, fl.F16)
    for j, v in enumerate(vals):
        t.set(0, j, v)
    want = f32_to_f16_ref(vals)
    _bits_equal(t.raw_bytes().view(np.uint16), want)
    for j in range(vals.size):
        got = np.float32(t.at(0, j))
        ref = f16_to_f32_ref(want[j:j + 1])[0]
        assert got.view(np.uint32) == ref.view(np.uint32) or (np.isnan(got) and np.isnan(ref))
    with pytest.raises(fl.FletcherError):
        t.at(1, 0)


def test_rne_mode_is_ieee(fl, be):
    x = half_conversion_probe(100_000, seed=3)
    x = x[np.isfinite(x)]
    be.set_half_conversion(fl.HALF_RNE)
    try:
        t = be.new_tensor(1, x.size, x, fl.F16)
        with np.errstate(over="ignore"):
            want = x.astype(np.float16)
        assert np.array_equal(t.raw_bytes().view(np.uint16), want.view(np.uint16))
        assert np.array_equal(t.to_host().ravel(), want.astype(np.float32))
    finally:
        be.set_half_conversion(fl.HALF_REFERENCE)


def test_model_fp16_weights_use_reference_bytes(fl, be):
    """LoadRaw of an fp16 model converts the fp32 blob as the reference's CopyFromFloat32 does
    (weights/loader.go:104,254 -> cuda_linux.go:158-169): a model loaded from the blob and one
    loaded from the blob already passed through Float32ToFloat16/Float16ToFloat32 on the host
    hold the same fp16 weights, so their outputs are bit-identical."""
    import dataclasses

    import synth
    cfg = dataclasses.replace(synth.NOMIC, num_layers=1)
    blob = synth.make_weights(cfg, 3)
    rt = f16_to_f32_ref(f32_to_f16_ref(blob))
    assert not np.array_equal(rt, blob)  # N(0, 0.02) weights have values in the flush band
    lens = np.array([40, 7, 130], np.int32)
    ids = synth.make_ids(lens, cfg.vocab_size, 9)
    outs = []
    for b in (blob, rt):
        m = fl.BertModel(be, cfg, "f16")
        m.load_raw(b)
        outs.append(m.forward_batch(ids, lens, fl.POOL_MEAN_L2))
        m.close()
    assert np.array_equal(outs[0], outs[1])
