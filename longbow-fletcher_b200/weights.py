"""Weight ingestion: SafeTensors and raw files -> the raw float32 blob Cuda_Model_LoadRaw takes.

The reference reads F32 SafeTensors only and rejects F16 (internal/embeddings/weights/loader.go:
155-296, rejection at :210-215).  This reader also takes F16 and BF16 files.  It keeps the
reference's tensor names (loader.go:257-293) and its transpose rule: a 2-D ".weight" outside the
embeddings and LayerNorms is a Linear weight stored (out, in) and is transposed to (in, out)
(loader.go:229-251).  The raw format is LoadFromRawBinary's: float32 little-endian tensors
back to back, in model order (loader.go:29-90).
"""
from __future__ import annotations

import json
import struct

import numpy as np

import synth

_DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2)}


def _bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even


def read_safetensors(path: str) -> dict:
    """name -> float32 ndarray with the file's shape."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if n > 100 * 1024 * 1024:  # loader.go:171-173
            raise ValueError(f"header size too large: {n}")
        header = json.loads(f.read(n))
        body = f.read()
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"tensor {name!r}: dtype {dt} not supported (F32, F16, BF16)")
        npdt, size = _DTYPES[dt]
        a, b = info["data_offsets"]
        count = int(np.prod(info["shape"])) if info["shape"] else 1
        if b - a != count * size:
            raise ValueError(f"tensor {name!r} byte size mismatch: {b - a} != {count * size}")
        arr = np.frombuffer(body[a:b], dtype=npdt).reshape(info["shape"])
        out[name] = _bf16_to_f32(arr) if dt == "BF16" else arr.astype(np.float32)
    return out


def write_safetensors(path: str, tensors: dict, dtype: str = "F32") -> None:
    """Writes float32 arrays as F32, F16 or BF16 SafeTensors."""
    header, chunks, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr, np.float32)
        if dtype == "F32":
            data = arr.tobytes()
        elif dtype == "F16":
            data = arr.astype(np.float16).tobytes()
        else:
            data = _f32_to_bf16(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(data)]}
        chunks.append(data)
        off += len(data)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for c in chunks:
            f.write(c)


def hf_names(cfg: synth.BertConfig):
    """[(HF tensor name, blob layout name)] in raw-file order (loader.go:257-293)."""
    out = [("embeddings.word_embeddings.weight", "word"), ("embeddings.position_embeddings.weight", "pos"),
           ("embeddings.token_type_embeddings.weight", "type"), ("embeddings.LayerNorm.weight", "emb_ln.gamma"),
           ("embeddings.LayerNorm.bias", "emb_ln.beta")]
    for l in range(cfg.num_layers):
        p, q = f"encoder.layer.{l}", f"layer{l}."
        out += [(p + ".attention.self.query.weight", q + "wq"), (p + ".attention.self.query.bias", q + "bq"),
                (p + ".attention.self.key.weight", q + "wk"), (p + ".attention.self.key.bias", q + "bk"),
                (p + ".attention.self.value.weight", q + "wv"), (p + ".attention.self.value.bias", q + "bv"),
                (p + ".attention.output.dense.weight", q + "wo"), (p + ".attention.output.dense.bias", q + "bo"),
                (p + ".attention.output.LayerNorm.weight", q + "ln1.gamma"),
                (p + ".attention.output.LayerNorm.bias", q + "ln1.beta"),
                (p + ".intermediate.dense.weight", q + "wi"), (p + ".intermediate.dense.bias", q + "bi"),
                (p + ".output.dense.weight", q + "wd"), (p + ".output.dense.bias", q + "bd"),
                (p + ".output.LayerNorm.weight", q + "ln2.gamma"), (p + ".output.LayerNorm.bias", q + "ln2.beta")]
    out += [("pooler.dense.weight", "pool.w"), ("pooler.dense.bias", "pool.b")]
    return out


def _is_linear_weight(name: str, arr: np.ndarray) -> bool:
    # loader.go:231-234
    return name.endswith(".weight") and arr.ndim == 2 and "embeddings" not in name and "LayerNorm" not in name


def read_safetensors_raw(path: str) -> dict:
    """name -> (raw ndarray in the stored dtype: float32, float16, or uint16 bfloat16 bits; dtype tag)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if n > 100 * 1024 * 1024:  # loader.go:171-173
            raise ValueError(f"header size too large: {n}")
        header = json.loads(f.read(n))
        body = f.read()
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"tensor {name!r}: dtype {dt} not supported (F32, F16, BF16)")
        npdt, size = _DTYPES[dt]
        a, b = info["data_offsets"]
        count = int(np.prod(info["shape"])) if info["shape"] else 1
        if b - a != count * size:
            raise ValueError(f"tensor {name!r} byte size mismatch: {b - a} != {count * size}")
        out[name] = (np.frombuffer(body[a:b], dtype=npdt).reshape(info["shape"]), dt)
    return out


def load_safetensors_direct(model, path: str) -> None:
    """Loads a SafeTensors checkpoint (F32, F16 or BF16) into a device model tensor by tensor
    through Cuda_Model_LoadTensor: the stored bytes go to the device as they are and are
    converted and packed there, so no fp32 copy of the model is built on the host.  The
    reference's names and transpose rule (loader.go:229-251) decide which tensors arrive
    (out, in)."""
    import fletcher
    codes = {"F32": fletcher.F32, "F16": fletcher.F16, "BF16": fletcher.BF16}
    tensors = read_safetensors_raw(path)
    for hf, _ in hf_names(model.cfg):
        if hf not in tensors:
            raise KeyError(f"tensor {hf!r} not found in SafeTensors file")  # loader.go:187-190
        arr, dt = tensors[hf]
        model.load_tensor(hf, arr, codes[dt], transposed=_is_linear_weight(hf, arr))
    if not model.is_loaded():
        raise RuntimeError("checkpoint did not cover every model tensor")


def blob_from_safetensors(path: str, cfg: synth.BertConfig) -> np.ndarray:
    """The raw float32 blob (LoadFromRawBinary order) from a SafeTensors checkpoint."""
    tensors = read_safetensors(path)
    blob = np.empty(synth.weight_count(cfg), np.float32)
    views = synth.weight_views(cfg, blob)
    for hf, ours in hf_names(cfg):
        if hf not in tensors:
            raise KeyError(f"tensor {hf!r} not found in SafeTensors file")  # loader.go:187-190
        t = tensors[hf]
        dest = views[ours]
        if t.size != dest.size:
            raise ValueError(f"tensor {hf!r} size mismatch: expected {dest.size}, got {t.size} (shape {t.shape})")
        if _is_linear_weight(hf, t):
            if t.shape != (dest.shape[1], dest.shape[0]):
                raise ValueError(f"tensor {hf!r} shape mismatch for transpose: header={list(t.shape)}, "
                                 f"expected {dest.shape[::-1]}")
            t = t.T
        dest[...] = t.reshape(dest.shape)
    return blob


def safetensors_from_blob(blob: np.ndarray, cfg: synth.BertConfig) -> dict:
    """HF-named tensors (Linear weights (out, in)) from a raw blob — the inverse mapping."""
    views = synth.weight_views(cfg, blob)
    out = {}
    for hf, ours in hf_names(cfg):
        v = views[ours]
        out[hf] = np.ascontiguousarray(v.T) if (v.ndim == 2 and _is_linear_weight(hf, v)) else v.copy()
    return out


def read_raw(path: str, cfg: synth.BertConfig) -> np.ndarray:
    """LoadFromRawBinary's file format (loader.go:29-90)."""
    blob = np.fromfile(path, dtype="<f4")
    if blob.size != synth.weight_count(cfg):
        raise ValueError(f"raw weight file holds {blob.size} floats, the model needs {synth.weight_count(cfg)}")
    return blob.astype(np.float32)
