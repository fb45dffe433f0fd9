"""Model presets and seeded synthetic inputs for the embedding forward pass.

The presets mirror the reference's BertConfig (internal/embeddings/model/bert.go:20-75)
with the overrides of the benchmark configurations (eps, RoPE base, vocab).  Weights are
one flat float32 blob in the order LoadFromRawBinary reads a raw weight file
(internal/embeddings/weights/loader.go:29-90, written by scripts/download_weights.py:21-71):

    word[V,H] pos[P,H] type[2,H] emb_ln.gamma[H] emb_ln.beta[H]
    per layer: Wq[H,H] bq[H] Wk[H,H] bk[H] Wv[H,H] bv[H] Wo[H,H] bo[H] ln1.gamma ln1.beta
               Wi[H,Iup] bi[Iup] Wd[I,H] bd[H] ln2.gamma ln2.beta
    pooler: Wp[H,H] bp[H]

Linear weights are stored (in, out), as the reference's Linear expects; Iup = 2*I for SwiGLU
(the fused gate|up projection, bert.go:768-779), else I.

There is no dataset: token ids, lengths and weights are all drawn from a seeded numpy
generator with the shapes and distributions of the benchmark configurations.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math

import numpy as np

ACT_IDENTITY, ACT_GELU, ACT_TANH, ACT_SOFTMAX, ACT_SWIGLU = 0, 1, 2, 3, 4  # device.go:126-134
POS_ABSOLUTE, POS_ROPE = 0, 1  # bert.go:12-17
CLS_ID, SEP_ID, PAD_ID = 101, 102, 0


@dataclasses.dataclass(frozen=True)
class BertConfig:
    vocab_size: int
    hidden: int
    num_layers: int
    num_heads: int
    intermediate: int
    max_positions: int
    activation: int
    position_type: int
    layer_norm_eps: float
    rope_base: float
    has_bias: bool = True

    @property
    def head_dim(self) -> int:
        return self.hidden // self.num_heads

    @property
    def up_width(self) -> int:
        return 2 * self.intermediate if self.activation == ACT_SWIGLU else self.intermediate

    def flops_per_sequence(self, length):
        """Algorithmic FLOPs of one sequence of `length` tokens (no padding):
        L * [2l(H*3H + H*H + H*Iup + I*H) + 4 l^2 H]."""
        H, I = self.hidden, self.intermediate
        lin = 2 * (H * 3 * H + H * H + H * self.up_width + I * H)
        return self.num_layers * (lin * np.asarray(length, np.float64)
                                  + 4.0 * H * np.asarray(length, np.float64) ** 2)


class CConfig(ctypes.Structure):
    """Matches FletcherBertConfig in include/fletcher_cuda.h."""
    _fields_ = [("vocab_size", ctypes.c_int32), ("hidden", ctypes.c_int32),
                ("num_layers", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("intermediate", ctypes.c_int32), ("max_positions", ctypes.c_int32),
                ("activation", ctypes.c_int32), ("position_type", ctypes.c_int32),
                ("layer_norm_eps", ctypes.c_float), ("rope_base", ctypes.c_float)]


def to_c(cfg: BertConfig) -> CConfig:
    return CConfig(cfg.vocab_size, cfg.hidden, cfg.num_layers, cfg.num_heads, cfg.intermediate,
                   cfg.max_positions, cfg.activation, cfg.position_type,
                   cfg.layer_norm_eps, cfg.rope_base)


# bert-tiny (bert.go:33-45) with the benchmark's eps 1e-12.
BERT_TINY = BertConfig(30522, 128, 2, 2, 512, 512, ACT_GELU, POS_ABSOLUTE, 1e-12, 10000.0, True)
# nomic-embed-text style (bert.go:48-60) with the benchmark's vocab 30528, eps 1e-12, RoPE base
# 1000 and no biases (the bias slots stay in the blob, zero-filled).
NOMIC = BertConfig(30528, 768, 12, 12, 3072, 8192, ACT_SWIGLU, POS_ROPE, 1e-12, 1000.0, False)


def weight_layout(cfg: BertConfig):
    """[(name, shape)] in raw-file order."""
    H, I, Iu = cfg.hidden, cfg.intermediate, cfg.up_width
    out = [("word", (cfg.vocab_size, H)), ("pos", (cfg.max_positions, H)), ("type", (2, H)),
           ("emb_ln.gamma", (H,)), ("emb_ln.beta", (H,))]
    for l in range(cfg.num_layers):
        p = f"layer{l}."
        out += [(p + "wq", (H, H)), (p + "bq", (H,)), (p + "wk", (H, H)), (p + "bk", (H,)),
                (p + "wv", (H, H)), (p + "bv", (H,)), (p + "wo", (H, H)), (p + "bo", (H,)),
                (p + "ln1.gamma", (H,)), (p + "ln1.beta", (H,)),
                (p + "wi", (H, Iu)), (p + "bi", (Iu,)), (p + "wd", (I, H)), (p + "bd", (H,)),
                (p + "ln2.gamma", (H,)), (p + "ln2.beta", (H,))]
    out += [("pool.w", (H, H)), ("pool.b", (H,))]
    return out


def weight_count(cfg: BertConfig) -> int:
    return sum(int(np.prod(s)) for _, s in weight_layout(cfg))


def weight_views(cfg: BertConfig, blob: np.ndarray):
    """name -> view into the blob."""
    views, off = {}, 0
    for name, shape in weight_layout(cfg):
        n = int(np.prod(shape))
        views[name] = blob[off:off + n].reshape(shape)
        off += n
    assert off == blob.size
    return views


def make_weights(cfg: BertConfig, seed: int, std: float = 0.02) -> np.ndarray:
    """Weights ~ N(0, std); LayerNorm gamma = 1, beta = 0; biases ~ N(0, std) when the
    model has biases, else 0."""
    rng = np.random.default_rng(seed)
    blob = rng.standard_normal(weight_count(cfg), dtype=np.float32)
    blob *= np.float32(std)
    v = weight_views(cfg, blob)
    for name, arr in v.items():
        if name.endswith(".gamma"):
            arr[...] = 1.0
        elif name.endswith(".beta"):
            arr[...] = 0.0
        elif not cfg.has_bias and (name.split(".")[-1] in ("bq", "bk", "bv", "bo", "bi", "bd")):
            arr[...] = 0.0
    return blob


def make_lengths(batch: int, lo: int, hi: int, seed: int, dist: str = "uniform") -> np.ndarray:
    rng = np.random.default_rng(seed + 1000)
    if dist == "uniform":
        return rng.integers(lo, hi + 1, size=batch).astype(np.int32)
    if dist == "loguniform":
        return np.exp(rng.uniform(math.log(lo), math.log(hi + 1), size=batch)).astype(np.int32).clip(lo, hi)
    raise ValueError(dist)


def make_ids(lengths: np.ndarray, vocab: int, seed: int, lo_id: int = 1000) -> np.ndarray:
    """Packed ids: per sequence [CLS] ids... [SEP] (embeddings.go:742-749), ids uniform in
    [lo_id, vocab).  Padding is packed away, so no PAD ids appear."""
    rng = np.random.default_rng(seed + 2000)
    T = int(lengths.sum())
    ids = rng.integers(lo_id, vocab, size=T).astype(np.int32)
    starts = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int64)
    ids[starts] = CLS_ID
    ends = starts + lengths.astype(np.int64) - 1
    ids[ends[lengths >= 2]] = SEP_ID
    return ids


@dataclasses.dataclass
class Workload:
    name: str
    cfg: BertConfig
    batch: int
    len_lo: int
    len_hi: int
    dist: str
    seed: int
    dtype: str  # "f32" | "bf16" | "f16"

    def lengths(self):
        return make_lengths(self.batch, self.len_lo, self.len_hi, self.seed, self.dist)


WORKLOADS = {
    "cfg1": Workload("bert-tiny fp32 B=32 S<=128", BERT_TINY, 32, 8, 128, "uniform", 0, "f32"),
    "cfg2": Workload("bert-tiny bf16 B=1024 S<=128", BERT_TINY, 1024, 8, 128, "uniform", 0, "bf16"),
    "cfg2_latency": Workload("bert-tiny bf16 B=1 l=16", BERT_TINY, 1, 16, 16, "uniform", 0, "bf16"),
    "cfg3": Workload("nomic-embed-text bf16 B=256 S<=512", NOMIC, 256, 32, 512, "uniform", 1, "bf16"),
    "cfg4": Workload("nomic-embed-text bf16 B=32 S<=2048 varlen", NOMIC, 32, 64, 2048, "loguniform", 1, "bf16"),
}
