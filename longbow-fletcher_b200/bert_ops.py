"""The reference's model code (internal/embeddings/model/bert.go) run unchanged, op by op,
through the tensor ABI of libcuda_fletcher.so.

This is the route an unmodified `bert.go` takes on this backend: every device.Tensor call it
makes (Gather, Add, LayerNorm, Linear, LinearActivation, ApplyRoPE, Attention, Slice, Scale,
Mul with a T() view, Softmax, Copy, AddLayerNorm, Cast) maps to one C-ABI call through
`fletcher.Tensor`, in the order and with the arguments bert.go uses.  It exists to show that
the op-level boundary is a drop-in (tests replay it against the oracle's literal mode) and to
time that route beside the fused whole-model entry point (`bench.py --route ops`).

Reference behaviour reproduced on purpose, because a drop-in must not change it:
  - LayerNorm eps is 1e-7 whatever the config says (bert.go:281);
  - RoPE uses base 10000 and position = row % lengths[0] over batch*lengths[0] rows
    (bert.go:619-624 -> cpu_backend.go:760-805);
  - ragged batches take the per-sequence fallback (bert.go:653-716), whose result is written
    into `output.Slice(...)`, a copy (cpu_backend.go:288-303), so the attention context of a
    ragged batch stays zero.
The only deviation: bert.go:255-259 casts the embeddings to Float32.  The fp16 CUDA backend of
the reference cannot run that Cast (cuda_linux.go:327-337 panics) and Linear here wants one
dtype, so in 16-bit mode the activations stay in the model dtype.
"""
from __future__ import annotations

import math

import numpy as np

import fletcher as fl
import synth

LITERAL_EPS = 1e-7  # bert.go:281


class OpsBertModel:
    """model.BertModel (bert.go:77-169) over fletcher.Tensor ops."""

    def __init__(self, be: fl.Backend, cfg: synth.BertConfig, blob: np.ndarray, dtype=fl.F32):
        self.be, self.cfg, self.dtype = be, cfg, dtype
        v = synth.weight_views(cfg, np.ascontiguousarray(blob, np.float32))

        def dev(name, f32=False):
            a = v[name]
            r, c = (1, a.shape[0]) if a.ndim == 1 else a.shape
            return be.new_tensor(r, c, a, fl.F32 if f32 else dtype)

        # NewBertEmbeddings / NewLayerNorm (bert.go:184-270): LayerNorm weights forced to fp32.
        self.word, self.pos, self.type = dev("word"), dev("pos"), dev("type")
        self.eln = (dev("emb_ln.gamma", True), dev("emb_ln.beta", True))
        self.layers = []
        for l in range(cfg.num_layers):
            p = f"layer{l}."
            self.layers.append({k: dev(p + k, k.startswith("ln")) for k in (
                "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln1.gamma", "ln1.beta",
                "wi", "bi", "wd", "bd", "ln2.gamma", "ln2.beta")})
        self.pool_w, self.pool_b = dev("pool.w"), dev("pool.b")

    # ---- BertEmbeddings.ForwardBatch (bert.go:215-261)
    def embeddings(self, ids, lengths):
        cfg = self.cfg
        T = len(ids)
        emb = self.word.gather(ids)
        if cfg.position_type == synth.POS_ABSOLUTE:
            pos = np.concatenate([np.minimum(np.arange(l), cfg.max_positions - 1) for l in lengths]).astype(np.int32)
            pe = self.pos.gather(pos)
            emb.add(pe)
        te = self.type.gather(np.zeros(T, np.int32))
        emb.add(te)
        emb.layer_norm(*self.eln, LITERAL_EPS)
        if emb.dtype != fl.F32 and self.dtype == fl.F32:
            emb = emb.cast(fl.F32)
        return emb

    # ---- BertSelfAttention.ForwardBatch (bert.go:610-728)
    def self_attention(self, L, h, lengths):
        cfg = self.cfg
        nh, dh = cfg.num_heads, cfg.head_dim
        q = h.linear(h, L["wq"], L["bq"])
        k = h.linear(h, L["wk"], L["bk"])
        val = h.linear(h, L["wv"], L["bv"])
        if cfg.position_type == synth.POS_ROPE:
            q.apply_rope(len(lengths), int(lengths[0]), nh, dh)
            k.apply_rope(len(lengths), int(lengths[0]), nh, dh)
        scale = np.float32(1.0 / math.sqrt(dh))
        if all(int(l) == int(lengths[0]) for l in lengths):
            return q.attention(q, k, val, len(lengths), int(lengths[0]), nh, float(scale))
        T, H = q.dims()
        output = self.be.new_tensor(T, H, None, q.dtype)
        off = 0
        sq = float(np.float32(math.sqrt(float(scale))))
        for l in (int(x) for x in lengths):
            if l == 0:
                continue
            qs = q.slice(off, off + l, 0, nh * dh)
            ks = k.slice(off, off + l, 0, nh * dh)
            vs = val.slice(off, off + l, 0, nh * dh)
            qs.scale(sq)
            ks.scale(sq)
            scores = self.be.new_tensor(l, l, None, q.dtype)
            scores.mul(qs, ks.T())
            scores.softmax()
            res = self.be.new_tensor(l, nh * dh, None, q.dtype)
            res.mul(scores, vs)
            out_slice = output.slice(off, off + l, 0, nh * dh)
            if res.dtype != out_slice.dtype:
                res = res.cast(out_slice.dtype)
            out_slice.copy(res)
            off += l
        return output

    # ---- BertLayer.ForwardBatch (bert.go:391-412) with BertSelfOutput / BertIntermediate /
    # BertOutput (bert.go:730-820).  LayerNorm.ForwardAdd: residual.AddLayerNorm(branch).
    def layer(self, L, h, lengths):
        ctx = self.self_attention(L, h, lengths)
        proj = ctx.linear(ctx, L["wo"], L["bo"])
        h.add_layer_norm(proj, L["ln1.gamma"], L["ln1.beta"], LITERAL_EPS)
        inter = h.linear(h, L["wi"], L["bi"], self.cfg.activation)
        proj = inter.linear(inter, L["wd"], L["bd"])
        h.add_layer_norm(proj, L["ln2.gamma"], L["ln2.beta"], LITERAL_EPS)
        return h

    # ---- BertPooler.ForwardBatch (bert.go:441-488): CLS rows -> Dense -> TanhFast
    def pooler(self, h, lengths):
        starts = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
        cls = h.gather(starts)
        if self.pool_w.dtype != fl.F32:  # the pooler runs in fp32 for 16-bit weights (bert.go:459-477)
            c32, w32, b32 = cls.cast(fl.F32), self.pool_w.cast(fl.F32), self.pool_b.cast(fl.F32)
            return w32.linear(c32, w32, b32, fl.ACT_TANH)
        return self.pool_w.linear(cls, self.pool_w, self.pool_b, fl.ACT_TANH)

    def forward_hidden(self, ids, lengths):
        lengths = [int(x) for x in lengths]
        h = self.embeddings(np.ascontiguousarray(ids, np.int32), lengths)
        for L in self.layers:
            h = self.layer(L, h, lengths)
        self.be.synchronize()  # bert.go:156
        return h

    def forward_batch(self, ids, lengths, pooling=fl.POOL_CLS_TANH):
        """BertModel.ForwardBatch (bert.go:149-169) -> host [B, H] float32.  POOL_MEAN_L2 runs the
        spec's mean-pool + L2 head in place of the pooler (the one model change)."""
        h = self.forward_hidden(ids, lengths)
        if pooling == fl.POOL_MEAN_L2:
            return h.mean_pool_l2(lengths).to_host()
        return self.pooler(h, lengths).to_host()
