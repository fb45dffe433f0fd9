"""Regenerates the golden fixtures in this directory from the CPU oracle (oracle/ref_cpu.cpp).

    python tests/golden/make_golden.py

The reference's own Go path cannot run in this environment (no Go toolchain), so these
fixtures pin the oracle itself: the tests check that the oracle still reproduces them and that
the CUDA library matches them.  Weights are not stored; they are regenerated from
(config, seed) by synth.make_weights.
"""
import dataclasses
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "longbow-fletcher_b200"), os.path.join(ROOT, "oracle")]
import oracle  # noqa: E402
import synth  # noqa: E402


def cases():
    tiny = synth.BERT_TINY
    tiny_lit = dataclasses.replace(tiny, layer_norm_eps=1e-7)
    nomic2 = dataclasses.replace(synth.NOMIC, num_layers=2)
    nomic2_lit = dataclasses.replace(nomic2, layer_norm_eps=1e-7, rope_base=10000.0)
    return {
        # name: (cfg, cfg-name, weight seed, lengths, ids seed, mode)
        "tiny_ragged_spec": (tiny, "BERT_TINY", 0, [8, 17, 64, 65, 128, 1, 127, 33], 5, oracle.MODE_SPEC),
        "tiny_ragged_literal": (tiny_lit, "BERT_TINY/eps1e-7", 0, [8, 17, 64, 65, 128, 1, 127, 33], 5, oracle.MODE_LITERAL),
        "tiny_uniform_literal": (tiny_lit, "BERT_TINY/eps1e-7", 0, [32] * 4, 6, oracle.MODE_LITERAL),
        "nomic2_ragged_spec": (nomic2, "NOMIC/2 layers", 1, [40, 77, 130, 64], 7, oracle.MODE_SPEC),
        "nomic2_uniform_literal": (nomic2_lit, "NOMIC/2 layers/eps1e-7/base1e4", 1, [48, 48, 48], 8, oracle.MODE_LITERAL),
    }


def main():
    for name, (cfg, cname, wseed, lengths, iseed, mode) in cases().items():
        blob = synth.make_weights(cfg, wseed)
        lens = np.array(lengths, np.int32)
        ids = synth.make_ids(lens, cfg.vocab_size, iseed)
        r = oracle.forward(cfg, blob, ids, lens, mode=mode, threads=1)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), ids=ids, lengths=lens, cls=r["cls"], mean=r["mean"],
                            weight_seed=np.int64(wseed), mode=np.int32(mode), config=np.array(cname),
                            cfg=np.array(dataclasses.astuple(cfg), dtype=object).astype(str))
        print(name, r["mean"].shape)


if __name__ == "__main__":
    main()
