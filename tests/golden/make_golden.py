"""Regenerate the golden fixtures from the compiled reference runtime.

    make -C oracle ref && python tests/golden/make_golden.py

Writes, next to this script:
  tt_gemv_cases.npz  -- TT-GEMV inputs and the reference's outputs
                        (tape_run on a one-instruction MATMUL_TT tape)
  tiny_decode.npz    -- a tiny chip's spec, a prompt, the reference's greedy
                        tokens (processor_infer) and per-step logits rows
The reference has no tests or golden vectors of its own for this path, so
these outputs of the reference binary are the pin.
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import harness  # noqa: E402
from kmap_b200 import chipgen  # noqa: E402

TT_CASES = [(1, 1, 5, 3), (1, 127, 33, 17), (2, 1000, 37, 400), (1, 1025, 24, 5461),
            (1, 2048, 24, 4096), (1, 5632, 8, 5461)]

TINY = dict(num_layers=2, hidden_size=128, num_attention_heads=4, num_key_value_heads=2,
            intermediate_size=256, vocab_size=600, max_seq=64, norm_weights="random", seed=11)


def main():
    ref = harness.Ref()
    out = {"n": len(TT_CASES)}
    for i, (rows, K, N, codes) in enumerate(TT_CASES):
        x, cb, idx = harness.tt_case(100 + i, K, N, codes, rows)
        tr = harness.TapeRun(ref, 3, {0: ("ext", x), 1: ("tt", cb, idx), 2: ("alloc", [1])},
                             [dict(tag=13, out_slot=2, in0=0, in1=1)])
        tr.run()
        y, _ = tr.read(2)
        tr.close()
        out.update({"x%d" % i: x, "cb%d" % i: cb, "idx%d" % i: idx, "y%d" % i: y.reshape(rows, N)})
    np.savez_compressed(os.path.join(HERE, "tt_gemv_cases.npz"), **out)

    spec = chipgen.ModelSpec(**TINY)
    with tempfile.TemporaryDirectory() as d:
        path = chipgen.ensure_chip(d, spec)
        h, info = ref.chip(path)
        prompt = np.random.default_rng(21).integers(3, spec.vocab_size, 9).astype(np.int32)
        max_new = 16
        toks = ref.infer(h, prompt, max_new)
        toks2, logits = ref.greedy_logits(h, prompt, max_new, spec.vocab_size)
        assert np.array_equal(toks, toks2)
        ref.L.refh_chip_destroy(h)
        # the first truth-table slot, for a checksum that detects generator drift
        rec =np.fromfile(os.path.join(path, "circuit", "slots.bin"), np.int32)[1:].reshape(-1, 10)
        tt_slot = int(np.nonzero(rec[:, 0] == 4)[0][0])
        idx = np.fromfile(os.path.join(path, "circuit", "const_%d_indices.bin" % tt_slot), np.uint16)
    keys = sorted(TINY)
    np.savez_compressed(os.path.join(HERE, "tiny_decode.npz"), spec_keys=np.array(keys),
                        spec_vals=np.array([str(TINY[k]) for k in keys]), prompt=prompt,
                        max_new=max_new, tokens=toks, logits=logits, tt_slot=tt_slot,
                        tt_checksum=int(idx.astype(np.uint64).sum()))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
