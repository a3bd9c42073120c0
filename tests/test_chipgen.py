"""The synthetic chip writer produces the reference compiler's exact files."""
import filecmp
import os
import shutil

import numpy as np
import pytest

from kmap_b200 import chipgen


@pytest.mark.parametrize("kv,norms", [(2, "random"), (4, "ones")])
def test_chip_bytes_equal_reference_compiler(ref, tmp_path, kv, norms):
    spec = chipgen.ModelSpec(num_layers=2, hidden_size=128, num_attention_heads=4,
                             num_key_value_heads=kv, intermediate_size=256, vocab_size=600,
                             max_seq=64, norm_weights=norms, seed=3)
    a, b = str(tmp_path / "mine"), str(tmp_path / "ref")
    chipgen.generate_chip(a, spec, write_weights=True)
    shutil.copytree(os.path.join(a, "weights"), os.path.join(b, "weights"))
    shutil.copytree(os.path.join(a, "tokenizer"), os.path.join(b, "tokenizer"))
    assert ref.L.compile_chip(b.encode(), spec.max_seq, spec.model_name.encode()) == 0
    n = 0
    for root, _, files in os.walk(b):
        if "/weights" in root or "/tokenizer" in root:
            continue
        for f in files:
            pb = os.path.join(root, f)
            pa = pb.replace(b, a, 1)
            assert os.path.exists(pa), pa
            assert filecmp.cmp(pa, pb, shallow=False), f
            n += 1
    assert n > 40


def test_tt_compress_matches_sort_unique():
    rng = np.random.default_rng(0)
    w = chipgen.bf16_round(rng.standard_normal((64, 80)).astype(np.float32) * 0.02)
    cb, idx = chipgen.tt_compress(w)
    u = np.unique(w)
    assert np.array_equal(cb, u)
    assert np.array_equal(cb[idx], w)
    # non-bf16 data takes the generic path
    w2 = rng.standard_normal((16, 8)).astype(np.float32)
    cb2, idx2 = chipgen.tt_compress(w2)
    assert np.array_equal(cb2[idx2], w2)


def test_tinyllama_shapes():
    s = chipgen.TINYLLAMA_1B
    assert (s.num_layers, s.hidden_size, s.head_dim, s.intermediate_size, s.vocab_size) == \
        (22, 2048, 64, 5632, 32000)
