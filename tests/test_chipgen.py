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


def test_device_generator_compresses_like_the_host_rule():
    """The device generation path (TorchWeightSource + the histogram
    compression, used for the 7B/8B chips) yields bf16 weights and the same
    codebook and indices as the host tt_compress of the same weights (run
    here on the CPU device)."""
    import torch

    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(hidden_size=64, intermediate_size=96)
    src = chipgen.TorchWeightSource(spec, torch.device("cpu"))
    w = src.matrix("layer_0/q_proj", 96, 64)
    again = src.matrix("layer_0/q_proj", 96, 64)
    assert torch.equal(w, again)   # seeded by name
    wt = torch.cat([w.t()], 1).contiguous()
    cb_d, idx_d = chipgen._tt_compress_torch(wt)
    cb_h, idx_h = chipgen.tt_compress(wt.numpy())
    assert np.array_equal(cb_d.view(np.uint32), cb_h.view(np.uint32))
    assert np.array_equal(idx_d, idx_h)
    assert not (wt.numpy().view(np.uint32) & 0xFFFF).any()


def test_device_generated_chip_loads(tmp_path):
    import torch

    import kmap_b200
    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(num_layers=1, hidden_size=64, num_attention_heads=4,
                             num_key_value_heads=2, intermediate_size=96, vocab_size=300,
                             max_seq=32)
    path = chipgen.ensure_chip(str(tmp_path), spec, device=torch.device("cpu"))
    assert path.endswith("_devrng")
    with kmap_b200.Chip(path) as chip:
        assert chip.info["vocab_size"] == 300 and chip.info["num_layers"] == 1
