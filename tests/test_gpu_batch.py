"""Batched greedy decode of several sequences (kllm_chip_infer_batch; the
reference's processor_infer runs one sequence, so every sequence of a
batch is checked against its own single-sequence run).

Each sequence's prompt goes through the batched prompt pass into its own KV
cache, then every step runs each projection as one TT-GEMM over the
sequences' rows (bit-identical per row to the TT-GEMV), attention per row
over its own cache.  Bar: every sequence's tokens identical to the oracle's
(and the compiled reference's) single-sequence greedy run, with the
projections on the tensor cores (the default for bf16 codebooks) and with
the exact FP32 TT-GEMM."""
import dataclasses

import numpy as np
import pytest

import harness

pytestmark = pytest.mark.gpu


def _prompts(V, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(3, V, n).astype(np.int32) for n in lens]


@pytest.mark.parametrize("name", ["gqa", "mha", "tl"])
@pytest.mark.parametrize("tc", ["1", "0"])
def test_batch_matches_single_sequence_oracle(gpu, oracle, chip_dir, name, tc, monkeypatch):
    """Tensor-core projections (the default where the codebooks are bf16
    numbers and the shapes fit) and the exact FP32 TT-GEMM."""
    import kmap_b200
    monkeypatch.setenv("KLLM_BATCH_TC", tc)
    path = chip_dir(name)
    max_new = 12
    with kmap_b200.Chip(path) as chip:
        V = chip.info["vocab_size"]
        prompts = _prompts(V, [1, 5, 9, 17, 3], 31)
        outs = chip.infer_batch(prompts, max_new)
    oc = harness.OracleChip(oracle, path)
    for p, toks in zip(prompts, outs):
        toks_o, _ = oc.infer(p, max_new)
        assert toks.tolist() == toks_o.tolist()
    oc.close()


def test_batch_eos_cuts_each_sequence(gpu, chip_dir):
    import kmap_b200
    path = chip_dir("gqa")
    with kmap_b200.Chip(path) as chip:
        V = chip.info["vocab_size"]
        prompts = _prompts(V, [4, 6], 2)
        full = chip.infer_batch(prompts, 10)
        eos = int(full[1][3])
        cut = chip.infer_batch(prompts, 10, eos=eos)
    for f, c in zip(full, cut):
        k = int(np.nonzero(f == eos)[0][0]) if (f == eos).any() else len(f)
        assert c.tolist() == f[:k].tolist()


def test_batch_without_graph_equals_graph(gpu, chip_dir):
    """Steps launched one by one give the tokens of the captured step graph."""
    import kmap_b200
    path = chip_dir("tl")
    with kmap_b200.Chip(path) as chip:
        prompts = _prompts(chip.info["vocab_size"], [7, 12, 2], 8)
        a = chip.infer_batch(prompts, 10)
        b = chip.infer_batch(prompts, 10, use_graphs=False)
    assert [x.tolist() for x in a] == [x.tolist() for x in b]


def test_batch_tinyllama_width_matches_reference(gpu, ref, tmp_path):
    import kmap_b200
    from kmap_b200 import chipgen
    spec = dataclasses.replace(chipgen.TINYLLAMA_1B, num_layers=2, max_seq=128)
    path = chipgen.ensure_chip(str(tmp_path), spec)
    prompts = _prompts(spec.vocab_size, [6, 20, 33], 17)
    with kmap_b200.Chip(path) as chip:
        outs = chip.infer_batch(prompts, 8)
    h, info = ref.chip(path)
    for p, toks in zip(prompts, outs):
        assert toks.tolist() == ref.infer(h, p, 8).tolist()
    ref.L.refh_chip_destroy(h)
