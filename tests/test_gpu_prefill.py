"""The batched prompt pass (kllm_infer_opts.prefill) on the GPU.

The prompt's positions but the last go through every layer at once (TT-GEMM
projections, row kernels); the last position and the generation run as
regular decode steps.  Bar (the north star's): greedy tokens identical to
the oracle / the compiled reference runtime, and the logits of the last step
within atol 1e-3 / rtol 1e-4 of the step-by-step run."""
import numpy as np
import pytest

import harness

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


@pytest.mark.parametrize("name", ["gqa", "mha", "tl", "tl-fp16", "tl-pool"])
def test_prefill_tokens_match_oracle(gpu, oracle, chip_dir, name):
    import kmap_b200
    path = chip_dir(name)
    oc = harness.OracleChip(oracle, path)
    with kmap_b200.Chip(path) as chip:
        V = chip.info["vocab_size"]
        prompt = np.random.default_rng(21).integers(3, V, 11)
        toks_o, _ = oc.infer(prompt, 12)
        oc.close()
        toks_s = chip.infer(prompt, 12)
        last_s = chip.final_logits()
    with kmap_b200.Chip(path, prefill=True) as chip:
        toks_p = chip.infer(prompt, 12)
        assert chip.stats()["fused"] == 1 and chip.stats()["step_kernel"] == 1
        last_p = chip.final_logits()
    assert toks_p.tolist() == toks_o.tolist()
    assert toks_s.tolist() == toks_o.tolist()
    np.testing.assert_allclose(last_p, last_s, rtol=RTOL, atol=ATOL)


def test_prefill_tinyllama_width_matches_reference(gpu, ref, tmp_path):
    """Two layers at the TinyLlama-1.1B widths, a 40-token prompt."""
    import kmap_b200
    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
    spec.num_layers = 2
    spec.max_seq = 256
    path = chipgen.ensure_chip(str(tmp_path), spec)
    prompt = np.random.default_rng(4).integers(3, spec.vocab_size, 40).astype(np.int32)
    h, info = ref.chip(path)
    toks_r, _ = ref.greedy_logits(h, prompt, 6, spec.vocab_size)
    ref.L.refh_chip_destroy(h)
    with kmap_b200.Chip(path, prefill=True) as chip:
        toks_p = chip.infer(prompt, 6)
    assert toks_p.tolist() == toks_r.tolist()
