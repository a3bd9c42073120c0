"""End-to-end generation on the device (needs a B200).

Bar (the north star's): greedy token IDs identical to the reference /
oracle, logits within max-abs 1e-3 and rel 1e-4 (np.allclose with
atol=1e-3, rtol=1e-4)."""
import numpy as np
import pytest

import harness

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4


def _oracle_run(oracle, path, prompt, max_new):
    oc = harness.OracleChip(oracle, path)
    toks, lg = oc.infer(prompt, max_new)
    oc.close()
    return toks, lg


@pytest.mark.parametrize("name", ["gqa", "mha", "tl", "tl-fp16", "tl-pool"])
@pytest.mark.parametrize("mode", ["generic", "auto", "auto-fast"])
def test_tiny_chip_tokens_and_logits(gpu, oracle, chip_dir, name, mode):
    import kmap_b200
    from conftest import TINY_STREAM_VALUES
    path = chip_dir(name)
    order = kmap_b200.ORDER_FAST if mode == "auto-fast" else kmap_b200.ORDER_EXACT
    with kmap_b200.Chip(path, order=order) as chip:
        V = chip.info["vocab_size"]
        prompt = np.random.default_rng(11).integers(3, V, 7)
        max_new = 20
        toks_o, lg_o = _oracle_run(oracle, path, prompt, max_new)
        m = kmap_b200.MODE_GENERIC if mode == "generic" else kmap_b200.MODE_AUTO
        toks_g, lg_g = chip.infer(prompt, max_new, mode=m, logits=True)
        st = chip.stats()
        if mode != "generic":
            assert st["fused"] == 1 and st["step_kernel"] == 1
            assert st["stream_values"] == TINY_STREAM_VALUES[name]
        assert toks_g.tolist() == toks_o.tolist()
        np.testing.assert_allclose(lg_g, lg_o, rtol=RTOL, atol=ATOL)


def test_slot_streams_forced_match_value_streams(gpu, chip_dir, monkeypatch):
    """A bf16 chip run with codebook-table streams (KLLM_TTX_VALUES=slot)
    gives the same bits as with bf16 value streams: both read the codebook
    entries themselves."""
    import kmap_b200
    path = chip_dir("tl")
    prompt = np.random.default_rng(5).integers(3, 2048, 5)
    with kmap_b200.Chip(path) as chip:
        t1, l1 = chip.infer(prompt, 10, logits=True)
        assert chip.stats()["stream_values"] == 1
    monkeypatch.setenv("KLLM_TTX_VALUES", "slot")
    with kmap_b200.Chip(path) as chip:
        t2, l2 = chip.infer(prompt, 10, logits=True)
        assert chip.stats()["step_kernel"] == 1 and chip.stats()["stream_values"] == 0
    assert t1.tolist() == t2.tolist()
    assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))


def test_eos_stops_generation(gpu, oracle, chip_dir):
    import kmap_b200
    path = chip_dir("gqa")
    with kmap_b200.Chip(path) as chip:
        prompt = np.array([5, 9, 13], np.int32)
        full = chip.infer(prompt, 12)
        eos = int(full[4])
        first = int(np.nonzero(full == eos)[0][0])
        cut = chip.infer(prompt, 12, eos=eos)
        assert cut.tolist() == full[:first].tolist()


def test_golden_tiny_decode_on_gpu(gpu, tmp_path):
    import os

    import kmap_b200
    from kmap_b200 import chipgen
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "tiny_decode.npz"))
    spec = chipgen.ModelSpec(**dict(zip(g["spec_keys"].tolist(), g["spec_vals"].tolist())))
    for k in ("num_layers", "hidden_size", "num_attention_heads", "num_key_value_heads",
              "intermediate_size", "vocab_size", "max_seq", "seed"):
        setattr(spec, k, int(getattr(spec, k)))
    path = chipgen.ensure_chip(str(tmp_path), spec)
    with kmap_b200.Chip(path) as chip:
        toks, lg = chip.infer(g["prompt"], int(g["max_new"]), logits=True)
    assert toks.tolist() == g["tokens"].tolist()
    np.testing.assert_allclose(lg, g["logits"], rtol=RTOL, atol=ATOL)


def test_infer_bytes_matches_reference(gpu, ref, chip_dir):
    import kmap_b200
    path = chip_dir("tl")
    h, info = ref.chip(path)
    text = b"<|user|>\nWhat is the capital of France?</s>\n<|assistant|>\n"
    out_r, gen_r = ref.infer_bytes(h, text, 12, int(info[5]))
    ref.L.refh_chip_destroy(h)
    with kmap_b200.Chip(path) as chip:
        out_g, gen_g, pieces = chip.infer_bytes(text, 12)
        assert gen_g == gen_r
        assert out_g == out_r
        # a callback that asks to stop ends generation after that token
        out_s, gen_s, _ = chip.infer_bytes(text, 12, stop_after=3)
        assert gen_s == 3 and out_s == b"".join(pieces[:3])


@pytest.mark.parametrize("order,values", [("exact", "bf16"), ("fast", "bf16"),
                                          ("exact", "fp16"), ("exact", "pool4096")])
def test_tinyllama_width_chip_matches_reference(gpu, ref, tmp_path, order, values):
    """Two layers at the TinyLlama-1.1B widths (K = 2048 and 5632, N up to
    32000, eight K-chunks per column): the fused step kernel's real tile,
    ring and stream geometry (bf16 / fp16 value streams, codebook tables
    for the 4096-value pools), against the compiled reference runtime on
    the same chip."""
    import kmap_b200
    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
    spec.num_layers = 2
    spec.max_seq = 256
    spec.weight_values = values
    path = chipgen.ensure_chip(str(tmp_path), spec)
    prompt = np.random.default_rng(3).integers(3, spec.vocab_size, 6).astype(np.int32)
    max_new = 6
    h, info = ref.chip(path)
    toks_r, lg_r = ref.greedy_logits(h, prompt, max_new, spec.vocab_size)
    ref.L.refh_chip_destroy(h)
    o = kmap_b200.ORDER_FAST if order == "fast" else kmap_b200.ORDER_EXACT
    with kmap_b200.Chip(path, order=o) as chip:
        toks_g, lg_g = chip.infer(prompt, max_new, logits=True)
        assert chip.stats()["fused"] == 1 and chip.stats()["step_kernel"] == 1
        assert chip.stats()["stream_values"] == {"bf16": 1, "fp16": 2, "pool4096": 0}[values]
    assert toks_g.tolist() == toks_r.tolist()
    n = len(prompt) + max_new - 1   # the last step's logits are not computed
    np.testing.assert_allclose(lg_g[:n], lg_r[:n], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("name", ["tl", "gqa", "mha"])
def test_split_attention_matches_oracle(gpu, oracle, chip_dir, monkeypatch, name):
    """Attention split over up to 4 CTAs per head once the context passes
    KLLM_ATT_SPLIT_MIN positions (32 here, 256 by default): each split's
    max, sum of exps and unnormalised P.V, combined in the O phase's input
    staging.  Tokens identical to the oracle, logits within 1e-3 / 1e-4."""
    import kmap_b200
    monkeypatch.setenv("KLLM_ATT_SPLIT_MIN", "32")
    path = chip_dir(name)
    with kmap_b200.Chip(path) as chip:
        V, S = chip.info["vocab_size"], chip.info["max_seq_len"]
        prompt = np.random.default_rng(21).integers(3, V, S // 2).astype(np.int32)
        max_new = S - len(prompt) - 1
        toks_o, lg_o = _oracle_run(oracle, path, prompt, max_new)
        toks_g, lg_g = chip.infer(prompt, max_new, logits=True)
        assert chip.stats()["step_kernel"] == 1
    assert toks_g.tolist() == toks_o.tolist()
    np.testing.assert_allclose(lg_g, lg_o, rtol=RTOL, atol=ATOL)


def test_long_context_matches_reference(gpu, ref, tmp_path):
    """700 positions on a 2-layer chip at the TinyLlama-1.1B widths: split
    attention (3 splits per head at the end) against the compiled reference
    runtime, token by token."""
    import kmap_b200
    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
    spec.num_layers = 2
    spec.max_seq = 1024
    path = chipgen.ensure_chip(str(tmp_path), spec)
    prompt = np.random.default_rng(8).integers(3, spec.vocab_size, 694).astype(np.int32)
    max_new = 6
    h, info = ref.chip(path)
    s = ref.session(h, prompt, max_new)
    lg_r = np.zeros((len(prompt) + max_new, spec.vocab_size), np.float32)
    s.run(len(prompt) + max_new, lg_r)
    toks_r = s.tokens()
    s.close()
    ref.L.refh_chip_destroy(h)
    with kmap_b200.Chip(path) as chip:
        toks_g, lg_g = chip.infer(prompt, max_new, logits=True)
    assert toks_g.tolist() == toks_r.tolist()
    n = len(prompt) + max_new - 1
    np.testing.assert_allclose(lg_g[:n], lg_r[:n], rtol=RTOL, atol=ATOL)


HD128 = dict(num_layers=2, hidden_size=512, num_attention_heads=4, num_key_value_heads=2,
             intermediate_size=1024, vocab_size=1000, max_seq=320, norm_weights="random", seed=9)


@pytest.mark.parametrize("mode", ["step", "split", "prefill"])
def test_head_dim_128_matches_oracle(gpu, oracle, tmp_path, monkeypatch, mode):
    """Head dim 128 (the 7B / 8B architectures' geometry) through the
    persistent step kernel's 128 instance: step by step, with attention
    splits forced (KLLM_ATT_SPLIT_MIN=32), and with the batched prompt pass
    (tensor-core projections, tiled attention); tokens identical to the
    oracle, logits within 1e-3 / 1e-4."""
    import kmap_b200
    from kmap_b200 import chipgen
    if mode == "split":
        monkeypatch.setenv("KLLM_ATT_SPLIT_MIN", "32")
    path = chipgen.ensure_chip(str(tmp_path), chipgen.ModelSpec(**HD128))
    prompt = np.random.default_rng(4).integers(3, 1000, 150).astype(np.int32)
    max_new = 40
    toks_o, lg_o = _oracle_run(oracle, path, prompt, max_new)
    with kmap_b200.Chip(path, prefill=(mode == "prefill")) as chip:
        if mode == "prefill":
            toks_g = chip.infer(prompt, max_new)
            lg_last = chip.final_logits()
            assert toks_g.tolist() == toks_o.tolist()
            np.testing.assert_allclose(lg_last, lg_o[len(prompt) + max_new - 1], rtol=RTOL,
                                       atol=ATOL)
            return
        toks_g, lg_g = chip.infer(prompt, max_new, logits=True)
        assert chip.stats()["step_kernel"] == 1
    assert toks_g.tolist() == toks_o.tolist()
    np.testing.assert_allclose(lg_g, lg_o, rtol=RTOL, atol=ATOL)
