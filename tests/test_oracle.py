"""The oracle pinned: its C restatement against the compiled reference and
against the committed golden vectors (CPU only)."""
import os

import numpy as np
import pytest

import harness
import opcases

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("K,N,codes,rows", [
    (1, 5, 3, 1), (100, 33, 17, 1), (127, 8, 100, 1), (128, 64, 50, 1), (1000, 37, 400, 2),
    (1023, 8, 4096, 1), (1024, 16, 4096, 1), (1025, 9, 5461, 1), (2048, 256, 4096, 1),
    (5632, 64, 5461, 1)])
def test_tt_gemv_bitexact_vs_reference(ref, oracle, K, N, codes, rows):
    x, cb, idx = harness.tt_case(K * 7 + N, K, N, codes, rows)
    y_o = oracle.tt_gemv(x, cb, idx)
    tr = harness.TapeRun(ref, 3, {0: ("ext", x), 1: ("tt", cb, idx), 2: ("alloc", [1])},
                         [dict(tag=13, out_slot=2, in0=0, in1=1)])
    tr.run()
    y_r, shape = tr.read(2)
    tr.close()
    assert shape == (rows, N)
    assert np.array_equal(_bits(y_o).ravel(), _bits(y_r))


@pytest.mark.parametrize("case", opcases.cases(), ids=lambda c: c[0])
def test_ops_vs_reference(ref, oracle, case):
    name, n_slots, slots, instrs, out_slot, exact = case
    res = []
    for api in (ref, oracle):
        tr = harness.TapeRun(api, n_slots, slots, instrs)
        tr.run()
        res.append(tr.read(out_slot))
        tr.close()
    (y_r, s_r), (y_o, s_o) = res
    assert s_r == s_o
    assert y_r.size == y_o.size
    if exact:
        assert np.array_equal(_bits(y_r), _bits(y_o))
    else:
        np.testing.assert_allclose(y_o, y_r, rtol=1e-5, atol=1e-5)


def test_tt_gemv_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "tt_gemv_cases.npz"))
    for i in range(int(g["n"])):
        x, cb, idx, y = g["x%d" % i], g["cb%d" % i], g["idx%d" % i], g["y%d" % i]
        assert np.array_equal(_bits(oracle.tt_gemv(x, cb, idx)), _bits(y)), i


def test_tiny_decode_golden(oracle, tmp_path):
    """Oracle greedy tokens + logits on the golden tiny chip (regenerated from
    its spec) equal the reference's recorded ones."""
    from kmap_b200 import chipgen
    g = np.load(os.path.join(GOLDEN, "tiny_decode.npz"))
    spec = chipgen.ModelSpec(**dict(zip(g["spec_keys"].tolist(), g["spec_vals"].tolist())))
    for k in ("num_layers", "hidden_size", "num_attention_heads", "num_key_value_heads",
              "intermediate_size", "vocab_size", "max_seq", "seed"):
        setattr(spec, k, int(getattr(spec, k)))
    path = chipgen.ensure_chip(str(tmp_path), spec)
    idx = np.fromfile(os.path.join(path, "circuit", "const_%d_indices.bin" % int(g["tt_slot"])),
                      np.uint16)
    assert int(idx.astype(np.uint64).sum()) == int(g["tt_checksum"]), "chip generator drifted"
    oc = harness.OracleChip(oracle, path)
    toks, lg = oc.infer(g["prompt"], int(g["max_new"]))
    oc.close()
    assert np.array_equal(toks, g["tokens"])
    np.testing.assert_allclose(lg, g["logits"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", ["gqa", "mha"])
def test_tiny_decode_vs_reference(ref, oracle, chip_dir, name):
    path = chip_dir(name)
    h, info = ref.chip(path)
    prompt = np.random.default_rng(3).integers(3, int(info[0]), 9)
    toks_r = ref.infer(h, prompt, 24)
    toks_l, lg_r = ref.greedy_logits(h, prompt, 24, int(info[0]))
    ref.L.refh_chip_destroy(h)
    assert np.array_equal(toks_l, toks_r)   # the logits loop is the reference loop
    oc = harness.OracleChip(oracle, path)
    toks_o, lg_o = oc.infer(prompt, 24)
    oc.close()
    assert np.array_equal(toks_o, toks_r)
    np.testing.assert_allclose(lg_o, lg_r, rtol=1e-4, atol=1e-5)


def test_reference_session_windows_equal_full_run(ref, chip_dir):
    """The windowed reference session (the benchmark's reference arm) runs
    the same greedy loop as processor_infer: cut into windows of 5 positions
    it gives the same tokens and the same logits bits."""
    path = chip_dir("gqa")
    h, info = ref.chip(path)
    V = int(info[0])
    prompt = np.random.default_rng(8).integers(3, V, 7)
    toks_r = ref.infer(h, prompt, 16)
    toks_l, lg_r = ref.greedy_logits(h, prompt, 16, V)
    s = ref.session(h, prompt, 16)
    rows = []
    while True:
        buf = np.zeros((5, V), np.float32)
        n = s.run(5, buf)
        if n == 0:
            break
        rows.append(buf[:n])
    toks_s = s.tokens()
    s.close()
    ref.L.refh_chip_destroy(h)
    assert np.array_equal(toks_s, toks_r)
    assert np.array_equal(np.concatenate(rows).view(np.uint32), lg_r.view(np.uint32))
