"""Parity at full size (needs a B200 and the compiled reference).

* Decode: the 22-layer TinyLlama-1.1B-architecture chip (every matrix
  N(0, 0.02) rounded to bf16), a 32-token uniform-random prompt and 128
  greedy tokens -- the benchmark's own workload -- against the compiled
  reference runtime on the same chip: identical token IDs and every step's
  logits within atol 1e-3 / rtol 1e-4, in the exact and the fast summation
  order.
* Prefill: a 2047-token prompt through the batched prompt pass against the
  step-by-step pass on the GPU (first token's logits within 1e-3 / 1e-4,
  same first token), and a 255-token prompt against the reference (first
  token's logits, then 8 generated tokens).

The chip is written once into KLLM_CHIP_CACHE (default /tmp/kllm_chips),
which the benchmark shares."""
import os

import numpy as np
import pytest


pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-4
PROMPT, GEN = 32, 128


@pytest.fixture(scope="module")
def chip0():
    from kmap_b200 import chipgen
    spec = chipgen.ModelSpec(**{**chipgen.TINYLLAMA_1B.__dict__})
    spec.max_seq = 2048
    root = os.environ.get("KLLM_CHIP_CACHE", "/tmp/kllm_chips")
    os.makedirs(root, exist_ok=True)
    import fcntl
    with open(os.path.join(root, ".lock"), "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        return chipgen.ensure_chip(root, spec)


def _prompt(n, seed=0):
    return np.random.default_rng(seed).integers(3, 32000, n).astype(np.int32)


@pytest.fixture(scope="module")
def ref_run(ref, chip0):
    """The reference's tokens and every position's logits for the workload."""
    h, info = ref.chip(chip0)
    s = ref.session(h, _prompt(PROMPT), GEN)
    lg = np.zeros((PROMPT + GEN, int(info[0])), np.float32)
    n = s.run(PROMPT + GEN, lg)
    toks = s.tokens()
    s.close()
    ref.L.refh_chip_destroy(h)
    assert n == PROMPT + GEN and len(toks) == GEN
    return toks, lg


@pytest.mark.parametrize("order", ["exact", "fast"])
def test_config0_decode_matches_reference(gpu, chip0, ref_run, order):
    import kmap_b200
    toks_r, lg_r = ref_run
    o = kmap_b200.ORDER_FAST if order == "fast" else kmap_b200.ORDER_EXACT
    with kmap_b200.Chip(chip0, order=o) as chip:
        toks, lg = chip.infer(_prompt(PROMPT), GEN, logits=True)
        st = chip.stats()
    assert st["fused"] == 1 and st["step_kernel"] == 1
    assert toks.tolist() == toks_r.tolist()
    rows = PROMPT + GEN - 1   # the last step's logits pick no token
    np.testing.assert_allclose(lg[:rows], lg_r[:rows], rtol=RTOL, atol=ATOL)


def test_config2_prefill_matches_step_by_step(gpu, chip0):
    import kmap_b200
    prompt = _prompt(2047, seed=2)
    first = {}
    for batched in (True, False):
        with kmap_b200.Chip(chip0, prefill=batched) as chip:
            chip.infer(prompt, 0)
            first[batched] = chip.final_logits()
    assert int(np.argmax(first[True])) == int(np.argmax(first[False]))
    np.testing.assert_allclose(first[True], first[False], rtol=RTOL, atol=ATOL)


def test_prefill_255_matches_reference(gpu, ref, chip0):
    import kmap_b200
    prompt = _prompt(255, seed=4)
    h, info = ref.chip(chip0)
    s = ref.session(h, prompt, 8)
    lg = np.zeros((255 + 8, int(info[0])), np.float32)
    assert s.run(255 + 8, lg) == 255 + 8
    toks_r = s.tokens()
    s.close()
    ref.L.refh_chip_destroy(h)
    with kmap_b200.Chip(chip0, prefill=True) as chip:
        chip.infer(prompt, 0)
        first = chip.final_logits()
        toks = chip.infer(prompt, 8)
    np.testing.assert_allclose(first, lg[254], rtol=RTOL, atol=ATOL)
    assert toks.tolist() == toks_r.tolist()
