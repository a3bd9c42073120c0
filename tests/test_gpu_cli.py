"""The drop-in check: the UNMODIFIED reference CLI (csrc/kllm.c), linked
against libkllm_cuda.so instead of the reference runtime, prints the same
`kllm infer` output as the reference CLI on the CPU (needs a B200 and the
binaries that oracle/Makefile builds where the reference sources exist)."""
import os
import subprocess

import pytest

import harness

pytestmark = pytest.mark.gpu

REF = os.path.join(harness.ROOT, "oracle", "_ref", "kllm_ref")
GPU = os.path.join(harness.ROOT, "oracle", "_ref", "kllm_gpu")


@pytest.mark.skipif(not (os.path.exists(REF) and os.path.exists(GPU)),
                    reason="reference CLI binaries not built")
@pytest.mark.parametrize("prompt", ["What is the capital of France?", "Hello world"])
def test_kllm_infer_same_text(gpu, chip_dir, prompt):
    path = chip_dir("tl")
    outs = []
    for exe in (REF, GPU):
        r = subprocess.run([exe, "infer", path, "--max-tokens", "12", *prompt.split()],
                           capture_output=True, timeout=300)
        assert r.returncode == 0, r.stderr.decode(errors="replace")
        outs.append(r.stdout)
    assert outs[0] == outs[1]
    assert len(outs[0].strip()) > 0
