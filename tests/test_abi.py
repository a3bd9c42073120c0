"""The C-ABI library without a GPU: it loads, exports every symbol the
headers declare, loads chips exactly like the reference loader, tokenizes
like the reference BPE, and fails loudly (no CPU fallback) where compute
would need a device."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import harness

ROOT = harness.ROOT


def _declared():
    names = set()
    for h in ("tape_runner.h", "kllm_cuda.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\(", src):
            if m.group(1) not in ("if", "for", "while", "sizeof", "return", "int", "void",
                                  "char", "float", "typedef", "const"):
                names.add(m.group(1))
    names.discard("token_callback_fn")
    return sorted(n for n in names if not n.startswith("_"))


def test_exports_every_declared_symbol(built_lib):
    names = _declared()
    assert "tape_run" in names and "kllm_tt_gemv" in names and "processor_infer_bytes" in names
    missing = [n for n in names if not hasattr(built_lib, n)]
    assert not missing, missing


def test_no_cpu_fallback_without_gpu(built_lib):
    import kmap_b200
    if kmap_b200.device_count() > 0:
        pytest.skip("a GPU is visible")
    x = np.ones((1, 4), np.float32)
    cb = np.ones(3, np.float32)
    idx = np.zeros((4, 2), np.uint16)
    with pytest.raises(kmap_b200.KllmError):
        kmap_b200.tt_gemv_host(x, cb, idx)


def test_chip_loader_matches_reference(ref, built_lib, chip_dir):
    import kmap_b200
    for name in ("gqa", "mha"):
        path = chip_dir(name)
        h, info = ref.chip(path)
        with kmap_b200.Chip(path) as chip:
            assert [chip.info[k] for k in kmap_b200.INFO_KEYS] == info.tolist()
        ref.L.refh_chip_destroy(h)


def test_chip_loader_rejects_truncated_files(built_lib, chip_dir, tmp_path):
    import shutil

    import kmap_b200
    src = chip_dir("gqa")
    dst = str(tmp_path / "bad")
    shutil.copytree(src, dst)
    rec = np.fromfile(os.path.join(dst, "circuit", "slots.bin"), np.int32)[1:].reshape(-1, 10)
    tt = int(np.nonzero(rec[:, 0] == 4)[0][0])
    p = os.path.join(dst, "circuit", "const_%d_indices.bin" % tt)
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-2])
    with pytest.raises(kmap_b200.KllmError, match="expected"):
        kmap_b200.Chip(dst)
    os.remove(p)
    with pytest.raises(kmap_b200.KllmError, match="cannot open"):
        kmap_b200.Chip(dst)


TEXTS = [b"", b"Hello", b"What is the capital of France?",
         b"Explain quantum computing in simple terms for a beginner.",
         b"<|user|>\nHello world</s>\n<|assistant|>\n", b"  double  spaces ",
         "café 世界 \U0001F600!".encode(), b"</s></s>x</s>", b"\x01\x02\xff tail",
         b"the the the model token chip", b"tok12 tok3 <s> inside"]


def test_bpe_encode_decode_match_reference(ref, built_lib, chip_dir):
    import kmap_b200
    path = chip_dir("tl")
    h, _ = ref.chip(path)
    with kmap_b200.Chip(path) as chip:
        for t in TEXTS:
            ids_r = ref.encode(h, t)
            ids_g = chip.encode(t)
            assert ids_g.tolist() == ids_r.tolist(), t
            for skip in (0, 1):
                assert chip.decode(ids_r, skip_leading_space=skip) == ref.decode(h, ids_r, skip=skip)
        # max_tokens truncation
        assert chip.encode(TEXTS[3], 5).tolist() == ref.encode(h, TEXTS[3], 5).tolist()
    ref.L.refh_chip_destroy(h)


def test_fused_plan_matches_compiler_tapes(built_lib, chip_dir):
    import kmap_b200
    for name in ("gqa", "mha", "tl"):
        with kmap_b200.Chip(chip_dir(name)) as chip:
            ok, why = chip.plan_match()
            assert ok, (name, why)


def test_fused_plan_rejects_changed_tapes(built_lib, chip_dir):
    """Any change to the template's wiring or parameters sends processor_infer
    to the per-instruction executor instead of the fused plan."""
    import ctypes as C

    import kmap_b200
    from kmap_b200 import chipgen
    with kmap_b200.Chip(chip_dir("tl")) as chip:
        lib = kmap_b200.lib()
        n = chip.info["n_instrs"]
        edits = [(3, "axis", 0), (3, "keepdims", 0), (12, "in0", 3), (n - 1, "in1", 0),
                 (30, "tag", 8), (9, "starts", 1)]
        for i, field, val in edits:
            p = lib.tape_get_instr(chip.ctx, i)
            rec = np.frombuffer(C.string_at(p, 276), chipgen.INSTR_DTYPE).copy()
            old = np.copy(rec[0][field])
            if np.ndim(old):
                rec[0][field][1] = old[1] + val
            else:
                rec[0][field] = val if old != val else val + 1
            C.memmove(p, rec.ctypes.data, 276)
            ok, why = chip.plan_match()
            assert not ok and why, (i, field)
            rec[0][field] = old
            C.memmove(p, rec.ctypes.data, 276)
        assert chip.plan_match()[0]
        # a KV output that differs from the slot map
        import json
        import os
        m = json.load(open(os.path.join(chip.path, "processor.json")))
        ko = [m["output_map"]["L%d/new_%s" % (l, c)] for l in range(2) for c in "kv"]
        ko[1], ko[0] = ko[0], ko[1]
        assert not chip.plan_match(kv_out=ko)[0]


def test_infer_batch_rejects_bad_arguments(built_lib):
    import ctypes as C

    import kmap_b200
    lib = kmap_b200.lib()
    one = (C.c_int * 4)(1, 1, 1, 1)
    assert lib.kllm_infer_batch(None, one, one, 1, 1, -1, one, one) == -1
    assert b"bad argument" in lib.kllm_last_error()
    lib.kllm_clear_error()
    assert lib.kllm_chip_infer_batch(None, one, one, 1, 1, -1, one, one) == -1
    lib.kllm_clear_error()
