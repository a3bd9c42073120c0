"""Test-side drivers for the three implementations of the tape ABI.

* ``Ref``    -- the unmodified reference runtime, compiled from its sources
                into oracle/_ref/libkllm_ref.so (present only where the
                reference could be built);
* ``Oracle`` -- this repository's C restatement (oracle/liboracle.so);
* ``Gpu``    -- the product, libkllm_cuda.so.

All three expose the same slot API (reference csrc/tape_runner.h), so a
test builds one tape and runs it on each.  Checker code only: nothing here
is imported by the product.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libkllm_ref.so")
ORACLE_SO = os.path.join(ROOT, "oracle", "liboracle.so")

import sys  # noqa: E402

sys.path.insert(0, ROOT)
from kmap_b200 import chipgen  # noqa: E402

INSTR = chipgen.INSTR_DTYPE
IP = C.POINTER(C.c_int)


def build_oracle():
    if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(
            os.path.join(ROOT, "oracle", "tape_oracle.c")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


def have_ref() -> bool:
    return os.path.exists(REF_SO)


class _Api:
    """Slot API over one library with a name prefix."""

    prefix = ""
    names = dict(create="tape_ctx_create", destroy="tape_ctx_destroy", alloc="tape_slot_alloc",
                 ext="tape_slot_set_external", tt="tape_slot_set_truth_table",
                 write="tape_slot_write", shape="tape_slot_set_shape", read="tape_slot_read",
                 rshape="tape_slot_read_shape", instr="tape_get_instr", run="tape_run")

    def __init__(self, so):
        self.L = C.CDLL(so)
        f = {k: getattr(self.L, v) for k, v in self.names.items()}
        f["create"].restype = C.c_void_p
        f["create"].argtypes = [C.c_int, C.c_int]
        f["destroy"].argtypes = [C.c_void_p]
        f["alloc"].argtypes = [C.c_void_p, C.c_int, IP, C.c_int]
        f["ext"].argtypes = [C.c_void_p, C.c_int, C.c_void_p, IP, C.c_int]
        f["tt"].argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int]
        f["write"].argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        f["shape"].argtypes = [C.c_void_p, C.c_int, IP, C.c_int]
        f["read"].restype = C.POINTER(C.c_float)
        f["read"].argtypes = [C.c_void_p, C.c_int, IP]
        f["rshape"].argtypes = [C.c_void_p, C.c_int, IP]
        f["instr"].restype = C.c_void_p
        f["instr"].argtypes = [C.c_void_p, C.c_int]
        f["run"].argtypes = [C.c_void_p]
        self.f = f


class Ref(_Api):
    def __init__(self):
        super().__init__(REF_SO)
        L = self.L
        L.refh_chip_load.restype = C.c_void_p
        L.refh_chip_load.argtypes = [C.c_char_p]
        L.refh_chip_destroy.argtypes = [C.c_void_p]
        L.refh_chip_info.argtypes = [C.c_void_p, IP]
        L.refh_processor_infer.argtypes = [C.c_void_p, IP, C.c_int, C.c_int, C.c_int, IP, IP]
        L.refh_greedy_logits.argtypes = [C.c_void_p, IP, C.c_int, C.c_int, IP, C.c_void_p]
        L.refh_infer_bytes.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_int,
                                       C.c_char_p, C.c_int, IP, IP]
        L.refh_bpe_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, IP]
        L.refh_bpe_decode.argtypes = [C.c_void_p, IP, C.c_int, C.c_int, C.c_int, C.c_char_p]
        L.compile_chip.argtypes = [C.c_char_p, C.c_int, C.c_char_p]
        L.refh_session_create.restype = C.c_void_p
        L.refh_session_create.argtypes = [C.c_void_p, IP, C.c_int, C.c_int]
        L.refh_session_run.restype = C.c_int
        L.refh_session_run.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.refh_session_tokens.restype = C.c_int
        L.refh_session_tokens.argtypes = [C.c_void_p, IP, C.c_int]
        L.refh_session_destroy.argtypes = [C.c_void_p]

    def session(self, h, prompt, max_new):
        """A resumable greedy run (refh_session_*): .run(n) advances it."""
        return RefSession(self, h, prompt, max_new)

    # chip-level helpers (the reference's own loader and drivers)
    def chip(self, path):
        h = self.L.refh_chip_load(path.encode())
        info = np.zeros(18, np.int32)
        self.L.refh_chip_info(h, info.ctypes.data_as(IP))
        return h, info

    def infer(self, h, prompt, max_new, eos=-1):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int(0)
        self.L.refh_processor_infer(h, p.ctypes.data_as(IP), len(p), max_new, eos,
                                    out.ctypes.data_as(IP), C.byref(n))
        return out[:n.value].copy()

    def greedy_logits(self, h, prompt, max_new, vocab):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        lg = np.zeros((len(p) + max_new, vocab), np.float32)
        self.L.refh_greedy_logits(h, p.ctypes.data_as(IP), len(p), max_new,
                                  out.ctypes.data_as(IP), lg.ctypes.data_as(C.c_void_p))
        return out[:max_new].copy(), lg

    def infer_bytes(self, h, text: bytes, max_new, max_seq):
        buf = C.create_string_buffer(1 << 16)
        n, g = C.c_int(0), C.c_int(0)
        self.L.refh_infer_bytes(h, text, len(text), max_new, max_seq, buf, 1 << 16,
                                C.byref(n), C.byref(g))
        return buf.raw[:n.value], g.value

    def encode(self, h, text: bytes, max_tokens=4096):
        out = np.zeros(max_tokens, np.int32)
        n = self.L.refh_bpe_encode(h, text, len(text), max_tokens, out.ctypes.data_as(IP))
        return out[:n].copy()

    def decode(self, h, ids, max_bytes=8192, skip=0):
        ids = np.ascontiguousarray(ids, np.int32)
        buf = C.create_string_buffer(max_bytes + 256)
        n = self.L.refh_bpe_decode(h, ids.ctypes.data_as(IP), len(ids), max_bytes, skip, buf)
        return buf.raw[:n]


class RefSession:
    """The reference greedy loop cut into windows of positions."""

    def __init__(self, ref: Ref, h, prompt, max_new):
        self.ref, self.max_new = ref, max_new
        self.p = np.ascontiguousarray(prompt, np.int32)
        self.total = len(self.p) + max_new
        self.s = ref.L.refh_session_create(h, self.p.ctypes.data_as(IP), len(self.p), max_new)

    def run(self, n, logits: np.ndarray | None = None) -> int:
        ptr = None
        if logits is not None:
            assert logits.dtype == np.float32 and logits.flags.c_contiguous and logits.shape[0] >= n
            ptr = logits.ctypes.data
        return self.ref.L.refh_session_run(self.s, n, ptr)

    def tokens(self) -> np.ndarray:
        out = np.zeros(max(self.max_new, 1), np.int32)
        n = self.ref.L.refh_session_tokens(self.s, out.ctypes.data_as(IP), len(out))
        return out[:n].copy()

    def close(self):
        if self.s:
            self.ref.L.refh_session_destroy(self.s)
            self.s = None


class Oracle(_Api):
    names = {k: "orc_" + v for k, v in dict(
        create="ctx_create", destroy="ctx_destroy", alloc="slot_alloc",
        ext="slot_set_external", tt="slot_set_truth_table", write="slot_write",
        shape="slot_set_shape", read="slot_read", rshape="slot_read_shape",
        instr="get_instr", run="tape_run").items()}

    def __init__(self):
        build_oracle()
        super().__init__(ORACLE_SO)
        L = self.L
        L.orc_tt_gemv.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                  C.c_int, C.c_int, C.c_void_p]
        L.orc_processor_infer.restype = C.c_int
        L.orc_processor_infer.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, IP,
                                          IP, C.c_int, C.c_int, C.c_int, IP, C.c_int, C.c_int,
                                          C.c_int, IP, IP, C.c_void_p]

    def tt_gemv(self, x, cb, idx):
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None]
        cb = np.ascontiguousarray(cb, np.float32)
        idx = np.ascontiguousarray(idx, np.uint16)
        K, N = idx.shape
        y = np.empty((x.shape[0], N), np.float32)
        self.L.orc_tt_gemv(x.ctypes.data, x.shape[0], cb.ctypes.data, cb.size, idx.ctypes.data,
                           K, N, y.ctypes.data)
        return y


class Gpu(_Api):
    def __init__(self):
        from kmap_b200 import LIB_PATH, lib
        lib()
        super().__init__(LIB_PATH)


# ------------------------------------------------------------- one tape --

class TapeRun:
    """One tape built through an implementation's slot API.

    ``slots`` maps slot id -> ("alloc", shape) | ("ext", array) |
    ("tt", codebook, indices); ``instrs`` is a list of INSTR field dicts.
    Keeps every host buffer alive for the context's lifetime."""

    def __init__(self, api: _Api, n_slots: int, slots: dict, instrs: list):
        self.api, self.keep = api, []
        f = api.f
        self.ctx = f["create"](n_slots, len(instrs))
        for s, spec in slots.items():
            if spec[0] == "alloc":
                sh = np.asarray(spec[1], np.int32)
                f["alloc"](self.ctx, s, sh.ctypes.data_as(IP), len(sh))
            elif spec[0] == "ext":
                a = np.ascontiguousarray(spec[1], np.float32)
                sh = np.asarray(a.shape, np.int32)
                self.keep += [a, sh]
                f["ext"](self.ctx, s, a.ctypes.data, sh.ctypes.data_as(IP), a.ndim)
            else:
                cb = np.ascontiguousarray(spec[1], np.float32)
                ix = np.ascontiguousarray(spec[2], np.uint16)
                self.keep += [cb, ix]
                f["tt"](self.ctx, s, cb.ctypes.data, cb.size, ix.ctypes.data, *ix.shape)
        for i, fields in enumerate(instrs):
            rec = np.zeros(1, INSTR)
            for k, v in fields.items():
                if isinstance(v, (list, tuple)):
                    rec[0][k][:len(v)] = v
                else:
                    rec[0][k] = v
            p = f["instr"](self.ctx, i)
            C.memmove(p, rec.ctypes.data, INSTR.itemsize)

    def set_ext(self, s, a):
        a = np.ascontiguousarray(a, np.float32)
        sh = np.asarray(a.shape, np.int32)
        self.keep += [a, sh]
        self.api.f["ext"](self.ctx, s, a.ctypes.data, sh.ctypes.data_as(IP), a.ndim)

    def run(self):
        self.api.f["run"](self.ctx)

    def read(self, s):
        n = C.c_int(0)
        p = self.api.f["read"](self.ctx, s, C.byref(n))
        sh = np.zeros(8, np.int32)
        nd = self.api.f["rshape"](self.ctx, s, sh.ctypes.data_as(IP))
        data = np.ctypeslib.as_array(p, (n.value,)).copy() if n.value > 0 and p else np.zeros(0, np.float32)
        return data, tuple(int(v) for v in sh[:nd])

    def close(self):
        if self.ctx:
            self.api.f["destroy"](self.ctx)
            self.ctx = None


# ------------------------------------------------------ chip for oracle --

class OracleChip:
    """A chip directory loaded into the oracle (Python restatement of the
    reference loader, kllm.c:152-388, for the C restatement)."""

    def __init__(self, oracle: Oracle, path: str):
        self.o, self.path = oracle, path
        pj = open(os.path.join(path, "processor.json")).read()
        self.meta = json.loads(pj)
        m = self.meta
        circ = os.path.join(path, "circuit")
        tape = np.fromfile(os.path.join(circ, "tape.bin"), np.int32)
        n_instr = int(tape[0])
        slots = np.fromfile(os.path.join(circ, "slots.bin"), np.int32)
        n_slots = int(slots[0])
        recs = slots[1:].reshape(n_slots, 10)
        self.ctx = oracle.f["create"](n_slots, n_instr)
        raw = tape[2:].view(np.uint8)
        C.memmove(oracle.f["instr"](self.ctx, 0), raw.ctypes.data, raw.nbytes)
        self.keep = [raw]
        for s in range(n_slots):
            typ, nd = int(recs[s, 0]), int(recs[s, 1])
            sh = np.ascontiguousarray(recs[s, 2:2 + nd], np.int32)
            self.keep.append(sh)
            if typ == 4:
                cb = np.fromfile(os.path.join(circ, "const_%d_codebook.bin" % s), np.float32)
                ix = np.fromfile(os.path.join(circ, "const_%d_indices.bin" % s), np.uint16)
                self.keep += [cb, ix]
                oracle.f["tt"](self.ctx, s, cb.ctypes.data, cb.size, ix.ctypes.data,
                               int(sh[0]), int(sh[1]))
            elif typ == 1:
                d = np.fromfile(os.path.join(circ, "const_%d.bin" % s), np.float32)
                self.keep.append(d)
                oracle.f["ext"](self.ctx, s, d.ctypes.data, sh.ctypes.data_as(IP), nd)
            elif typ in (2, 3):
                oracle.f["alloc"](self.ctx, s, sh.ctypes.data_as(IP), nd)
        tab = os.path.join(path, "tables")
        self.embed = np.fromfile(os.path.join(tab, "embed_table.bin"), np.float32)
        self.cos = np.fromfile(os.path.join(tab, "rope_cos.bin"), np.float32)
        self.sin = np.fromfile(os.path.join(tab, "rope_sin.bin"), np.float32)
        L = m["num_layers"]
        self.kv_in = np.array([m["input_map"]["L%d/cache_%s" % (l, kv)] for l in range(L)
                               for kv in "kv"], np.int32)
        self.kv_out = np.array([m["output_map"]["L%d/new_%s" % (l, kv)] for l in range(L)
                                for kv in "kv"], np.int32)

    def infer(self, prompt, max_new, eos=-1):
        m = self.meta
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int(0)
        lg = np.zeros((len(p) + max_new, m["vocab_size"]), np.float32)
        steps = self.o.L.orc_processor_infer(
            self.ctx, self.embed.ctypes.data, m["vocab_size"], m["hidden_dim"],
            self.cos.ctypes.data, self.sin.ctypes.data, m["head_dim"],
            m["input_map"]["token_embed"], m["input_map"]["rope_cos"],
            m["input_map"]["rope_sin"], self.kv_in.ctypes.data_as(IP),
            self.kv_out.ctypes.data_as(IP), m["output_map"]["logits"], m["num_layers"],
            m["num_kv_heads"], p.ctypes.data_as(IP), len(p), max_new, eos,
            out.ctypes.data_as(IP), C.byref(n), lg.ctypes.data)
        return out[:n.value].copy(), lg[:steps]

    def close(self):
        if self.ctx:
            self.o.f["destroy"](self.ctx)
            self.ctx = None


gaussian_rank_indices = chipgen.gaussian_rank_indices
tt_case = chipgen.tt_case
