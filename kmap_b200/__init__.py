"""kmap_b200 -- B200-native executor for kllm chips.

The product is ``libkllm_cuda.so``: a C-ABI library (``include/tape_runner.h``
drop-in surface + ``include/kllm_cuda.h`` extensions) whose tape steps run
as hand-written sm_100a kernels.  This module is a thin ctypes binding of
that ABI for Python callers, tests and benchmarks; it adds no compute of its
own, and every call fails loudly when the library or a GPU is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkllm_cuda.so")

_lib = None


class KllmError(RuntimeError):
    pass


def _fp(t):
    return C.POINTER(t)


_SIGS = {
    "kllm_last_error": (C.c_char_p, []),
    "kllm_clear_error": (None, []),
    "kllm_version": (C.c_char_p, []),
    "kllm_device_count": (C.c_int, []),
    "kllm_set_device": (C.c_int, [C.c_int]),
    "kllm_tape_run": (C.c_int, [C.c_void_p]),
    "kllm_launch_count": (C.c_longlong, []),
    "kllm_set_infer_opts": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kllm_get_infer_stats": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kllm_default_infer_opts": (None, [C.c_void_p]),
    "kllm_tt_gemv": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "kllm_tt_gemm": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                               C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "kllm_tt_gemv_host": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                     C.c_int, C.c_int, C.c_void_p]),
    "kllm_tt_gemm_tc": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                  C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "kllm_chip_open": (C.c_void_p, [C.c_char_p]),
    "kllm_chip_close": (None, [C.c_void_p]),
    "kllm_chip_plan_prepare": (C.c_int, [C.c_void_p]),
    "kllm_shard_set": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "kllm_shard_export": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t,
                                    C.POINTER(C.c_size_t)]),
    "kllm_shard_connect": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "kllm_chip_ctx": (C.c_void_p, [C.c_void_p]),
    "kllm_chip_info": (C.c_int, [C.c_void_p, _fp(C.c_int)]),
    "kllm_chip_infer": (C.c_int, [C.c_void_p, _fp(C.c_int), C.c_int, C.c_int, C.c_int,
                                   _fp(C.c_int), _fp(C.c_int)]),
    "kllm_chip_infer_bytes": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_int,
                                         C.c_void_p, C.c_void_p, _fp(C.c_int)]),
    "kllm_chip_encode": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_int, _fp(C.c_int32)]),
    "kllm_chip_infer_batch": (C.c_int, [C.c_void_p, _fp(C.c_int), _fp(C.c_int), C.c_int, C.c_int,
                                         C.c_int, _fp(C.c_int), _fp(C.c_int)]),
    "kllm_infer_batch": (C.c_int, [C.c_void_p, _fp(C.c_int), _fp(C.c_int), C.c_int, C.c_int,
                                    C.c_int, _fp(C.c_int), _fp(C.c_int)]),
    "kllm_chip_decode": (C.c_int, [C.c_void_p, _fp(C.c_int32), C.c_int, C.c_int, C.c_int,
                                    C.c_char_p]),
    "kllm_plan_match": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, _fp(C.c_int), _fp(C.c_int), C.c_int, C.c_int,
                                  C.c_int, C.c_char_p, C.c_int]),
    "tape_ctx_create": (C.c_void_p, [C.c_int, C.c_int]),
    "tape_ctx_destroy": (None, [C.c_void_p]),
    "tape_ctx_n_instrs": (C.c_int, [C.c_void_p]),
    "tape_ctx_n_slots": (C.c_int, [C.c_void_p]),
    "tape_slot_alloc": (None, [C.c_void_p, C.c_int, _fp(C.c_int), C.c_int]),
    "tape_slot_set_external": (None, [C.c_void_p, C.c_int, C.c_void_p, _fp(C.c_int), C.c_int]),
    "tape_slot_set_truth_table": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                         C.c_int, C.c_int]),
    "tape_slot_write": (None, [C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
    "tape_slot_set_shape": (None, [C.c_void_p, C.c_int, _fp(C.c_int), C.c_int]),
    "tape_slot_read": (_fp(C.c_float), [C.c_void_p, C.c_int, _fp(C.c_int)]),
    "tape_slot_read_shape": (C.c_int, [C.c_void_p, C.c_int, _fp(C.c_int)]),
    "tape_get_instr": (C.c_void_p, [C.c_void_p, C.c_int]),
    "tape_run": (None, [C.c_void_p]),
    "processor_infer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                  C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                  C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                  C.c_int, C.c_int, C.c_void_p, _fp(C.c_int)]),
    "bpe_encode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                             C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                             C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                             C.c_void_p]),
    "bpe_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                             C.c_int, C.c_int, C.c_int, C.c_void_p]),
}


def lib():
    """The loaded libkllm_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise KllmError("libkllm_cuda.so is not built: run `python -m kmap_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def last_error() -> str | None:
    e = lib().kllm_last_error()
    return e.decode() if e else None


def check(rc, what="call"):
    if rc != 0:
        msg = last_error() or "unknown error"
        lib().kllm_clear_error()
        raise KllmError("%s failed: %s" % (what, msg))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _iptr(a: np.ndarray):
    return a.ctypes.data_as(_fp(C.c_int))


def device_count() -> int:
    return lib().kllm_device_count()


def require_gpu():
    if device_count() < 1:
        raise KllmError("no CUDA device visible: the kllm executor has no CPU fallback")


# --------------------------------------------------------- infer options --

class InferOpts(C.Structure):
    _fields_ = [("mode", C.c_int), ("logits_out", C.c_void_p), ("logits_rows", C.c_int),
                ("use_graphs", C.c_int), ("order", C.c_int), ("prefill", C.c_int),
                ("reserved", C.c_int * 6)]


class InferStats(C.Structure):
    _fields_ = [("fused", C.c_int), ("steps", C.c_int), ("prefill_ms", C.c_double),
                ("decode_ms", C.c_double), ("total_ms", C.c_double),
                ("launches", C.c_longlong), ("step_kernel", C.c_int),
                ("stream_values", C.c_int), ("reserved", C.c_int * 6)]


MODE_AUTO, MODE_GENERIC, MODE_FUSED = 0, 1, 2


def exchange_blocks(block: bytes, group=None) -> list:
    """All ranks' shard blocks, in rank order, over torch.distributed (any
    backend: the blocks are a few hundred bytes of host data)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, block, group=group)
    return out

ORDER_EXACT, ORDER_FAST = 0, 1


def tt_gemv_host(x: np.ndarray, codebook: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """y = x @ codebook[idx] in the reference TT-GEMV order (host buffers)."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    cb = np.ascontiguousarray(codebook, np.float32)
    idx = np.ascontiguousarray(idx, np.uint16)
    K, N = idx.shape
    assert x.shape[1] == K
    y = np.empty((x.shape[0], N), np.float32)
    check(lib().kllm_tt_gemv_host(_ptr(x), x.shape[0], _ptr(cb), cb.size, _ptr(idx), K, N,
                                  _ptr(y)), "kllm_tt_gemv_host")
    return y


# ----------------------------------------------------------------- chips --

INFO_KEYS = ("vocab_size", "hidden_dim", "num_layers", "num_kv_heads", "head_dim",
             "max_seq_len", "eos_token_id", "logits_slot", "token_embed_slot",
             "rope_cos_slot", "rope_sin_slot", "n_slots", "n_instrs", "bos_token_id",
             "table_size", "max_piece_len", "num_merges", "num_special")


class Chip:
    """A chip directory loaded into a device tape context."""

    def __init__(self, path: str, order: int = 0, prefill: bool = False):
        self.path = path
        self.order = order        # ORDER_EXACT / ORDER_FAST for the fused decode step
        self.prefill = prefill    # batched prompt pass (kllm_infer_opts.prefill)
        h = lib().kllm_chip_open(path.encode())
        if not h:
            msg = last_error()
            lib().kllm_clear_error()
            raise KllmError("kllm_chip_open(%s): %s" % (path, msg))
        self.h = h
        info = np.zeros(18, np.int32)
        lib().kllm_chip_info(h, _iptr(info))
        self.info = dict(zip(INFO_KEYS, (int(v) for v in info)))

    @property
    def ctx(self):
        return lib().kllm_chip_ctx(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().kllm_chip_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def set_opts(self, mode=MODE_AUTO, logits: np.ndarray | None = None, use_graphs=True,
                 order=None):
        o = InferOpts()
        lib().kllm_default_infer_opts(C.byref(o))
        o.mode = mode
        o.use_graphs = 1 if use_graphs else 0
        o.order = self.order if order is None else order
        o.prefill = 1 if self.prefill else 0
        if logits is not None:
            assert logits.dtype == np.float32 and logits.flags.c_contiguous
            o.logits_out = logits.ctypes.data
            o.logits_rows = logits.shape[0]
        check(lib().kllm_set_infer_opts(self.ctx, C.byref(o)), "kllm_set_infer_opts")

    def plan_match(self, kv_in=None, kv_out=None):
        """(matched, reason): whether processor_infer takes the fused plan."""
        import json
        m = json.load(open(os.path.join(self.path, "processor.json")))
        L = m["num_layers"]
        if kv_in is None:
            kv_in = [m["input_map"]["L%d/cache_%s" % (l, c)] for l in range(L) for c in "kv"]
        if kv_out is None:
            kv_out = [m["output_map"]["L%d/new_%s" % (l, c)] for l in range(L) for c in "kv"]
        ki = np.asarray(kv_in, np.int32)
        ko = np.asarray(kv_out, np.int32)
        why = C.create_string_buffer(512)
        i = self.info
        r = lib().kllm_plan_match(self.ctx, i["vocab_size"], i["hidden_dim"], i["head_dim"],
                                  i["token_embed_slot"], i["rope_cos_slot"], i["rope_sin_slot"],
                                  _iptr(ki), _iptr(ko), i["logits_slot"], i["num_layers"],
                                  i["num_kv_heads"], why, 512)
        return r == 1, why.value.decode()

    # ------------------------------------------------ column-sharded decode
    def shard(self, rank: int, world: int) -> bytes:
        """Make this chip rank `rank` of a `world`-GPU column-sharded decode:
        build its plan (this rank's column groups only) and return the block
        every other rank needs (pass all blocks, in rank order, to connect)."""
        check(lib().kllm_shard_set(self.ctx, rank, world), "kllm_shard_set")
        self.set_opts()
        check(lib().kllm_chip_plan_prepare(self.h), "kllm_chip_plan_prepare")
        n = C.c_size_t(0)
        lib().kllm_shard_export(self.ctx, None, 0, C.byref(n))
        buf = C.create_string_buffer(n.value)
        check(lib().kllm_shard_export(self.ctx, buf, n.value, C.byref(n)), "kllm_shard_export")
        return buf.raw[:n.value]

    def final_logits(self) -> np.ndarray:
        """The logits slot after the last processor_infer step ([vocab])."""
        n = C.c_int(0)
        ptr = lib().tape_slot_read(self.ctx, int(self.info["logits_slot"]), C.byref(n))
        if not ptr:
            raise KllmError("tape_slot_read: " + last_error())
        V = int(self.info["vocab_size"])
        a = np.ctypeslib.as_array(ptr, shape=(n.value,))
        return a[max(n.value - V, 0):].copy()

    def connect(self, blocks: list) -> None:
        """Map the other ranks' buffers (blocks from every rank's shard())."""
        per = len(blocks[0])
        assert all(len(b) == per for b in blocks)
        data = b"".join(blocks)
        check(lib().kllm_shard_connect(self.ctx, data, per), "kllm_shard_connect")

    def stats(self) -> dict:
        s = InferStats()
        check(lib().kllm_get_infer_stats(self.ctx, C.byref(s)), "kllm_get_infer_stats")
        return {k: getattr(s, k) for k, _ in InferStats._fields_ if k != "reserved"}

    def infer(self, prompt, max_new: int, eos: int = -1, mode=MODE_AUTO,
              logits: bool = False):
        """Greedy generation from token IDs (processor_infer).

        Returns the generated IDs, plus the per-step logits rows
        ``[len(prompt) + max_new][vocab]`` when ``logits`` is set."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int(0)
        lg = None
        if logits:
            lg = np.zeros((len(p) + max_new, self.info["vocab_size"]), np.float32)
        self.set_opts(mode=mode, logits=lg)
        rc = lib().kllm_chip_infer(self.h, _iptr(p), len(p), max_new, eos, _iptr(out),
                                   C.byref(n))
        self.set_opts(mode=MODE_AUTO)
        check(rc, "processor_infer")
        toks = out[:n.value].copy()
        return (toks, lg) if logits else toks

    def infer_batch(self, prompts, max_new: int, eos: int = -1, use_graphs: bool = True):
        """Greedy generation for several sequences at once
        (kllm_chip_infer_batch): returns one token array per sequence, each
        cut before its first `eos`."""
        lens = np.array([len(p) for p in prompts], np.int32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]),
                                    np.int32)
        out = np.zeros((len(prompts), max_new), np.int32)
        n = np.zeros(len(prompts), np.int32)
        self.set_opts(use_graphs=use_graphs)
        check(lib().kllm_chip_infer_batch(self.h, _iptr(flat), _iptr(lens), len(prompts), max_new,
                                          eos, _iptr(out), _iptr(n)), "kllm_chip_infer_batch")
        return [out[i, :n[i]].copy() for i in range(len(prompts))]

    def infer_bytes(self, text: bytes, max_new: int, max_seq: int = 0, stop_after: int = -1):
        """Bytes in, streamed bytes out (processor_infer_bytes)."""
        pieces = []
        CB = C.CFUNCTYPE(C.c_int, C.POINTER(C.c_uint8), C.c_int, C.c_void_p)

        def cb(ptr, n, ud):
            pieces.append(C.string_at(ptr, n))
            return 1 if (stop_after >= 0 and len(pieces) >= stop_after) else 0

        ccb = CB(cb)
        gen = C.c_int(0)
        check(lib().kllm_chip_infer_bytes(self.h, text, len(text), max_new, max_seq,
                                          C.cast(ccb, C.c_void_p), None, C.byref(gen)),
              "processor_infer_bytes")
        return b"".join(pieces), gen.value, pieces

    def encode(self, text: bytes, max_tokens: int = 4096) -> np.ndarray:
        out = np.zeros(max_tokens, np.int32)
        n = lib().kllm_chip_encode(self.h, text, len(text), max_tokens,
                                   out.ctypes.data_as(_fp(C.c_int32)))
        return out[:n].copy()

    def decode(self, ids, max_bytes: int = 8192, skip_leading_space: bool = False) -> bytes:
        ids = np.ascontiguousarray(ids, np.int32)
        buf = C.create_string_buffer(max_bytes + 256)
        n = lib().kllm_chip_decode(self.h, ids.ctypes.data_as(_fp(C.c_int32)), len(ids),
                                   max_bytes, 1 if skip_leading_space else 0, buf)
        return buf.raw[:n]
