"""Synthetic kllm chip writer.

Writes a complete chip directory in the on-disk layout that the kllm
compiler produces and the kllm runtime reads (reference
``csrc/kllm_compile.c:1705-1890`` writes it, ``csrc/kllm.c:152-388`` reads
it), for a random-init LLaMA-family model:

* ``circuit/tape.bin``   -- ``[n_instrs, 276, TapeInstr...]`` emitted in the
  exact order of the compiler's fixed decode template
  (``kllm_compile.c:1143-1385`` subgraphs, driven by ``:1427-1690``);
* ``circuit/slots.bin``  -- ``[n, {type, ndim, shape[8]}...]``;
* ``circuit/const_<slot>.bin`` (fp32), ``const_<slot>_codebook.bin`` (fp32
  sorted unique values) and ``const_<slot>_indices.bin`` (uint16 ``[K][N]``)
  -- the truth-table form of ``tt_compress`` (``kllm_compile.c:778-822``);
* ``tables/{embed_table,rope_cos,rope_sin}.bin`` (``build_rope``
  ``kllm_compile.c:829-855``), ``bpe/*`` ROMs (``build_bpe_roms``
  ``kllm_compile.c:634-728``), ``processor.json`` and ``chip.json``.

The weights follow the benchmark recipe: each matrix is drawn N(0, 0.02) in
float32 from a seeded generator, rounded to bf16 (round-to-nearest-even) and
stored back as float32, so each matrix has a few thousand unique values.
Because every value is a bf16 pattern, the sorted-unique codebook and the
uint16 ranks are computed in O(n) from a 65536-bin histogram of the bit
patterns instead of a sort; the result is the same codebook and indices the
compiler's qsort + binary search produce (pinned byte-for-byte against the
reference compiler in ``tests/test_chipgen.py``).

This is input synthesis for tests and benchmarks.  The executor itself only
reads chips; it never calls this module.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import json
import os
from dataclasses import dataclass, field

import numpy as np

# ---------------------------------------------------------------- formats --

MAX_DIMS = 8
MAX_CONCAT_INPUTS = 8

#: Tape opcodes (``_tape_runner.c:29-54``, ``kllm_compile.c:870-878``).
T_LUT_SILU, T_LUT_EXP, T_LUT_RSQRT, T_LUT_COS, T_LUT_SIN = 0, 1, 2, 3, 4
T_ADD, T_SUB, T_MUL, T_DIV, T_MAX = 5, 6, 7, 8, 9
T_NEG, T_SQUARE, T_MATMUL, T_MATMUL_TT = 10, 11, 12, 13
T_SUM, T_MAX_RED, T_MEAN, T_ARGMAX = 14, 15, 16, 17
T_RESHAPE, T_TRANSPOSE, T_CONCAT, T_REPEAT, T_SLICE, T_COPY = 18, 19, 20, 21, 22, 23

OPCODE_NAMES = [
    "SILU", "EXP", "RSQRT", "COS", "SIN", "ADD", "SUB", "MUL", "DIV", "MAX",
    "NEG", "SQUARE", "MATMUL", "MATMUL_TT", "SUM", "MAX_RED", "MEAN", "ARGMAX",
    "RESHAPE", "TRANSPOSE", "CONCAT", "REPEAT", "SLICE", "COPY",
]

#: ``TapeInstr`` (``tape_runner.h:30-49``): 69 int32 = 276 bytes.
INSTR_DTYPE = np.dtype([
    ("tag", "<i4"), ("out_slot", "<i4"), ("in0", "<i4"), ("in1", "<i4"),
    ("in2", "<i4"), ("axis", "<i4"), ("keepdims", "<i4"), ("repeats", "<i4"),
    ("out_shape", "<i4", (8,)), ("out_ndim", "<i4"), ("out_size", "<i4"),
    ("axes", "<i4", (8,)), ("starts", "<i4", (8,)), ("stops", "<i4", (8,)),
    ("steps", "<i4", (8,)), ("slice_out_shape", "<i4", (8,)),
    ("slice_out_ndim", "<i4"), ("concat_inputs", "<i4", (8,)),
    ("concat_n_inputs", "<i4"), ("tt_weight_slot", "<i4"),
])
assert INSTR_DTYPE.itemsize == 276

#: slots.bin record: type, ndim, shape[8] (``kllm_compile.c:1727-1742``).
SLOT_DTYPE = np.dtype([("type", "<i4"), ("ndim", "<i4"), ("shape", "<i4", (8,))])

SLOT_UNUSED, SLOT_CONST, SLOT_INPUT, SLOT_INTER, SLOT_TT = 0, 1, 2, 3, 4


@dataclass
class ModelSpec:
    """A LLaMA-family architecture (the keys of ``weights/config.json``)."""

    num_layers: int = 2
    hidden_size: int = 256
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    intermediate_size: int = 512
    vocab_size: int = 1024
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_seq: int = 256
    seed: int = 0
    weight_std: float = 0.02
    #: "ones" (HF init) or "random" (1 + N(0, 0.1), bf16-rounded): the
    #: random form makes norm-weight handling visible in parity tests.
    norm_weights: str = "ones"
    #: number format of the matrix weights: "bf16" (the checkpoints the
    #: benchmarks stand for), "fp16", or "pool4096" (every matrix draws from
    #: its own 4096 fp32 values, as a quantised codebook would: neither bf16
    #: nor fp16 numbers).
    weight_values: str = "bf16"
    model_name: str = "random-init"

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


#: Benchmark architectures (random-init weights, TT-compressed).
TINYLLAMA_1B = ModelSpec(num_layers=22, hidden_size=2048, num_attention_heads=32,
                         num_key_value_heads=4, intermediate_size=5632,
                         vocab_size=32000, rope_theta=10000.0, max_seq=2048,
                         model_name="random-init TinyLlama-1.1B architecture")
LLAMA2_7B = ModelSpec(num_layers=32, hidden_size=4096, num_attention_heads=32,
                      num_key_value_heads=32, intermediate_size=11008,
                      vocab_size=32000, rope_theta=10000.0, max_seq=4352,
                      model_name="random-init Llama-2-7B architecture")
LLAMA3_8B = ModelSpec(num_layers=32, hidden_size=4096, num_attention_heads=32,
                      num_key_value_heads=8, intermediate_size=14336,
                      vocab_size=128256, rope_theta=500000.0, max_seq=1152,
                      model_name="random-init Llama-3-8B architecture")


# ------------------------------------------------------------ weight draws --

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bf16 value (ties to even), as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    # -0.0 and +0.0 compare equal, so the compiler keeps one zero code; keep
    # the generated data free of -0.0 so that choice never arises.
    out[out == 0] = 0.0
    return out


class WeightSource:
    """Seeded, per-matrix-named weight draws (independent streams)."""

    def __init__(self, spec: ModelSpec):
        self.spec = spec

    def _rng(self, name: str) -> np.random.Generator:
        h = np.frombuffer(name.encode(), dtype=np.uint8).astype(np.uint64)
        key = int((h * np.uint64(1099511628211)).sum() % np.uint64(2**61 - 1))
        return np.random.default_rng([self.spec.seed, key, len(name)])

    def matrix(self, name: str, rows: int, cols: int) -> np.ndarray:
        """HF-layout ``(out, in)`` weight: N(0, std) in the spec's number format."""
        rng = self._rng(name)
        std = np.float32(self.spec.weight_std)
        kind = self.spec.weight_values
        if kind == "pool4096":
            pool = np.sort(rng.standard_normal(4096, dtype=np.float32) * std)
            return pool[rng.integers(0, 4096, (rows, cols))]
        g = rng.standard_normal((rows, cols), dtype=np.float32)
        g *= std
        if kind == "fp16":
            out = g.astype(np.float16).astype(np.float32)
            out[out == 0] = 0.0
            return out
        if kind != "bf16":
            raise ValueError("weight_values must be bf16, fp16 or pool4096")
        return bf16_round(g)

    def norm(self, name: str, n: int) -> np.ndarray:
        if self.spec.norm_weights == "ones":
            return np.ones(n, np.float32)
        g = self._rng(name).standard_normal(n, dtype=np.float32) * np.float32(0.1)
        return bf16_round(np.float32(1.0) + g)


class TorchWeightSource(WeightSource):
    """Seeded draws on a CUDA device, for chips too large to draw on the
    host in reasonable time (the 7B/8B architectures): N(0, std) from
    torch's generator, rounded to bf16 with round-to-nearest-even, -0.0
    replaced by +0.0.  Same distribution and number format as
    WeightSource's bf16 draws, different values (another generator)."""

    def __init__(self, spec: ModelSpec, device):
        super().__init__(spec)
        if spec.weight_values != "bf16":
            raise ValueError("the device generator draws bf16 weights only")
        self.device = device

    def _gen(self, name: str):
        import torch
        h = np.frombuffer(name.encode(), dtype=np.uint8).astype(np.uint64)
        key = int((h * np.uint64(1099511628211)).sum() % np.uint64(2**61 - 1))
        g = torch.Generator(device=self.device)
        g.manual_seed((self.spec.seed * 1000003 + key * 31 + len(name)) % (2**63 - 1))
        return g

    def matrix(self, name: str, rows: int, cols: int):
        import torch
        w = torch.randn((rows, cols), generator=self._gen(name), device=self.device,
                        dtype=torch.float32)
        w *= float(np.float32(self.spec.weight_std))
        w = w.to(torch.bfloat16).to(torch.float32)
        w[w == 0] = 0.0
        return w


def _tt_compress_torch(w):
    """tt_compress of a bf16-exact float32 CUDA tensor [K][N]: the sorted
    distinct values and each weight's rank among them (the compiler's rule,
    kllm_compile.c:778-822), from a histogram of the 16-bit patterns."""
    global _BF16_ORDER
    import torch
    if _BF16_ORDER is None:
        _BF16_ORDER = _bf16_order()
    bits = w.contiguous().view(torch.int32)
    if bool(((bits & 0xFFFF) != 0).any()):
        raise ValueError("device compression needs bf16-exact weights")
    hi = ((bits >> 16) & 0xFFFF).to(torch.int64)
    present = torch.bincount(hi.flatten(), minlength=65536) > 0
    if bool(present[0x8000]):
        raise ValueError("-0.0 in the weights")
    order_all = torch.from_numpy(_BF16_ORDER.astype(np.int64)).to(w.device)
    order = order_all[present[order_all]]
    rank = torch.zeros(65536, dtype=torch.int32, device=w.device)
    rank[order] = torch.arange(order.numel(), dtype=torch.int32, device=w.device)
    idx = rank[hi].to(torch.int16).cpu().numpy().view(np.uint16)
    codebook = (order.cpu().numpy().astype(np.uint32) << np.uint32(16)).view(np.float32)
    return codebook.copy(), idx


# ------------------------------------------------------- TT compression --

def _bf16_order() -> np.ndarray:
    """All 65536 bf16 patterns sorted by value (NaNs last, -0 before +0)."""
    pats = np.arange(65536, dtype=np.uint32)
    vals = (pats << np.uint32(16)).view(np.float32)
    return np.argsort(vals, kind="stable").astype(np.uint32)


_BF16_ORDER = None


def tt_compress(w: np.ndarray):
    """Codebook (sorted unique fp32) + uint16 index matrix of ``w`` [K][N].

    Same result as the compiler's ``tt_compress`` (``kllm_compile.c:778-822``):
    codebook[i] is the i-th smallest distinct value, ``indices[k][n]`` the
    position of ``w[k][n]`` in it.  Returns None when there are more than
    65536 distinct values (the compiler then stores the matrix dense).
    """
    global _BF16_ORDER
    w = np.ascontiguousarray(w, dtype=np.float32)
    u = w.view(np.uint32)
    if not np.any(u & np.uint32(0xFFFF)):
        # bf16-exact data: O(n) histogram of the 16-bit patterns.
        if _BF16_ORDER is None:
            _BF16_ORDER = _bf16_order()
        hi = (u >> np.uint32(16)).astype(np.uint16)
        present = np.bincount(hi.ravel(), minlength=65536) > 0
        # -0.0 equals +0.0 and NaN equals nothing: leave those to np.unique.
        nan_pats = np.isnan((np.arange(65536, dtype=np.uint32) << np.uint32(16)).view(np.float32))
        if not (present[0x8000] or np.any(present & nan_pats)):
            order = _BF16_ORDER[present[_BF16_ORDER]]
            rank = np.zeros(65536, np.uint16)
            rank[order] = np.arange(order.size, dtype=np.uint32).astype(np.uint16)
            codebook = (order.astype(np.uint32) << np.uint32(16)).view(np.float32)
            return codebook.copy(), rank[hi]
    codebook, inv = np.unique(w, return_inverse=True)
    if codebook.size > 65536:
        return None
    return codebook.astype(np.float32), inv.reshape(w.shape).astype(np.uint16)


# ------------------------------------------------------------- tokenizer --

_WORDS = (
    "the of and to in is you that it he was for on are as with his they at be "
    "this have from or one had by word but not what all were we when your can "
    "said there use an each which she do how their if will up other about out "
    "many then them these so some her would make like him into time has look "
    "two more write go see number no way could people my than first water been "
    "call who oil its now find long down day did get come made may part hello "
    "world capital france paris explain quantum computing simple terms beginner "
    "model token chip tape table truth kernel memory bandwidth user assistant"
).split()


@dataclass
class Tokenizer:
    """A SentencePiece-style vocabulary: specials, byte fallback, merges."""

    pieces: list = field(default_factory=list)      # bytes per id
    merges: list = field(default_factory=list)      # (a_bytes, b_bytes)
    special: tuple = (0, 1, 2)
    bos: int = 1
    eos: int = 2


def make_tokenizer(vocab_size: int) -> Tokenizer:
    """Deterministic vocabulary of exactly ``vocab_size`` pieces.

    ids 0-2 ``<unk> <s> </s>``; 3-258 byte fallback ``<0xHH>``; then the
    metaspace, printable ASCII characters and the left-to-right merge chains
    of a small word list (``▁word`` -> ``▁w``+``o`` ...); filler ``tokN``
    pieces pad to ``vocab_size``.  Tiny vocabularies keep the prefix.
    """
    meta = "▁".encode()
    pieces = [b"<unk>", b"<s>", b"</s>"] + [("<0x%02X>" % b).encode() for b in range(256)]
    seen = set(pieces)
    merges = []

    def add(p):
        if p not in seen:
            seen.add(p)
            pieces.append(p)

    add(meta)
    for c in range(33, 127):
        add(bytes([c]))
    for w in _WORDS:
        syms = [meta] + [bytes([c]) for c in w.encode()]
        cur = syms[0]
        for s in syms[1:]:
            merged = cur + s
            if merged not in seen:
                merges.append((cur, s))
                add(merged)
            cur = merged
    n = 0
    while len(pieces) < vocab_size:
        add(("tok%d" % n).encode())
        n += 1
    pieces = pieces[:vocab_size]
    keep = set(pieces)
    merges = [(a, b) for a, b in merges if a in keep and b in keep and a + b in keep]
    return Tokenizer(pieces=pieces, merges=merges)


def _fnv1a(data: bytes) -> int:
    h = 2166136261
    for b in data:
        h ^= b
        h = (h * 16777619) & 0xFFFFFFFF
    return h


def bpe_roms(tok: Tokenizer) -> dict:
    """The BPE ROM arrays for ``tok`` (``build_bpe_roms``, kllm_compile.c:634-728)."""
    V = len(tok.pieces)
    max_piece_len = 64
    offsets = np.zeros((V, 2), np.int32)
    blob = bytearray()
    for i, p in enumerate(tok.pieces):
        offsets[i] = (len(blob), len(p))
        blob += p
    ids = {p: i for i, p in reversed(list(enumerate(tok.pieces)))}
    ma = np.array([ids.get(a, -1) for a, b in tok.merges], np.int32)
    mb = np.array([ids.get(b, -1) for a, b in tok.merges], np.int32)
    mr = np.array([ids.get(a + b, -1) for a, b in tok.merges], np.int32)
    n = V
    table_size = int(n / 0.6) + 1
    ts = 1
    while ts < table_size:
        ts <<= 1
    keys = np.zeros((ts, max_piece_len), np.uint8)
    vals = np.full(ts, -1, np.int32)
    lens = np.zeros(ts, np.int32)
    for tid, p in enumerate(tok.pieces):
        if len(p) > max_piece_len:
            continue
        idx = _fnv1a(p) % ts
        for _ in range(ts):
            if lens[idx] == 0:
                keys[idx, :len(p)] = np.frombuffer(p, np.uint8)
                vals[idx] = tid
                lens[idx] = len(p)
                break
            idx = (idx + 1) % ts
    return dict(hash_keys=keys, hash_vals=vals, hash_lens=lens, table_size=ts,
                max_piece_len=max_piece_len, merge_a=ma, merge_b=mb,
                merge_result=mr, special_ids=np.array(sorted(tok.special), np.int32),
                id_to_bytes=bytes(blob), id_to_offsets=offsets)


def tokenizer_json(tok: Tokenizer) -> tuple[str, str]:
    """``tokenizer.json`` / ``tokenizer_config.json`` texts for ``tok``."""
    dec = [p.decode("utf-8", "surrogateescape") for p in tok.pieces]
    added = [{"id": i, "content": dec[i]} for i in tok.special]
    body = {"added_tokens": added,
            "model": {"vocab": {d: i for i, d in enumerate(dec)},
                      "merges": [a.decode() + " " + b.decode() for a, b in tok.merges]}}
    cfg = {"bos_token": dec[tok.bos], "eos_token": dec[tok.eos]}
    return json.dumps(body), json.dumps(cfg)


# ------------------------------------------------------------- rope table --

def rope_tables(max_seq: int, head_dim: int, theta: float):
    """cos/sin tables ``[max_seq][head_dim]`` as ``build_rope`` makes them
    (``kllm_compile.c:829-855``): float ``powf``/``cosf``/``sinf`` from the C
    math library, the half-dimension block duplicated."""
    libm = ctypes.CDLL(ctypes.util.find_library("m"))
    libm.powf.restype = libm.cosf.restype = libm.sinf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    libm.cosf.argtypes = libm.sinf.argtypes = [ctypes.c_float]
    half = head_dim // 2
    inv = np.empty(half, np.float32)
    for i in range(half):
        e = np.float32(np.float32(i * 2) / np.float32(head_dim))
        inv[i] = np.float32(1.0) / np.float32(libm.powf(float(np.float32(theta)), float(e)))
    ang = (np.arange(max_seq, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cosf, sinf = libm.cosf, libm.sinf
    flat = ang.ravel().tolist()
    c = np.fromiter((cosf(a) for a in flat), np.float32, len(flat)).reshape(ang.shape)
    s = np.fromiter((sinf(a) for a in flat), np.float32, len(flat)).reshape(ang.shape)
    return np.concatenate([c, c], 1), np.concatenate([s, s], 1)


# ----------------------------------------------------------- tape builder --

class TapeBuilder:
    """Slot allocator + instruction emitter with the compiler's conventions
    (``kllm_compile.c:884-1125``): instructions start zeroed, so unary ops
    carry ``in1 = 0``; slices record ``starts``/``steps``/``slice_out_shape``
    and leave ``stops`` zero; matmuls record only their operands."""

    def __init__(self):
        self.slot_type, self.slot_shape = [], []
        self.instrs = []

    def slot(self, typ, shape):
        self.slot_type.append(typ)
        self.slot_shape.append(list(shape))
        return len(self.slot_type) - 1

    def emit(self, **f):
        self.instrs.append(f)

    def _shaped(self, tag, out, shape, **f):
        f.update(out_shape=list(shape), out_ndim=len(shape),
                 out_size=int(np.prod(shape)))
        self.emit(tag=tag, out_slot=out, **f)

    def binop(self, tag, a, b, shape):
        out = self.slot(SLOT_INTER, shape)
        self._shaped(tag, out, shape, in0=a, in1=b)
        return out

    def unary(self, tag, a, shape):
        out = self.slot(SLOT_INTER, shape)
        self._shaped(tag, out, shape, in0=a)
        return out

    def matmul(self, tag, a, b, shape):
        out = self.slot(SLOT_INTER, shape)
        self.emit(tag=tag, out_slot=out, in0=a, in1=b)
        return out

    def reshape(self, a, shape):
        out = self.slot(SLOT_INTER, shape)
        self._shaped(T_RESHAPE, out, shape, in0=a)
        return out

    def transpose(self, a, axes, shape):
        out = self.slot(SLOT_INTER, shape)
        self.emit(tag=T_TRANSPOSE, out_slot=out, in0=a, axes=list(axes))
        return out

    def concat(self, ins, axis, shape):
        out = self.slot(SLOT_INTER, shape)
        self.emit(tag=T_CONCAT, out_slot=out, in0=ins[0], axis=axis,
                  concat_n_inputs=len(ins), concat_inputs=list(ins))
        return out

    def repeat(self, a, reps, axis, shape):
        out = self.slot(SLOT_INTER, shape)
        self.emit(tag=T_REPEAT, out_slot=out, in0=a, repeats=reps, axis=axis)
        return out

    def slice(self, a, starts, stops, shape):
        out = self.slot(SLOT_INTER, shape)
        n = len(starts)
        self.emit(tag=T_SLICE, out_slot=out, in0=a, starts=list(starts),
                  steps=[1] * n, slice_out_shape=[e - s for s, e in zip(starts, stops)],
                  slice_out_ndim=n)
        return out

    def copy(self, a, shape):
        out = self.slot(SLOT_INTER, shape)
        self._shaped(T_COPY, out, shape, in0=a)
        return out

    def reduce(self, tag, a, axis, shape):
        out = self.slot(SLOT_INTER, shape)
        self.emit(tag=tag, out_slot=out, in0=a, axis=axis, keepdims=1)
        return out

    def tape_array(self) -> np.ndarray:
        arr = np.zeros(len(self.instrs), INSTR_DTYPE)
        for i, f in enumerate(self.instrs):
            for k, v in f.items():
                if isinstance(v, list):
                    arr[i][k][:len(v)] = v
                else:
                    arr[i][k] = v
        return arr

    def slots_array(self) -> np.ndarray:
        arr = np.zeros(len(self.slot_type), SLOT_DTYPE)
        for i, (t, s) in enumerate(zip(self.slot_type, self.slot_shape)):
            arr[i]["type"] = t
            arr[i]["ndim"] = len(s)
            arr[i]["shape"][:len(s)] = s
        return arr


# ------------------------------------------------------------ chip writer --

def _write(path, data):
    with open(path, "wb") as f:
        f.write(data if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data).tobytes())


def generate_chip(out_dir: str, spec: ModelSpec, write_weights: bool = False,
                  log=None, device=None) -> dict:
    """Write a chip for ``spec`` into ``out_dir``; returns a small summary.

    With ``write_weights`` the HF-layout ``weights/*.npy`` and
    ``tokenizer/*.json`` inputs of the kllm compiler are written too, so the
    reference compiler can build the same chip from the same numbers.
    """
    c = spec
    H, nh, nkv, hd, F, V, L = (c.hidden_size, c.num_attention_heads, c.num_key_value_heads,
                               c.head_dim, c.intermediate_size, c.vocab_size, c.num_layers)
    groups = nh // nkv
    q_dim, kv_dim = nh * hd, nkv * hd
    circuit = os.path.join(out_dir, "circuit")
    for d in ("circuit", "bpe", "tables") + (("weights", "tokenizer") if write_weights else ()):
        os.makedirs(os.path.join(out_dir, d), exist_ok=True)
    src = TorchWeightSource(spec, device) if device is not None else WeightSource(spec)
    if device is not None and write_weights:
        raise ValueError("write_weights needs the host generator")
    wdir = os.path.join(out_dir, "weights")

    def cat_t(mats):   # [m.T for m in mats] side by side, host or device
        if device is None:
            return np.concatenate([m.T for m in mats], 1)
        import torch
        return torch.cat([m.t() for m in mats], 1).contiguous()

    def host(m):
        return m if device is None else m.cpu().numpy()
    if write_weights:
        with open(os.path.join(wdir, "config.json"), "w") as f:
            json.dump(dict(model_name=c.model_name, num_layers=L, hidden_size=H,
                           num_attention_heads=nh, num_key_value_heads=nkv,
                           intermediate_size=F, vocab_size=V, rms_norm_eps=c.rms_norm_eps,
                           rope_theta=c.rope_theta), f)

    tb = TapeBuilder()
    consts = {}

    def const(arr, shape):
        s = tb.slot(SLOT_CONST, shape)
        consts[s] = np.asarray(arr, np.float32)
        return s

    n_idx_bytes = 0

    def tt(wt: np.ndarray):
        nonlocal n_idx_bytes
        K, N = wt.shape
        res = tt_compress(wt) if device is None else _tt_compress_torch(wt)
        if res is None:  # dense fallback, kllm_compile.c:1516-1524
            return const(wt, [K, N]), False
        cb, idx = res
        s = tb.slot(SLOT_TT, [K, N])
        _write(os.path.join(circuit, "const_%d_codebook.bin" % s), cb)
        _write(os.path.join(circuit, "const_%d_indices.bin" % s), idx)
        n_idx_bytes += idx.nbytes
        return s, True

    def save_npy(rel, arr):
        if write_weights:
            p = os.path.join(wdir, rel)
            os.makedirs(os.path.dirname(p), exist_ok=True)
            np.save(p, arr)

    def rms_norm(hidden, w_slot):
        sq = tb.binop(T_MUL, hidden, hidden, [1, H])
        ms = tb.reduce(T_MEAN, sq, 1, [1, 1])
        eps = const(np.array([np.float32(c.rms_norm_eps)]), [1])
        add = tb.binop(T_ADD, ms, eps, [1, 1])
        rsq = tb.unary(T_LUT_RSQRT, add, [1, 1])
        nrm = tb.binop(T_MUL, hidden, rsq, [1, H])
        return tb.binop(T_MUL, nrm, w_slot, [1, H])

    def rope(x, cos_b, sin_b, heads):
        half = hd // 2
        x1 = tb.slice(x, [0, 0, 0], [heads, 1, half], [heads, 1, half])
        x2 = tb.slice(x, [0, 0, half], [heads, 1, hd], [heads, 1, half])
        neg = tb.unary(T_NEG, x2, [heads, 1, half])
        rot = tb.concat([neg, x1], 2, [heads, 1, hd])
        xc = tb.binop(T_MUL, x, cos_b, [heads, 1, hd])
        rs = tb.binop(T_MUL, rot, sin_b, [heads, 1, hd])
        return tb.binop(T_ADD, xc, rs, [heads, 1, hd])

    tok_embed = tb.slot(SLOT_INPUT, [1, H])
    rope_cos_in = tb.slot(SLOT_INPUT, [1, hd])
    rope_sin_in = tb.slot(SLOT_INPUT, [1, hd])
    kv_in = []
    for li in range(L):
        kv_in.append(tb.slot(SLOT_INPUT, [nkv, 1, hd]))
        kv_in.append(tb.slot(SLOT_INPUT, [nkv, 1, hd]))
    one = np.float32(1.0)
    scale = const(np.array([one / np.sqrt(np.float32(hd))], np.float32), [1])
    cos_b = tb.copy(rope_cos_in, [1, 1, hd])
    sin_b = tb.copy(rope_sin_in, [1, 1, hd])
    kv_out = [0] * (2 * L)
    hidden = tok_embed
    for li in range(L):
        if log:
            log("layer %d/%d" % (li + 1, L))
        ln = "layer_%d/" % li
        wq = src.matrix(ln + "q_proj", q_dim, H)
        wk = src.matrix(ln + "k_proj", kv_dim, H)
        wv = src.matrix(ln + "v_proj", kv_dim, H)
        for n_, w_ in (("q_proj", wq), ("k_proj", wk), ("v_proj", wv)):
            save_npy(ln + n_ + ".npy", w_)
        qkv_slot, _ = tt(cat_t([wq, wk, wv]))
        del wq, wk, wv
        wo = src.matrix(ln + "o_proj", H, q_dim)
        save_npy(ln + "o_proj.npy", wo)
        o_slot, _ = tt(cat_t([wo]))
        del wo
        wg = src.matrix(ln + "gate_proj", F, H)
        wu = src.matrix(ln + "up_proj", F, H)
        save_npy(ln + "gate_proj.npy", wg)
        save_npy(ln + "up_proj.npy", wu)
        gu_slot, _ = tt(cat_t([wg, wu]))
        del wg, wu
        wd = src.matrix(ln + "down_proj", H, F)
        save_npy(ln + "down_proj.npy", wd)
        d_slot, _ = tt(cat_t([wd]))
        del wd
        n1 = src.norm(ln + "input_layernorm", H)
        n2 = src.norm(ln + "post_attention_layernorm", H)
        save_npy(ln + "input_layernorm_weight.npy", n1)
        save_npy(ln + "post_attention_layernorm_weight.npy", n2)
        ln1 = const(n1, [H])
        ln2 = const(n2, [H])

        residual = hidden
        h = rms_norm(hidden, ln1)
        # attention (kllm_compile.c:1216-1343)
        qkv = tb.matmul(T_MATMUL_TT, h, qkv_slot, [1, q_dim + 2 * kv_dim])
        q = tb.slice(qkv, [0, 0], [1, q_dim], [1, q_dim])
        k = tb.slice(qkv, [0, q_dim], [1, q_dim + kv_dim], [1, kv_dim])
        v = tb.slice(qkv, [0, q_dim + kv_dim], [1, q_dim + 2 * kv_dim], [1, kv_dim])
        q = tb.reshape(q, [1, nh, hd])
        q = tb.transpose(q, [1, 0, 2], [nh, 1, hd])
        k = tb.reshape(k, [1, nkv, hd])
        k = tb.transpose(k, [1, 0, 2], [nkv, 1, hd])
        v = tb.reshape(v, [1, nkv, hd])
        v = tb.transpose(v, [1, 0, 2], [nkv, 1, hd])
        q = rope(q, cos_b, sin_b, nh)
        k = rope(k, cos_b, sin_b, nkv)
        k_full = tb.concat([kv_in[2 * li], k], 1, [nkv, 2, hd])
        v_full = tb.concat([kv_in[2 * li + 1], v], 1, [nkv, 2, hd])
        kv_out[2 * li], kv_out[2 * li + 1] = k_full, v_full
        if groups > 1:
            k_exp = tb.repeat(k_full, groups, 0, [nh, 2, hd])
            v_exp = tb.repeat(v_full, groups, 0, [nh, 2, hd])
        else:
            k_exp, v_exp = k_full, v_full
        kt = tb.transpose(k_exp, [0, 2, 1], [nh, hd, 2])
        sc = tb.matmul(T_MATMUL, q, kt, [nh, 1, 2])
        sc = tb.binop(T_MUL, sc, scale, [nh, 1, 2])
        mx = tb.reduce(T_MAX_RED, sc, 2, [nh, 1, 1])
        sub = tb.binop(T_SUB, sc, mx, [nh, 1, 2])
        ex = tb.unary(T_LUT_EXP, sub, [nh, 1, 2])
        sm = tb.reduce(T_SUM, ex, 2, [nh, 1, 1])
        aw = tb.binop(T_DIV, ex, sm, [nh, 1, 2])
        ctx = tb.matmul(T_MATMUL, aw, v_exp, [nh, 1, hd])
        ctx = tb.transpose(ctx, [1, 0, 2], [1, nh, hd])
        ctx = tb.reshape(ctx, [1, q_dim])
        attn = tb.matmul(T_MATMUL_TT, ctx, o_slot, [1, nh * hd])
        hidden = tb.binop(T_ADD, residual, attn, [1, H])
        residual = hidden
        h = rms_norm(hidden, ln2)
        # MLP (kllm_compile.c:1350-1385)
        gu = tb.matmul(T_MATMUL_TT, h, gu_slot, [1, 2 * F])
        gate = tb.slice(gu, [0, 0], [1, F], [1, F])
        up = tb.slice(gu, [0, F], [1, 2 * F], [1, F])
        ga = tb.unary(T_LUT_SILU, gate, [1, F])
        gated = tb.binop(T_MUL, ga, up, [1, F])
        mlp = tb.matmul(T_MATMUL_TT, gated, d_slot, [1, H])
        hidden = tb.binop(T_ADD, residual, mlp, [1, H])

    fn = src.norm("final_norm", H)
    save_npy("final_norm_weight.npy", fn)
    fln = const(fn, [H])
    hidden = rms_norm(hidden, fln)
    lm = src.matrix("lm_head", V, H)
    save_npy("lm_head.npy", lm)
    lm_slot, _ = tt(cat_t([lm]))
    del lm
    logits = tb.matmul(T_MATMUL_TT, hidden, lm_slot, [1, V])

    _write(os.path.join(circuit, "tape.bin"),
           np.array([len(tb.instrs), INSTR_DTYPE.itemsize], np.int32).tobytes()
           + tb.tape_array().tobytes())
    _write(os.path.join(circuit, "slots.bin"),
           np.array([len(tb.slot_type)], np.int32).tobytes() + tb.slots_array().tobytes())
    for s, arr in consts.items():
        _write(os.path.join(circuit, "const_%d.bin" % s), arr)

    tok = make_tokenizer(V)
    roms = bpe_roms(tok)
    bpe = os.path.join(out_dir, "bpe")
    _write(os.path.join(bpe, "vocab_hash_keys.bin"), roms["hash_keys"])
    with open(os.path.join(bpe, "vocab_hash_keys.json"), "w") as f:
        f.write('{"shape": [%d, %d], "dtype": "uint8"}\n' % (roms["table_size"], roms["max_piece_len"]))
    for name in ("hash_vals", "hash_lens"):
        _write(os.path.join(bpe, "vocab_%s.bin" % name), roms[name])
    for name in ("merge_a", "merge_b", "merge_result", "special_ids", "id_to_bytes", "id_to_offsets"):
        _write(os.path.join(bpe, name + ".bin"), roms[name])
    if write_weights:
        tj, tc = tokenizer_json(tok)
        with open(os.path.join(out_dir, "tokenizer", "tokenizer.json"), "w") as f:
            f.write(tj)
        with open(os.path.join(out_dir, "tokenizer", "tokenizer_config.json"), "w") as f:
            f.write(tc)

    embed = host(src.matrix("embed_tokens", V, H))
    save_npy("embed_tokens.npy", embed)
    tables = os.path.join(out_dir, "tables")
    _write(os.path.join(tables, "embed_table.bin"), embed)
    del embed
    rc, rs = rope_tables(c.max_seq, hd, c.rope_theta)
    _write(os.path.join(tables, "rope_cos.bin"), rc)
    _write(os.path.join(tables, "rope_sin.bin"), rs)

    pj = ["{", '  "vocab_size": %d,' % V, '  "hidden_dim": %d,' % H,
          '  "num_layers": %d,' % L, '  "num_kv_heads": %d,' % nkv,
          '  "head_dim": %d,' % hd, '  "max_seq_len": %d,' % c.max_seq,
          '  "eos_token_id": %d,' % tok.eos, '  "input_map": {',
          '    "token_embed": %d,' % tok_embed, '    "rope_cos": %d,' % rope_cos_in,
          '    "rope_sin": %d,' % rope_sin_in]
    for li in range(L):
        pj.append('    "L%d/cache_k": %d,' % (li, kv_in[2 * li]))
        pj.append('    "L%d/cache_v": %d%s' % (li, kv_in[2 * li + 1], "," if li < L - 1 else ""))
    pj += ["  },", '  "output_map": {', '    "logits": %d,' % logits]
    for li in range(L):
        pj.append('    "L%d/new_k": %d,' % (li, kv_out[2 * li]))
        pj.append('    "L%d/new_v": %d%s' % (li, kv_out[2 * li + 1], "," if li < L - 1 else ""))
    pj += ["  }", "}"]
    with open(os.path.join(out_dir, "processor.json"), "w") as f:
        f.write("\n".join(pj) + "\n")
    with open(os.path.join(out_dir, "chip.json"), "w") as f:
        f.write("{\n")
        f.write('  "kllm_version": "0.3.0",\n')
        f.write('  "model_name": "%s",\n' % c.model_name)
        f.write('  "eos_token_id": %d,\n' % tok.eos)
        f.write('  "max_seq_len": %d,\n' % c.max_seq)
        f.write('  "vocab_size": %d,\n' % V)
        f.write('  "hidden_dim": %d,\n' % H)
        f.write('  "num_layers": %d,\n' % L)
        f.write('  "head_dim": %d\n' % hd)
        f.write("}\n")
    return dict(n_instrs=len(tb.instrs), n_slots=len(tb.slot_type),
                index_bytes=n_idx_bytes, logits_slot=logits)


def ensure_chip(cache_root: str, spec: ModelSpec, log=None, device=None) -> str:
    """Generate ``spec``'s chip under ``cache_root`` once; return its path.
    With ``device`` (a CUDA device) the weights are drawn there
    (TorchWeightSource): a different chip, cached under its own name."""
    key = "chip_L%d_H%d_h%d_kv%d_F%d_V%d_S%d_seed%d_%s" % (
        spec.num_layers, spec.hidden_size, spec.num_attention_heads,
        spec.num_key_value_heads, spec.intermediate_size, spec.vocab_size,
        spec.max_seq, spec.seed, spec.norm_weights)
    if spec.weight_values != "bf16":
        key += "_" + spec.weight_values
    if device is not None:
        key += "_devrng"
    path = os.path.join(cache_root, key)
    done = os.path.join(path, ".complete")
    if not os.path.exists(done):
        generate_chip(path, spec, log=log, device=device)
        open(done, "w").close()
    return path


# ------------------------------------------------------ TT-GEMV inputs --

def gaussian_rank_indices(rng, K, N, n_codes, sigma=0.02, codebook=None):
    """uint16 indices whose code frequencies follow the Gaussian rank that
    bf16-rounding N(0, sigma) produces: draw w ~ N(0, sigma) and take the
    nearest entry of the sorted codebook."""
    if n_codes == 1:
        return np.zeros((K, N), np.uint16)
    w = rng.standard_normal((K, N), dtype=np.float32) * np.float32(sigma)
    pos = np.clip(np.searchsorted(codebook, w), 1, n_codes - 1)
    left, right = codebook[pos - 1], codebook[pos]
    pick = np.where(np.abs(w - left) <= np.abs(right - w), pos - 1, pos)
    return pick.astype(np.uint16)


def tt_case(seed, K, N, n_codes, rows=1):
    """A TT-GEMV microbenchmark input: sorted seeded N(0, 0.02) codebook of
    n_codes entries, Gaussian-rank uint16 indices [K][N], x ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    cb = np.sort(rng.standard_normal(n_codes).astype(np.float32) * np.float32(0.02))
    idx = gaussian_rank_indices(rng, K, N, n_codes, codebook=cb)
    x = rng.standard_normal((rows, K), dtype=np.float32)
    return x, cb, idx
