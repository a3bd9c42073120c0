"""Single-instruction tape cases covering every opcode (test data only).

Each case is (name, n_slots, slots, instrs, out_slot, exact) in the form
harness.TapeRun takes.  ``exact`` is False only for MATMUL, whose reference
implementation is BLAS with an unspecified summation order.
"""
from __future__ import annotations

import numpy as np

from kmap_b200.chipgen import (T_ADD, T_ARGMAX, T_CONCAT, T_COPY, T_DIV, T_LUT_COS,
                               T_LUT_EXP, T_LUT_RSQRT, T_LUT_SILU, T_LUT_SIN, T_MATMUL,
                               T_MATMUL_TT, T_MAX, T_MAX_RED, T_MEAN, T_MUL, T_NEG, T_REPEAT,
                               T_RESHAPE, T_SLICE, T_SQUARE, T_SUB, T_SUM, T_TRANSPOSE)


def _arr(rng, *shape, scale=1.0, positive=False):
    a = rng.standard_normal(shape).astype(np.float32) * np.float32(scale)
    return np.abs(a) + np.float32(0.1) if positive else a


def cases(seed=0):
    rng = np.random.default_rng(seed)
    out = []

    def add(name, slots, instr, out_slot, exact=True):
        out.append((name, max(slots) + 1 if slots else out_slot + 1, slots, [instr], out_slot,
                    exact))

    # unary (double-precision evaluation, rounded to float)
    for tag, nm, kw in [(T_LUT_SILU, "silu", {}), (T_LUT_EXP, "exp", {}),
                        (T_LUT_RSQRT, "rsqrt", dict(positive=True)), (T_LUT_COS, "cos", {}),
                        (T_LUT_SIN, "sin", {}), (T_NEG, "neg", {}), (T_SQUARE, "square", {})]:
        for shp in [(1, 7), (3, 5, 11), (2048,)]:
            x = _arr(rng, *shp, scale=3.0, **kw)
            add("%s_%s" % (nm, "x".join(map(str, shp))),
                {0: ("ext", x), 1: ("alloc", [1])}, dict(tag=tag, out_slot=1, in0=0, in1=0), 1)
    # binary with broadcasting
    bshapes = [((4, 6), (4, 6)), ((4, 6), (6,)), ((4, 1), (1, 6)), ((2, 3, 4), (1,)),
               ((5, 1, 7), (3, 1)), ((1, 2048), (2048,)), ((32, 1, 33), (1, 1, 1))]
    for tag, nm in [(T_ADD, "add"), (T_SUB, "sub"), (T_MUL, "mul"), (T_DIV, "div"),
                    (T_MAX, "max")]:
        for sa, sb in bshapes:
            a = _arr(rng, *sa)
            b = _arr(rng, *sb, positive=(tag == T_DIV))
            add("%s_%s_%s" % (nm, "x".join(map(str, sa)), "x".join(map(str, sb))),
                {0: ("ext", a), 1: ("ext", b), 2: ("alloc", [1])},
                dict(tag=tag, out_slot=2, in0=0, in1=1), 2)
    # reductions over every axis, keepdims on and off
    for tag, nm in [(T_SUM, "sum"), (T_MAX_RED, "maxred"), (T_MEAN, "mean"),
                    (T_ARGMAX, "argmax")]:
        for shp in [(3, 4, 5), (1, 2048), (32, 1, 37)]:
            x = _arr(rng, *shp)
            if tag == T_ARGMAX:
                x[..., 0] = x.max() + 1  # a tie-free maximum plus...
                x[..., -1] = x.max()     # ...an equal later one (first wins)
            for ax in range(len(shp)):
                add("%s_%s_ax%d" % (nm, "x".join(map(str, shp)), ax),
                    {0: ("ext", x), 1: ("alloc", [1])},
                    dict(tag=tag, out_slot=1, in0=0, axis=ax, keepdims=ax % 2), 1)
    # data movement
    x = _arr(rng, 2, 3, 4, 5)
    for axes in [(1, 0, 2, 3), (0, 2, 1, 3), (3, 2, 1, 0), (0, 1, 3, 2)]:
        add("transpose_%s" % "".join(map(str, axes)), {0: ("ext", x), 1: ("alloc", [1])},
            dict(tag=T_TRANSPOSE, out_slot=1, in0=0, axes=list(axes)), 1)
    for ax, reps in [(0, 8), (1, 3), (3, 2)]:
        add("repeat_ax%d_r%d" % (ax, reps), {0: ("ext", x), 1: ("alloc", [1])},
            dict(tag=T_REPEAT, out_slot=1, in0=0, axis=ax, repeats=reps), 1)
    for starts, so, steps in [((0, 1, 0, 2), (2, 2, 4, 3), (1, 1, 1, 1)),
                              ((1, 0, 1, 0), (1, 3, 2, 5), (1, 1, 2, 1)),
                              ((0, 0, 0, 1), (0, 0, 0, 2), (1, 1, 1, 2))]:
        add("slice_%s" % "".join(map(str, starts + so)), {0: ("ext", x), 1: ("alloc", [1])},
            dict(tag=T_SLICE, out_slot=1, in0=0, starts=list(starts), steps=list(steps),
                 slice_out_shape=list(so), slice_out_ndim=4), 1)
    add("reshape", {0: ("ext", x), 1: ("alloc", [1])},
        dict(tag=T_RESHAPE, out_slot=1, in0=0, out_shape=[6, 20], out_ndim=2, out_size=120), 1)
    add("copy", {0: ("ext", x), 1: ("alloc", [1])}, dict(tag=T_COPY, out_slot=1, in0=0), 1)
    # concat: KV-cache append (axis 1, including an empty cache), rope rotate
    # (axis 2), flat (axis 0)
    for seq in (0, 1, 7):
        cache = _arr(rng, 4, seq, 64)
        new = _arr(rng, 4, 1, 64)
        add("concat_kv_seq%d" % seq, {0: ("ext", cache), 1: ("ext", new), 2: ("alloc", [4, 2, 64])},
            dict(tag=T_CONCAT, out_slot=2, in0=0, axis=1, concat_n_inputs=2,
                 concat_inputs=[0, 1]), 2)
    a, b = _arr(rng, 32, 1, 32), _arr(rng, 32, 1, 32)
    add("concat_rot", {0: ("ext", a), 1: ("ext", b), 2: ("alloc", [1])},
        dict(tag=T_CONCAT, out_slot=2, in0=0, axis=2, concat_n_inputs=2, concat_inputs=[0, 1]), 2)
    p, q, r = _arr(rng, 3, 5), _arr(rng, 1, 5), _arr(rng, 2, 5)
    add("concat_flat3", {0: ("ext", p), 1: ("ext", q), 2: ("ext", r), 3: ("alloc", [1])},
        dict(tag=T_CONCAT, out_slot=3, in0=0, axis=0, concat_n_inputs=3,
             concat_inputs=[0, 1, 2]), 3)
    # dense matmul (attention shapes) -- tolerance only
    for (bt, m, k, n) in [(32, 1, 64, 9), (32, 1, 9, 64), (1, 3, 17, 5)]:
        A, B = _arr(rng, bt, m, k), _arr(rng, bt, k, n)
        add("matmul_%dx%dx%dx%d" % (bt, m, k, n), {0: ("ext", A), 1: ("ext", B), 2: ("alloc", [1])},
            dict(tag=T_MATMUL, out_slot=2, in0=0, in1=1), 2, exact=False)
    # truth-table matmul, 1 and 3 rows, K across the chunking thresholds
    for (rows, K, N, codes) in [(1, 64, 40, 30), (1, 1000, 33, 500), (3, 1030, 17, 2000),
                                (1, 2048, 64, 4096)]:
        cb = np.sort(_arr(rng, codes, scale=0.02))
        ix = rng.integers(0, codes, (K, N)).astype(np.uint16)
        xx = _arr(rng, rows, K)
        add("tt_%dx%dx%d" % (rows, K, N), {0: ("ext", xx), 1: ("tt", cb, ix), 2: ("alloc", [1])},
            dict(tag=T_MATMUL_TT, out_slot=2, in0=0, in1=1), 2)
    return out
