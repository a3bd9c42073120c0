/*
 * tape_oracle.c -- CPU restatement of the kllm tape semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load this library, and only as the checker;
 * the product library never links it.
 *
 * It restates, in this repository's own code, what the reference runtime
 * computes (file:line below are in the reference's csrc/):
 *   orc_tt_gemv        TT-GEMV order: T = min(8, ceil(K/128)) chunks, the
 *                      first K%T one row longer, rounded products summed row
 *                      by row from 0.0f per chunk, chunk sums added in order
 *                      (_tape_runner.c:495-663)
 *   orc_tape_run       all 24 opcodes with the reference's dynamic-shape
 *                      rules (_tape_runner.c:665-995); MATMUL is a plain
 *                      k-ascending dot product (the reference calls BLAS,
 *                      whose order is unspecified)
 *   orc_processor_infer the prefill/decode loop of processor_infer
 *                      (_tape_runner.c:1602-1763), capturing logits rows
 *   slot API           _tape_runner.c:306-435
 * Its results are pinned against the compiled reference (oracle/_ref) in
 * tests/test_oracle.py.  Built with -ffp-contract=off: no FMA contraction.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MAXD 8

typedef struct {
    float *data;
    int shape[MAXD];
    int ndim;
    int size;
    int owns_data;
    float *codebook;
    uint16_t *w_indices;
    int n_codes;
    int tt_K;
    int tt_N;
} OSlot;

typedef struct {
    int tag, out_slot, in0, in1, in2, axis, keepdims, repeats;
    int out_shape[MAXD];
    int out_ndim, out_size;
    int axes[MAXD], starts[MAXD], stops[MAXD], steps[MAXD];
    int slice_out_shape[MAXD];
    int slice_out_ndim;
    int concat_inputs[MAXD];
    int concat_n_inputs;
    int tt_weight_slot;
} OInstr;

typedef struct {
    OSlot *slots;
    int n_slots;
    OInstr *tape;
    int n_instrs;
} OCtx;

_Static_assert(sizeof(OInstr) == 276, "tape record is 276 bytes");

/* ------------------------------------------------------------ TT-GEMV -- */

static int tt_chunks(int K)
{
    int t = 8;
    if (K < 128 * t) t = (K + 127) / 128;
    return t < 1 ? 1 : t;
}

void orc_tt_gemv(const float *x, int rows, const float *cb, int n_codes,
                 const uint16_t *idx, int K, int N, float *y)
{
    (void)n_codes;
    int T = tt_chunks(K);
    float *acc = malloc((size_t)N * sizeof(float));
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * K;
        float *yr = y + (size_t)r * N;
        int k0 = 0;
        for (int t = 0; t < T; t++) {
            int len = K / T + (t < K % T ? 1 : 0);
            for (int n = 0; n < N; n++) acc[n] = 0.0f;
            for (int k = k0; k < k0 + len; k++) {
                float xk = xr[k];
                const uint16_t *row = idx + (size_t)k * N;
                for (int n = 0; n < N; n++) {
                    float p = xk * cb[row[n]];
                    acc[n] = acc[n] + p;
                }
            }
            if (t == 0)
                memcpy(yr, acc, (size_t)N * sizeof(float));
            else
                for (int n = 0; n < N; n++) yr[n] = yr[n] + acc[n];
            k0 += len;
        }
    }
    free(acc);
}

/* ------------------------------------------------------------- slots --- */

OCtx *orc_ctx_create(int n_slots, int n_instrs)
{
    OCtx *c = calloc(1, sizeof(OCtx));
    c->n_slots = n_slots;
    c->n_instrs = n_instrs;
    c->slots = calloc(n_slots > 0 ? n_slots : 1, sizeof(OSlot));
    c->tape = calloc(n_instrs > 0 ? n_instrs : 1, sizeof(OInstr));
    return c;
}

void orc_ctx_destroy(OCtx *c)
{
    if (!c) return;
    for (int i = 0; i < c->n_slots; i++)
        if (c->slots[i].owns_data) free(c->slots[i].data);
    free(c->slots);
    free(c->tape);
    free(c);
}

static void set_dims(OSlot *s, const int *shape, int nd)
{
    s->ndim = nd;
    s->size = 1;
    for (int d = 0; d < nd; d++) {
        s->shape[d] = shape[d];
        s->size *= shape[d];
    }
}

void orc_slot_alloc(OCtx *c, int i, const int *shape, int nd)
{
    OSlot *s = &c->slots[i];
    if (s->owns_data) free(s->data);
    set_dims(s, shape, nd);
    s->data = calloc(s->size > 0 ? s->size : 1, sizeof(float));
    s->owns_data = 1;
}

void orc_slot_set_external(OCtx *c, int i, float *data, const int *shape, int nd)
{
    OSlot *s = &c->slots[i];
    if (s->owns_data) free(s->data);
    s->data = data;
    s->owns_data = 0;
    set_dims(s, shape, nd);
}

void orc_slot_set_truth_table(OCtx *c, int i, float *cb, int n_codes, uint16_t *idx,
                              int K, int N)
{
    OSlot *s = &c->slots[i];
    s->codebook = cb;
    s->w_indices = idx;
    s->n_codes = n_codes;
    s->tt_K = K;
    s->tt_N = N;
    int sh[2] = {K, N};
    set_dims(s, sh, 2);
}

void orc_slot_write(OCtx *c, int i, const float *data, int n)
{
    OSlot *s = &c->slots[i];
    if (n <= 0) return;
    if (n > s->size) {
        if (s->owns_data) free(s->data);
        s->data = malloc((size_t)n * sizeof(float));
        s->owns_data = 1;
        s->size = n;
    }
    memcpy(s->data, data, (size_t)n * sizeof(float));
}

void orc_slot_set_shape(OCtx *c, int i, const int *shape, int nd)
{
    set_dims(&c->slots[i], shape, nd);
}

const float *orc_slot_read(OCtx *c, int i, int *size)
{
    *size = c->slots[i].size;
    return c->slots[i].data;
}

int orc_slot_read_shape(OCtx *c, int i, int *shape)
{
    for (int d = 0; d < c->slots[i].ndim; d++) shape[d] = c->slots[i].shape[d];
    return c->slots[i].ndim;
}

void *orc_get_instr(OCtx *c, int i) { return &c->tape[i]; }

/* output buffer with room for `need` floats; the size field grows only */
static void grow(OSlot *s, int need)
{
    if (need < 1) need = 1;
    if (need > s->size) {
        if (s->owns_data) free(s->data);
        s->data = malloc((size_t)need * sizeof(float));
        s->owns_data = 1;
        s->size = need;
    }
}

/* --------------------------------------------------------------- ops --- */

/* Source offset of output element `o` for an input of shape `ish` broadcast
 * (right-aligned) into an output of shape `osh`. */
static long bcast_src(long o, const int *osh, int ond, const int *ish, int ind)
{
    long src = 0, stride = 1;
    for (int d = ond - 1, j = ind - 1; d >= 0; d--, j--) {
        long q = o % osh[d];
        o /= osh[d];
        if (j >= 0) {
            if (ish[j] != 1) src += q * stride;
            stride *= ish[j];
        }
    }
    return src;
}

static float apply2(int tag, float a, float b)
{
    switch (tag) {
    case 5: return a + b;
    case 6: return a - b;
    case 7: return a * b;
    case 8: return a / b;
    default: return a > b ? a : b;
    }
}

static void op_binary(OCtx *c, const OInstr *op)
{
    OSlot *a = &c->slots[op->in0], *b = &c->slots[op->in1], *y = &c->slots[op->out_slot];
    int nd = a->ndim > b->ndim ? a->ndim : b->ndim, osh[MAXD];
    long n = 1;
    for (int k = 0; k < nd; k++) {
        int da = k < a->ndim ? a->shape[a->ndim - 1 - k] : 1;
        int db = k < b->ndim ? b->shape[b->ndim - 1 - k] : 1;
        osh[nd - 1 - k] = da > db ? da : db;
        n *= osh[nd - 1 - k];
    }
    int ash[MAXD], bsh[MAXD], and_ = a->ndim, bnd = b->ndim;
    memcpy(ash, a->shape, sizeof ash);
    memcpy(bsh, b->shape, sizeof bsh);
    const float *ad = a->data, *bd = b->data;
    grow(y, (int)n);
    for (long o = 0; o < n; o++)
        y->data[o] = apply2(op->tag, ad[bcast_src(o, osh, nd, ash, and_)],
                            bd[bcast_src(o, osh, nd, bsh, bnd)]);
    set_dims(y, osh, nd);
}

static void op_unary(OCtx *c, const OInstr *op)
{
    OSlot *x = &c->slots[op->in0], *y = &c->slots[op->out_slot];
    int n = x->size;
    grow(y, n);
    for (int i = 0; i < n; i++) {
        float v = x->data[i];
        double d = v;
        float r;
        switch (op->tag) {
        case 0: r = (float)(d / (1.0 + exp(-d))); break;
        case 1: r = (float)exp(d); break;
        case 2: r = (float)(1.0 / sqrt(d)); break;
        case 3: r = (float)cos(d); break;
        case 4: r = (float)sin(d); break;
        case 10: { uint32_t u; memcpy(&u, &v, 4); u ^= 0x80000000u; memcpy(&r, &u, 4); } break;
        default: r = v * v; break;
        }
        y->data[i] = r;
    }
    set_dims(y, x->shape, x->ndim);
}

static void op_reduce(OCtx *c, const OInstr *op)
{
    OSlot *x = &c->slots[op->in0], *y = &c->slots[op->out_slot];
    int ax = op->axis, an = x->shape[ax];
    long outer = 1, inner = 1;
    for (int d = 0; d < ax; d++) outer *= x->shape[d];
    for (int d = ax + 1; d < x->ndim; d++) inner *= x->shape[d];
    int cnt = x->size / an, osh[MAXD], od = 0;
    for (int d = 0; d < x->ndim; d++) {
        if (d != ax) osh[od++] = x->shape[d];
        else if (op->keepdims && op->tag != 17) osh[od++] = 1;
    }
    const float *xd = x->data;
    grow(y, cnt);
    for (long o = 0; o < outer; o++)
        for (long i = 0; i < inner; i++) {
            const float *p = xd + o * an * inner + i;
            float r;
            if (op->tag == 14 || op->tag == 16) {
                float s = 0.0f;
                for (int a = 0; a < an; a++) s = s + p[a * inner];
                r = op->tag == 16 ? s * (1.0f / (float)an) : s;
            } else {
                float m = p[0];
                int mi = 0;
                for (int a = 1; a < an; a++)
                    if (p[a * inner] > m) { m = p[a * inner]; mi = a; }
                r = op->tag == 15 ? m : (float)mi;
            }
            y->data[o * inner + i] = r;
        }
    set_dims(y, osh, od);
}

/* y[o] = x[src(o)] with per-dimension (stride, divisor, offset) rules. */
static void gather(const float *x, float *y, const int *osh, int nd, const long *istr,
                   const int *div, const int *off)
{
    long n = 1;
    for (int d = 0; d < nd; d++) n *= osh[d];
    for (long o = 0; o < n; o++) {
        long rem = o, src = 0;
        for (int d = nd - 1; d >= 0; d--) {
            long q = rem % osh[d];
            rem /= osh[d];
            src += (q / div[d] + off[d]) * istr[d];
        }
        y[o] = x[src];
    }
}

static void strides_of(const int *sh, int nd, long *st)
{
    long acc = 1;
    for (int d = nd - 1; d >= 0; d--) { st[d] = acc; acc *= sh[d]; }
}

static void op_move(OCtx *c, const OInstr *op)
{
    OSlot *x = &c->slots[op->in0], *y = &c->slots[op->out_slot];
    int nd = x->ndim, osh[MAXD], div[MAXD], off[MAXD], sh[MAXD];
    long st[MAXD], istr[MAXD];
    memcpy(sh, x->shape, sizeof sh);
    strides_of(sh, nd, st);
    int outn = x->size;
    for (int d = 0; d < nd; d++) { div[d] = 1; off[d] = 0; istr[d] = st[d]; osh[d] = sh[d]; }
    if (op->tag == 19) {                       /* TRANSPOSE */
        for (int d = 0; d < nd; d++) { osh[d] = sh[op->axes[d]]; istr[d] = st[op->axes[d]]; }
    } else if (op->tag == 21) {                /* REPEAT */
        osh[op->axis] *= op->repeats;
        div[op->axis] = op->repeats;
        outn = x->size * op->repeats;
    } else {                                   /* SLICE: x[start + q*step] */
        outn = 1;
        for (int d = 0; d < nd; d++) {
            int start = op->starts[d], step = op->steps[d], stop = sh[d];
            if (d < op->slice_out_ndim && op->slice_out_shape[d] > 0 &&
                op->slice_out_shape[d] <= sh[d])
                stop = start + op->slice_out_shape[d] * step;
            int dim = (stop - start + step - 1) / step;
            osh[d] = dim < 0 ? 0 : dim;
            outn *= osh[d];
        }
        const float *xd = x->data;
        grow(y, outn);
        for (long o = 0; o < outn; o++) {
            long rem = o, src = 0;
            for (int d = nd - 1; d >= 0; d--) {
                long q = rem % osh[d];
                rem /= osh[d];
                src += (op->starts[d] + q * op->steps[d]) * st[d];
            }
            y->data[o] = xd[src];
        }
        set_dims(y, osh, nd);
        return;
    }
    const float *xd = x->data;
    grow(y, outn);
    gather(xd, y->data, osh, nd, istr, div, off);
    set_dims(y, osh, nd);
}

static void op_concat(OCtx *c, const OInstr *op)
{
    OSlot *y = &c->slots[op->out_slot];
    OSlot *first = &c->slots[op->concat_inputs[0]];
    int nc = op->concat_n_inputs, ax = op->axis;
    int need = 0;
    for (int i = 0; i < nc; i++) need += c->slots[op->concat_inputs[i]].size;
    if (need > y->size) {
        if (y->owns_data) free(y->data);
        y->data = malloc((size_t)(need > 0 ? need : 1) * sizeof(float));
        y->owns_data = 1;
        y->size = need;
    }
    int nd = first->ndim, sh[MAXD], tot = 0;
    memcpy(sh, first->shape, sizeof sh);
    for (int i = 0; i < nc; i++) tot += c->slots[op->concat_inputs[i]].shape[ax];
    float *w = y->data;
    if (ax == 0 || nd == 1) {
        for (int i = 0; i < nc; i++) {
            OSlot *s = &c->slots[op->concat_inputs[i]];
            memcpy(w, s->data, (size_t)s->size * sizeof(float));
            w += s->size;
        }
    } else {
        long outer = 1, inner = 1;
        for (int d = 0; d < ax; d++) outer *= sh[d];
        for (int d = ax + 1; d < nd; d++) inner *= sh[d];
        for (long o = 0; o < outer; o++)
            for (int i = 0; i < nc; i++) {
                OSlot *s = &c->slots[op->concat_inputs[i]];
                long ch = (long)s->shape[ax] * inner;
                memcpy(w, s->data + o * ch, (size_t)ch * sizeof(float));
                w += ch;
            }
    }
    y->ndim = nd;
    for (int d = 0; d < nd; d++) y->shape[d] = sh[d];
    y->shape[ax] = tot;
}

static void op_matmul(OCtx *c, const OInstr *op)
{
    OSlot *a = &c->slots[op->in0], *b = &c->slots[op->in1], *y = &c->slots[op->out_slot];
    int an = a->ndim, bn = b->ndim;
    int m = a->shape[an - 2], k = a->shape[an - 1];
    int batch = 1, osh[MAXD];
    for (int d = 0; d < an - 2; d++) { batch *= a->shape[d]; osh[d] = a->shape[d]; }
    if (op->tag == 13) {
        int K = b->tt_K, N = b->tt_N;
        osh[an - 2] = m;
        osh[an - 1] = N;
        long tot = (long)batch * m * N;
        float *x = a->data;
        grow(y, (int)tot);
        if (tot > 0 && (K == 0))
            memset(y->data, 0, (size_t)tot * sizeof(float));
        else if (tot > 0)
            orc_tt_gemv(x, batch * m, b->codebook, b->n_codes, b->w_indices, K, N, y->data);
        set_dims(y, osh, an);
        return;
    }
    int n = b->shape[bn - 1];
    osh[an - 2] = m;
    osh[an - 1] = n;
    long tot = (long)batch * m * n;
    const float *ad = a->data, *bd = b->data;
    grow(y, (int)tot);
    for (int bi = 0; bi < batch; bi++)
        for (int i = 0; i < m; i++)
            for (int j = 0; j < n; j++) {
                float s = 0.0f;
                for (int kk = 0; kk < k; kk++)
                    s = s + ad[((long)bi * m + i) * k + kk] * bd[((long)bi * k + kk) * n + j];
                y->data[((long)bi * m + i) * n + j] = s;
            }
    set_dims(y, osh, an);
}

void orc_tape_run(OCtx *c)
{
    for (int i = 0; i < c->n_instrs; i++) {
        const OInstr *op = &c->tape[i];
        OSlot *y = &c->slots[op->out_slot];
        switch (op->tag) {
        case 0: case 1: case 2: case 3: case 4: case 10: case 11: op_unary(c, op); break;
        case 5: case 6: case 7: case 8: case 9: op_binary(c, op); break;
        case 12: case 13: op_matmul(c, op); break;
        case 14: case 15: case 16: case 17: op_reduce(c, op); break;
        case 18: case 23: {
            OSlot *x = &c->slots[op->in0];
            int n = x->size, sh[MAXD], nd = x->ndim;
            memcpy(sh, x->shape, sizeof sh);
            grow(y, n);
            if (y->data != x->data) memcpy(y->data, x->data, (size_t)n * sizeof(float));
            if (op->tag == 18) set_dims(y, op->out_shape, op->out_ndim);
            else set_dims(y, sh, nd);
            y->size = n;
            break;
        }
        case 19: case 21: case 22: op_move(c, op); break;
        case 20: op_concat(c, op); break;
        default: break;
        }
    }
}

/* Prefill + greedy decode (processor_infer's loop) with logits capture:
 * logits gets one row per tape step ([prompt_len + max_new][vocab]). */
int orc_processor_infer(OCtx *c, const float *embed, int vocab, int hidden,
                        const float *rcos, const float *rsin, int hd, int embed_slot,
                        int cos_slot, int sin_slot, const int *kv_in, const int *kv_out,
                        int logits_slot, int layers, int nkv, const int *prompt,
                        int prompt_len, int max_new, int eos, int *out, int *out_len,
                        float *logits)
{
    int total = prompt_len + max_new, kvd = nkv * hd;
    float **kb = calloc(layers, sizeof(float *)), **vb = calloc(layers, sizeof(float *));
    for (int l = 0; l < layers; l++) {
        kb[l] = calloc((size_t)kvd * (total > 64 ? total : 64), sizeof(float));
        vb[l] = calloc((size_t)kvd * (total > 64 ? total : 64), sizeof(float));
    }
    int es[2] = {1, hidden}, rs[2] = {1, hd}, gen = 0, steps = 0;
    int tok = prompt[0];
    for (int pos = 0; pos < total; pos++) {
        if (pos < prompt_len) {
            tok = prompt[pos];
        } else {
            int sz;
            const float *lg = orc_slot_read(c, logits_slot, &sz);
            const float *row = lg + (sz > vocab ? sz - vocab : 0);
            int best = 0;
            for (int v = 1; v < vocab; v++)
                if (row[v] > row[best]) best = v;
            if (best == eos) break;
            out[gen++] = best;
            tok = best;
        }
        orc_slot_write(c, embed_slot, embed + (size_t)tok * hidden, hidden);
        orc_slot_set_shape(c, embed_slot, es, 2);
        orc_slot_write(c, cos_slot, rcos + (size_t)pos * hd, hd);
        orc_slot_set_shape(c, cos_slot, rs, 2);
        orc_slot_write(c, sin_slot, rsin + (size_t)pos * hd, hd);
        orc_slot_set_shape(c, sin_slot, rs, 2);
        for (int l = 0; l < layers; l++) {
            int ks[3] = {nkv, pos, hd};
            orc_slot_set_external(c, kv_in[2 * l], kb[l], ks, 3);
            orc_slot_set_external(c, kv_in[2 * l + 1], vb[l], ks, 3);
        }
        orc_tape_run(c);
        for (int l = 0; l < layers; l++) {
            int sz;
            size_t n = (size_t)kvd * (pos + 1);
            memcpy(kb[l], orc_slot_read(c, kv_out[2 * l], &sz), n * sizeof(float));
            memcpy(vb[l], orc_slot_read(c, kv_out[2 * l + 1], &sz), n * sizeof(float));
        }
        if (logits) {
            int sz;
            const float *lg = orc_slot_read(c, logits_slot, &sz);
            memcpy(logits + (size_t)steps * vocab, lg + (sz > vocab ? sz - vocab : 0),
                   (size_t)vocab * sizeof(float));
        }
        steps++;
    }
    for (int l = 0; l < layers; l++) { free(kb[l]); free(vb[l]); }
    free(kb);
    free(vb);
    *out_len = gen;
    return steps;
}
