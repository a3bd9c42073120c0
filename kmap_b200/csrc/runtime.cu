// runtime.cu -- context and slot API of the drop-in ABI, and the generic
// executor that runs every tape instruction as one device kernel.
//
// Host-side bookkeeping (Slot.shape / ndim / size / owns_data) follows the
// reference runtime rule for rule, because callers observe it through
// tape_slot_read / tape_slot_read_shape:
//   slot API          reference _tape_runner.c:306-435
//   per-op shapes     reference _tape_runner.c:665-995 (tape_run)
// The data itself lives in HBM (DevSlot) and is copied to the host only when
// a caller reads a slot.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"

namespace kllm {

long long g_launches = 0;

static thread_local std::string t_err;
static thread_local bool t_has_err = false;
static thread_local int t_device = -1;

void set_error(const char *fmt, ...) {
    if (t_has_err) return;
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    t_has_err = true;
    fprintf(stderr, "[kllm] error: %s\n", buf);
}

bool cuda_ok(cudaError_t e, const char *what, const char *file, int line) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    return false;
}

bool select_device(CtxImpl *c) {
    if (!KLLM_CUDA(cudaSetDevice(c->device))) return false;
    if (!c->stream) {
        if (!KLLM_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)))
            return false;
    }
    return true;
}

// Device buffer of `slot` with room for `need` floats (at least one); the
// current contents survive a growth.
bool ensure_device(CtxImpl *c, int slot, size_t need) {
    DevSlot &d = c->ds[slot];
    if (need < 1) need = 1;
    if (d.d && d.cap >= need) return true;
    size_t cap = std::max(need, d.cap + d.cap / 2);
    float *p = nullptr;
    if (!KLLM_CUDA(cudaMallocAsync((void **)&p, cap * sizeof(float), c->stream))) return false;
    if (d.d) {
        if (!KLLM_CUDA(cudaMemcpyAsync(p, d.d, d.cap * sizeof(float),
                                       cudaMemcpyDeviceToDevice, c->stream)))
            return false;
        KLLM_CUDA(cudaFreeAsync(d.d, c->stream));
    }
    d.d = p;
    d.cap = cap;
    return true;
}

bool ensure_part(CtxImpl *c, size_t floats) {
    if (c->d_part && c->part_cap >= floats) return true;
    if (c->d_part) KLLM_CUDA(cudaFreeAsync(c->d_part, c->stream));
    c->d_part = nullptr;
    size_t cap = std::max(floats, (size_t)1 << 16);
    if (!KLLM_CUDA(cudaMallocAsync((void **)&c->d_part, cap * sizeof(float), c->stream)))
        return false;
    c->part_cap = cap;
    return true;
}

// Host copy of a device-newer slot (tape_slot_read).
static bool download(CtxImpl *c, int slot) {
    Slot &s = c->base.slots[slot];
    DevSlot &d = c->ds[slot];
    if (!d.dev_newer) return true;
    size_t n = s.size > 0 ? (size_t)s.size : 0;
    if (n > d.cap) n = d.cap;
    if (!s.data || (s.owns_data && d.host_cap < n) || (!s.owns_data && (size_t)s.size < n)) {
        if (s.owns_data) free(s.data);
        s.data = (float *)malloc(std::max<size_t>(n, 1) * sizeof(float));
        s.owns_data = 1;
        d.host_cap = std::max<size_t>(n, 1);
    }
    if (n && !KLLM_CUDA(cudaMemcpyAsync(s.data, d.d, n * sizeof(float),
                                        cudaMemcpyDeviceToHost, c->stream)))
        return false;
    if (!KLLM_CUDA(cudaStreamSynchronize(c->stream))) return false;
    d.dev_newer = false;
    return true;
}

// Index-range check of a truth-table matrix, once at upload: every index
// must address the codebook (the reference reads out of bounds instead).
__global__ void k_max_index(const uint16_t *idx, size_t n, unsigned int *out) {
    unsigned int m = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        m = max(m, (unsigned int)idx[i]);
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

bool upload_tt(CtxImpl *c, int slot) {
    Slot &s = c->base.slots[slot];
    DevSlot &d = c->ds[slot];
    if (d.tt_ready && d.tt_src_idx == s.w_indices && d.tt_src_cb == s.codebook &&
        d.tt_K == s.tt_K && d.tt_N == s.tt_N && d.tt_codes == s.n_codes)
        return true;
    if (!s.w_indices || !s.codebook || s.n_codes <= 0 || s.tt_K < 0 || s.tt_N < 0) {
        set_error("slot %d: truth-table matrix is not set", slot);
        return false;
    }
    if (d.d_idx) KLLM_CUDA(cudaFreeAsync(d.d_idx, c->stream));
    if (d.d_cb) KLLM_CUDA(cudaFreeAsync(d.d_cb, c->stream));
    d.d_idx = nullptr;
    d.d_cb = nullptr;
    size_t n = (size_t)s.tt_K * s.tt_N;
    size_t cbn = ((size_t)s.n_codes + 3) & ~(size_t)3;
    if (!KLLM_CUDA(cudaMallocAsync((void **)&d.d_idx, std::max<size_t>(n, 8) * 2, c->stream)))
        return false;
    if (!KLLM_CUDA(cudaMallocAsync((void **)&d.d_cb, cbn * 4, c->stream))) return false;
    if (!KLLM_CUDA(cudaMemsetAsync(d.d_cb, 0, cbn * 4, c->stream))) return false;
    if (n && !KLLM_CUDA(cudaMemcpyAsync(d.d_idx, s.w_indices, n * 2,
                                        cudaMemcpyHostToDevice, c->stream)))
        return false;
    if (!KLLM_CUDA(cudaMemcpyAsync(d.d_cb, s.codebook, (size_t)s.n_codes * 4,
                                   cudaMemcpyHostToDevice, c->stream)))
        return false;
    if (n) {
        unsigned int *dm = nullptr, hm = 0;
        if (!KLLM_CUDA(cudaMallocAsync((void **)&dm, 4, c->stream))) return false;
        KLLM_CUDA(cudaMemsetAsync(dm, 0, 4, c->stream));
        k_max_index<<<296, 256, 0, c->stream>>>(d.d_idx, n, dm);
        g_launches++;
        KLLM_CUDA(cudaMemcpyAsync(&hm, dm, 4, cudaMemcpyDeviceToHost, c->stream));
        KLLM_CUDA(cudaFreeAsync(dm, c->stream));
        if (!KLLM_CUDA(cudaStreamSynchronize(c->stream))) return false;
        if ((int)hm >= s.n_codes) {
            set_error("slot %d: index %u outside its codebook of %d entries", slot, hm,
                      s.n_codes);
            return false;
        }
    }
    d.tt_src_idx = s.w_indices;
    d.tt_src_cb = s.codebook;
    d.tt_K = s.tt_K;
    d.tt_N = s.tt_N;
    d.tt_codes = s.n_codes;
    d.tt_ready = true;
    return true;
}

// Copy host-newer slots to the device (before a tape step).
bool sync_inputs(CtxImpl *c) {
    for (int i = 0; i < c->base.n_slots; i++) {
        Slot &s = c->base.slots[i];
        DevSlot &d = c->ds[i];
        if (d.zero_pending) {
            if (!ensure_device(c, i, (size_t)std::max(s.size, 1))) return false;
            if (!KLLM_CUDA(cudaMemsetAsync(d.d, 0, d.cap * sizeof(float), c->stream)))
                return false;
            d.zero_pending = false;
        }
        if (d.host_dirty) {
            size_t n = s.size > 0 ? (size_t)s.size : 0;
            if (!ensure_device(c, i, n)) return false;
            if (n && s.data &&
                !KLLM_CUDA(cudaMemcpyAsync(d.d, s.data, n * sizeof(float),
                                           cudaMemcpyHostToDevice, c->stream)))
                return false;
            d.host_dirty = false;
            d.dev_newer = false;
        }
    }
    // Pageable host sources are staged by the driver; make sure none of
    // them is touched again before the copies finish.
    return KLLM_CUDA(cudaStreamSynchronize(c->stream));
}

}  // namespace kllm

using namespace kllm;

// ================================================================ C ABI ===

extern "C" {

const char *kllm_last_error(void) { return t_has_err ? t_err.c_str() : nullptr; }

void kllm_clear_error(void) {
    t_has_err = false;
    t_err.clear();
}

const char *kllm_version(void) { return "kllm-b200 0.1.0 (sm_100a)"; }

int kllm_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int kllm_set_device(int device) {
    if (device < 0 || device >= kllm_device_count()) {
        set_error("kllm_set_device: no CUDA device %d", device);
        return -1;
    }
    t_device = device;
    return 0;
}

long long kllm_launch_count(void) { return g_launches; }

void kllm_default_infer_opts(kllm_infer_opts *o) {
    memset(o, 0, sizeof *o);
    o->mode = KLLM_MODE_AUTO;
    o->use_graphs = 1;
}

TapeCtx *tape_ctx_create(int n_slots, int n_instrs) {
    if (n_slots < 0) n_slots = 0;
    if (n_instrs < 0) n_instrs = 0;
    CtxImpl *c = new CtxImpl();
    c->base.n_slots = n_slots;
    c->base.n_instrs = n_instrs;
    c->base.slots = (Slot *)calloc(std::max(n_slots, 1), sizeof(Slot));
    c->base.tape = (TapeInstr *)calloc(std::max(n_instrs, 1), sizeof(TapeInstr));
    c->ds.resize(n_slots);
    kllm_default_infer_opts(&c->opts);
    memset(&c->stats, 0, sizeof c->stats);
    int dev = t_device;
    if (dev < 0) {
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            dev = 0;
        }
    }
    c->device = dev;
    return &c->base;
}

void tape_ctx_destroy(TapeCtx *ctx) {
    if (!ctx) return;
    CtxImpl *c = impl(ctx);
    if (c->stream) cudaSetDevice(c->device);
    plan_destroy(c);
    for (int i = 0; i < ctx->n_slots; i++) {
        if (ctx->slots[i].owns_data && ctx->slots[i].data) free(ctx->slots[i].data);
        DevSlot &d = c->ds[i];
        if (c->stream) {
            if (d.d) cudaFreeAsync(d.d, c->stream);
            if (d.d_idx) cudaFreeAsync(d.d_idx, c->stream);
            if (d.d_cb) cudaFreeAsync(d.d_cb, c->stream);
        }
    }
    if (c->stream) {
        if (c->d_part) cudaFreeAsync(c->d_part, c->stream);
        if (c->d_counters) cudaFreeAsync(c->d_counters, c->stream);
        cudaStreamSynchronize(c->stream);
        cudaStreamDestroy(c->stream);
    }
    free(ctx->slots);
    free(ctx->tape);
    delete c;
}

int tape_ctx_n_instrs(TapeCtx *ctx) { return ctx->n_instrs; }
int tape_ctx_n_slots(TapeCtx *ctx) { return ctx->n_slots; }

static bool slot_ok(TapeCtx *ctx, int i, const char *fn) {
    if (!ctx || i < 0 || i >= ctx->n_slots) {
        set_error("%s: slot %d out of range", fn, i);
        return false;
    }
    return true;
}

static bool ndim_ok(int ndim, const char *fn) {
    if (ndim < 0 || ndim > MAX_DIMS) {
        set_error("%s: ndim %d outside 0..%d", fn, ndim, MAX_DIMS);
        return false;
    }
    return true;
}

// Reference _tape_runner.c:328-340.
void tape_slot_alloc(TapeCtx *ctx, int slot_idx, const int *shape, int ndim) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_alloc") || !ndim_ok(ndim, "tape_slot_alloc")) return;
    Slot *s = &ctx->slots[slot_idx];
    DevSlot &d = impl(ctx)->ds[slot_idx];
    if (s->owns_data && s->data) free(s->data);
    s->ndim = ndim;
    s->size = 1;
    for (int i = 0; i < ndim; i++) {
        s->shape[i] = shape[i];
        s->size *= shape[i];
    }
    s->data = (float *)calloc(std::max(s->size, 1), sizeof(float));
    s->owns_data = 1;
    d.host_cap = std::max(s->size, 1);
    d.zero_pending = true;
    d.host_dirty = false;
    d.dev_newer = false;
}

// Reference _tape_runner.c:343-355.
void tape_slot_set_external(TapeCtx *ctx, int slot_idx, float *data, const int *shape,
                            int ndim) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_set_external") ||
        !ndim_ok(ndim, "tape_slot_set_external"))
        return;
    Slot *s = &ctx->slots[slot_idx];
    DevSlot &d = impl(ctx)->ds[slot_idx];
    if (s->owns_data && s->data) free(s->data);
    s->data = data;
    s->ndim = ndim;
    s->size = 1;
    for (int i = 0; i < ndim; i++) {
        s->shape[i] = shape[i];
        s->size *= shape[i];
    }
    s->owns_data = 0;
    d.host_cap = 0;
    d.host_dirty = true;
    d.dev_newer = false;
    d.zero_pending = false;
}

// Reference _tape_runner.c:362-375.
void tape_slot_set_truth_table(TapeCtx *ctx, int slot_idx, float *codebook, int n_codes,
                               uint16_t *w_indices, int K, int N) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_set_truth_table")) return;
    Slot *s = &ctx->slots[slot_idx];
    s->codebook = codebook;
    s->w_indices = w_indices;
    s->n_codes = n_codes;
    s->tt_K = K;
    s->tt_N = N;
    s->shape[0] = K;
    s->shape[1] = N;
    s->ndim = 2;
    s->size = K * N;
    impl(ctx)->ds[slot_idx].tt_ready = false;
}

// Reference _tape_runner.c:378-390.
void tape_slot_write(TapeCtx *ctx, int slot_idx, const float *data, int n) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_write")) return;
    Slot *s = &ctx->slots[slot_idx];
    CtxImpl *c = impl(ctx);
    DevSlot &d = c->ds[slot_idx];
    if (n <= 0) return;
    if (d.dev_newer) {
        if (!select_device(c) || !download(c, slot_idx)) return;
    }
    if (n > s->size) {
        if (s->owns_data && s->data) free(s->data);
        s->data = (float *)malloc((size_t)n * sizeof(float));
        s->size = n;
        s->owns_data = 1;
        d.host_cap = n;
    } else if (s->owns_data && d.host_cap < (size_t)n) {
        s->data = (float *)realloc(s->data, (size_t)n * sizeof(float));
        d.host_cap = n;
    }
    memcpy(s->data, data, (size_t)n * sizeof(float));
    d.host_dirty = true;
    d.dev_newer = false;
    d.zero_pending = false;
}

// Reference _tape_runner.c:393-402.
void tape_slot_set_shape(TapeCtx *ctx, int slot_idx, const int *shape, int ndim) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_set_shape") || !ndim_ok(ndim, "tape_slot_set_shape"))
        return;
    Slot *s = &ctx->slots[slot_idx];
    s->ndim = ndim;
    s->size = 1;
    for (int i = 0; i < ndim; i++) {
        s->shape[i] = shape[i];
        s->size *= shape[i];
    }
}

// Reference _tape_runner.c:405-408; the data comes back from the device.
const float *tape_slot_read(TapeCtx *ctx, int slot_idx, int *out_size) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_read")) {
        if (out_size) *out_size = 0;
        return nullptr;
    }
    CtxImpl *c = impl(ctx);
    if (c->ds[slot_idx].dev_newer) {
        if (!select_device(c) || !download(c, slot_idx)) {
            if (out_size) *out_size = 0;
            return nullptr;
        }
    }
    if (out_size) *out_size = ctx->slots[slot_idx].size;
    return ctx->slots[slot_idx].data;
}

// Reference _tape_runner.c:411-415.
int tape_slot_read_shape(TapeCtx *ctx, int slot_idx, int *out_shape) {
    if (!slot_ok(ctx, slot_idx, "tape_slot_read_shape")) return 0;
    Slot *s = &ctx->slots[slot_idx];
    for (int d = 0; d < s->ndim; d++) out_shape[d] = s->shape[d];
    return s->ndim;
}

TapeInstr *tape_get_instr(TapeCtx *ctx, int instr_idx) {
    if (!ctx || instr_idx < 0 || instr_idx >= ctx->n_instrs) {
        set_error("tape_get_instr: instruction %d out of range", instr_idx);
        return nullptr;
    }
    return &ctx->tape[instr_idx];
}

int kllm_tape_run(TapeCtx *ctx) {
    if (!ctx) {
        set_error("kllm_tape_run: NULL context");
        return -1;
    }
    CtxImpl *c = impl(ctx);
    if (!select_device(c)) return -1;
    if (!sync_inputs(c)) return -1;
    if (!run_generic(c)) return -1;
    return 0;
}

void tape_run(TapeCtx *ctx) { (void)kllm_tape_run(ctx); }

int kllm_set_infer_opts(TapeCtx *ctx, const kllm_infer_opts *o) {
    if (!ctx || !o) {
        set_error("kllm_set_infer_opts: NULL argument");
        return -1;
    }
    if (o->order != KLLM_ORDER_EXACT && o->order != KLLM_ORDER_FAST) {
        set_error("kllm_set_infer_opts: order %d is not KLLM_ORDER_EXACT or KLLM_ORDER_FAST",
                  o->order);
        return -1;
    }
    impl(ctx)->opts = *o;
    return 0;
}

int kllm_get_infer_stats(TapeCtx *ctx, kllm_infer_stats *s) {
    if (!ctx || !s) {
        set_error("kllm_get_infer_stats: NULL argument");
        return -1;
    }
    *s = impl(ctx)->stats;
    return 0;
}

}  // extern "C"

// ======================================================= generic steps ===

namespace kllm {

static void copy_shape(Slot *dst, const Slot *src) {
    dst->ndim = src->ndim;
    int sz = 1;
    for (int d = 0; d < src->ndim; d++) {
        dst->shape[d] = src->shape[d];
        sz *= src->shape[d];
    }
    dst->size = sz;
}

static Dims dims_of(const int *shape, int nd) {
    Dims d;
    d.nd = nd;
    for (int i = 0; i < MAX_DIMS; i++) d.d[i] = i < nd ? shape[i] : 1;
    return d;
}

// Reference ensure_slot (_tape_runner.c:437-445): the size field only ever
// grows here; the device buffer follows it.
static bool ensure_out(CtxImpl *c, int slot, int need) {
    Slot *s = &c->base.slots[slot];
    if (need < 1) need = 1;
    if (need > s->size) s->size = need;
    return ensure_device(c, slot, (size_t)need);
}

static inline float *D(CtxImpl *c, int slot) { return c->ds[slot].d; }

static void mark_out(CtxImpl *c, int slot) {
    DevSlot &d = c->ds[slot];
    d.dev_newer = true;
    d.host_dirty = false;
    d.zero_pending = false;
}

static bool in_ok(CtxImpl *c, int i, int slot, const char *what) {
    if (slot < 0 || slot >= c->base.n_slots) {
        set_error("instruction %d: %s slot %d out of range", i, what, slot);
        return false;
    }
    if (!c->ds[slot].d) {
        // an input never written: the reference would read its (absent)
        // buffer; give it a zeroed device buffer instead
        Slot &s = c->base.slots[slot];
        if (!ensure_device(c, slot, (size_t)std::max(s.size, 1))) return false;
        if (!KLLM_CUDA(cudaMemsetAsync(c->ds[slot].d, 0, c->ds[slot].cap * 4, c->stream)))
            return false;
    }
    return true;
}

bool run_generic(CtxImpl *c) {
    TapeCtx *ctx = &c->base;
    Slot *slots = ctx->slots;
    cudaStream_t st = c->stream;
    for (int i = 0; i < ctx->n_instrs; i++) {
        const TapeInstr *op = &ctx->tape[i];
        if (op->out_slot < 0 || op->out_slot >= ctx->n_slots) {
            set_error("instruction %d: output slot %d out of range", i, op->out_slot);
            return false;
        }
        Slot *out = &slots[op->out_slot];
        int tag = op->tag;
        bool unary = tag <= OP_SIN || tag == OP_NEG || tag == OP_SQUARE || tag == OP_SUM ||
                     tag == OP_MAX_RED || tag == OP_MEAN || tag == OP_ARGMAX ||
                     tag == OP_RESHAPE || tag == OP_TRANSPOSE || tag == OP_REPEAT ||
                     tag == OP_SLICE || tag == OP_COPY;
        bool binary = (tag >= OP_ADD && tag <= OP_MAX) || tag == OP_MATMUL ||
                      tag == OP_MATMUL_TT;
        if ((unary || binary) && !in_ok(c, i, op->in0, "input")) return false;
        if (binary && tag != OP_MATMUL_TT && !in_ok(c, i, op->in1, "second input"))
            return false;
        Slot *s0 = (unary || binary) ? &slots[op->in0] : nullptr;
        Slot *s1 = binary ? &slots[op->in1] : nullptr;
        const int o = op->out_slot;

        switch (tag) {
        case OP_SILU: case OP_EXP: case OP_RSQRT: case OP_COS: case OP_SIN:
        case OP_NEG: case OP_SQUARE: {
            if (!ensure_out(c, o, s0->size)) return false;
            copy_shape(out, s0);
            if (!launch_unary(st, tag, D(c, op->in0), D(c, o), s0->size)) return false;
            break;
        }
        case OP_ADD: case OP_SUB: case OP_MUL: case OP_DIV: case OP_MAX: {
            int bs[MAX_DIMS], bnd = std::max(s0->ndim, s1->ndim);
            long long bsz = 1;
            for (int d = 0; d < bnd; d++) {
                int ad = d < s0->ndim ? s0->shape[s0->ndim - 1 - d] : 1;
                int bd = d < s1->ndim ? s1->shape[s1->ndim - 1 - d] : 1;
                if ((ad != bd && ad != 1 && bd != 1)) {
                    set_error("instruction %d: shapes do not broadcast", i);
                    return false;
                }
                bs[bnd - 1 - d] = std::max(ad, bd);
                bsz *= bs[bnd - 1 - d];
            }
            if (!ensure_out(c, o, (int)bsz)) return false;
            Dims da = dims_of(s0->shape, s0->ndim), db = dims_of(s1->shape, s1->ndim),
                 dy = dims_of(bs, bnd);
            if (!launch_binop(st, tag, D(c, op->in0), da, D(c, op->in1), db, D(c, o), dy))
                return false;
            out->ndim = bnd;
            for (int d = 0; d < bnd; d++) out->shape[d] = bs[d];
            out->size = (int)bsz;
            break;
        }
        case OP_MATMUL: {
            int an = s0->ndim, bn = s1->ndim;
            if (an < 2 || bn < 2) {
                set_error("instruction %d: MATMUL needs 2-D operands", i);
                return false;
            }
            int m = s0->shape[an - 2], k = s0->shape[an - 1], nn = s1->shape[bn - 1];
            int batch = 1;
            for (int d = 0; d < an - 2; d++) batch *= s0->shape[d];
            long long tot = (long long)batch * m * nn;
            if (!ensure_out(c, o, (int)tot)) return false;
            out->ndim = an;
            for (int d = 0; d < an - 2; d++) out->shape[d] = s0->shape[d];
            out->shape[an - 2] = m;
            out->shape[an - 1] = nn;
            out->size = (int)tot;
            if (m == 0 || k == 0 || nn == 0 || batch == 0) {
                if (tot > 0 && !launch_fill(st, D(c, o), tot, 0.f)) return false;
                break;
            }
            if ((long long)s1->size < (long long)batch * k * nn ||
                (long long)s0->size < (long long)batch * m * k) {
                set_error("instruction %d: MATMUL operand smaller than its shape", i);
                return false;
            }
            if (!launch_matmul(st, D(c, op->in0), D(c, op->in1), D(c, o), batch, m, k, nn))
                return false;
            break;
        }
        case OP_MATMUL_TT: {
            if (op->in1 < 0 || op->in1 >= ctx->n_slots) {
                set_error("instruction %d: weight slot %d out of range", i, op->in1);
                return false;
            }
            int an = s0->ndim;
            if (an < 2) {
                set_error("instruction %d: MATMUL_TT needs a 2-D input", i);
                return false;
            }
            int K = s1->tt_K, N = s1->tt_N, m = s0->shape[an - 2];
            int batch = 1;
            for (int d = 0; d < an - 2; d++) batch *= s0->shape[d];
            long long tot = (long long)batch * m * N;
            if (!ensure_out(c, o, (int)tot)) return false;
            out->ndim = an;
            for (int d = 0; d < an - 2; d++) out->shape[d] = s0->shape[d];
            out->shape[an - 2] = m;
            out->shape[an - 1] = N;
            out->size = (int)tot;
            if (m == 0 || K == 0 || N == 0 || batch == 0) {
                if (tot > 0 && !launch_fill(st, D(c, o), tot, 0.f)) return false;
                break;
            }
            if (!upload_tt(c, op->in1)) return false;
            int rows = batch * m;
            if ((long long)s0->size < (long long)rows * K) {
                set_error("instruction %d: MATMUL_TT input smaller than rows x K", i);
                return false;
            }
            int T = tt_chunks(K);
            if (!ensure_part(c, (size_t)T * rows * N)) return false;
            const DevSlot &w = c->ds[op->in1];
            if (rows == 1 && tt_fused_applies(w.d_idx, w.d_cb, K, N, s1->n_codes)) {
                if (!c->d_counters) {
                    if (!KLLM_CUDA(cudaMallocAsync((void **)&c->d_counters, 4096 * 4, st)) ||
                        !KLLM_CUDA(cudaMemsetAsync(c->d_counters, 0, 4096 * 4, st)))
                        return false;
                }
                if (N / 64 + 1 > 4096) {
                    set_error("instruction %d: MATMUL_TT wider than the counter table", i);
                    return false;
                }
                if (!tt_gemv_fused_y(st, D(c, op->in0), w.d_cb, s1->n_codes, w.d_idx, K, N,
                                     c->d_part, c->d_counters, D(c, o), nullptr))
                    return false;
                break;
            }
            if (!tt_gemv_partials(st, D(c, op->in0), rows, w.d_cb, s1->n_codes, w.d_idx, K, N,
                                  c->d_part))
                return false;
            if (!tt_reduce_partials(st, c->d_part, T, rows, N, D(c, o))) return false;
            break;
        }
        case OP_SUM: case OP_MAX_RED: case OP_MEAN: case OP_ARGMAX: {
            int ax = op->axis;
            if (ax < 0 || ax >= s0->ndim || s0->shape[ax] <= 0) {
                set_error("instruction %d: reduction axis %d invalid", i, ax);
                return false;
            }
            int red = s0->size / s0->shape[ax];
            if (!ensure_out(c, o, red)) return false;
            int od = 0;
            for (int d = 0; d < s0->ndim; d++) {
                if (d == ax) {
                    if (op->keepdims && tag != OP_ARGMAX) out->shape[od++] = 1;
                } else {
                    out->shape[od++] = s0->shape[d];
                }
            }
            out->ndim = od;
            out->size = red;
            long long outer = 1, inner = 1;
            for (int d = 0; d < ax; d++) outer *= s0->shape[d];
            for (int d = ax + 1; d < s0->ndim; d++) inner *= s0->shape[d];
            if (!launch_reduce(st, tag, D(c, op->in0), D(c, o), outer, s0->shape[ax], inner))
                return false;
            break;
        }
        case OP_RESHAPE: {
            if (!ensure_out(c, o, s0->size)) return false;
            if (o != op->in0 && s0->size > 0 &&
                !KLLM_CUDA(cudaMemcpyAsync(D(c, o), D(c, op->in0), (size_t)s0->size * 4,
                                           cudaMemcpyDeviceToDevice, st)))
                return false;
            if (op->out_ndim < 0 || op->out_ndim > MAX_DIMS) {
                set_error("instruction %d: RESHAPE ndim %d invalid", i, op->out_ndim);
                return false;
            }
            out->ndim = op->out_ndim;
            for (int d = 0; d < op->out_ndim; d++) out->shape[d] = op->out_shape[d];
            out->size = s0->size;
            break;
        }
        case OP_TRANSPOSE: {
            int nd = s0->ndim;
            unsigned seen = 0;
            for (int d = 0; d < nd; d++) {
                int a = op->axes[d];
                if (a < 0 || a >= nd || (seen >> a & 1u)) {
                    set_error("instruction %d: TRANSPOSE axes are not a permutation", i);
                    return false;
                }
                seen |= 1u << a;
            }
            int sz = s0->size;
            if (!ensure_out(c, o, sz)) return false;
            int ish[MAX_DIMS];
            for (int d = 0; d < nd; d++) ish[d] = s0->shape[d];
            out->ndim = nd;
            out->size = sz;
            for (int d = 0; d < nd; d++) out->shape[d] = ish[op->axes[d]];
            if (!launch_transpose(st, D(c, op->in0), dims_of(ish, nd), op->axes, D(c, o)))
                return false;
            break;
        }
        case OP_CONCAT: {
            int ax = op->axis, nc = op->concat_n_inputs;
            if (nc < 1 || nc > MAX_CONCAT_INPUTS) {
                set_error("instruction %d: CONCAT of %d inputs", i, nc);
                return false;
            }
            long long need = 0;
            for (int ci = 0; ci < nc; ci++) {
                if (!in_ok(c, i, op->concat_inputs[ci], "concat input")) return false;
                need += slots[op->concat_inputs[ci]].size;
            }
            Slot *first = &slots[op->concat_inputs[0]];
            if (ax < 0 || (first->ndim > 0 && ax >= first->ndim)) {
                set_error("instruction %d: CONCAT axis %d invalid", i, ax);
                return false;
            }
            // the reference grows the size field only when the result is
            // larger (_tape_runner.c:903-908)
            if (need > out->size) out->size = (int)need;
            if (!ensure_device(c, o, (size_t)std::max<long long>(need, 1))) return false;
            int fnd = first->ndim, fsh[MAX_DIMS];
            for (int d = 0; d < fnd; d++) fsh[d] = first->shape[d];
            int total_ax = 0;
            for (int ci = 0; ci < nc; ci++) total_ax += slots[op->concat_inputs[ci]].shape[ax];
            const float *xs[MAX_CONCAT_INPUTS];
            long long chunk[MAX_CONCAT_INPUTS];
            long long outer = 1, inner = 1;
            bool flat = (ax == 0 || fnd == 1);
            if (!flat) {
                for (int d = 0; d < ax; d++) outer *= fsh[d];
                for (int d = ax + 1; d < fnd; d++) inner *= fsh[d];
            }
            for (int ci = 0; ci < nc; ci++) {
                Slot *si = &slots[op->concat_inputs[ci]];
                xs[ci] = D(c, op->concat_inputs[ci]);
                chunk[ci] = flat ? si->size : (long long)si->shape[ax] * inner;
                if (!flat && outer * chunk[ci] > si->size) {
                    set_error("instruction %d: CONCAT input %d smaller than its shape", i, ci);
                    return false;
                }
            }
            if (flat) outer = 1;
            out->ndim = fnd;
            for (int d = 0; d < fnd; d++) out->shape[d] = fsh[d];
            out->shape[ax] = total_ax;
            if (!launch_concat(st, xs, chunk, nc, outer, D(c, o))) return false;
            break;
        }
        case OP_REPEAT: {
            int ax = op->axis, r = op->repeats;
            if (ax < 0 || ax >= s0->ndim || r < 0) {
                set_error("instruction %d: REPEAT axis %d / repeats %d invalid", i, ax, r);
                return false;
            }
            int rsz = s0->size * r;
            if (!ensure_out(c, o, rsz)) return false;
            Dims din = dims_of(s0->shape, s0->ndim);
            copy_shape(out, s0);
            out->shape[ax] *= r;
            out->size = rsz;
            if (rsz > 0 && !launch_repeat(st, D(c, op->in0), din, r, ax, D(c, o))) return false;
            break;
        }
        case OP_SLICE: {
            int nd = s0->ndim, sl[MAX_DIMS];
            long long sz = 1;
            for (int d = 0; d < nd; d++) {
                int start = op->starts[d], step = op->steps[d], stop = s0->shape[d];
                if (step <= 0) {
                    set_error("instruction %d: SLICE step %d invalid", i, step);
                    return false;
                }
                if (d < op->slice_out_ndim) {
                    int sd = op->slice_out_shape[d];
                    if (sd > 0 && sd <= s0->shape[d]) stop = start + sd * step;
                }
                int dim = (stop - start + step - 1) / step;
                if (dim < 0) dim = 0;
                if (dim > 0 && (start < 0 || start + (long long)(dim - 1) * step >= s0->shape[d])) {
                    set_error("instruction %d: SLICE reads outside its input", i);
                    return false;
                }
                sl[d] = dim;
                sz *= dim;
            }
            if (!ensure_out(c, o, (int)sz)) return false;
            Dims din = dims_of(s0->shape, nd);
            out->ndim = nd;
            out->size = (int)sz;
            for (int d = 0; d < nd; d++) out->shape[d] = sl[d];
            if (sz > 0 && !launch_slice(st, D(c, op->in0), din, op->starts, op->steps,
                                        dims_of(sl, nd), D(c, o)))
                return false;
            break;
        }
        case OP_COPY: {
            if (!ensure_out(c, o, s0->size)) return false;
            int sz = s0->size;
            if (o != op->in0 && sz > 0 &&
                !KLLM_CUDA(cudaMemcpyAsync(D(c, o), D(c, op->in0), (size_t)sz * 4,
                                           cudaMemcpyDeviceToDevice, st)))
                return false;
            copy_shape(out, s0);
            break;
        }
        default:
            set_error("instruction %d: unknown opcode %d", i, tag);
            return false;
        }
        mark_out(c, o);
    }
    return KLLM_CUDA(cudaGetLastError());
}

}  // namespace kllm
