// plan.cu -- fused decode plan for the compiler's LLaMA decode template.
//
// processor_infer drives one tape step per token (reference
// _tape_runner.c:1602-1763).  When the tape is exactly the template the
// kllm compiler emits (kllm_compile.c:1143-1385 per layer, driven by
// :1427-1690), the plan replaces its ~60 instructions per layer by 5 fused
// kernels over device-resident state (tt_fused.cuh for the TT-GEMVs):
//
//   qkv        x = rmsnorm(h) * w1 (h = embedding row in layer 0), TT-GEMV
//   attention  RoPE(q,k), KV append in place, softmax(q.K^T * scale).V
//   o          TT-GEMV of the attention output, h += y
//   gate_up    x = rmsnorm(h) * w2, TT-GEMV, act = silu(gate) * up
//   down       TT-GEMV of act, h += y
// then the lm_head TT-GEMV (final rmsnorm in its prologue) whose epilogue
// forms the logits and the first-maximum argmax that feeds the next step's
// embedding lookup.
//
// Arithmetic follows the tape op for op: every elementwise step is the
// same float operation (no FMA contraction), SILU / EXP / RSQRT evaluate in
// double, and the TT-GEMV keeps the reference's chunked order, so results
// differ from the reference only where its summation order is not
// reproducible at speed: the RMSNorm mean and softmax sums (a tree instead
// of a serial loop) and the attention dot products (BLAS in the reference).
//
// Every kernel is launched with programmatic dependent launch: weight
// streams and codebooks start before griddepcontrol.wait, so they overlap
// the previous kernel.  Each step is captured once as a CUDA graph and
// replayed; the step position and token live in device memory.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <type_traits>
#include <chrono>
#include <set>
#include <vector>

#include "pfgemm.cuh"
#include "plan.cuh"
#include "sm100.cuh"
#include "tt_fused.cuh"
#include "persist.cuh"
#include "batch.cuh"
#include "prefill.cuh"

namespace kllm {


// ============================================================ matching ===

struct LayerSlots {
    int ln1 = -1, ln2 = -1, eps1 = -1, eps2 = -1;
    int qkv = -1, o = -1, gu = -1, dn = -1;
};

struct TemplateInfo {
    int H = 0, nh = 0, nkv = 0, hd = 0, F = 0, V = 0, L = 0, groups = 1;
    int scale = -1, fln = -1, feps = -1, lm = -1;
    std::vector<LayerSlots> layers;
};

namespace {

struct Matcher {
    const TapeCtx *ctx;
    int pc = 0;
    std::string why;
    std::set<int> written;

    const TapeInstr *next(int tag) {
        if (!why.empty()) return nullptr;
        if (pc >= ctx->n_instrs) {
            why = "tape ends early";
            return nullptr;
        }
        const TapeInstr *op = &ctx->tape[pc];
        if (op->tag != tag) {
            why = "instruction " + std::to_string(pc) + ": opcode " + std::to_string(op->tag) +
                  ", template expects " + std::to_string(tag);
            return nullptr;
        }
        if (op->out_slot < 0 || op->out_slot >= ctx->n_slots || written.count(op->out_slot)) {
            why = "instruction " + std::to_string(pc) + ": output slot is not fresh";
            return nullptr;
        }
        written.insert(op->out_slot);
        pc++;
        return op;
    }
    bool fail(const std::string &w) {
        if (why.empty()) why = "instruction " + std::to_string(pc - 1) + ": " + w;
        return false;
    }
    int unary(int tag, int in) {
        const TapeInstr *op = next(tag);
        if (!op) return -1;
        if (op->in0 != in) return fail("unexpected operand"), -1;
        return op->out_slot;
    }
    int binop(int tag, int a, int b) {   // b < 0: any slot, returned via *cap
        const TapeInstr *op = next(tag);
        if (!op) return -1;
        if (op->in0 != a || (b >= 0 && op->in1 != b)) return fail("unexpected operands"), -1;
        return op->out_slot;
    }
    const TapeInstr *binop_any(int tag, int a) {
        const TapeInstr *op = next(tag);
        if (op && op->in0 != a) return fail("unexpected operand"), nullptr;
        return op;
    }
    int reduce(int tag, int in, int axis) {
        const TapeInstr *op = next(tag);
        if (!op) return -1;
        if (op->in0 != in || op->axis != axis || op->keepdims != 1)
            return fail("unexpected reduction"), -1;
        return op->out_slot;
    }
    int slice(int in, std::initializer_list<int> starts, std::initializer_list<int> sizes) {
        const TapeInstr *op = next(22);
        if (!op) return -1;
        int nd = (int)starts.size();
        if (op->in0 != in || op->slice_out_ndim != nd) return fail("unexpected slice"), -1;
        int d = 0;
        for (int s : starts) {
            if (op->starts[d] != s || op->steps[d] != 1) return fail("unexpected slice start"), -1;
            d++;
        }
        d = 0;
        for (int z : sizes) {
            if (op->slice_out_shape[d] != z) return fail("unexpected slice size"), -1;
            d++;
        }
        return op->out_slot;
    }
    int reshape(int in, std::initializer_list<int> shape) {
        const TapeInstr *op = next(18);
        if (!op) return -1;
        if (op->in0 != in || op->out_ndim != (int)shape.size()) return fail("unexpected reshape"), -1;
        int d = 0;
        for (int z : shape)
            if (op->out_shape[d++] != z) return fail("unexpected reshape shape"), -1;
        return op->out_slot;
    }
    int transpose(int in, int a0, int a1, int a2) {
        const TapeInstr *op = next(19);
        if (!op) return -1;
        if (op->in0 != in || op->axes[0] != a0 || op->axes[1] != a1 || op->axes[2] != a2)
            return fail("unexpected transpose"), -1;
        return op->out_slot;
    }
    int concat2(int a, int b, int axis) {
        const TapeInstr *op = next(20);
        if (!op) return -1;
        if (op->concat_n_inputs != 2 || op->concat_inputs[0] != a || op->concat_inputs[1] != b ||
            op->axis != axis)
            return fail("unexpected concat"), -1;
        return op->out_slot;
    }
    int repeat(int in, int reps, int axis) {
        const TapeInstr *op = next(21);
        if (!op) return -1;
        if (op->in0 != in || op->repeats != reps || op->axis != axis)
            return fail("unexpected repeat"), -1;
        return op->out_slot;
    }
    int matmul(int a, int b) {
        const TapeInstr *op = next(12);
        if (!op) return -1;
        if (op->in0 != a || op->in1 != b) return fail("unexpected matmul"), -1;
        return op->out_slot;
    }
    // MATMUL_TT: returns out slot, weight slot via *w (must be a TT slot, K rows)
    int matmul_tt(int a, int K, int *w) {
        const TapeInstr *op = next(13);
        if (!op) return -1;
        if (op->in0 != a || op->in1 < 0 || op->in1 >= ctx->n_slots)
            return fail("unexpected TT matmul"), -1;
        const Slot &s = ctx->slots[op->in1];
        if (!s.codebook || !s.w_indices || s.tt_K != K || s.n_codes <= 0)
            return fail("TT weight slot missing or of the wrong shape"), -1;
        *w = op->in1;
        return op->out_slot;
    }
};

bool const_slot(const TapeCtx *c, int s, int size) {
    return s >= 0 && s < c->n_slots && c->slots[s].data && c->slots[s].size == size;
}

// RMSNorm of the template (kllm_compile.c:1143-1164): returns xn slot.
int match_norm(Matcher &m, const TapeCtx *c, int h, int H, int *w_slot, int *eps_slot) {
    int sq = m.binop(7, h, h);
    int ms = m.reduce(16, sq, 1);
    const TapeInstr *add = m.binop_any(5, ms);
    if (!add) return -1;
    *eps_slot = add->in1;
    int rs = m.unary(2, add->out_slot);
    int nm = m.binop(7, h, rs);
    const TapeInstr *mw = m.binop_any(7, nm);
    if (!mw) return -1;
    *w_slot = mw->in1;
    if (!const_slot(c, *eps_slot, 1) || !const_slot(c, *w_slot, H)) {
        m.fail("norm constants missing");
        return -1;
    }
    return mw->out_slot;
}

// RoPE of the template (kllm_compile.c:1172-1203).
int match_rope(Matcher &m, int x, int cos_b, int sin_b, int heads, int hd) {
    int half = hd / 2;
    int x1 = m.slice(x, {0, 0, 0}, {heads, 1, half});
    int x2 = m.slice(x, {0, 0, half}, {heads, 1, half});
    int ng = m.unary(10, x2);
    int rot = m.concat2(ng, x1, 2);
    int xc = m.binop(7, x, cos_b);
    int rs = m.binop(7, rot, sin_b);
    return m.binop(5, xc, rs);
}

}  // namespace

static bool match_template(const TapeCtx *ctx, const PlanDesc &d, TemplateInfo *ti,
                           std::string *why) {
    Matcher m{ctx};
    TemplateInfo &t = *ti;
    t.H = d.hidden;
    t.hd = d.head_dim;
    t.nkv = d.n_kv;
    t.V = d.vocab;
    t.L = d.n_layers;
    if (t.H <= 0 || t.hd <= 0 || (t.hd & 1) || t.nkv <= 0 || t.V <= 0 || t.L <= 0) {
        *why = "machine dimensions invalid";
        return false;
    }
    int cos_b = -1, sin_b = -1;
    {
        const TapeInstr *c1 = m.next(23);
        if (c1 && c1->in0 != d.cos_slot) m.fail("cos broadcast copy");
        if (c1) cos_b = c1->out_slot;
        const TapeInstr *c2 = m.next(23);
        if (c2 && c2->in0 != d.sin_slot) m.fail("sin broadcast copy");
        if (c2) sin_b = c2->out_slot;
    }
    int h = d.embed_slot;
    for (int l = 0; l < t.L && m.why.empty(); l++) {
        LayerSlots ls;
        int xn = match_norm(m, ctx, h, t.H, &ls.ln1, &ls.eps1);
        int qkv = m.matmul_tt(xn, t.H, &ls.qkv);
        if (!m.why.empty()) break;
        int nq = ctx->slots[ls.qkv].tt_N;
        if (l == 0) {
            int qd = nq - 2 * t.nkv * t.hd;
            if (qd <= 0 || qd % t.hd) {
                m.fail("QKV width does not split into heads");
                break;
            }
            t.nh = qd / t.hd;
            if (t.nh % t.nkv) {
                m.fail("query heads not a multiple of KV heads");
                break;
            }
            t.groups = t.nh / t.nkv;
        }
        int qd = t.nh * t.hd, kvd = t.nkv * t.hd;
        if (nq != qd + 2 * kvd) {
            m.fail("QKV width differs between layers");
            break;
        }
        int q = m.slice(qkv, {0, 0}, {1, qd});
        int k = m.slice(qkv, {0, qd}, {1, kvd});
        int v = m.slice(qkv, {0, qd + kvd}, {1, kvd});
        q = m.reshape(q, {1, t.nh, t.hd});
        q = m.transpose(q, 1, 0, 2);
        k = m.reshape(k, {1, t.nkv, t.hd});
        k = m.transpose(k, 1, 0, 2);
        v = m.reshape(v, {1, t.nkv, t.hd});
        v = m.transpose(v, 1, 0, 2);
        q = match_rope(m, q, cos_b, sin_b, t.nh, t.hd);
        k = match_rope(m, k, cos_b, sin_b, t.nkv, t.hd);
        int kf = m.concat2(d.kv_in[2 * l], k, 1);
        int vf = m.concat2(d.kv_in[2 * l + 1], v, 1);
        if (m.why.empty() && (kf != d.kv_out[2 * l] || vf != d.kv_out[2 * l + 1])) {
            m.fail("KV outputs differ from the slot map");
            break;
        }
        int ke = kf, ve = vf;
        if (t.groups > 1) {
            ke = m.repeat(kf, t.groups, 0);
            ve = m.repeat(vf, t.groups, 0);
        }
        int kt = m.transpose(ke, 0, 2, 1);
        int sc = m.matmul(q, kt);
        const TapeInstr *scl = m.binop_any(7, sc);
        if (!scl) break;
        if (t.scale < 0) t.scale = scl->in1;
        if (scl->in1 != t.scale || !const_slot(ctx, t.scale, 1)) {
            m.fail("attention scale constant");
            break;
        }
        int mx = m.reduce(15, scl->out_slot, 2);
        int sub = m.binop(6, scl->out_slot, mx);
        int ex = m.unary(1, sub);
        int sm = m.reduce(14, ex, 2);
        int aw = m.binop(8, ex, sm);
        int cx = m.matmul(aw, ve);
        cx = m.transpose(cx, 1, 0, 2);
        cx = m.reshape(cx, {1, qd});
        int at = m.matmul_tt(cx, qd, &ls.o);
        int h1 = m.binop(5, h, at);
        int xn2 = match_norm(m, ctx, h1, t.H, &ls.ln2, &ls.eps2);
        int gu = m.matmul_tt(xn2, t.H, &ls.gu);
        if (!m.why.empty()) break;
        int F2 = ctx->slots[ls.gu].tt_N;
        if (F2 % 2) {
            m.fail("gate_up width is odd");
            break;
        }
        if (l == 0) t.F = F2 / 2;
        if (F2 != 2 * t.F) {
            m.fail("gate_up width differs between layers");
            break;
        }
        int g = m.slice(gu, {0, 0}, {1, t.F});
        int u = m.slice(gu, {0, t.F}, {1, t.F});
        int ga = m.unary(0, g);
        int gd = m.binop(7, ga, u);
        int dn = m.matmul_tt(gd, t.F, &ls.dn);
        if (m.why.empty() && ctx->slots[ls.o].tt_N != t.H) m.fail("O projection width");
        if (m.why.empty() && ctx->slots[ls.dn].tt_N != t.H) m.fail("down projection width");
        h = m.binop(5, h1, dn);
        t.layers.push_back(ls);
    }
    if (m.why.empty()) {
        int xn = match_norm(m, ctx, h, t.H, &t.fln, &t.feps);
        int lg = m.matmul_tt(xn, t.H, &t.lm);
        if (m.why.empty() && (lg != d.logits_slot || ctx->slots[t.lm].tt_N != t.V))
            m.fail("logits slot / vocabulary width");
        if (m.why.empty() && m.pc != ctx->n_instrs) m.fail("tape continues after the logits");
    }
    if (!m.why.empty()) {
        *why = m.why;
        return false;
    }
    return true;
}

// ============================================================= kernels ===

// Attention for one query head (kllm_compile.c:1216-1343 after the QKV
// projection): ordered chunk sums of the QKV partials, RoPE of q and k,
// append of k/v at `pos` (by the first query head of each KV group),
// scores q.k_j * scale over positions 0..pos, max-subtracted exp in double,
// sum, divide, and the weighted sum of V.
template <int HD, int THREADS>
__global__ void __launch_bounds__(THREADS)
k_attention(const StepState *st, const float *__restrict__ qkv_part, int T, int nq,
            const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
            float *__restrict__ kc, float *__restrict__ vc, int max_pos, int groups, int nkv,
            float scale, float *__restrict__ ctx_out) {
    static_assert(HD % 32 == 0 && THREADS % HD == 0, "head_dim layout");
    constexpr int DPL = HD / 32;          // dims per lane in the score loop
    constexpr int NG = THREADS / HD;      // position groups in the V loop
    extern __shared__ float sc[];         // [pos + 1] scores / weights
    __shared__ float q[HD], k[HD], v[HD], red[THREADS / 32], part_ctx[NG][HD];
    __shared__ float s_max, s_sum;
    pdl_launch_dependents();
    pdl_wait();
    const int hq = blockIdx.x, g = hq / groups, tid = threadIdx.x;
    const int pos = st->pos;
    if (pos >= max_pos) return;   // the host never launches past the KV capacity
    const int qd = gridDim.x * HD, kvd = nkv * HD;
    for (int i = tid; i < 3 * HD; i += THREADS) {
        int which = i / HD, d = i % HD;
        int col = which == 0 ? hq * HD + d : (which == 1 ? qd + g * HD + d : qd + kvd + g * HD + d);
        (which == 0 ? q : which == 1 ? k : v)[d] = sum_parts(qkv_part + col, nq, T);
    }
    __syncthreads();
    // RoPE: x*cos + rotate_half(x)*sin, rotate_half = concat(-x2, x1)
    float qr = 0.f, kr = 0.f;
    if (tid < HD) {
        const float c = rope_cos[(size_t)pos * HD + tid], s = rope_sin[(size_t)pos * HD + tid];
        const int half = HD / 2;
        float rq = tid < half ? -q[tid + half] : q[tid - half];
        float rk = tid < half ? -k[tid + half] : k[tid - half];
        qr = __fadd_rn(__fmul_rn(q[tid], c), __fmul_rn(rq, s));
        kr = __fadd_rn(__fmul_rn(k[tid], c), __fmul_rn(rk, s));
    }
    __syncthreads();
    if (tid < HD) {
        q[tid] = qr;
        k[tid] = kr;
        if (hq % groups == 0) {
            size_t o = ((size_t)g * max_pos + pos) * HD + tid;
            kc[o] = kr;
            vc[o] = v[tid];
        }
    }
    __syncthreads();
    // scores: one warp per position, DPL dims per lane, xor-tree sum
    const int warp = tid >> 5, lane = tid & 31;
    float qv[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) qv[i] = q[lane + 32 * i];
    for (int j = warp; j <= pos; j += THREADS / 32) {
        const float *kj = j == pos ? k : kc + ((size_t)g * max_pos + j) * HD;
        float dot = __fmul_rn(qv[0], kj[lane]);
#pragma unroll
        for (int i = 1; i < DPL; i++) dot = __fadd_rn(dot, __fmul_rn(qv[i], kj[lane + 32 * i]));
        for (int o = 16; o; o >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
        if (lane == 0) sc[j] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = tid; j <= pos; j += THREADS) m = fmaxf(m, sc[j]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int i = 1; i < THREADS / 32; i++) mm = fmaxf(mm, red[i]);
        s_max = mm;
    }
    __syncthreads();
    const float mx = s_max;
    float sum = 0.f;
    for (int j = tid; j <= pos; j += THREADS) {
        float e = (float)exp((double)__fsub_rn(sc[j], mx));
        sc[j] = e;
        sum = __fadd_rn(sum, e);
    }
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        float ss = red[0];
        for (int i = 1; i < THREADS / 32; i++) ss = __fadd_rn(ss, red[i]);
        s_sum = ss;
    }
    __syncthreads();
    const float tot = s_sum;
    for (int j = tid; j <= pos; j += THREADS) sc[j] = __fdiv_rn(sc[j], tot);
    __syncthreads();
    // ctx[d] = sum_j p_j * v_j[d]: NG position groups per dim
    const int d = tid % HD, grp = tid / HD;
    float acc = 0.f;
    for (int j = grp; j <= pos; j += NG) {
        float vj = j == pos ? v[d] : vc[((size_t)g * max_pos + j) * HD + d];
        acc = __fadd_rn(acc, __fmul_rn(sc[j], vj));
    }
    part_ctx[grp][d] = acc;
    __syncthreads();
    if (tid < HD) {
        float a = part_ctx[0][tid];
        for (int i = 1; i < NG; i++) a = __fadd_rn(a, part_ctx[i][tid]);
        ctx_out[hq * HD + tid] = a;
    }
}

// ================================================================ plan ===

struct DecodePlan {
    TemplateInfo ti;
    int max_pos = 0;
    int T_h = 0, T_qd = 0, T_f = 0;   // chunk counts by K
    const float *src_embed = nullptr;
    const float *src_cos = nullptr, *src_sin = nullptr;
    // device state
    float *embed = nullptr, *rcos = nullptr, *rsin = nullptr;
    float *h = nullptr, *qkv = nullptr, *ctx = nullptr, *act = nullptr, *logits = nullptr;
    float *part = nullptr;          // [T][N] chunk partials, shared by the GEMVs
    int *counters = nullptr;        // column-block arrival counters (zero at rest)
    float *kc = nullptr, *vc = nullptr;
    float *cand_v = nullptr;
    int *cand_i = nullptr;
    StepState *st = nullptr;
    int *prompt = nullptr, *gen = nullptr, *status = nullptr;
    int *gen_host = nullptr;   // mapped pinned
    int *gen_host_dev = nullptr;
    float *hist = nullptr;
    int hist_rows = 0;
    std::vector<float> norm_w;   // not used on device; kept for checks
    std::vector<float *> dev_norm;
    std::vector<float> eps;
    float scale = 0.f, f_eps = 0.f;
    std::vector<CUtensorMap> maps;   // per layer: qkv, o, gu, dn ; then lm
    std::vector<TFConfig> cfgs;      // launch geometry per map
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    float *graph_hist = nullptr;   // history buffer baked into the graph
    // persistent step kernel
    bool persist = false;
    int order = 0;                 // KLLM_ORDER_* the layouts were built for
    int task_warps = 8;            // consumer warps taking GEMV tasks
    int vm = TTX_VSLOT;            // what the device streams hold (TTXVals)
    int ds_grid = 0, ds_stages = 0;
    size_t ds_smem = 0;
    DSArgs ds = {};
    std::vector<DSPhase> phases;
    DSPhase *d_phases = nullptr;
    int *d_cnt = nullptr;          // done[phases] then the epoch (zero only when built)
    size_t cnt_n = 0;
    int *d_abort = nullptr;
    std::vector<void *> ds_bufs;   // device layouts, partials, activations
    std::vector<std::pair<void *, size_t>> ll_bufs;   // tagged activations (zeroed on reset)
    // column shard: every rank's copy of the shared buffers ([kind][rank])
    int rank = 0, world = 1;
    bool connected = false;
    std::vector<void *> peer_host;   // host copy of the table
    void **d_peers = nullptr;
    std::vector<void *> opened;      // peers' buffers mapped into this process
    long long kernels_per_step = 0;
    int graph_hist_rows = 0;
    int logits_slot = -1;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr;
    std::vector<cudaEvent_t> step_ev;
    // batched prompt pass: activation arena, grown to the longest prompt seen
    float *pf_arena = nullptr;
    size_t pf_cap = 0;   // floats
    // tensor-core projections: per layer the bf16 weights transposed
    // ([N][K], 4 per layer: qkv, o, gate_up, down), built at the first pass
    std::vector<void *> pf_wt;
    bool pf_wt_tried = false;
    int pf_terms = 0;    // bf16 terms of x (0: the exact FP32 TT-GEMM)
    // batched decode of several sequences: caches and rows, grown as needed
    float *bd_arena = nullptr;
    size_t bd_cap = 0;   // floats
    void *bd_lm_wt = nullptr;   // lm_head as bf16 Wt (tensor-core batches)
#ifdef KLLM_DS_PROFILE
    unsigned long long *prof = nullptr;   // step timestamps (profiling build)
    size_t prof_n = 0;
#endif
};

static void free_plan(DecodePlan *p) {
    if (!p) return;
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    void *bufs[] = {p->embed, p->rcos, p->rsin, p->h, p->qkv, p->ctx, p->act, p->logits,
                    p->part, p->counters, p->kc, p->vc, p->cand_v, p->cand_i,
                    p->st, p->prompt, p->gen, p->status, p->hist, p->pf_arena, p->bd_arena,
                    p->bd_lm_wt
#ifdef KLLM_DS_PROFILE
                    , p->prof
#endif
    };
    for (void *b : bufs)
        if (b) cudaFree(b);
    for (float *b : p->dev_norm)
        if (b) cudaFree(b);
    for (void *b : p->ds_bufs)
        if (b) cudaFree(b);
    for (void *b : p->pf_wt)
        if (b) cudaFree(b);
    for (void *b : p->opened)
        if (b) cudaIpcCloseMemHandle(b);
    for (void *b : {(void *)p->d_phases, (void *)p->d_cnt, (void *)p->d_abort, (void *)p->d_peers})
        if (b) cudaFree(b);
    if (p->gen_host) cudaFreeHost(p->gen_host);
    for (cudaEvent_t e : {p->ev0, p->ev1, p->ev2})
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : p->step_ev) cudaEventDestroy(e);
    delete p;
}

void plan_kind(const CtxImpl *c, int *persist, int *values) {
    const DecodePlan *p = c->plan;
    *persist = p && p->persist ? 1 : 0;
    *values = p && p->persist ? p->vm : 0;
}

void plan_destroy(CtxImpl *c) {
    if (c->plan) {
        cudaSetDevice(c->device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        free_plan(c->plan);
    }
    c->plan = nullptr;
}

template <class T>
static bool dalloc(T **p, size_t n) {
    return KLLM_CUDA(cudaMalloc((void **)p, std::max<size_t>(n, 1) * sizeof(T)));
}

// Persistent step kernel: phase list, tensor maps with each phase's box,
// scratch, shared-memory layout and co-residency check.  Returns false (no
// error recorded) when the kernel cannot be used; the per-kernel plan stays.
static bool env_on(const char *name, bool dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    return *v != '0';
}

typedef void (*DSKernel)(const DSArgs);

template <int HD>
static DSKernel ds_kernel_hd(int vm) {
    return vm == TTX_VBF16 ? k_decode_step<HD, TTX_VBF16>
         : vm == TTX_VF16  ? k_decode_step<HD, TTX_VF16>
                           : k_decode_step<HD, TTX_VSLOT>;
}

static DSKernel ds_kernel(int hd, int vm) {
    return hd == 32 ? ds_kernel_hd<32>(vm) : hd == 64 ? ds_kernel_hd<64>(vm) : ds_kernel_hd<128>(vm);
}

static bool persist_prepare(CtxImpl *c, DecodePlan *p, const std::vector<int> &tts) {
    if (!env_on("KLLM_PERSIST", true)) return false;
    const TapeCtx *ctx = &c->base;
    const TemplateInfo &t = p->ti;
    if (t.hd != 32 && t.hd != 64 && t.hd != 128) return false;   // the step kernel's instances
    const int H = t.H, hd = t.hd, nkv = t.nkv, qd = t.nh * hd, kvd = nkv * hd;
    const int V = t.V, L = t.L;
    const int nmat = (int)tts.size();
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device);
    // Value streams when every codebook holds only bf16 (or only fp16)
    // numbers -- the compiler's codebooks of bf16 / fp16 checkpoints; table
    // slots otherwise.  KLLM_TTX_VALUES=slot keeps the slot streams.
    unsigned modes = (1u << TTX_VBF16) | (1u << TTX_VF16);
    {
        for (int ti : tts) {   // the host codebooks the device copies were made from
            const Slot &sl = ctx->slots[ti];
            modes &= ttx_value_modes(sl.codebook, sl.n_codes);
            if (!modes) break;
        }
        const char *e = getenv("KLLM_TTX_VALUES");
        if (e && !strcmp(e, "slot")) modes = 0;
    }
    const int vm = modes & (1u << TTX_VBF16) ? TTX_VBF16 : modes & (1u << TTX_VF16) ? TTX_VF16 : TTX_VSLOT;
    p->vm = vm;
    // GEMV task warps per CTA (KLLM_TASK_WARPS, 1..8)
    p->task_warps = 6;
    if (const char *e = getenv("KLLM_TASK_WARPS")) p->task_warps = std::max(1, std::min(DS_NCW, atoi(e)));
    auto kern = ds_kernel(hd, vm);
    cudaFuncAttributes fa = {};
    if (!KLLM_CUDA(cudaFuncGetAttributes(&fa, kern))) return false;
    int smem_optin = 0;
    cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device);
    const size_t avail = (size_t)smem_optin - fa.sharedSizeBytes;
    // device layouts (ttx.cuh), one per matrix
    // two tables (this phase's and the next's), R <= 2 copies each
    int max_r = 2;
    if (const char *e = getenv("KLLM_TTX_R")) max_r = std::max(1, std::min(4, atoi(e)));
    const int max_table = 48 * 1024;
    std::vector<TTXDesc> desc(nmat);
    std::vector<uint8_t *> streams(nmat);
    std::vector<float *> tables(nmat);
    std::vector<int> xsz(nmat), groups_all(nmat);
    const int rank = c->shard_rank, world = c->shard_world;
    int tab_cap = 0, xc_cap = (p->max_pos + 3) & ~3;
    auto own = [&](void *b) { p->ds_bufs.push_back(b); };
    for (int i = 0; i < nmat; i++) {
        const Slot &sl = ctx->slots[tts[i]];
        const DevSlot &w = c->ds[tts[i]];
        const int role = i + 1 == nmat ? 4 : i % 4;   // 0 qkv 1 o 2 gate_up 3 down 4 lm_head
        const int mode = role == 0 ? TTX_ROPE : role == 2 ? TTX_GATE_UP : TTX_IDENT;
        // fast order: split a group over W warps while the phase still fits
        // one round of warp tasks (decode tolerance instead of bit-exact sums)
        int W = 1;
        if (p->order == KLLM_ORDER_FAST) {
            const int ng =
                ((mode == TTX_GATE_UP ? (sl.tt_N / 2 + 3) / 4 : (sl.tt_N + 7) / 8) + world - 1) / world;
            while (W < 8 && 2 * W <= p->task_warps &&
                   (long long)ng * 2 * W <= (long long)sms * p->task_warps &&
                   sl.tt_K % (16 * 8 * W) == 0)
                W *= 2;
        }
        if (!ttx_describe(sl.tt_K, sl.tt_N, sl.n_codes, mode, vm, hd, t.nh + nkv, max_table, max_r,
                          W, &desc[i]))
            return false;
        groups_all[i] = desc[i].ngroups;
        if (c->shard_world > 1) ttx_shard(&desc[i], c->shard_rank, c->shard_world);
        const TTXDesc &d = desc[i];
        if (!KLLM_CUDA(cudaMalloc((void **)&streams[i], d.stream_bytes()))) return false;
        own(streams[i]);
        tables[i] = nullptr;
        if (d.table_elems()) {
            if (!KLLM_CUDA(cudaMalloc((void **)&tables[i], d.table_elems() * 4))) return false;
            own(tables[i]);
        }
        if (!ttx_build(c->stream, w.d_idx, w.d_cb, d, streams[i], tables[i])) return false;
        tab_cap = std::max(tab_cap, (int)d.table_elems());
        // staged x: chunk rows of 8 * ns floats, padded to 4 mod 32 floats so
        // that the 8 chunks' float4 reads fall in different banks
        const int r8 = 8 * d.ns;
        xsz[i] = r8 + ((4 - r8 % 32) + 32) % 32;
        xc_cap = std::max(xc_cap, d.T * xsz[i]);
    }
    if (!KLLM_CUDA(cudaStreamSynchronize(c->stream))) return false;
    // shared memory: ring | 2 tables | 2 norm weight vectors | staged x
    // (attention scores alias it) | saved raw x | mbarriers
    if (H % 4) return false;   // norm weights arrive by bulk copy
    xc_cap = (xc_cap + 3) & ~3;
    const int wn_cap = (H + 3) & ~3;
    const size_t fixed = (size_t)4 * (2 * tab_cap + 3 * wn_cap + xc_cap) + 8 * 5 + 16;
    if (avail <= fixed + 2 * ((size_t)DS_STAGE + 16)) return false;
    const int S = (int)std::min<size_t>(DS_MAX_STAGES, (avail - fixed) / (DS_STAGE + 20));
    const size_t smem = (size_t)S * DS_STAGE + fixed + (size_t)8 * (2 * S) + (size_t)4 * S;
    if (S < 2 || smem > avail) return false;
    if (!KLLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem)))
        return false;
    int per_sm = 0;
    if (!KLLM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, DS_THREADS, smem)) ||
        per_sm < 1)
        return false;
    // tagged activations (one allocation each: each is a peer buffer);
    // zero tags never match a step's (ds_tag >= 256)
    auto llbuf = [&](size_t n) -> ll_t * {
        ll_t *b = nullptr;
        const size_t bytes = std::max<size_t>(n, 1) * sizeof(ll_t);
        if (!KLLM_CUDA(cudaMalloc((void **)&b, bytes)) || !KLLM_CUDA(cudaMemset(b, 0, bytes)))
            return nullptr;
        own(b);
        p->ll_bufs.push_back({b, bytes});
        return b;
    };
    ll_t *qb = llbuf(qd), *act = llbuf(t.F), *hA = llbuf(H), *hB = llbuf(H);
    ll_t *kn = llbuf(kvd), *vn = llbuf(kvd), *ctxl = llbuf(qd);
    if (!qb || !act || !hA || !hB || !kn || !vn || !ctxl) return false;
    // Split attention for long contexts: up to att_spmax CTAs per head
    // (KLLM_ATT_SPLITS; default the CTAs per head the grid allows, at most
    // 8), one more split every KLLM_ATT_SPLIT_MIN positions (default 256).
    int att_spmax = std::max(1, std::min(8, sms / std::max(1, t.nh)));
    if (const char *e = getenv("KLLM_ATT_SPLITS")) att_spmax = std::max(1, std::min(8, atoi(e)));
    if (att_spmax * t.nh > sms) att_spmax = std::max(1, sms / t.nh);
    int att_split_min = 256;
    if (const char *e = getenv("KLLM_ATT_SPLIT_MIN")) att_split_min = std::max(16, atoi(e));
    if (p->max_pos <= att_split_min) att_spmax = 1;
    ll_t *att_part = llbuf((size_t)att_spmax * qd), *att_ml = llbuf((size_t)att_spmax * t.nh * 2);
    if (!att_part || !att_ml) return false;
    if (L > 255) return false;   // ds_tag keeps the layer in 8 bits
    if ((size_t)sms * world > 4096) return false;   // lm_head candidates, one per CTA and rank
    // phases
    std::vector<DSPhase> ph;
    // The residual epilogues of O and down read the raw x that the same CTA
    // staged for QKV and gate_up: every CTA with O (down) work must have
    // QKV (gate_up) work.
    auto local_groups = [&](int mi) {
        return rank < groups_all[mi] ? (groups_all[mi] - rank + world - 1) / world : 0;
    };
    for (int l = 0; l < L; l++)
        if (std::min(sms, local_groups(4 * l + 1)) > std::min(sms, local_groups(4 * l)) ||
            std::min(sms, local_groups(4 * l + 3)) > std::min(sms, local_groups(4 * l + 2)))
            return false;
    // KLLM_COL_SPLIT: 0 never, 1 (default) phases with few groups per CTA,
    // 2 every phase of the reference order
    int split_mode = 1;
    if (const char *e = getenv("KLLM_COL_SPLIT")) split_mode = std::max(0, std::min(2, atoi(e)));
    auto gemv = [&](int mi, int xmode, const ll_t *x, const float *nw, float eps, int emode,
                    int save_x, float *out, int out_kind, int layer, int x_layer) {
        const TTXDesc &d = desc[mi];
        DSPhase m = {};
        m.kind = DS_GEMV;
        m.ntasks = d.ngroups;
        m.d = d;
        m.npieces = (d.ns + DS_PIECE_STEPS - 1) / DS_PIECE_STEPS;
        m.xs = xsz[mi];
        m.lmagic = (unsigned)((((unsigned long long)1 << 32) + d.base - 1) / d.base);
        m.stream = streams[mi];
        m.table = tables[mi];
        m.table_bytes = (int)(d.table_elems() * 4);
        m.xmode = xmode;
        m.emode = emode;
        m.x = x;
        m.norm_w = nw;
        m.eps = eps;
        m.x_layer = x_layer;
        m.save_x = save_x;
        m.out = out;
        m.out_kind = out_kind;
        m.groups_all = groups_all[mi];
        m.layer = layer;
        // a group's two columns per lane on two warps when the phase has few
        // groups per CTA (the reference order per column is unchanged)
        const int per_cta = (d.ngroups + sms - 1) / sms * d.W;
        m.csplit = split_mode && d.W == 1 &&
                           (split_mode == 2 || (emode != DE_LM && 2 * per_cta <= p->task_warps))
                       ? 2
                       : 1;
        ph.push_back(m);
        return (int)ph.size() - 1;
    };
    // Each phase reads its input words with the tag of the layer that wrote
    // them: QKV of layer l the residual of down l-1 (layer 0: the embedding
    // row), attention and the rest of layer l the outputs of layer l.
    for (int l = 0; l < L; l++) {
        const int mq = 4 * l;
        gemv(mq, l == 0 ? DX_EMBED : DX_NORM, l == 0 ? nullptr : hA, p->dev_norm[2 * l],
             p->eps[2 * l], DE_QKV, 1, nullptr, DSP_Q, l, l - 1);
        DSPhase at = {};
        at.kind = DS_ATT;
        at.ntasks = t.nh * att_spmax;   // task tk: head tk % nh, split tk / nh
        at.layer = l;
        ph.push_back(at);
        gemv(mq + 1, DX_ATT, ctxl, nullptr, 0.f, DE_RESID, 0, nullptr, DSP_HB, l, l);
        gemv(mq + 2, DX_NORM, hB, p->dev_norm[2 * l + 1], p->eps[2 * l + 1], DE_SWIGLU, 1, nullptr,
             DSP_ACT, l, l);
        gemv(mq + 3, DX_VEC, act, nullptr, 0.f, DE_RESID, 0, nullptr, DSP_HA, l, l);
    }
    gemv(nmat - 1, DX_NORM, hA, p->dev_norm.back(), p->f_eps, DE_LM, 0, p->logits, DSP_LOGITS, L,
         L - 1);
    const size_t nph = ph.size();
    p->cnt_n = nph + 2;   // done[phases], epoch, this rank's lm_head arrivals
    if (!KLLM_CUDA(cudaMalloc((void **)&p->d_cnt, p->cnt_n * sizeof(int))) ||
        !KLLM_CUDA(cudaMemset(p->d_cnt, 0, p->cnt_n * sizeof(int))) ||
        !KLLM_CUDA(cudaMalloc((void **)&p->d_phases, nph * sizeof(DSPhase))) ||
        !KLLM_CUDA(cudaMemcpy(p->d_phases, ph.data(), nph * sizeof(DSPhase),
                              cudaMemcpyHostToDevice)) ||
        !KLLM_CUDA(cudaMalloc((void **)&p->d_abort, sizeof(int))) ||
        !KLLM_CUDA(cudaMemset(p->d_abort, 0, sizeof(int))))
        return false;
    p->phases = ph;
    // this rank's shared buffers; the other ranks' arrive with shard_connect
    p->rank = rank;
    p->world = world;
    p->peer_host.assign((size_t)DSP_KINDS * world, nullptr);
    {
        void *mine[DSP_KINDS] = {qb, p->kc, p->vc, hA, hB, act, p->logits, p->cand_v, p->cand_i,
                                 kn, vn, p->d_cnt};
        for (int k = 0; k < DSP_KINDS; k++) p->peer_host[(size_t)k * world + rank] = mine[k];
    }
    if (!KLLM_CUDA(cudaMalloc((void **)&p->d_peers, p->peer_host.size() * sizeof(void *))) ||
        !KLLM_CUDA(cudaMemcpy(p->d_peers, p->peer_host.data(), p->peer_host.size() * sizeof(void *),
                              cudaMemcpyHostToDevice)))
        return false;
    p->connected = world == 1;
    DSArgs &a = p->ds;
    a.phases = p->d_phases;
    a.nphases = (int)nph;
    a.done = p->d_cnt;
    a.epoch = p->d_cnt + nph;
    a.lm_local = p->d_cnt + nph + 1;
    a.status = p->status;
    a.abort = p->d_abort;
    a.stages = S;
    a.tab_cap = tab_cap;
    a.wn_cap = wn_cap;
    a.xc_cap = xc_cap;
    a.st = p->st;
    a.embed = p->embed;
    a.prompt = p->prompt;
    a.gen = p->gen;
    a.gen_host = (volatile int *)p->gen_host_dev;
    a.vocab = V;
    a.max_gen = p->max_pos;
    a.H = H;
    a.q = qb;
    a.nh = t.nh;
    a.nkv = nkv;
    a.groups = t.groups;
    a.max_pos = p->max_pos;
    a.qd = qd;
    a.kvd = kvd;
    a.rope_cos = p->rcos;
    a.rope_sin = p->rsin;
    a.kc = p->kc;
    a.vc = p->vc;
    a.scale = p->scale;
    a.ctx = ctxl;
    a.cand_v = p->cand_v;
    a.cand_i = p->cand_i;
    a.rank = rank;
    a.world = world;
    a.peers = p->d_peers;
#ifdef KLLM_DS_PROFILE
    {
        const size_t n = (size_t)sms * nph * 16;
        if (!dalloc(&p->prof, n) || !KLLM_CUDA(cudaMemset(p->prof, 0, n * 8))) return false;
        p->prof_n = n;
        a.prof = p->prof;
        const char *e = getenv("KLLM_PROF_POS");
        a.prof_pos = e ? atoi(e) : 100;
    }
#endif
    // every device wait of the step gives up after this long (default 2 s);
    // KLLM_WAIT_LIMIT_MS shortens it, e.g. for a test that makes one run out
    a.wait_ns = kWaitLimitNs;
    if (const char *e = getenv("KLLM_WAIT_LIMIT_MS")) {
        const long long ms = atoll(e);
        if (ms > 0 && ms <= 60000) a.wait_ns = (unsigned long long)ms * 1000000ull;
    }
    a.task_warps = p->task_warps;
    a.kv_prefetch = env_on("KLLM_KV_PREFETCH", true) ? 1 : 0;
    a.gpu_scope = env_on("KLLM_GPU_SCOPE", true) ? 1 : 0;
    a.unroll = env_on("KLLM_UNROLL", true) ? 1 : 0;
    a.att_part = att_part;
    a.att_ml = att_ml;
    a.att_spmax = att_spmax;
    a.att_split_min = att_split_min;
    a.l2_pf = 0;
    if (const char *e = getenv("KLLM_L2_PREFETCH")) a.l2_pf = std::max(0, std::min(512, atoi(e)));
    p->ds_grid = sms;
    p->ds_stages = S;
    p->ds_smem = smem;
    p->persist = true;
    return true;
}

// Column shard: IPC handles of this rank's shared buffers, in DSPeer order.
bool plan_shard_export(CtxImpl *c, void *out, size_t cap, size_t *len) {
    DecodePlan *p = c->plan;
    const size_t need = (size_t)DSP_KINDS * sizeof(cudaIpcMemHandle_t);
    if (len) *len = need;
    if (!p || !p->persist) {
        set_error("kllm_shard_export: no fused decode plan (prepare it first)");
        return false;
    }
    if (!out && cap == 0) return true;   // size query
    if (!out || cap < need) {
        set_error("kllm_shard_export: buffer of %zu bytes, %zu needed", cap, need);
        return false;
    }
    cudaSetDevice(c->device);
    for (int k = 0; k < DSP_KINDS; k++) {
        cudaIpcMemHandle_t h;
        if (!KLLM_CUDA(cudaIpcGetMemHandle(&h, p->peer_host[(size_t)k * p->world + p->rank])))
            return false;
        memcpy(static_cast<char *>(out) + k * sizeof h, &h, sizeof h);
    }
    return true;
}

// Map every other rank's shared buffers (world blocks of the export format,
// rank order) and publish the full table to the kernel.
bool plan_shard_connect(CtxImpl *c, const void *all, size_t per_rank) {
    DecodePlan *p = c->plan;
    if (!p || !p->persist) {
        set_error("kllm_shard_connect: no fused decode plan (prepare it first)");
        return false;
    }
    if (!all || per_rank < (size_t)DSP_KINDS * sizeof(cudaIpcMemHandle_t)) {
        set_error("kllm_shard_connect: malformed handle block");
        return false;
    }
    if (p->connected) return true;
    cudaSetDevice(c->device);
    for (int r = 0; r < p->world; r++) {
        if (r == p->rank) continue;
        for (int k = 0; k < DSP_KINDS; k++) {
            cudaIpcMemHandle_t h;
            memcpy(&h, static_cast<const char *>(all) + r * per_rank + k * sizeof h, sizeof h);
            void *ptr = nullptr;
            if (!KLLM_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess)))
                return false;
            p->opened.push_back(ptr);
            p->peer_host[(size_t)k * p->world + r] = ptr;
        }
    }
    if (!KLLM_CUDA(cudaMemcpy(p->d_peers, p->peer_host.data(), p->peer_host.size() * sizeof(void *),
                              cudaMemcpyHostToDevice)))
        return false;
    p->connected = true;
    return true;
}

bool plan_match(const TapeCtx *ctx, const PlanDesc &d, std::string *why) {
    TemplateInfo ti;
    return match_template(ctx, d, &ti, why);
}

// The summation order a plan is built with: the fast order (groups split
// over W warps) only on one GPU; a column-sharded context always runs the
// reference order.  (A 2-GPU test of the fast order on a sharded context ran
// past its time limit without a fault; until its cause is found that
// combination is not built.)
static int plan_order(const CtxImpl *c) {
    return c->shard_world > 1 ? KLLM_ORDER_EXACT : c->opts.order;
}

bool plan_prepare(CtxImpl *c, const PlanDesc &d, int max_pos, std::string *why) {
    TapeCtx *ctx = &c->base;
    DecodePlan *old = c->plan;
    if (old && old->max_pos >= max_pos && old->src_embed == d.embed &&
        old->src_cos == d.rope_cos && old->src_sin == d.rope_sin && old->ti.H == d.hidden &&
        old->ti.V == d.vocab && old->order == plan_order(c) && old->rank == c->shard_rank &&
        old->world == c->shard_world) {
        return true;   // reuse (weights are re-checked by upload_tt below)
    }
    TemplateInfo ti;
    if (!match_template(ctx, d, &ti, why)) return false;
    if (ti.hd != 32 && ti.hd != 64 && ti.hd != 128) {
        *why = "head_dim " + std::to_string(ti.hd) + " (fused attention covers 32, 64, 128)";
        return false;
    }
    if ((size_t)max_pos * 4 > 160 * 1024) {
        *why = "context longer than the fused attention's score buffer";
        return false;
    }
    static bool att_attr[64] = {};
    if (!att_attr[c->device & 63]) {
        for (auto f : {k_attention<32, 256>, k_attention<64, 256>, k_attention<128, 256>})
            if (!KLLM_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                160 * 1024)))
                return false;
        att_attr[c->device & 63] = true;
    }
    plan_destroy(c);
    DecodePlan *p = new DecodePlan();
    p->ti = ti;
    p->order = plan_order(c);
    if (p->order != c->opts.order && env_on("KLLM_VERBOSE", false))
        fprintf(stderr, "kllm: column-sharded decode runs the reference summation order\n");
    p->max_pos = max_pos;
    p->src_embed = d.embed;
    p->src_cos = d.rope_cos;
    p->src_sin = d.rope_sin;
    p->logits_slot = d.logits_slot;
    const int H = ti.H, V = ti.V, L = ti.L, hd = ti.hd, nkv = ti.nkv;
    const int qd = ti.nh * hd, nq = qd + 2 * nkv * hd, F = ti.F;
    p->T_h = tt_chunks(H);
    p->T_qd = tt_chunks(qd);
    p->T_f = tt_chunks(F);
    auto fail = [&]() {
        free_plan(p);
        return false;
    };
    // weights: the context's device copies of the TT slots
    std::vector<int> tts;
    for (auto &ls : ti.layers) tts.insert(tts.end(), {ls.qkv, ls.o, ls.gu, ls.dn});
    tts.push_back(ti.lm);
    for (int s : tts) {
        if (!upload_tt(c, s)) return fail();
        const Slot &sl = ctx->slots[s];
        (void)sl;
    }
    // The per-kernel plan (fallback of the persistent step) reads the
    // index matrices by TMA tiles; the persistent step needs neither.
    std::string tf_why;
    p->maps.resize(tts.size());
    p->cfgs.resize(tts.size());
    for (size_t i = 0; i < tts.size(); i++) {
        const Slot &sl = ctx->slots[tts[i]];
        const int em = (i + 1 == tts.size()) ? E_ARGMAX : (i % 4 == 2 ? E_SWIGLU : E_Y);
        p->cfgs[i] = tf_config(sl.tt_K, sl.tt_N, sl.n_codes, em);
        if (!tf_tma_ok(c->ds[tts[i]].d_idx, c->ds[tts[i]].d_cb, sl.tt_K, sl.tt_N, sl.n_codes,
                       p->cfgs[i]))
            tf_why = "a weight matrix does not meet the TMA alignment rules";
    }
    // the up half of each gate_up tile starts at column F: a TMA x
    // coordinate must be a multiple of 8 uint16
    if (F % 8) tf_why = "intermediate size not a multiple of 8";
    for (size_t i = 0; i < tts.size() && tf_why.empty(); i++) {
        const Slot &sl = ctx->slots[tts[i]];
        if (!make_idx_tmap(&p->maps[i], c->ds[tts[i]].d_idx, sl.tt_K, sl.tt_N,
                           p->cfgs[i].bw(), 32))
            return fail();
    }
    // norm weights and constants
    for (auto &ls : ti.layers) {
        for (int s : {ls.ln1, ls.ln2}) {
            float *dw = nullptr;
            if (!dalloc(&dw, H)) return fail();
            p->dev_norm.push_back(dw);
            if (!KLLM_CUDA(cudaMemcpy(dw, ctx->slots[s].data, (size_t)H * 4,
                                      cudaMemcpyHostToDevice)))
                return fail();
        }
        p->eps.push_back(ctx->slots[ls.eps1].data[0]);
        p->eps.push_back(ctx->slots[ls.eps2].data[0]);
    }
    {
        float *dw = nullptr;
        if (!dalloc(&dw, H)) return fail();
        p->dev_norm.push_back(dw);
        if (!KLLM_CUDA(cudaMemcpy(dw, ctx->slots[ti.fln].data, (size_t)H * 4,
                                  cudaMemcpyHostToDevice)))
            return fail();
        p->f_eps = ctx->slots[ti.feps].data[0];
    }
    p->scale = ctx->slots[ti.scale].data[0];
    // tables
    if (!dalloc(&p->embed, (size_t)V * H) ||
        !KLLM_CUDA(cudaMemcpy(p->embed, d.embed, (size_t)V * H * 4, cudaMemcpyHostToDevice)) ||
        !dalloc(&p->rcos, (size_t)max_pos * hd) || !dalloc(&p->rsin, (size_t)max_pos * hd) ||
        !KLLM_CUDA(cudaMemcpy(p->rcos, d.rope_cos, (size_t)max_pos * hd * 4,
                              cudaMemcpyHostToDevice)) ||
        !KLLM_CUDA(cudaMemcpy(p->rsin, d.rope_sin, (size_t)max_pos * hd * 4,
                              cudaMemcpyHostToDevice)))
        return fail();
    // activations, partials, KV cache, step state
    size_t kv = (size_t)L * nkv * max_pos * hd;
    size_t part_n = std::max({(size_t)p->T_h * nq, (size_t)p->T_qd * H, (size_t)p->T_h * 2 * F,
                              (size_t)p->T_f * H, (size_t)p->T_h * V});
    const int n_cnt = 4096;
    int nblk = 0;
    for (size_t i = 0; i < tts.size(); i++) {
        const Slot &sl = ctx->slots[tts[i]];
        const int em = (i + 1 == tts.size()) ? E_ARGMAX : (i % 4 == 2 ? E_SWIGLU : E_Y);
        nblk = std::max(nblk, tf_blocks(p->cfgs[i], sl.tt_N, sl.tt_N / 2, em));
    }
    if (nblk > 1024 || nblk > n_cnt) tf_why = "too many column blocks for the argmax candidates";
    if (!dalloc(&p->h, H) || !dalloc(&p->qkv, nq) || !dalloc(&p->ctx, qd) ||
        !dalloc(&p->act, F) || !dalloc(&p->logits, V) || !dalloc(&p->part, part_n) ||
        !dalloc(&p->counters, n_cnt) || !dalloc(&p->kc, kv) || !dalloc(&p->vc, kv) ||
        !dalloc(&p->cand_v, 4096) || !dalloc(&p->cand_i, 4096) || !dalloc(&p->st, 1) ||
        !dalloc(&p->prompt, max_pos) || !dalloc(&p->gen, max_pos) || !dalloc(&p->status, 1))
        return fail();
    if (!KLLM_CUDA(cudaMemset(p->kc, 0, kv * 4)) || !KLLM_CUDA(cudaMemset(p->vc, 0, kv * 4)) ||
        !KLLM_CUDA(cudaMemset(p->st, 0, sizeof(StepState))) ||
        !KLLM_CUDA(cudaMemset(p->counters, 0, n_cnt * sizeof(int))))
        return fail();
    if (!KLLM_CUDA(cudaHostAlloc((void **)&p->gen_host, (size_t)max_pos * 4,
                                 cudaHostAllocMapped)) ||
        !KLLM_CUDA(cudaHostGetDevicePointer((void **)&p->gen_host_dev, p->gen_host, 0)))
        return fail();
    if (!KLLM_CUDA(cudaEventCreate(&p->ev0)) || !KLLM_CUDA(cudaEventCreate(&p->ev1)) ||
        !KLLM_CUDA(cudaEventCreate(&p->ev2)))
        return fail();
    if (!persist_prepare(c, p, tts)) {
        // the per-kernel plan remains available; KLLM_VERBOSE=1 says why
        if (env_on("KLLM_VERBOSE", false))
            fprintf(stderr, "kllm: persistent decode step unavailable: %s\n",
                    kllm_last_error() ? kllm_last_error() : "shape or resource limit");
        kllm_clear_error();
        p->persist = false;
        if (!tf_why.empty()) {
            *why = tf_why;
            free_plan(p);
            return false;
        }
    }
    c->plan = p;
    return true;
}

// Programmatic dependent launch (KLLM_PDL=1).  Off by default: measured on
// B200, the early-resident dependent CTAs slowed a decode step from 1.56 ms
// to 2.45 ms (graph replay, TinyLlama-architecture chip).
bool pdl_enabled() {
    static int on = [] {
        const char *v = getenv("KLLM_PDL");
        return v && *v == '1' ? 1 : 0;
    }();
    return on != 0;
}

template <class Kern, class... Args>
static bool launch_pdl(cudaStream_t s, Kern kern, dim3 grid, dim3 block, size_t smem,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    g_launches++;
    return KLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
}

// One tape step as a single cooperative launch (arrival counters cleared
// first).
static bool record_step_persist(CtxImpl *c, DecodePlan *p) {
    if (!p->connected) {
        set_error("column-sharded decode: the ranks' buffers are not connected "
                  "(kllm_shard_export / kllm_shard_connect)");
        return false;
    }
    DSArgs a = p->ds;
    a.hist = p->hist;
    a.hist_rows = p->hist_rows;
    auto kern = ds_kernel(p->ti.hd, p->vm);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->ds_grid);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = p->ds_smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    g_launches++;
    return KLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
}

// All kernels of one tape step, in stream order.
static bool record_step(CtxImpl *c, DecodePlan *p) {
    if (p->persist) return record_step_persist(c, p);
    cudaStream_t s = c->stream;
    const TemplateInfo &t = p->ti;
    const int H = t.H, hd = t.hd, nkv = t.nkv, qd = t.nh * hd, nq = qd + 2 * nkv * hd;
    const int F = t.F, V = t.V;
    const TapeCtx *ctx = &c->base;
    auto gemv = [&](int mi, int w_slot, int K, int N, int xmode, const float *x, int norm_i,
                    float eps, bool embed, int emode, float *y) -> bool {
        const DevSlot &w = c->ds[w_slot];
        TTArgs a = {};
        a.cb = w.d_cb;
        a.n_codes = ctx->slots[w_slot].n_codes;
        a.K = K;
        a.N = N;
        a.T = tt_chunks(K);
        a.F = F;
        a.xmode = xmode;
        a.x = x;
        a.norm_w = norm_i >= 0 ? p->dev_norm[norm_i] : nullptr;
        a.eps = eps;
        a.inv_k = 1.0f / (float)K;
        if (embed) {
            a.embed = p->embed;
            a.h_init = p->h;
        }
        a.st = p->st;
        a.prompt = p->prompt;
        a.gen = p->gen;
        a.vocab = V;
        a.emode = emode;
        a.part = p->part;
        a.counters = p->counters;
        a.y = y;
        a.logits = p->logits;
        a.hist = p->hist;
        a.hist_rows = p->hist_rows;
        a.cand_v = p->cand_v;
        a.cand_i = p->cand_i;
        a.stw = p->st;
        a.gen_dev = p->gen;
        a.gen_host = (volatile int *)p->gen_host_dev;
        a.max_gen = p->max_pos;
        a.status = p->status;
        return launch_tt_fused(s, p->cfgs[mi], p->maps[mi], a, pdl_enabled());
    };
    for (int l = 0; l < t.L; l++) {
        const LayerSlots &ls = t.layers[l];
        // x = rmsnorm(h) * w1 (the embedding row in layer 0) -> qkv
        if (!gemv(4 * l + 0, ls.qkv, H, nq, X_NORM, p->h, 2 * l, p->eps[2 * l], l == 0, E_Y,
                  p->qkv))
            return false;
        size_t smem_att = (size_t)p->max_pos * 4;
        auto att = hd == 32 ? k_attention<32, 256> : hd == 64 ? k_attention<64, 256>
                                                              : k_attention<128, 256>;
        if (!launch_pdl(s, att, dim3(t.nh), dim3(256), smem_att, (const StepState *)p->st,
                        (const float *)p->qkv, 1, nq, (const float *)p->rcos,
                        (const float *)p->rsin, p->kc + (size_t)l * nkv * p->max_pos * hd,
                        p->vc + (size_t)l * nkv * p->max_pos * hd, p->max_pos, t.groups, nkv,
                        p->scale, p->ctx))
            return false;
        // h += ctx @ Wo
        if (!gemv(4 * l + 1, ls.o, qd, H, X_PLAIN, p->ctx, -1, 0.f, false, E_RESID, p->h))
            return false;
        // x = rmsnorm(h) * w2 -> act = silu(gate) * up
        if (!gemv(4 * l + 2, ls.gu, H, 2 * F, X_NORM, p->h, 2 * l + 1, p->eps[2 * l + 1], false,
                  E_SWIGLU, p->act))
            return false;
        // h += act @ Wdown
        if (!gemv(4 * l + 3, ls.dn, F, H, X_PLAIN, p->act, -1, 0.f, false, E_RESID, p->h))
            return false;
    }
    // logits = rmsnorm(h) * wf @ Wlm, greedy token
    return gemv((int)p->maps.size() - 1, t.lm, H, V, X_NORM, p->h, 2 * t.L, p->f_eps, false,
                E_ARGMAX, nullptr);
}

static bool ensure_graph(CtxImpl *c, DecodePlan *p) {
    if (p->exec && p->graph_hist == p->hist && p->graph_hist_rows == p->hist_rows) return true;
    if (p->exec) cudaGraphExecDestroy(p->exec);
    if (p->graph) cudaGraphDestroy(p->graph);
    p->exec = nullptr;
    p->graph = nullptr;
    if (!KLLM_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal)))
        return false;
    long long l0 = g_launches;
    bool ok = record_step(c, p);
    p->kernels_per_step = g_launches - l0;
    g_launches = l0;   // counted when the graph is replayed
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (!ok || !KLLM_CUDA(e)) {
        if (g) cudaGraphDestroy(g);
        return false;
    }
    p->graph = g;
    if (!KLLM_CUDA(cudaGraphInstantiate(&p->exec, g, 0))) return false;
    p->graph_hist = p->hist;
    p->graph_hist_rows = p->hist_rows;
    return true;
}

// The layers' projection weights as bf16 Wt[N][K] for the tensor-core
// GEMMs, built once per plan, when the plan's value streams are bf16 (every
// codebook entry a bf16 number) and every projection's shape fits; pf_wt
// stays empty otherwise.  False only on a CUDA error.
static bool plan_layer_wt(CtxImpl *c, DecodePlan *p, cudaStream_t s) {
    if (!p->pf_wt.empty() || p->pf_wt_tried) return true;
    p->pf_wt_tried = true;
    const TemplateInfo &t = p->ti;
    const TapeCtx *ctx = &c->base;
    bool tc = p->vm == TTX_VBF16;
    for (int l = 0; tc && l < t.L; l++)
        for (int sl : {t.layers[l].qkv, t.layers[l].o, t.layers[l].gu, t.layers[l].dn})
            tc = tc && pf_gemm_applies(ctx->slots[sl].tt_K, ctx->slots[sl].tt_N);
    if (!tc) return true;
    p->pf_wt.assign((size_t)4 * t.L, nullptr);
    for (int l = 0; l < t.L; l++) {
        const LayerSlots &ls = t.layers[l];
        const int mats[4] = {ls.qkv, ls.o, ls.gu, ls.dn};
        for (int i = 0; i < 4; i++) {
            const Slot &sl = ctx->slots[mats[i]];
            const DevSlot &w = c->ds[mats[i]];
            void *&wt = p->pf_wt[(size_t)4 * l + i];
            if (!KLLM_CUDA(cudaMalloc(&wt, (size_t)sl.tt_K * sl.tt_N * 2)) ||
                !pf_build_wt(s, w.d_idx, w.d_cb, sl.tt_K, sl.tt_N, wt)) {
                cudaStreamSynchronize(s);
                for (void *b : p->pf_wt)
                    if (b) cudaFree(b);
                p->pf_wt.clear();
                return false;
            }
        }
    }
    return true;
}

// Batched prompt pass (KLLM infer option `prefill`): positions 0..R-1 of
// the prompt through every layer at once -- projections as TT-GEMMs (rows
// bit-identical to the TT-GEMV), norms, RoPE, causal attention, residuals
// and SwiGLU as row kernels -- leaving the KV cache of those positions as
// the per-token steps would.  The last layer needs only its k and v.  The
// prompt's last position then runs as a regular decode step, which picks
// the first token.  Its activations live in one arena of the plan, grown
// (once) to the longest prompt seen and freed with the plan.
static bool plan_prefill(CtxImpl *c, DecodePlan *p, int R, const int *prompt_dev, float *kc_base,
                         float *vc_base, cudaStream_t s) {
    const TemplateInfo &t = p->ti;
    const TapeCtx *ctx = &c->base;
    const int H = t.H, hd = t.hd, nh = t.nh, nkv = t.nkv, F = t.F, L = t.L;
    const int qd = nh * hd, kvd = nkv * hd, nq = qd + 2 * kvd, mp = p->max_pos;
    if (R <= 0) return true;
    if (!((hd == 64 || hd == 128) && env_on("KLLM_PREFILL_FLASH", true)) &&
        (size_t)(R + 1) * 4 > 200 * 1024) {
        set_error("prefill: %d positions exceed the attention kernel's score buffer", R);
        return false;
    }
    // Tensor-core projections (pfgemm.cu) when every codebook is bf16 (the
    // plan's value streams are bf16) and the shapes fit; KLLM_PREFILL_TC=0
    // keeps the exact FP32 TT-GEMM, KLLM_PREFILL_TERMS picks 2 or 3 (the
    // default) bf16 terms of x.
    if (p->pf_terms == 0 && env_on("KLLM_PREFILL_TC", true)) {
        if (!plan_layer_wt(c, p, s)) return false;
        if (!p->pf_wt.empty()) {
            const char *te = getenv("KLLM_PREFILL_TERMS");
            p->pf_terms = te && atoi(te) == 2 ? 2 : 3;
        }
    }
    // arena: hA, hB, xn [R][H]; big [R][max(nq, 2F, H)]; qr, cx [R][qd];
    // act [R][F]; the bf16 terms of a projection's x [terms][R][max(H, F, qd)]
    // (every piece a multiple of 4 floats: 16-byte aligned)
    auto up4 = [](size_t n) { return (n + 3) & ~(size_t)3; };
    const size_t wide = up4((size_t)R * std::max({(size_t)nq, (size_t)2 * F, (size_t)H}));
    const size_t rh = up4((size_t)R * H), rq = up4((size_t)R * qd), rf = up4((size_t)R * F);
    const size_t rxs = p->pf_terms ? up4(((size_t)p->pf_terms * R *
                                          std::max({(size_t)H, (size_t)F, (size_t)qd}) + 1) / 2)
                                   : 0;
    const size_t need = 3 * rh + wide + 2 * rq + rf + rxs;
    if (p->pf_cap < need) {
        if (p->pf_arena) {
            if (!KLLM_CUDA(cudaStreamSynchronize(s))) return false;
            cudaFree(p->pf_arena);
        }
        p->pf_arena = nullptr;
        p->pf_cap = 0;
        if (!dalloc(&p->pf_arena, need)) return false;
        p->pf_cap = need;
    }
    float *hA = p->pf_arena, *hB = hA + rh, *xn = hB + rh, *big = xn + rh, *qr = big + wide,
          *cx = qr + rq, *act = cx + rq, *xs = act + rf;
    bool ok = true;
    int cur_layer = 0;
    auto gemm = [&](int slot, const float *x, float *y) {
        const Slot &sl = ctx->slots[slot];
        const DevSlot &w = c->ds[slot];
        if (p->pf_terms) {
            const LayerSlots &ls = t.layers[cur_layer];
            const int i = slot == ls.qkv ? 0 : slot == ls.o ? 1 : slot == ls.gu ? 2 : 3;
            return pf_split(s, x, (long long)R * sl.tt_K, p->pf_terms, xs) &&
                   pf_gemm_tc(s, xs, p->pf_terms, R, sl.tt_K, p->pf_wt[(size_t)4 * cur_layer + i],
                              sl.tt_N, y, p->status);
        }
        return kllm_tt_gemm(x, R, w.d_cb, sl.n_codes, w.d_idx, sl.tt_K, sl.tt_N, y, s) == 0;
    };
    const int ew_blocks = 148 * 8;
    // attention: the tiled kernel for head dims 64 and 128 (KLLM_PREFILL_FLASH=0:
    // the row kernel, one block per position and head)
    const bool flash = (hd == 64 || hd == 128) && env_on("KLLM_PREFILL_FLASH", true);
    const size_t att_smem = flash ? (hd == 64 ? pf_flash_smem<64>() : pf_flash_smem<128>())
                                  : (size_t)(R + 1) * 4;
    if (ok && att_smem > 48 * 1024) {
        const void *fn = !flash ? (const void *)k_pf_attention
                         : hd == 64 ? (const void *)k_pf_flash<64> : (const void *)k_pf_flash<128>;
        ok = KLLM_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)att_smem));
    }
    if (ok) {
        k_pf_embed<<<R, PF_THREADS, 0, s>>>(p->embed, prompt_dev, H, hA);
        g_launches++;
    }
    for (int l = 0; ok && l < L; l++) {
        const LayerSlots &ls = t.layers[l];
        cur_layer = l;
        float *kc = kc_base + (size_t)l * nkv * mp * hd, *vc = vc_base + (size_t)l * nkv * mp * hd;
        k_pf_rmsnorm<<<R, PF_THREADS, 0, s>>>(hA, p->dev_norm[2 * l], p->eps[2 * l], H, xn);
        ok = gemm(ls.qkv, xn, big);
        if (!ok) break;
        k_pf_rope_kv<<<R, PF_THREADS, 0, s>>>(big, nq, nh, nkv, hd, p->rcos, p->rsin, mp, qr, kc, vc);
        g_launches += 2;
        if (l + 1 == L) break;   // later positions need only this layer's k and v
        if (!flash)
            k_pf_attention<<<dim3(R, nh), PF_THREADS, att_smem, s>>>(
                qr, kc, vc, nh, t.groups, hd, mp, p->scale, cx);
        else if (hd == 64)
            k_pf_flash<64><<<dim3((R + PFA_BQ - 1) / PFA_BQ, nh), 256, att_smem, s>>>(
                qr, kc, vc, R, nh, t.groups, mp, p->scale, cx);
        else
            k_pf_flash<128><<<dim3((R + PFA_BQ - 1) / PFA_BQ, nh), 256, att_smem, s>>>(
                qr, kc, vc, R, nh, t.groups, mp, p->scale, cx);
        ok = gemm(ls.o, cx, big);
        if (!ok) break;
        k_pf_add<<<ew_blocks, 256, 0, s>>>(hA, big, (long long)R * H, hB);
        k_pf_rmsnorm<<<R, PF_THREADS, 0, s>>>(hB, p->dev_norm[2 * l + 1], p->eps[2 * l + 1], H, xn);
        ok = gemm(ls.gu, xn, big);
        if (!ok) break;
        k_pf_swiglu<<<ew_blocks, 256, 0, s>>>(big, F, (long long)R * F, act);
        ok = gemm(ls.dn, act, big);
        if (!ok) break;
        k_pf_add<<<ew_blocks, 256, 0, s>>>(hB, big, (long long)R * H, hA);
        g_launches += 5;
        ok = KLLM_CUDA(cudaGetLastError());
    }
    return ok && KLLM_CUDA(cudaGetLastError());
}

// Batched greedy decode of nseq independent sequences (no counterpart in the
// reference: its processor_infer, _tape_runner.c:1602-1763, runs one
// sequence; this is that loop for many sequences at once).  Each prompt but
// its last position goes through the batched prompt pass into the
// sequence's own KV cache; then every step feeds one token per sequence:
// embedding rows, per layer row RMSNorm, the QKV / O / gate_up / down
// projections as one GEMM over the nseq rows (the few-row tensor-core GEMM
// where the codebooks hold bf16 numbers, up to 128 rows; the exact TT-GEMM,
// each row bit-identical to the TT-GEMV, otherwise or with
// KLLM_BATCH_TC=0), RoPE and the append at each row's own position,
// attention over each row's own cache, residual adds and SwiGLU (batch.cuh);
// final norm, lm_head, the first-maximum pick per row.  One step is
// captured as a CUDA graph and replayed.  Sequences run the full max_new
// steps; out_lens cut each at its first EOS (the reference stops there and
// emits nothing after it).
bool plan_infer_batch(CtxImpl *c, const int *prompts, const int *lens, int nseq, int max_new,
                      int eos, int *out, int *out_lens, double *prefill_ms, double *decode_ms) {
    DecodePlan *p = c->plan;
    if (!p || !p->persist) {
        set_error("batched decode: no fused decode plan");
        return false;
    }
    if (p->world != 1) {
        set_error("batched decode runs on one GPU (the context is column-sharded)");
        return false;
    }
    const TemplateInfo &t = p->ti;
    const TapeCtx *ctx = &c->base;
    const int H = t.H, hd = t.hd, nh = t.nh, nkv = t.nkv, F = t.F, L = t.L, V = t.V;
    const int qd = nh * hd, kvd = nkv * hd, nq = qd + 2 * kvd, mp = p->max_pos;
    if (nseq < 1 || max_new < 1 || PF_THREADS % hd) {
        set_error("batched decode: %d sequences, %d new tokens, head dim %d", nseq, max_new, hd);
        return false;
    }
    size_t total = 0;
    for (int i = 0; i < nseq; i++) {
        if (lens[i] < 1 || lens[i] + max_new > mp) {
            set_error("batched decode: sequence %d has %d prompt tokens (+%d) for %d positions", i,
                      lens[i], max_new, mp);
            return false;
        }
        for (int j = 0; j < lens[i]; j++)
            if (prompts[total + j] < 0 || prompts[total + j] >= V) {
                set_error("batched decode: prompt token %d of sequence %d outside the vocabulary",
                          j, i);
                return false;
            }
        total += lens[i];
    }
    cudaStream_t s = c->stream;
    // tensor-core projections by default when the codebooks are bf16 numbers
    // (KLLM_BATCH_TC=0: the exact FP32 TT-GEMM, each row bit-identical to
    // the TT-GEMV)
    bool tc = env_on("KLLM_BATCH_TC", true) && p->vm == TTX_VBF16 && nseq <= 128;
    if (tc && !plan_layer_wt(c, p, s)) return false;
    const Slot &lms = ctx->slots[t.lm];
    const bool layer_tc = tc && !p->pf_wt.empty();
    const bool lm_tc = tc && pf_gemm_applies(lms.tt_K, lms.tt_N);
    // split-K partial tiles of the skinny tensor-core GEMM
    size_t part_n = 0;
    if (tc) {
        const LayerSlots &l0 = t.layers[0];
        for (int sl : {l0.qkv, l0.o, l0.gu, l0.dn, t.lm}) {
            const Slot &x = ctx->slots[sl];
            if (!pf_gemm_applies(x.tt_K, x.tt_N)) continue;
            const int ks = bd_gemm_splits(x.tt_K, x.tt_N);
            if (ks > 1) part_n = std::max(part_n, (size_t)ks * nseq * x.tt_N);
        }
    }
    const size_t att_smem = bd_att_smem(t.groups, hd, mp);
    if (att_smem > 227 * 1024) {
        set_error("batched decode: %d positions of %d query heads exceed the attention block's "
                  "shared memory", mp, t.groups);
        return false;
    }
    // arena (floats, each piece a multiple of 4): K and V caches of every
    // sequence; residual rows h, hB [nseq][H]; big [nseq][max(nq, 2F, V)]
    // (a GEMM output in one piece); qr [nseq][qd]; xs, a GEMM's input (fp32
    // rows or three bf16 terms); split-K partials; the greedy pick's slice
    // maxima; ints: prompts, tokens, positions, first positions, generated
    // tokens, the slice maxima's indices
    auto up4 = [](size_t n) { return (n + 3) & ~(size_t)3; };
    const size_t seq_stride = (size_t)L * nkv * mp * hd;
    const size_t kv = up4((size_t)nseq * seq_stride);
    const size_t rh = up4((size_t)nseq * H), rq = up4((size_t)nseq * qd);
    const size_t wide = up4((size_t)nseq * std::max({(size_t)nq, (size_t)2 * F, (size_t)H, (size_t)V}));
    const size_t rxs = up4(((size_t)3 * nseq * std::max({(size_t)H, (size_t)F, (size_t)qd}) + 1) / 2);
    const size_t rpart = up4(part_n), rcand = up4((size_t)nseq * BD_AC);
    const size_t ints = up4(total + 3 * (size_t)nseq + (size_t)nseq * max_new) + rcand;
    const size_t need = 2 * kv + 2 * rh + wide + rq + rxs + rpart + rcand + ints;
    if (p->bd_cap < need) {
        if (!KLLM_CUDA(cudaStreamSynchronize(s))) return false;
        if (p->bd_arena) cudaFree(p->bd_arena);
        p->bd_arena = nullptr;
        p->bd_cap = 0;
        if (!dalloc(&p->bd_arena, need)) return false;
        p->bd_cap = need;
    }
    float *kcs = p->bd_arena, *vcs = kcs + kv, *h = vcs + kv, *hB = h + rh, *big = hB + rh,
          *qr = big + wide, *xs = qr + rq, *part = xs + rxs, *cand_v = part + rpart;
    int *d_cand_i = reinterpret_cast<int *>(cand_v + rcand), *d_prompts = d_cand_i + rcand,
        *d_tok = d_prompts + total, *d_pos = d_tok + nseq, *d_start = d_pos + nseq,
        *d_gen = d_start + nseq;
    std::vector<int> tok0(nseq), pos0(nseq);
    {
        size_t off = 0;
        for (int i = 0; i < nseq; i++) {
            tok0[i] = prompts[off + lens[i] - 1];
            pos0[i] = lens[i] - 1;
            off += lens[i];
        }
    }
    if (!KLLM_CUDA(cudaMemcpyAsync(d_prompts, prompts, total * 4, cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemcpyAsync(d_tok, tok0.data(), nseq * 4, cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemcpyAsync(d_pos, pos0.data(), nseq * 4, cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemcpyAsync(d_start, pos0.data(), nseq * 4, cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemsetAsync(p->status, 0, 4, s)))
        return false;
    // the lm_head as bf16 Wt for the tensor-core form (built once)
    if (lm_tc && !p->bd_lm_wt) {
        if (!KLLM_CUDA(cudaMalloc(&p->bd_lm_wt, (size_t)lms.tt_K * lms.tt_N * 2)) ||
            !pf_build_wt(s, c->ds[t.lm].d_idx, c->ds[t.lm].d_cb, lms.tt_K, lms.tt_N, p->bd_lm_wt))
            return false;
    }
    if (!KLLM_CUDA(cudaEventRecord(p->ev0, s))) return false;
    // prompt passes, one sequence after another, into the sequences' caches
    {
        size_t off = 0;
        for (int i = 0; i < nseq; i++) {
            if (lens[i] >= 2 && !plan_prefill(c, p, lens[i] - 1, d_prompts + off,
                                              kcs + (size_t)i * seq_stride,
                                              vcs + (size_t)i * seq_stride, s))
                return false;
            off += lens[i];
        }
    }
    if (!KLLM_CUDA(cudaEventRecord(p->ev1, s))) return false;
    // The projections: the few-row tensor-core GEMM from the bf16 terms in
    // xs, its K-range partial tiles left in `part` (nz of them; one range
    // writes `big`), or the exact TT-GEMM from fp32 rows in xs into `big`.
    // Each returns where its output is and in how many tiles.
    auto gemm = [&](int slot, int layer, int which, const float **y, int *nz) {
        const Slot &sl = ctx->slots[slot];
        const DevSlot &w = c->ds[slot];
        const void *wt = which < 4 ? (layer_tc ? p->pf_wt[(size_t)4 * layer + which] : nullptr)
                                   : (lm_tc ? p->bd_lm_wt : nullptr);
        if (wt) {
            if (!bd_gemm_tc(s, xs, 3, nseq, sl.tt_K, wt, sl.tt_N, big, part, p->status, nz))
                return false;
            *y = *nz > 1 ? part : big;
            return true;
        }
        *nz = 1;
        *y = big;
        return kllm_tt_gemm(reinterpret_cast<const float *>(xs), nseq, w.d_cb, sl.n_codes,
                            w.d_idx, sl.tt_K, sl.tt_N, big, s) == 0;
    };
    // terms of each GEMM's input: 3 for the tensor cores, 0 (fp32) for the
    // exact TT-GEMM
    const int lt = layer_tc ? 3 : 0, lmt = lm_tc ? 3 : 0;
    if (tc && !bd_gemm_prepare()) return false;
    const int ew_blocks = 148 * 8;
    auto att_for = [](auto hdc, int groups) {
        constexpr int D = decltype(hdc)::value;
        return groups == 1 ? k_bd_attn_group<D, 1> : groups == 2 ? k_bd_attn_group<D, 2>
             : groups == 4 ? k_bd_attn_group<D, 4> : groups == 8 ? k_bd_attn_group<D, 8>
                           : k_bd_attn_group<D, 0>;
    };
    auto att = hd == 32 ? att_for(std::integral_constant<int, 32>(), t.groups)
             : hd == 64 ? att_for(std::integral_constant<int, 64>(), t.groups)
                        : att_for(std::integral_constant<int, 128>(), t.groups);
    if (att_smem > 48 * 1024 &&
        !KLLM_CUDA(cudaFuncSetAttribute(att, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)att_smem)))
        return false;
    // one decode step of every sequence: positions, tokens and the generated
    // token's slot are read on the device, so the same launches (a graph)
    // serve every step.  Per layer: QKV GEMM, RoPE + append, attention, O
    // GEMM, residual add + RMSNorm, gate_up GEMM, SwiGLU, down GEMM, and the
    // residual add + the next RMSNorm (the next layer's, or the final one).
    auto record_step = [&]() -> bool {
        const float *y = nullptr;
        int nz = 1;
        k_bd_add_norm<<<nseq * BD_CL, PF_THREADS, 0, s>>>(nullptr, p->embed, d_tok, nullptr, 1,
                                                  p->dev_norm[0], p->eps[0], H, h, lt, xs);
        g_launches++;
        for (int l = 0; l < L; l++) {
            const LayerSlots &ls = t.layers[l];
            float *kc = kcs + (size_t)l * nkv * mp * hd, *vc = vcs + (size_t)l * nkv * mp * hd;
            if (!gemm(ls.qkv, l, 0, &y, &nz)) return false;
            k_bd_rope_kv<<<dim3(nseq, 8), PF_THREADS, 0, s>>>(y, nz, d_pos, nq, nh, nkv, hd, p->rcos,
                                                     p->rsin, mp, seq_stride, qr, kc, vc);
            att<<<dim3(nseq, nkv), BD_ATT_THREADS, att_smem, s>>>(
                qr, kc, vc, d_pos, nh, t.groups, mp, seq_stride, p->scale, lt, xs);
            if (!gemm(ls.o, l, 1, &y, &nz)) return false;
            k_bd_add_norm<<<nseq * BD_CL, PF_THREADS, 0, s>>>(h, nullptr, nullptr, y, nz,
                                                      p->dev_norm[2 * l + 1], p->eps[2 * l + 1],
                                                      H, hB, lt, xs);
            if (!gemm(ls.gu, l, 2, &y, &nz)) return false;
            k_bd_swiglu<<<ew_blocks, 256, 0, s>>>(y, nz, nseq, F, lt, xs);
            if (!gemm(ls.dn, l, 3, &y, &nz)) return false;
            const bool last = l + 1 == L;
            k_bd_add_norm<<<nseq * BD_CL, PF_THREADS, 0, s>>>(
                hB, nullptr, nullptr, y, nz, last ? p->dev_norm.back() : p->dev_norm[2 * l + 2],
                last ? p->f_eps : p->eps[2 * l + 2], H, h, last ? lmt : lt, xs);
            g_launches += 5;
        }
        if (!gemm(t.lm, 0, 4, &y, &nz)) return false;
        k_bd_argmax_part<<<dim3(nseq, BD_AC), PF_THREADS, 0, s>>>(y, nz, V, cand_v, d_cand_i);
        k_bd_argmax_pick<<<(nseq + 31) / 32, 32, 0, s>>>(y, nz, V, nseq, cand_v, d_cand_i, d_start,
                                                        max_new, d_tok, d_pos, d_gen);
        g_launches += 2;
        return KLLM_CUDA(cudaGetLastError());
    };
    bool ok = true;
    if (c->opts.use_graphs && max_new > 1) {
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        const long long g0 = g_launches;
        ok = KLLM_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        if (ok) {
            const bool rec = record_step();
            ok = KLLM_CUDA(cudaStreamEndCapture(s, &graph)) && rec;
        }
        const long long per_step = g_launches - g0;
        ok = ok && KLLM_CUDA(cudaGraphInstantiate(&exec, graph, 0));
        for (int step = 0; ok && step < max_new; step++) ok = KLLM_CUDA(cudaGraphLaunch(exec, s));
        if (ok) g_launches += per_step * (max_new - 1);
        if (exec) {
            cudaStreamSynchronize(s);
            cudaGraphExecDestroy(exec);
        }
        if (graph) cudaGraphDestroy(graph);
    } else {
        for (int step = 0; ok && step < max_new; step++) ok = record_step();
    }
    if (!ok || !KLLM_CUDA(cudaEventRecord(p->ev2, s))) return false;
    std::vector<int> gen((size_t)nseq * max_new);
    int status = 0;
    if (!KLLM_CUDA(cudaMemcpyAsync(gen.data(), d_gen, gen.size() * 4, cudaMemcpyDeviceToHost, s)) ||
        !KLLM_CUDA(cudaMemcpyAsync(&status, p->status, 4, cudaMemcpyDeviceToHost, s)) ||
        !KLLM_CUDA(cudaStreamSynchronize(s)))
        return false;
    if (status) {
        set_error("batched decode kernels reported status 0x%x", status);
        return false;
    }
    for (int i = 0; i < nseq; i++) {
        int n = 0;
        while (n < max_new && gen[(size_t)i * max_new + n] != eos) n++;
        memcpy(out + (size_t)i * max_new, gen.data() + (size_t)i * max_new, (size_t)max_new * 4);
        out_lens[i] = n;
    }
    float pre = 0.f, dec = 0.f;
    cudaEventElapsedTime(&pre, p->ev0, p->ev1);
    cudaEventElapsedTime(&dec, p->ev1, p->ev2);
    if (prefill_ms) *prefill_ms = pre;
    if (decode_ms) *decode_ms = dec;
    return true;
}

bool plan_infer(CtxImpl *c, const int *prompt, int prompt_len, int max_new, int max_pos,
                int eos, const std::function<bool(int, int)> &emit, int *generated) {
    DecodePlan *p = c->plan;
    *generated = 0;
    if (!p || max_pos > p->max_pos) {
        set_error("decode plan not prepared");
        return false;
    }
    const int V = p->ti.V;
    for (int i = 0; i < prompt_len; i++)
        if (prompt[i] < 0 || prompt[i] >= V) {
            set_error("prompt token %d (%d) outside the vocabulary of %d", i, prompt[i], V);
            return false;
        }
    cudaStream_t s = c->stream;
    // logits history for callers that asked for every step's logits
    int want_rows = c->opts.logits_out ? std::min(c->opts.logits_rows, max_pos) : 0;
    if (want_rows > 0 && (!p->hist || p->hist_rows < want_rows)) {
        if (p->hist) cudaFree(p->hist);
        p->hist = nullptr;
        if (!dalloc(&p->hist, (size_t)want_rows * V)) return false;
        p->hist_rows = want_rows;
    } else if (want_rows == 0 && p->hist) {
        cudaFree(p->hist);
        p->hist = nullptr;
        p->hist_rows = 0;
    }
    StepState st0 = {0, prompt_len, 0, 0};
    if (!KLLM_CUDA(cudaMemcpyAsync(p->prompt, prompt, (size_t)prompt_len * 4,
                                   cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemcpyAsync(p->st, &st0, sizeof st0, cudaMemcpyHostToDevice, s)) ||
        !KLLM_CUDA(cudaMemsetAsync(p->status, 0, 4, s)) ||
        (p->d_abort && !KLLM_CUDA(cudaMemsetAsync(p->d_abort, 0, 4, s))) ||
        !KLLM_CUDA(cudaStreamSynchronize(s)))
        return false;
    for (int i = 0; i < max_pos; i++) p->gen_host[i] = -1;
    bool graphs = c->opts.use_graphs != 0;
    if (graphs && !ensure_graph(c, p)) return false;
    // positions are capped at max_pos (the bytes driver's max_seq_tokens,
    // _tape_runner.c:1537): at most max_pos - prompt_len tokens
    const int max_gen = std::max(0, std::min(max_new, max_pos - prompt_len));
    const int total = prompt_len + max_gen;
    if ((int)p->step_ev.size() < total) {
        size_t old = p->step_ev.size();
        p->step_ev.resize(total);
        for (size_t i = old; i < p->step_ev.size(); i++)
            if (!KLLM_CUDA(cudaEventCreateWithFlags(&p->step_ev[i], cudaEventDisableTiming)))
                return false;
    }
    auto launch_step = [&](int i) -> bool {
        bool ok;
        if (graphs) {
            ok = KLLM_CUDA(cudaGraphLaunch(p->exec, s));
            g_launches += p->kernels_per_step;
        } else {
            ok = record_step(c, p);
        }
        return ok && KLLM_CUDA(cudaEventRecord(p->step_ev[i], s));
    };
    if (!KLLM_CUDA(cudaEventRecord(p->ev0, s))) return false;
    int launched = 0;
    // batched prompt pass for all prompt positions but the last (persistent
    // plan, no per-step logits requested).  A column-sharded rank runs the
    // whole pass itself from its full matrices: it fills its own copy of the
    // KV cache, the state every rank holds in full.
    if (c->opts.prefill && p->persist && want_rows == 0 && prompt_len >= 2) {
        const int R = prompt_len - 1;
        StepState st1 = {R, prompt_len, 0, 0};
        if (!plan_prefill(c, p, R, p->prompt, p->kc, p->vc, s) ||
            !KLLM_CUDA(cudaMemcpyAsync(p->st, &st1, sizeof st1, cudaMemcpyHostToDevice, s)))
            return false;
        launched = R;
    }
    for (; launched < prompt_len; launched++)
        if (!launch_step(launched)) return false;
    if (!KLLM_CUDA(cudaEventRecord(p->ev1, s))) return false;
    // decode: keep the device ahead of the host by up to `window` steps
    const int window = 64;
    int gen = 0;
    bool stop = false;
    while (!stop && gen < max_gen) {
        while (launched < total && launched - (prompt_len - 1 + gen) <= window)
            if (!launch_step(launched++)) return false;
        // token `gen` is produced by step prompt_len - 1 + gen
        if (!KLLM_CUDA(cudaEventSynchronize(p->step_ev[prompt_len - 1 + gen]))) return false;
        int tok = ((volatile int *)p->gen_host)[gen];
        if (tok == eos) break;
        gen++;
        if (!emit(tok, gen - 1)) stop = true;
    }
    // the reference also feeds the last generated token (one more step)
    if (!stop && gen == max_gen) {
        while (launched < total)
            if (!launch_step(launched++)) return false;
    }
    if (!KLLM_CUDA(cudaEventRecord(p->ev2, s)) || !KLLM_CUDA(cudaStreamSynchronize(s)))
        return false;
    int status = 0;
    if (!KLLM_CUDA(cudaMemcpy(&status, p->status, 4, cudaMemcpyDeviceToHost))) return false;
    if (status) {
        // an aborted step leaves the counters mid-step and tagged words of
        // step numbers that will be reused: start over
        if (p->d_cnt) cudaMemset(p->d_cnt, 0, p->cnt_n * sizeof(int));
        if (p->d_abort) cudaMemset(p->d_abort, 0, sizeof(int));
        for (auto &b : p->ll_bufs) cudaMemset(b.first, 0, b.second);
        set_error("decode kernels reported status 0x%x (%s)", status,
                  (status & ST_WAIT_TIMEOUT) ? "a wait timed out" : "a token was out of range");
        return false;
    }
    float pre = 0.f, dec = 0.f;
    cudaEventElapsedTime(&pre, p->ev0, p->ev1);
    cudaEventElapsedTime(&dec, p->ev1, p->ev2);
    c->stats.prefill_ms = pre;
    c->stats.decode_ms = dec;
    c->stats.steps = prompt_len + gen;
    *generated = gen;
    if (want_rows > 0) {
        int rows = std::min(want_rows, prompt_len + gen);
        if (!KLLM_CUDA(cudaMemcpy(c->opts.logits_out, p->hist, (size_t)rows * V * 4,
                                  cudaMemcpyDeviceToHost)))
            return false;
    }
    // leave the last step's logits in the logits slot, as the tape would
    // (only when no step ran past it)
    int ls = p->logits_slot;
    if (ls >= 0 && launched == prompt_len + gen) {
        Slot &sl = c->base.slots[ls];
        if (ensure_device(c, ls, (size_t)V) &&
            KLLM_CUDA(cudaMemcpyAsync(c->ds[ls].d, p->logits, (size_t)V * 4,
                                      cudaMemcpyDeviceToDevice, s))) {
            sl.ndim = 2;
            sl.shape[0] = 1;
            sl.shape[1] = V;
            if (sl.size < V) sl.size = V;
            c->ds[ls].dev_newer = true;
            c->ds[ls].host_dirty = false;
        }
    }
    return KLLM_CUDA(cudaStreamSynchronize(s));
}

}  // namespace kllm

#ifdef KLLM_DS_PROFILE
// Profiling build: copy the decode step's timestamps ([cta][phase][16]) to
// out; returns the number of values (cta count * phases * 16), -1 without a
// persistent plan.
extern "C" int kllm_ds_profile(TapeCtx *ctx, unsigned long long *out, int cap, int *grid,
                               int *nphases) {
    using namespace kllm;
    CtxImpl *c = impl(ctx);
    DecodePlan *p = c ? c->plan : nullptr;
    if (!p || !p->persist || !p->prof) return -1;
    *grid = p->ds_grid;
    *nphases = (int)p->phases.size();
    const size_t n = std::min<size_t>(p->prof_n, (size_t)cap);
    cudaSetDevice(c->device);
    if (!KLLM_CUDA(cudaMemcpy(out, p->prof, n * 8, cudaMemcpyDeviceToHost))) return -1;
    return (int)n;
}
#endif
