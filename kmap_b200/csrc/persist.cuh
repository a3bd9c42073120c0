// persist.cuh -- the persistent decode step: one cooperative launch runs a
// whole tape step of the compiler's LLaMA template.
//
// Grid = one CTA per SM (co-resident: cooperative launch).  Each CTA has
// eight consumer warps, a producer warp and a table warp.  The step is a
// list of phases; per layer QKV, attention, O, gate_up, down; then lm_head.
// A GEMV task is one column group (8 columns x all chunks, ttx.cuh) for one
// warp, or one of its W sub-tasks in the fast order; group i of a phase
// goes to CTA i mod G, and a CTA deals its tasks to its warps in turn.
//
// Producer warp: lane 0 streams the CTA's tasks through a ring of 16 KB
// stages with bulk copies, in the order the warps consume them (rounds of
// up to eight tasks, piece by piece).  Weights do not depend on
// activations, so the stream runs ahead across phase boundaries.  Table
// warp: bulk-copies each phase's codebook table (slot streams only) and
// norm weights into one of two slots, two phases ahead.
//
// Consumers, per phase: stage x in shared memory, chunk by chunk, by
// polling the tagged words the producing phase stores (waiting for the
// input and reading it are one poll, bounded in time); then rmsnorm of the
// residual, the embedding row in layer 0, or a plain vector (ctx, act).
// GEMV task, lane = 8 * pair + chunk, two columns per lane:
//   rows   acc = fl(acc + fl(x[k] * w[k][n])) over the chunk's rows in
//          order -- the reference's serial chunk sum (_tape_runner.c:530-545);
//          w[k][n] is codebook[idx[k][n]], read from the stream's value
//          pattern or gathered from the table;
//   sum    chunk sums added in chunk order through shuffles
//          (_tape_runner.c:646-662): every TT-GEMV result is bit-identical
//          to the reference's (fast order: W partial sums in w order);
//   out    RoPE + KV append (QKV), residual add (O, down), silu(gate) * up
//          (gate_up), logits + first maximum (lm_head; the CTA that arrives
//          last on the lm_head counter, the step's only counter, picks the
//          token).
// Attention: one head per task; q and this position's k, v are polled as
// tagged words, earlier positions read from the cache.
//
// Every wait is bounded; a wait that gives up raises the abort flag, and
// the consumers of every CTA leave at the next phase boundary together
// (named barriers are never split).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tt_fused.cuh"
#include "ttx.cuh"

namespace kllm {

enum DSKind : int { DS_GEMV = 0, DS_ATT = 1 };
// Buffers every rank of a column-sharded decode holds a full copy of; a rank
// stores its columns' results into all copies (DSArgs::peers).  Q, HA, HB,
// ACT, KN and VN hold tagged words (ll_t).
enum DSPeer : int {
    DSP_Q = 0, DSP_KC, DSP_VC, DSP_HA, DSP_HB, DSP_ACT, DSP_LOGITS, DSP_CANDV, DSP_CANDI,
    DSP_KN, DSP_VN, DSP_DONE, DSP_KINDS
};

// An activation word: the float's bits in the low half, the tag of the
// (step, layer) that wrote it in the high half, stored and loaded as one
// 8-byte access.  A reader that sees its tag sees the value: waiting for an
// input and reading it are one poll, with no counter, fence or second load.
typedef unsigned long long ll_t;
enum DSX : int { DX_EMBED = 0, DX_NORM = 1, DX_VEC = 2, DX_ATT = 3 };
enum DSE : int { DE_QKV = 0, DE_RESID = 1, DE_SWIGLU = 2, DE_LM = 3 };

struct DSPhase {
    int kind, ntasks;          // GEMV: column groups; attention: heads
    TTXDesc d;                 // GEMV layout (ttx.cuh)
    int npieces;               // 16-step pieces per group
    int xs;                    // floats per chunk row of the staged x
    unsigned lmagic;           // ceil(2^32 / L): r / L for equal chunks of L rows
    const uint8_t *stream;
    const float *table;        // replicated codebook table (ttx.cuh), built at upload
    int table_bytes;
    int xmode, emode;
    const ll_t *x;             // DX_NORM: residual; DX_VEC: input vector (tagged words)
    const float *norm_w;
    float eps;
    int x_layer;               // the layer whose tag x carries
    int save_x;                // keep the raw x: the residual of a later epilogue
    float *out;                // logits (DE_LM, this rank's copy)
    int out_kind;              // DSPeer of the output
    int groups_all;            // column groups of the matrix over all ranks
    int layer;
    int csplit;                // 2: the two columns of a lane pair go to two warps
                               // (phases with few groups per CTA), 1: one warp
    int pad_[2];               // 16-byte multiple: copied into shared memory in 16-byte pieces
};
static_assert(sizeof(DSPhase) % 16 == 0, "DSPhase is copied in 16-byte pieces");

struct DSArgs {
    const DSPhase *phases;
    int nphases;
    int *done;                 // [nphases] arrivals, counting up across steps (only the
                               // lm_head phase's entry is used)
    int *epoch;                // steps completed since the counters were zeroed
    int *lm_local;             // lm_head arrivals of this rank's CTAs only
    int *status;
    int *abort;
    int stages, tab_cap, wn_cap, xc_cap;
    // step state and embedding
    StepState *st;
    const float *embed;
    const int *prompt;
    int *gen;
    volatile int *gen_host;
    int vocab, max_gen, H;
    // attention
    const ll_t *q;             // this rank's copy
    int nh, nkv, groups, max_pos, qd, kvd;
    const float *rope_cos, *rope_sin;
    float *kc, *vc;            // [L][nkv][max_pos][hd]
    float scale;
    ll_t *ctx;
    // lm_head
    float *hist;
    int hist_rows;
    float *cand_v;             // [world][G] per-CTA first maxima
    int *cand_i;
    // column sharding: this rank, the ranks, and [DSP_KINDS][world] pointers
    // to every rank's copy of the shared buffers (this rank's own included)
    int rank, world;
    void *const *peers;
    // bound of every wait (ns of %globaltimer); a wait that runs out sets
    // ST_WAIT_TIMEOUT and the abort flag
    unsigned long long wait_ns;
    // consumer warps that take GEMV tasks (1..8; the others only stage x
    // and run attention): each task warp holds the ring stage it computes
    // on, so fewer task warps leave more stages for loads in flight
    int task_warps;
    int kv_prefetch;           // L2 prefetch of the cached k, v rows (0: off)
    int gpu_scope;             // tagged words at GPU scope (one rank only)
    int l2_pf;                 // L2 prefetch distance in pieces ahead of the ring loads (0: off)
    int unroll;                // whole pieces through the unrolled scalar loops
    // split attention: up to att_spmax CTAs per head, one more split per
    // att_split_min positions; partial P.V rows [spmax][qd] and (max, sum)
    // pairs [spmax][nh][2] as tagged words (this rank's own)
    ll_t *att_part, *att_ml;
    int att_spmax, att_split_min;
#ifdef KLLM_DS_PROFILE
    // profiling build only: %globaltimer stamps of the step at position
    // prof_pos, [cta][phase][8] (DS_STAMP slots below)
    unsigned long long *prof;
    int prof_pos;
#endif
};

// Profiling build (-DKLLM_DS_PROFILE): timestamps of one step, per CTA and
// phase.  Consumer slots 0 phase start, 1 warp 0's input words in, 2 input
// staged and normalised (all warps), 3 warp 0's tasks done, 4 phase done
// (all warps); producer slots 5 first piece issued, 6 last piece issued,
// 7 ns spent waiting for a free stage; warp 0 (SM clock cycles) slots 8
// waiting for its pieces to land, 9 computing on landed pieces, 10 pieces,
// 11 pieces it had to wait for, 12 chunk sums and epilogues, 13 slot 2 to
// slot 3, 15 slot 0 to slot 2; 14 (CTA 0, phase 0) the %globaltimer step.
// Compiled out otherwise.
#ifdef KLLM_DS_PROFILE
// ds_prof_on: set once per role at kernel start (this step is the profiled one)
#define DS_STAMP(cond, slot, val)                                                         \
    do {                                                                                 \
        if ((cond) && ds_prof_on)                                                        \
            a.prof[((size_t)blockIdx.x * a.nphases + p) * 16 + (slot)] = (val);          \
    } while (0)
#define DS_PROF_INIT() const bool ds_prof_on = a.prof && a.st->pos == a.prof_pos
#else
#define DS_STAMP(cond, slot, val) \
    do {                          \
    } while (0)
#define DS_PROF_INIT() \
    do {               \
    } while (0)
#endif

constexpr int DS_MAX_WORLD = 8;
// DSArgs::peers, copied into shared memory when a step starts: every
// epilogue store goes through it.
__shared__ void *ds_speers[DSP_KINDS * DS_MAX_WORLD];

template <class T>
__device__ __forceinline__ T *ds_peer(const DSArgs &a, int kind, int r) {
    return reinterpret_cast<T *>(ds_speers[kind * a.world + r]);
}

// Store v at index i of every rank's copy of buffer `kind`.
__device__ __forceinline__ void ds_put(const DSArgs &a, int kind, size_t i, float v) {
    for (int r = 0; r < a.world; r++) ds_peer<float>(a, kind, r)[i] = v;
}

__device__ __forceinline__ uint32_t ds_tag(int ep1, int layer) {
    return (uint32_t)ep1 * 256u + (uint32_t)layer;
}

// Scope of the tagged-word accesses: the GPU when every reader and writer
// is on this GPU (one rank), the system when peers store over NVLink.
__shared__ int ds_gpu_scope;

__device__ __forceinline__ void st_ll(ll_t *p, float v, uint32_t tag) {
    const ll_t w = ((ll_t)tag << 32) | __float_as_uint(v);
    if (ds_gpu_scope)
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
    else
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ ll_t ld_ll(const ll_t *p) {
    ll_t w;
    if (ds_gpu_scope)
        asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Store v with its tag at index i of every rank's copy of buffer `kind`.
__device__ __forceinline__ void ds_put_ll(const DSArgs &a, int kind, size_t i, float v,
                                          uint32_t tag) {
    for (int r = 0; r < a.world; r++) st_ll(ds_peer<ll_t>(a, kind, r) + i, v, tag);
}

// CTAs of rank r with work in a phase of `groups_all` column groups.
__device__ __forceinline__ int ds_ncta(const DSArgs &a, int groups_all, int r, int G) {
    const int local = r < groups_all ? (groups_all - r + a.world - 1) / a.world : 0;
    return min(G, local);
}

constexpr int DS_NCW = 8;                    // consumer warps
constexpr int DS_TCH = 8;                    // K chunks of one warp task (lane = 8 * pair + chunk)
constexpr int DS_NC = DS_NCW * 32;
constexpr int DS_PRODUCER = DS_NCW;          // warp: streams the ring
constexpr int DS_TABLER = DS_NCW + 1;        // warp: builds codebook tables
constexpr int DS_THREADS = (DS_NCW + 2) * 32;
constexpr int DS_MAX_STAGES = 32;
constexpr int DS_PIECE_STEPS = 16;           // steps per ring stage (16 KB: one issuing
                                             // thread keeps HBM busy only with pieces this big)
constexpr int DS_STAGE = DS_PIECE_STEPS * TTX_STEP;

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *ctr >= target; false on abort or timeout (which raises abort).
__device__ __forceinline__ bool ds_wait_counter(const int *ctr, int target, int *status,
                                                int *abort, unsigned long long limit) {
    if (ld_acquire(ctr) >= target) return true;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire(ctr) < target) {
        if (ld_acquire(abort)) return false;
        if (globaltimer() - t0 > limit) {
            atomicOr(status, ST_WAIT_TIMEOUT);
            atomicExch(abort, 1);
            return false;
        }
        __nanosleep(20);
    }
    return true;
}

// mbar_wait for the support warps (producer, table builder): their waits are
// long, so they sleep between polls instead of taking issue slots from the
// consumer warps on the same scheduler.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t *bar, uint32_t parity, int *status,
                                               unsigned long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > limit) {
            if (status) atomicOr(status, ST_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Wait until the stage tag says the stage holds piece `seq`.
__device__ __forceinline__ bool ds_wait_tag(volatile int *tag, int seq, int *status,
                                            unsigned long long limit) {
    if (*tag == seq) return true;
    const unsigned long long t0 = globaltimer();
    while (*tag != seq) {
        if (globaltimer() - t0 > limit) {
            atomicOr(status, ST_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Give up a poll: record the timeout and raise the abort flag.
__device__ __forceinline__ bool ds_poll_expired(unsigned long long &t0, const DSArgs &a) {
    const unsigned long long now = globaltimer();
    if (!t0) t0 = now;
    if (now - t0 <= a.wait_ns) return false;
    atomicOr(a.status, ST_WAIT_TIMEOUT);
    atomicExch(a.abort, 1);
    return true;
}

constexpr int LL_BATCH = 16;   // words in flight per thread

// Read n (<= LL_BATCH) activation words src[32 u], u < n, written with
// `tag`: one batch of loads, then batches of reloads of the words not
// written yet.  False when the wait ran out or another CTA aborted.
__device__ __forceinline__ bool ll_fetch(const ll_t *src, int n, uint32_t tag,
                                         float (&out)[LL_BATCH], const DSArgs &a) {
    ll_t w[LL_BATCH];
    unsigned pend = 0;
#pragma unroll
    for (int u = 0; u < LL_BATCH; u++) {
        w[u] = u < n ? ld_ll(src + 32 * u) : 0ull;
        if (u < n) pend |= 1u << u;
    }
    unsigned long long t0 = 0;
    for (;;) {
#pragma unroll
        for (int u = 0; u < LL_BATCH; u++)
            if ((uint32_t)(w[u] >> 32) == tag) pend &= ~(1u << u);
        if (!pend) break;
#pragma unroll
        for (int u = 0; u < LL_BATCH; u++)
            if (pend >> u & 1u) w[u] = ld_ll(src + 32 * u);
        if (ld_acquire(a.abort) || ds_poll_expired(t0, a)) return false;
    }
#pragma unroll
    for (int u = 0; u < LL_BATCH; u++) out[u] = __uint_as_float((uint32_t)w[u]);
    return true;
}

// One activation word written with `tag`.
__device__ __forceinline__ bool ll_fetch1(const ll_t *src, uint32_t tag, float *out,
                                          const DSArgs &a) {
    ll_t w = ld_ll(src);
    unsigned long long t0 = 0;
    while ((uint32_t)(w >> 32) != tag) {
        __nanosleep(32);
        w = ld_ll(src);
        if (ld_acquire(a.abort) || ds_poll_expired(t0, a)) return false;
    }
    *out = __uint_as_float((uint32_t)w);
    return true;
}

__device__ __forceinline__ void cbar_sync() {   // the consumer warps
    asm volatile("bar.sync 1, %0;" ::"n"(DS_NC) : "memory");
}

// Fixed-shape sum over the consumer threads: the same bits in every CTA.
__device__ __forceinline__ float ds_block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    cbar_sync();   // red[] may still be read from its previous use
    if (l == 0) red[w] = v;
    cbar_sync();
    float r = red[0];
    for (int i = 1; i < DS_NCW; i++) r = __fadd_rn(r, red[i]);
    return r;
}

// Attention splits per head at this position (1 up to att_split_min
// positions, then one more per att_split_min, at most att_spmax).
__device__ __forceinline__ int ds_nsplit(const DSArgs &a, int pos) {
    if (a.att_spmax <= 1) return 1;
    return min(a.att_spmax, (pos + a.att_split_min) / a.att_split_min);
}

// Token fed at the current position (-1: outside the vocabulary).
__device__ __forceinline__ int ds_token(const DSArgs &a) {
    const int pos = a.st->pos, P = a.st->prompt_len;
    const int tok = pos < P ? a.prompt[pos] : __ldcg(a.gen + pos - P);
    return (tok < 0 || tok >= a.vocab) ? -1 : tok;
}

__device__ __forceinline__ uint32_t lo16(uint32_t w) { return w & 0xffffu; }
__device__ __forceinline__ uint32_t hi16(uint32_t w) { return w >> 16; }

// Table word at a slot (a byte offset into the table).
__device__ __forceinline__ float ds_tab(const float *tab, uint32_t off) {
    return *reinterpret_cast<const float *>(reinterpret_cast<const char *>(tab) + off);
}

// The two columns' values for the low or high halves of two stream words.
__device__ __forceinline__ float2 ds_gather(const float *tab, uint32_t w0, uint32_t w1, int hi) {
    return hi ? make_float2(ds_tab(tab, hi16(w0)), ds_tab(tab, hi16(w1)))
              : make_float2(ds_tab(tab, lo16(w0)), ds_tab(tab, lo16(w1)));
}

// The 8 gathered (column 0, column 1) pairs of one step.
struct DSVals {
    float2 v[8];
};

__device__ __forceinline__ DSVals ds_gather_step(const float *tab, const uint4 &q0, const uint4 &q1) {
    DSVals r;
    r.v[0] = ds_gather(tab, q0.x, q1.x, 0);
    r.v[1] = ds_gather(tab, q0.x, q1.x, 1);
    r.v[2] = ds_gather(tab, q0.y, q1.y, 0);
    r.v[3] = ds_gather(tab, q0.y, q1.y, 1);
    r.v[4] = ds_gather(tab, q0.z, q1.z, 0);
    r.v[5] = ds_gather(tab, q0.z, q1.z, 1);
    r.v[6] = ds_gather(tab, q0.w, q1.w, 0);
    r.v[7] = ds_gather(tab, q0.w, q1.w, 1);
    return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float f16_lo(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
}
__device__ __forceinline__ float f16_hi(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// The 8 (column 0, column 1) values of one step from its two stream words
// per lane: table gathers (slot streams) or the patterns themselves.
template <int VM>
__device__ __forceinline__ DSVals ds_step_vals(const float *tab, const uint4 &q0, const uint4 &q1) {
    if constexpr (VM == TTX_VSLOT) {
        return ds_gather_step(tab, q0, q1);
    } else {
        const uint32_t a[4] = {q0.x, q0.y, q0.z, q0.w}, b[4] = {q1.x, q1.y, q1.z, q1.w};
        DSVals r;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            if constexpr (VM == TTX_VBF16) {
                r.v[2 * c] = make_float2(bf16_lo(a[c]), bf16_lo(b[c]));
                r.v[2 * c + 1] = make_float2(bf16_hi(a[c]), bf16_hi(b[c]));
            } else {
                r.v[2 * c] = make_float2(f16_lo(a[c]), f16_lo(b[c]));
                r.v[2 * c + 1] = make_float2(f16_hi(a[c]), f16_hi(b[c]));
            }
        }
        return r;
    }
}

template <int VM>
__device__ __forceinline__ DSVals ds_load_step(const uint8_t *lp, const float *tab) {
    const uint4 q0 = *reinterpret_cast<const uint4 *>(lp);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(lp + 512);
    return ds_step_vals<VM>(tab, q0, q1);
}

__device__ __forceinline__ float2 ds_mac_step(const float *xr, const DSVals &v, float2 acc) {
    const float4 xa = *reinterpret_cast<const float4 *>(xr);
    const float4 xb = *reinterpret_cast<const float4 *>(xr + 4);
    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    float2 p[8];
#pragma unroll
    for (int e = 0; e < 8; e++) p[e] = __fmul2_rn(make_float2(xv[e], xv[e]), v.v[e]);
#pragma unroll
    for (int e = 0; e < 8; e++) acc = __fadd2_rn(acc, p[e]);
    return acc;
}

// One step of a value stream as loaded: the lane's two stream words and
// its 8 x values.
struct DSRaw {
    uint4 q0, q1;
    float4 xa, xb;
};

__device__ __forceinline__ DSRaw ds_load_raw(const uint8_t *lp, const float *xr) {
    DSRaw r;
    r.q0 = *reinterpret_cast<const uint4 *>(lp);
    r.q1 = *reinterpret_cast<const uint4 *>(lp + 512);
    r.xa = *reinterpret_cast<const float4 *>(xr);
    r.xb = *reinterpret_cast<const float4 *>(xr + 4);
    return r;
}

template <int VM>
__device__ __forceinline__ float2 ds_mac_raw(const DSRaw &r, float2 acc) {
    const DSVals v = ds_step_vals<VM>(nullptr, r.q0, r.q1);
    const float xv[8] = {r.xa.x, r.xa.y, r.xa.z, r.xa.w, r.xb.x, r.xb.y, r.xb.z, r.xb.w};
    float2 pr[8];
#pragma unroll
    for (int e = 0; e < 8; e++) pr[e] = __fmul2_rn(make_float2(xv[e], xv[e]), v.v[e]);
#pragma unroll
    for (int e = 0; e < 8; e++) acc = __fadd2_rn(acc, pr[e]);
    return acc;
}

// Steps [0, n) of a piece whose every row is inside the lane's chunk, in
// order.  Two register sets of two steps each: the next two steps' weights
// (and, for value streams, x) are in flight while the current two are
// multiplied and added in row order.
template <int VM>
__device__ __forceinline__ float2 ds_steps_full(const uint8_t *pc, int lane, const float *xr,
                                                int n, const float *tab, float2 acc) {
    const uint8_t *lp = pc + lane * 16;
    int i = 0;
    if constexpr (VM != TTX_VSLOT) {
        if (n >= 4) {
            DSRaw a0 = ds_load_raw(lp, xr), a1 = ds_load_raw(lp + TTX_STEP, xr + 8);
            for (; i + 4 <= n; i += 4) {
                const DSRaw b0 = ds_load_raw(lp + (i + 2) * TTX_STEP, xr + 8 * i + 16);
                const DSRaw b1 = ds_load_raw(lp + (i + 3) * TTX_STEP, xr + 8 * i + 24);
                acc = ds_mac_raw<VM>(a0, acc);
                acc = ds_mac_raw<VM>(a1, acc);
                if (i + 6 <= n) {
                    a0 = ds_load_raw(lp + (i + 4) * TTX_STEP, xr + 8 * i + 32);
                    a1 = ds_load_raw(lp + (i + 5) * TTX_STEP, xr + 8 * i + 40);
                }
                acc = ds_mac_raw<VM>(b0, acc);
                acc = ds_mac_raw<VM>(b1, acc);
            }
        }
        for (; i < n; i++) acc = ds_mac_raw<VM>(ds_load_raw(lp + i * TTX_STEP, xr + 8 * i), acc);
        return acc;
    }
    if (n >= 4) {
        DSVals a0 = ds_load_step<VM>(lp, tab), a1 = ds_load_step<VM>(lp + TTX_STEP, tab);
        for (; i + 4 <= n; i += 4) {
            const DSVals b0 = ds_load_step<VM>(lp + (i + 2) * TTX_STEP, tab);
            const DSVals b1 = ds_load_step<VM>(lp + (i + 3) * TTX_STEP, tab);
            acc = ds_mac_step(xr + 8 * i, a0, acc);
            acc = ds_mac_step(xr + 8 * i + 8, a1, acc);
            if (i + 6 <= n) {
                a0 = ds_load_step<VM>(lp + (i + 4) * TTX_STEP, tab);
                a1 = ds_load_step<VM>(lp + (i + 5) * TTX_STEP, tab);
            }
            acc = ds_mac_step(xr + 8 * i + 16, b0, acc);
            acc = ds_mac_step(xr + 8 * i + 24, b1, acc);
        }
    }
    for (; i < n; i++) acc = ds_mac_step(xr + 8 * i, ds_load_step<VM>(lp + i * TTX_STEP, tab), acc);
    return acc;
}

// Split groups: one column of the lane's pair (pc points at that column's
// 512 bytes of each step).  The 8 values of one step's word q, in row order.
template <int VM>
__device__ __forceinline__ void ds_half_vals(const float *tab, const uint4 &q, float (&v)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        if constexpr (VM == TTX_VSLOT) {
            v[2 * c] = ds_tab(tab, lo16(w[c]));
            v[2 * c + 1] = ds_tab(tab, hi16(w[c]));
        } else if constexpr (VM == TTX_VBF16) {
            v[2 * c] = bf16_lo(w[c]);
            v[2 * c + 1] = bf16_hi(w[c]);
        } else {
            v[2 * c] = f16_lo(w[c]);
            v[2 * c + 1] = f16_hi(w[c]);
        }
    }
}

struct DSHalfRaw {
    uint4 q;
    float4 xa, xb;
};

__device__ __forceinline__ DSHalfRaw ds_load_half(const uint8_t *lp, const float *xr) {
    DSHalfRaw r;
    r.q = *reinterpret_cast<const uint4 *>(lp);
    r.xa = *reinterpret_cast<const float4 *>(xr);
    r.xb = *reinterpret_cast<const float4 *>(xr + 4);
    return r;
}

// acc = fl(acc + fl(x[k] * w[k])) over the step's 8 rows, in order.
template <int VM>
__device__ __forceinline__ float ds_mac_half(const DSHalfRaw &r, const float *tab, float acc) {
    float v[8];
    ds_half_vals<VM>(tab, r.q, v);
    const float xv[8] = {r.xa.x, r.xa.y, r.xa.z, r.xa.w, r.xb.x, r.xb.y, r.xb.z, r.xb.w};
    float p[8];
#pragma unroll
    for (int e = 0; e < 8; e++) p[e] = __fmul_rn(xv[e], v[e]);
#pragma unroll
    for (int e = 0; e < 8; e++) acc = __fadd_rn(acc, p[e]);
    return acc;
}

// Steps [0, n) of a piece, every row inside the lane's chunk, in order; the
// next two steps' words and x are in flight while the current two are added.
template <int VM>
__device__ __forceinline__ float ds_steps_half(const uint8_t *pc, int lane, const float *xr,
                                               int n, const float *tab, float acc) {
    const uint8_t *lp = pc + lane * 16;
    int i = 0;
    if (n >= 4) {
        DSHalfRaw a0 = ds_load_half(lp, xr), a1 = ds_load_half(lp + TTX_STEP, xr + 8);
        for (; i + 4 <= n; i += 4) {
            const DSHalfRaw b0 = ds_load_half(lp + (i + 2) * TTX_STEP, xr + 8 * i + 16);
            const DSHalfRaw b1 = ds_load_half(lp + (i + 3) * TTX_STEP, xr + 8 * i + 24);
            acc = ds_mac_half<VM>(a0, tab, acc);
            acc = ds_mac_half<VM>(a1, tab, acc);
            if (i + 6 <= n) {
                a0 = ds_load_half(lp + (i + 4) * TTX_STEP, xr + 8 * i + 32);
                a1 = ds_load_half(lp + (i + 5) * TTX_STEP, xr + 8 * i + 40);
            }
            acc = ds_mac_half<VM>(b0, tab, acc);
            acc = ds_mac_half<VM>(b1, tab, acc);
        }
    }
    for (; i < n; i++) acc = ds_mac_half<VM>(ds_load_half(lp + i * TTX_STEP, xr + 8 * i), tab, acc);
    return acc;
}

// A whole piece (DS_PIECE_STEPS steps, every row inside the lane's chunk),
// one column: fully unrolled so the loads are issued ahead of the dependent
// add chain (scalar adds: the f32x2 add's dependent latency is about twice
// the scalar one's).
template <int VM>
__device__ __forceinline__ float ds_piece_half(const uint8_t *pc, int lane, const float *xr,
                                               const float *tab, float acc) {
    const uint8_t *lp = pc + lane * 16;
    constexpr int AHEAD = 4;
    DSHalfRaw r[AHEAD];
#pragma unroll
    for (int i = 0; i < AHEAD; i++) r[i] = ds_load_half(lp + i * TTX_STEP, xr + 8 * i);
#pragma unroll
    for (int i = 0; i < DS_PIECE_STEPS; i++) {
        const DSHalfRaw cur = r[i % AHEAD];
        if (i + AHEAD < DS_PIECE_STEPS)
            r[i % AHEAD] = ds_load_half(lp + (i + AHEAD) * TTX_STEP, xr + 8 * (i + AHEAD));
        acc = ds_mac_half<VM>(cur, tab, acc);
    }
    return acc;
}

// The same for both columns of the lane's pair, as two scalar chains.
template <int VM>
__device__ __forceinline__ float2 ds_piece_full(const uint8_t *pc, int lane, const float *xr,
                                                const float *tab, float2 acc) {
    const uint8_t *lp = pc + lane * 16;
    constexpr int AHEAD = 3;
    DSRaw r[AHEAD];
#pragma unroll
    for (int i = 0; i < AHEAD; i++) r[i] = ds_load_raw(lp + i * TTX_STEP, xr + 8 * i);
#pragma unroll
    for (int i = 0; i < DS_PIECE_STEPS; i++) {
        const DSRaw cur = r[i % AHEAD];
        if (i + AHEAD < DS_PIECE_STEPS)
            r[i % AHEAD] = ds_load_raw(lp + (i + AHEAD) * TTX_STEP, xr + 8 * (i + AHEAD));
        float v0[8], v1[8];
        {
            DSHalfRaw h0 = {cur.q0, cur.xa, cur.xb}, h1 = {cur.q1, cur.xa, cur.xb};
            ds_half_vals<VM>(tab, h0.q, v0);
            ds_half_vals<VM>(tab, h1.q, v1);
        }
        const float xv[8] = {cur.xa.x, cur.xa.y, cur.xa.z, cur.xa.w,
                             cur.xb.x, cur.xb.y, cur.xb.z, cur.xb.w};
        float p0[8], p1[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            p0[e] = __fmul_rn(xv[e], v0[e]);
            p1[e] = __fmul_rn(xv[e], v1[e]);
        }
#pragma unroll
        for (int e = 0; e < 8; e++) {
            acc.x = __fadd_rn(acc.x, p0[e]);
            acc.y = __fadd_rn(acc.y, p1[e]);
        }
    }
    return acc;
}

// One step of which only the first `rows` rows (< 8, may be <= 0) are in
// the lane's chunk (split groups).
template <int VM>
__device__ __forceinline__ float ds_step_tail_half(const uint8_t *stp, int lane, const float *xr,
                                                   int rows, const float *tab, float acc) {
    if (rows <= 0) return acc;
    const uint4 q = *reinterpret_cast<const uint4 *>(stp + lane * 16);
    float v[8];
    ds_half_vals<VM>(tab, q, v);
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < rows) acc = __fadd_rn(acc, __fmul_rn(xr[e], v[e]));
    return acc;
}

// One step of which only the first `rows` rows (< 8, may be <= 0) are in
// the lane's chunk.
template <int VM>
__device__ __forceinline__ float2 ds_step_tail(const uint8_t *stp, int lane, const float *xr,
                                               int rows, const float *tab, float2 acc) {
    if (rows <= 0) return acc;
    const uint4 q0 = *reinterpret_cast<const uint4 *>(stp + lane * 16);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(stp + 512 + lane * 16);
    const DSVals v = ds_step_vals<VM>(tab, q0, q1);
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (e < rows) acc = __fadd2_rn(acc, __fmul2_rn(make_float2(xr[e], xr[e]), v.v[e]));
    return acc;
}

// ttx_col with the head dim a compile-time constant (no divisions).
template <int HD>
__device__ __forceinline__ int ds_col(const TTXDesc &d, int g, int c) {
    if (d.colmode == TTX_GATE_UP) {
        const int n = 4 * g + (c & 3);
        if (n >= d.F) return -1;
        return c < 4 ? n : d.F + n;
    }
    if (d.colmode == TTX_ROPE) {
        constexpr int PH = HD / 8;   // groups per rotated head
        const int rg = d.rope_heads * PH;
        if (g < rg) {
            const int head = g / PH, d0 = (g % PH) * 4;
            return head * HD + (c < 4 ? d0 + c : d0 + HD / 2 + (c - 4));
        }
        const int n = rg * 8 + (g - rg) * 8 + c;
        return n < d.N ? n : -1;
    }
    const int n = g * TTX_GCOLS + c;
    return n < d.N ? n : -1;
}

// Walks a CTA's weight pieces in the order its producer loads them from the
// shared ring (phase, task round, piece, task of the round), continuing
// with the first phase after the last (the next step's weights are the
// same): the L2 prefetch cursor.
struct DSPieceCursor {
    int p = 0, r = 0, b = 0, j = 0, wraps = 0;
    int J = 0, W = 1, ns = 0, np = 0, nr = 0, NW = 1;
    const uint8_t *stream = nullptr;

    // the first GEMV phase with work for this CTA at or after `from`
    __device__ bool enter(const DSArgs &a, int from, int cta, int G) {
        for (int k = 0; k < a.nphases; k++) {
            int q = from + k;
            if (q >= a.nphases) q -= a.nphases;
            const DSPhase &ph = a.phases[q];
            if (ph.kind != DS_GEMV || cta >= ph.ntasks) continue;
            if (q < from) wraps++;
            p = q;
            NW = a.task_warps;
            W = ph.d.W;
            J = (ph.ntasks - cta + G - 1) / G * W;
            ns = ph.d.ns;
            np = ph.npieces;
            stream = ph.stream;
            r = b = j = 0;
            nr = min(NW, J);
            return true;
        }
        return false;
    }
    __device__ const uint8_t *addr(int cta, int G, uint32_t *bytes) const {
        *bytes = (uint32_t)min(DS_PIECE_STEPS, ns - DS_PIECE_STEPS * b) * TTX_STEP;
        const int jj = NW * r + j;
        const size_t gw = (size_t)(cta + (jj / W) * G) * W + (jj % W);
        return stream + (gw * ns + (size_t)DS_PIECE_STEPS * b) * TTX_STEP;
    }
    __device__ bool next(const DSArgs &a, int cta, int G) {
        if (++j < nr) return true;
        j = 0;
        if (++b < np) return true;
        b = 0;
        if (NW * ++r < J) {
            nr = min(NW, J - NW * r);
            return true;
        }
        return enter(a, p + 1, cta, G);
    }
};

// HD: head dim; VM: what the streams hold (TTXVals, the same for every
// matrix of the step).
template <int HD, int VM>
__global__ void __launch_bounds__(DS_THREADS, 1) k_decode_step(const __grid_constant__ DSArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NQ = HD / 4;                 // float4 per head row
    constexpr int NPG = DS_NC / NQ;            // position groups in P.V
    __shared__ float red[DS_NCW + 1];
    __shared__ __align__(16) float qv[HD];
    __shared__ __align__(16) float knv[2][HD];   // this position's k and v (attention)
    __shared__ __align__(16) float pctx[NPG][HD];
    __shared__ float rcs[2][HD];               // RoPE cos / sin of this position
    __shared__ int s_bad;                      // a consumer warp gave up a wait
    __shared__ int s_prod;                     // pieces the producer has issued (shared ring)
    __shared__ int s_prod_done;
    __shared__ __align__(16) DSPhase s_ph[2];  // consumers: this phase's and the next one's
    __shared__ int ri[DS_NCW];
    __shared__ float2 sub_y[DS_NCW][4];        // split groups: each warp's column sums

    const int G = gridDim.x, cta = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    uint8_t *ring = smem;
    float *tabs = reinterpret_cast<float *>(smem + (size_t)S * DS_STAGE);   // 2 tables
    float *wns = tabs + 2 * a.tab_cap; // 2 phases' norm weights
    float *xc = wns + 2 * a.wn_cap;    // staged x, chunk-major
    float *sc = xc;                    // attention scores (no GEMV then)
    float *hsave = xc + a.xc_cap;      // raw x of QKV / gate_up: the residual of O / down
    uint64_t *full = reinterpret_cast<uint64_t *>(hsave + a.wn_cap);
    uint64_t *empty = full + S;
    uint64_t *tready = empty + S;      // [2] table built
    uint64_t *tfree = tready + 2;      // [2] table no longer read
    uint64_t *rawfull = tfree + 2;     // codebook bulk copy landed
    // Sequence number of the piece each stage holds or awaits.  A consumer
    // may run a whole ring ahead of another; full[s]'s parity alone cannot
    // tell its piece from the stage's previous one, the tag can.
    volatile int *stage_seq = reinterpret_cast<volatile int *>(rawfull + 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);   // two arrivals: the pair of warps of a split
                                       // group, or one warp arriving twice
            stage_seq[s] = -1;
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tready[i], 1);
            mbar_init(&tfree[i], 1);
        }
        mbar_init(rawfull, 1);
        mbar_fence_init();
        s_bad = 0;
        s_prod = 0;
        s_prod_done = 0;
    }
    for (int i = threadIdx.x; i < DSP_KINDS * a.world; i += blockDim.x) ds_speers[i] = a.peers[i];
    if (threadIdx.x == 0) ds_gpu_scope = a.world == 1 && a.gpu_scope;
    __syncthreads();

    // ================================================================ producer
    if (warp == DS_TABLER && lane != 0) {
        // Lanes 1..31: keep the weight pieces up to l2_pf past the producer's
        // on their way into L2 (plain L2 prefetches, not the copy engine the
        // ring loads use), so HBM keeps streaming while the ring is full and
        // the consumers wait for a phase's input.  The cursor runs on into
        // the next step's first pieces.
        if (a.l2_pf <= 0) return;
        DSPieceCursor c;
        if (!c.enter(a, 0, cta, G)) return;
        const volatile int *prod = &s_prod;
        const volatile int *pdone = &s_prod_done;
        int pf = 0, last = -1;
        unsigned long long t_last = globaltimer();
        while (c.wraps <= 1) {
            const int pr = *prod;
            const bool done = *pdone != 0;
            if (pr != last) {
                last = pr;
                t_last = globaltimer();
            }
            if (pf > pr + a.l2_pf) {   // far enough ahead: wait for the producer
                if (done || ld_acquire(a.abort) || globaltimer() - t_last > a.wait_ns) break;
                __nanosleep(256);
                continue;
            }
            if (pf >= max(pr, S)) {    // not loaded yet, nor about to be
                uint32_t nb;
                const uint8_t *base = c.addr(cta, G, &nb);
                for (uint32_t o = (uint32_t)(lane - 1) * 128u; o < nb; o += 31u * 128u)
                    prefetch_l2_line(base + o);
            }
            if (!c.next(a, cta, G)) break;
            pf++;
        }
        return;
    }
    if (warp == DS_TABLER) {
        {
            // The tables, two phases deep, by bulk copy of the replicated
            // table built at upload (lane 0).
            int q = 0;
            const int kpos = a.st->pos;
            for (int p = 0; p < a.nphases; p++) {
                const DSPhase &ph = a.phases[p];
                if (ph.kind == DS_ATT) {
                    // this CTA's attention tasks read cached k and v rows of
                    // their head's group, positions [j0, j1) of the split:
                    // into L2 while the QKV phase runs (the first head of
                    // each group asks for the rows of the cache, which holds
                    // positions before kpos)
                    if (lane == 0 && a.kv_prefetch && kpos > 0 && kpos < a.max_pos) {
                        const int nsp = ds_nsplit(a, kpos);
                        for (int tk = cta; tk < ph.ntasks; tk += G) {
                            const int hq = tk % a.nh, sp = tk / a.nh;
                            if (sp >= nsp || hq % a.groups) continue;
                            const int span = (kpos + nsp) / nsp;
                            const int j0 = sp * span, j1 = min(kpos, j0 + span);   // cached rows only
                            if (j1 <= j0) continue;
                            const size_t off = (((size_t)ph.layer * a.nkv + hq / a.groups) *
                                                    a.max_pos + j0) * HD;
                            const uint32_t nb = (uint32_t)(j1 - j0) * HD * 4;
                            for (uint32_t o = 0; o < nb; o += 65536) {
                                prefetch_l2_bulk(reinterpret_cast<const uint8_t *>(a.kc + off) + o,
                                                 min(65536u, nb - o));
                                prefetch_l2_bulk(reinterpret_cast<const uint8_t *>(a.vc + off) + o,
                                                 min(65536u, nb - o));
                            }
                        }
                    }
                    continue;
                }
                if (ph.kind != DS_GEMV || cta >= ph.ntasks) continue;
                if (ld_acquire(a.abort)) return;
                const int slot = q & 1;
                float *tab = tabs + slot * a.tab_cap;
                if (q >= 2 && !mbar_wait_idle(&tfree[slot], ((q >> 1) - 1) & 1, a.status, a.wait_ns)) {
                    atomicExch(a.abort, 1);
                    return;
                }
                if (lane == 0) {   // the table, and the norm weights the prologue reads
                    const uint32_t cb = (uint32_t)ph.table_bytes;
                    const uint32_t wb =
                        ph.xmode == DX_EMBED || ph.xmode == DX_NORM ? (uint32_t)ph.d.K * 4 : 0u;
                    mbar_expect_tx(rawfull, cb + wb);
                    for (uint32_t off = 0; off < cb; off += 32768)
                        bulk_load(reinterpret_cast<uint8_t *>(tab) + off,
                                  reinterpret_cast<const uint8_t *>(ph.table) + off,
                                  min(32768u, cb - off), rawfull);
                    for (uint32_t off = 0; off < wb; off += 32768)
                        bulk_load(reinterpret_cast<uint8_t *>(wns + slot * a.wn_cap) + off,
                                  reinterpret_cast<const uint8_t *>(ph.norm_w) + off,
                                  min(32768u, wb - off), rawfull);
                }
                if (!mbar_wait_idle(rawfull, q & 1, a.status, a.wait_ns)) {
                    atomicExch(a.abort, 1);
                    return;
                }
                mbar_arrive(&tready[slot]);
                q++;
            }
            return;
        }
    }
    if (warp == DS_PRODUCER) {
        if (lane != 0) return;
        DS_PROF_INIT();
        int seq = 0;   // slot streams, in the consumers' order
        const uint64_t pol = l2_evict_first();
        const int NW = a.task_warps;
        for (int p = 0; p < a.nphases; p++) {
            const DSPhase &ph = a.phases[p];
            if (ph.kind != DS_GEMV || cta >= ph.ntasks) continue;
            if (ld_acquire(a.abort)) return;
            const int W = ph.d.W;
            const int J = (ph.ntasks - cta + G - 1) / G * W, ns = ph.d.ns, np = ph.npieces;
#ifdef KLLM_DS_PROFILE
            unsigned long long pw = 0;   // ns waiting for free stages in this phase
            bool first = true;
#endif
            const int NWt = NW / ph.csplit;   // tasks per round
            for (int r = 0; NWt * r < J; r++) {
                const int nr = min(NWt, J - NWt * r);
                for (int b = 0; b < np; b++) {
                    const uint32_t bytes = (uint32_t)min(DS_PIECE_STEPS, ns - DS_PIECE_STEPS * b) * TTX_STEP;
                    for (int j = NWt * r; j < NWt * r + nr; j++, seq++) {
                        const size_t gw = (size_t)(cta + (j / W) * G) * W + (j % W);
                        const int s = seq % S;
#ifdef KLLM_DS_PROFILE
                        const unsigned long long tw = globaltimer();
#endif
                        if (seq >= S && !mbar_wait_idle(&empty[s], ((seq / S) - 1) & 1, a.status, a.wait_ns)) {
                            atomicExch(a.abort, 1);
                            return;
                        }
#ifdef KLLM_DS_PROFILE
                        const unsigned long long tn = globaltimer();
                        pw += tn - tw;
                        DS_STAMP(first, 5, tn);
                        first = false;
                        DS_STAMP(true, 6, tn);
                        DS_STAMP(true, 7, pw);
#endif
                        stage_seq[s] = seq;
                        mbar_expect_tx(&full[s], bytes);
                        bulk_load_hint(ring + (size_t)s * DS_STAGE,
                                       ph.stream + (gw * ns + (size_t)DS_PIECE_STEPS * b) * TTX_STEP,
                                       bytes, &full[s], pol);
                        *reinterpret_cast<volatile int *>(&s_prod) = seq + 1;

                    }
                }
            }
        }
        *reinterpret_cast<volatile int *>(&s_prod_done) = 1;
        return;
    }

    // =============================================================== consumers
    const int tid = threadIdx.x;
    const int t = lane & 7, cp = lane >> 3;    // chunk, column pair
    // This step's number: the tag of every activation word written in it,
    // and (times a phase's arrivals) the lm_head counter's target.
    const int ep1 = *a.epoch + 1;
    const int pos = a.st->pos;
    DS_PROF_INIT();
    if (pos < a.max_pos)   // read by the QKV epilogues, after the first barrier
        for (int d = tid; d < HD; d += DS_NC) {
            rcs[0][d] = __ldg(a.rope_cos + (size_t)pos * HD + d);
            rcs[1][d] = __ldg(a.rope_sin + (size_t)pos * HD + d);
        }
    // The phase descriptors come through shared memory: warp 0 copies the
    // next one while the current phase runs (cp.async, waited for before
    // the phase's closing barrier).
    auto ph_fetch = [&](int p) {
        if (warp == 0 && p < a.nphases) {
            const char *src = reinterpret_cast<const char *>(a.phases + p);
            char *dst = reinterpret_cast<char *>(&s_ph[p & 1]);
            for (int i = lane; i < (int)sizeof(DSPhase) / 16; i += 32) cp_async16(dst + 16 * i, src + 16 * i);
            cp_async_commit();
        }
    };
    auto ph_ready = [&]() {
        if (warp == 0) cp_async_wait_all();
    };
    ph_fetch(0);
    ph_ready();
    cbar_sync();
    int seq_base = 0, q = 0;
    float lm_v = -INFINITY;                    // this warp's first maximum
    int lm_i = -1;
    bool bad = false;                          // this warp gave up a wait
    for (int p = 0; p < a.nphases; p++) {
        // Warp 0 refills the other slot while this phase runs, so that slot
        // (the previous phase's) is not read from here on, and this one is
        // not read after the phase's closing barrier except by the last
        // phase (lm_head: nothing is fetched after it).
        const DSPhase &ph = s_ph[p & 1];
        const int ntasks = ph.ntasks, emode = ph.emode;
        ph_fetch(p + 1);
        DS_STAMP(tid == 0, 0, globaltimer());
#ifdef KLLM_DS_PROFILE
        const unsigned long long c0 = clock64();
        if (p == 0 && cta == 0 && tid == 0) {   // the %globaltimer step
            const unsigned long long g0 = globaltimer();
            unsigned long long g1 = g0;
            for (int i = 0; i < 100000 && g1 == g0; i++) g1 = globaltimer();
            DS_STAMP(true, 14, g1 - g0);
        }
#endif
        if (cta >= ntasks) {
            ph_ready();
            cbar_sync();
            continue;
        }
        const uint32_t otag = ds_tag(ep1, ph.layer);
        if (ph.kind == DS_GEMV) {
            const TTXDesc &d = ph.d;
            const int K = d.K, xs = ph.xs, xmode = ph.xmode;
            // ------------------------------------------------ stage x
            // Warp w stages its rows of x -- chunk w (reference order,
            // T <= 8) or chunks W*w .. W*w + W - 1 (fast order: equal chunks
            // of L rows, one contiguous range) -- then rmsnorm in place:
            // x * rsqrt(mean(x^2) + eps) * w.  Tagged inputs are polled:
            // the wait for the producing phase and the read are one.
            const bool norm = xmode == DX_EMBED || xmode == DX_NORM;
            const int CH = (d.T + DS_NCW - 1) / DS_NCW;   // chunks per warp
            const int wrows = CH == 1 ? (warp < d.T ? d.chunk_len(warp) : 0) : CH * d.base;
            const int wk0 = CH == 1 ? (warp < d.T ? d.chunk_start(warp) : 0) : warp * CH * d.base;
            // row r of the warp's range -> its slot in xc
            auto slot_of = [&](int r) {
                const int cq = CH == 1 ? 0 : (int)__umulhi((unsigned)r, ph.lmagic);
                return (CH * warp + cq) * xs + (r - cq * d.base);
            };
            const float *emb = nullptr;
            if (xmode == DX_EMBED) {
                int tok = lane == 0 ? ds_token(a) : 0;
                tok = __shfl_sync(0xffffffffu, tok, 0);
                if (tok < 0) {
                    if (lane == 0) atomicOr(a.status, ST_BAD_TOKEN);
                    tok = 0;
                }
                emb = a.embed + (size_t)tok * K;
            }
            const uint32_t xtag = ds_tag(ep1, ph.x_layer);
            // Input of O after split attention: per head, M = max of the
            // splits' maxima, weights w_s = exp(m_s - M) and 1 / sum_s l_s w_s
            // (shared, in pctx), then each row is sum_s P.V_s w_s / that sum.
            const int nsp = xmode == DX_ATT ? ds_nsplit(a, pos) : 1;
            float *atab = &pctx[0][0];                 // [nsp][nh][2] (max, sum)
            float *awt = atab + 2 * nsp * a.nh;        // [nh][nsp + 1]: weights, 1 / denominator
            if (nsp > 1) {
                for (int i = tid; i < 2 * nsp * a.nh && !bad; i += DS_NC)
                    if (!ll_fetch1(a.att_ml + i, xtag, atab + i, a)) bad = true;
                cbar_sync();
                for (int h = tid; h < a.nh; h += DS_NC) {
                    float M = atab[2 * h];
                    for (int sp = 1; sp < nsp; sp++) M = fmaxf(M, atab[2 * (sp * a.nh + h)]);
                    float den = 0.f;
                    for (int sp = 0; sp < nsp; sp++) {
                        const float w = (float)exp((double)__fsub_rn(atab[2 * (sp * a.nh + h)], M));
                        awt[h * (nsp + 1) + sp] = w;
                        den = __fadd_rn(den, __fmul_rn(atab[2 * (sp * a.nh + h) + 1], w));
                    }
                    awt[h * (nsp + 1) + nsp] = __fdiv_rn(1.0f, den);
                }
                cbar_sync();
            }
            float ss = 0.f;
            for (int b0 = 0; b0 < wrows; b0 += 32 * LL_BATCH) {
                float v[LL_BATCH];
                const int nu = min(LL_BATCH, (wrows - b0 - lane + 31) / 32);   // rows b0 + lane + 32u
                if (emb) {
#pragma unroll
                    for (int u = 0; u < LL_BATCH; u++)
                        v[u] = u < nu ? __ldcg(emb + wk0 + b0 + lane + 32 * u) : 0.f;
                } else if (nsp > 1) {
                    float num[LL_BATCH], part[LL_BATCH];
#pragma unroll
                    for (int u = 0; u < LL_BATCH; u++) num[u] = 0.f;
                    for (int sp = 0; sp < nsp && !bad; sp++) {
                        if (!ll_fetch(a.att_part + (size_t)sp * a.qd + wk0 + b0 + lane, nu, xtag,
                                      part, a)) {
                            bad = true;
                            break;
                        }
#pragma unroll
                        for (int u = 0; u < LL_BATCH; u++) {
                            const int h = (wk0 + b0 + lane + 32 * u) / HD;
                            if (u < nu)
                                num[u] = __fadd_rn(num[u], __fmul_rn(part[u], awt[h * (nsp + 1) + sp]));
                        }
                    }
#pragma unroll
                    for (int u = 0; u < LL_BATCH; u++) {
                        const int h = (wk0 + b0 + lane + 32 * u) / HD;
                        v[u] = u < nu ? __fmul_rn(num[u], awt[h * (nsp + 1) + nsp]) : 0.f;
                    }
                } else if (!bad && !ll_fetch(ph.x + wk0 + b0 + lane, nu, xtag, v, a)) {
                    bad = true;
                }
                if (bad) continue;
#pragma unroll
                for (int u = 0; u < LL_BATCH; u++)
                    if (u < nu) {
                        const int r = b0 + lane + 32 * u;
                        xc[slot_of(r)] = v[u];
                        ss = __fadd_rn(ss, __fmul_rn(v[u], v[u]));
                        if (ph.save_x) hsave[wk0 + r] = v[u];
                    }
            }
            DS_STAMP(tid == 0, 1, globaltimer());
            const int slot = q & 1;
            const float *tab = tabs + slot * a.tab_cap;
            if (!bad && !mbar_wait(&tready[slot], (q >> 1) & 1, a.status, a.wait_ns)) {
                bad = true;
                atomicExch(a.abort, 1);
            }
            if (bad) s_bad = 1;
            if (norm) {
                const float *wn = wns + slot * a.wn_cap;   // staged with the table
                const float tot = ds_block_sum(ss, red);
                const float add = __fadd_rn(__fmul_rn(tot, 1.0f / (float)K), ph.eps);
                const float rsq = (float)(1.0 / sqrt((double)add));
#pragma unroll 4
                for (int r = lane; r < wrows; r += 32) {
                    const int o = slot_of(r);
                    xc[o] = __fmul_rn(__fmul_rn(xc[o], rsq), wn[wk0 + r]);
                }
            }
            cbar_sync();
            DS_STAMP(tid == 0, 2, globaltimer());
            if (s_bad) break;   // uniform: every consumer warp leaves together
            // ------------------------------------------------ tasks
            const int W = d.W, lw = __ffs(W) - 1;   // W is 1, 2, 4 or 8 (<= task warps)
            const int J = (ph.ntasks - cta + G - 1) / G * W, ns = d.ns, np = ph.npieces;
            const int nfull = d.base / 8;             // steps inside every chunk
            const int NW = a.task_warps;
#ifdef KLLM_DS_PROFILE
            unsigned long long pf_wait = 0, pf_comp = 0, pf_n = 0, pf_nw = 0, pf_epi = 0, pf_redo = 0;
            const unsigned long long c2 = clock64();
#endif
            // warp task j: sub-task w = j % W of group m = j / W; a group's W
            // sub-tasks sit on W adjacent warps of one round of NWt tasks.  A
            // split group (csplit 2) has two warps, `half` 0 for the first
            // column of every lane pair, 1 for the second.
            const int cs = ph.csplit, NWt = NW / cs, half = warp % cs;
            for (int j = warp / cs; warp < NWt * cs && j < J; j += NWt) {
                const int r = j / NWt, nr = min(NWt, J - NWt * r);
                const int m = j >> lw, w = j & (W - 1);
                const int g = (cta + m * G) * a.world + a.rank;   // the matrix's group
                const int ch = DS_TCH * w + t;        // this lane's chunk
                const int len = d.chunk_len(ch);
                const float *xr = ch < d.T ? xc + ch * xs : xc;
                const int nch = min(DS_TCH, d.T - DS_TCH * w);   // chunks in this sub-task
                const int n0 = ds_col<HD>(d, g, 2 * cp), n1 = ds_col<HD>(d, g, 2 * cp + 1);
                float2 acc = make_float2(0.f, 0.f);
                for (int b = 0; b < np; b++) {
                    const int seq = seq_base + r * NWt * np + b * nr + (j - NWt * r);
                    const int s = seq % S, par = (seq / S) & 1;
#ifdef KLLM_DS_PROFILE
                    const unsigned long long tw0 = clock64();
                    const bool landed = mbar_try_wait(&full[s], par);
#endif
                    if (!bad && (!ds_wait_tag(stage_seq + s, seq, a.status, a.wait_ns) ||
                                 !mbar_wait(&full[s], par, a.status, a.wait_ns))) {
                        bad = true;
                        s_bad = 1;
                        atomicExch(a.abort, 1);
                    }
#ifdef KLLM_DS_PROFILE
                    const unsigned long long tl = clock64();
#endif
                    if (!bad) {
                        const uint8_t *st = ring + (size_t)s * DS_STAGE;
                        const int s0 = DS_PIECE_STEPS * b, s1 = min(ns, s0 + DS_PIECE_STEPS);
                        const int sf = min(s1, max(s0, nfull));
                        if (cs == 1 && sf - s0 == DS_PIECE_STEPS && a.unroll) {
                            acc = ds_piece_full<VM>(st, lane, xr + 8 * s0, tab, acc);
                        } else if (cs == 2 && sf - s0 == DS_PIECE_STEPS && a.unroll) {
                            acc.x = ds_piece_half<VM>(st + half * 512, lane, xr + 8 * s0, tab, acc.x);
#ifdef KLLM_DS_PROFILE
                            if (warp == 0 && ds_prof_on) {   // the same piece again, timed alone
                                __syncwarp();
                                const unsigned long long r0 = clock64();
                                const float again =
                                    ds_piece_half<VM>(st + half * 512, lane, xr + 8 * s0, tab, 0.f);
                                __syncwarp();
                                const unsigned long long r1 = clock64();
                                if (lane == 0) pf_redo += r1 - r0 + (again == 12345.f ? 1 : 0);
                            }
#endif
                        } else if (cs == 1) {
                            acc = ds_steps_full<VM>(st, lane, xr + 8 * s0, sf - s0, tab, acc);
                            for (int sg = sf; sg < s1; sg++)
                                acc = ds_step_tail<VM>(st + (sg - s0) * TTX_STEP, lane, xr + 8 * sg,
                                                       len - 8 * sg, tab, acc);
                        } else {
                            acc.x = ds_steps_half<VM>(st + half * 512, lane, xr + 8 * s0, sf - s0,
                                                      tab, acc.x);
                            for (int sg = sf; sg < s1; sg++)
                                acc.x = ds_step_tail_half<VM>(st + (sg - s0) * TTX_STEP + half * 512,
                                                              lane, xr + 8 * sg, len - 8 * sg, tab,
                                                              acc.x);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {   // two arrivals free the stage
                        if (cs == 2)
                            mbar_arrive(&empty[s]);
                        else
                            mbar_arrive_cnt(&empty[s], 2);
                    }
#ifdef KLLM_DS_PROFILE
                    if (warp == 0 && lane == 0) {
                        const unsigned long long tw2 = clock64();
                        pf_wait += tl - tw0;
                        pf_comp += tw2 - tl;
                        pf_n++;
                        pf_nw += landed ? 0 : 1;
                    }
#endif
                }
#ifdef KLLM_DS_PROFILE
                const unsigned long long te0 = clock64();
#endif
                // chunk sums in chunk order (every lane of the pair gets them)
                float2 y;
                if (cs == 1) {
                    y.x = __shfl_sync(0xffffffffu, acc.x, cp * 8);
                    y.y = __shfl_sync(0xffffffffu, acc.y, cp * 8);
#pragma unroll
                    for (int tt = 1; tt < DS_TCH; tt++) {
                        float2 o;
                        o.x = __shfl_sync(0xffffffffu, acc.x, cp * 8 + tt);
                        o.y = __shfl_sync(0xffffffffu, acc.y, cp * 8 + tt);
                        if (tt < nch) y = __fadd2_rn(y, o);
                    }
                } else {   // this warp's column of every pair, in both halves of y
                    float v = __shfl_sync(0xffffffffu, acc.x, cp * 8);
#pragma unroll
                    for (int tt = 1; tt < DS_TCH; tt++) {
                        const float o = __shfl_sync(0xffffffffu, acc.x, cp * 8 + tt);
                        if (tt < nch) v = __fadd_rn(v, o);
                    }
                    y = make_float2(v, v);
                }
                if (W > 1) {   // sub-task sums of the group, in w order
                    const int bar_id = 2 + warp / W;
                    if (t == 0) sub_y[warp][cp] = y;
                    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(32 * W) : "memory");
                    if (w == 0)
                        for (int ww = 1; ww < W; ww++) y = __fadd2_rn(y, sub_y[warp + ww][cp]);
                    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(32 * W) : "memory");
                    if (w != 0) continue;   // the group's first warp stores the result
                }
                // Epilogue: lane t = k of each pair stores column k of it (a
                // split group: lane t = 0 stores this warp's column).
                const int ek = cs == 1 ? t : (t == 0 ? half : 2);   // 2: no column
                const int n = ek ? n1 : n0;
                const float yk = ek ? y.y : y.x;
                if (ph.emode == DE_QKV) {
                    float2 pr;   // rotate-half partner (pair cp ^ 2)
                    pr.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
                    pr.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
                    if (ek < 2 && n >= 0 && !bad && pos < a.max_pos) {
                        if (g < d.rope_heads * (HD / 8)) {
                            const int head = n / HD, dim = n % HD;
                            const float pk = ek ? pr.y : pr.x;
                            const float rt = cp < 2 ? -pk : pk;
                            const float v = __fadd_rn(__fmul_rn(yk, rcs[0][dim]),
                                                      __fmul_rn(rt, rcs[1][dim]));
                            if (head < a.nh) {
                                ds_put_ll(a, DSP_Q, n, v, otag);
                            } else {
                                const int kh = head - a.nh;
                                ds_put(a, DSP_KC, (((size_t)ph.layer * a.nkv + kh) * a.max_pos + pos) * HD + dim, v);
                                ds_put_ll(a, DSP_KN, kh * HD + dim, v, otag);
                            }
                        } else {
                            const int vi = n - a.qd - a.kvd;
                            ds_put(a, DSP_VC, (((size_t)ph.layer * a.nkv + vi / HD) * a.max_pos + pos) * HD + vi % HD, yk);
                            ds_put_ll(a, DSP_VN, vi, yk, otag);
                        }
                    }
                } else if (ph.emode == DE_RESID) {
                    // the residual: the raw x this CTA staged for QKV / gate_up
                    if (ek < 2 && n >= 0 && !bad)
                        ds_put_ll(a, ph.out_kind, n, __fadd_rn(hsave[n], yk), otag);
                } else if (ph.emode == DE_SWIGLU) {
                    float2 up;
                    up.x = __shfl_xor_sync(0xffffffffu, y.x, 16);
                    up.y = __shfl_xor_sync(0xffffffffu, y.y, 16);
                    if (ek < 2 && cp < 2 && n >= 0 && !bad) {
                        const double dg = (double)yk;
                        ds_put_ll(a, ph.out_kind, n,
                                  __fmul_rn((float)(dg / (1.0 + exp(-dg))), ek ? up.y : up.x), otag);
                    }
                } else {   // DE_LM
                    if (ek < 2 && n >= 0 && !bad) {
                        ds_put(a, ph.out_kind, n, yk);
                        if (a.hist && pos < a.hist_rows) a.hist[(size_t)pos * d.N + n] = yk;
                        if (yk > lm_v || (yk == lm_v && lm_i >= 0 && n < lm_i)) {
                            lm_v = yk;
                            lm_i = n;
                        }
                    }
                }
#ifdef KLLM_DS_PROFILE
                if (warp == 0) pf_epi += clock64() - te0;
#endif
            }
            seq_base += J * np;
#ifdef KLLM_DS_PROFILE
            const unsigned long long c3 = clock64();
#endif
            DS_STAMP(tid == 0, 3, globaltimer());
#ifdef KLLM_DS_PROFILE
            DS_STAMP(tid == 0, 8, pf_wait);
            DS_STAMP(tid == 0, 9, pf_comp);
            DS_STAMP(tid == 0, 10, pf_n);
            DS_STAMP(tid == 0, 11, pf_nw);
            DS_STAMP(tid == 0, 12, pf_epi);
            DS_STAMP(tid == 0, 13, c3 - c2);
            DS_STAMP(tid == 0, 15, c2 - c0);
            if (p > 0) DS_STAMP(tid == 0, 14, pf_redo);
#endif
            ph_ready();
            cbar_sync();   // every warp's outputs are stored and the table is free
            DS_STAMP(tid == 0, 4, globaltimer());
            if (tid == 0) mbar_arrive(&tfree[slot]);
            q++;
            if (emode != DE_LM) continue;
            // ------------------------------------------------ token pick
            {   // this CTA's first maximum
                float bv = lm_v;
                int bi = lm_i;
                for (int o = 16; o; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    red[warp] = bv;
                    ri[warp] = bi;
                }
                cbar_sync();
                if (tid == 0) {
                    for (int w2 = 1; w2 < DS_NCW; w2++) {
                        const int oi = ri[w2];
                        const float ov = red[w2];
                        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                            bv = ov;
                            bi = oi;
                        }
                    }
                    for (int r = 0; r < a.world; r++) {
                        ds_peer<float>(a, DSP_CANDV, r)[a.rank * G + cta] = bv;
                        ds_peer<int>(a, DSP_CANDI, r)[a.rank * G + cta] = bi;
                    }
                }
            }
            if (tid == 0) {
                // arrive at every rank's lm_head counter
                int ncta = 0;
                for (int r = 0; r < a.world; r++) ncta += ds_ncta(a, ph.groups_all, r, G);
                bool pick;
                if (a.world == 1) {
                    __threadfence();
                    pick = atomicAdd(a.done + p, 1) == ncta * ep1 - 1;
                } else {
                    __threadfence_system();
                    for (int r = 0; r < a.world; r++)
                        atomicAdd_system(ds_peer<int>(a, DSP_DONE, r) + p, 1);
                    // the token pick runs on every rank: by the last CTA of
                    // this rank to arrive, once every rank's candidates are in
                    const int pl = atomicAdd(a.lm_local, 1);
                    pick = pl == ds_ncta(a, ph.groups_all, a.rank, G) * ep1 - 1 &&
                           ds_wait_counter(a.done + p, ncta * ep1, a.status, a.abort, a.wait_ns);
                }
                if (pick) {
                    // the reference's greedy pick: best = logits[0], then
                    // strict > over the rest in index order
                    __threadfence_system();
                    const float l0 = __ldcg(ph.out);
                    int bidx = 0;
                    if (!(l0 != l0)) {
                        float best = l0;
                        for (int r = 0; r < a.world; r++)
                            for (int c = 0; c < ds_ncta(a, ph.groups_all, r, G); c++) {
                                const float cv = __ldcg(a.cand_v + r * G + c);
                                const int ci = __ldcg(a.cand_i + r * G + c);
                                if (ci >= 0 && (cv > best || (cv == best && ci < bidx))) {
                                    best = cv;
                                    bidx = ci;
                                }
                            }
                    }
                    const int P0 = a.st->prompt_len;
                    if (pos >= P0 - 1) {
                        const int gi = pos - (P0 - 1);
                        if (gi < a.max_gen) {
                            a.gen[gi] = bidx;
                            a.gen_host[gi] = bidx;
                            __threadfence_system();
                        }
                        a.st->n_gen = gi + 1;
                    }
                    a.st->pos = pos + 1;
                    *a.epoch = ep1;
                }
            }
        } else {   // ============================================ attention
            const int l = ph.layer;
            const float *kcl = a.kc + (size_t)l * a.nkv * a.max_pos * HD;
            const float *vcl = a.vc + (size_t)l * a.nkv * a.max_pos * HD;
            const ll_t *knl = ds_peer<ll_t>(a, DSP_KN, a.rank);
            const ll_t *vnl = ds_peer<ll_t>(a, DSP_VN, a.rank);
            // Task tk: head tk % nh, split tk / nh.  Up to 256 positions one
            // split per head (the whole softmax here, ctx words out); longer
            // contexts go to nsp splits of consecutive positions, each
            // leaving its max, its sum of exps and its unnormalised P.V
            // (the O phase's input staging combines them).
            const int nsp = ds_nsplit(a, pos);
            for (int tk = cta; tk < ntasks; tk += G) {
                const int hq = tk % a.nh, sp = tk / a.nh;
                const int g = hq / a.groups;
                const int span = (pos + nsp) / nsp;   // ceil((pos + 1) / nsp)
                const int j0 = sp * span, j1 = min(pos + 1, j0 + span), n = j1 - j0;
                if (pos < a.max_pos && sp < nsp && n > 0) {   // uniform in the CTA
                    // q of this head and this position's k and v of its
                    // group (positions before it come from the cache)
                    for (int i = tid; i < 3 * HD && !bad; i += DS_NC) {
                        const int part = i / HD, dd = i % HD;
                        const ll_t *src = part == 0 ? a.q + hq * HD + dd
                                        : (part == 1 ? knl : vnl) + g * HD + dd;
                        float *dst = part == 0 ? qv + dd : knv[part - 1] + dd;
                        if (!ll_fetch1(src, otag, dst, a)) bad = true;
                    }
                    if (bad) s_bad = 1;
                    cbar_sync();
                    DS_STAMP(tid == 0, 2, globaltimer());
                    if (s_bad) break;
                    // scores: 8 threads per position (HD / 8 dims each, summed in
                    // order, then combined by a fixed butterfly), four
                    // positions per thread in flight
                    {
                        constexpr int TPP = 8, DQ = NQ / TPP;   // float4 per thread and row
                        const int sub = tid % TPP, pl = tid / TPP;   // 32 position lanes
                        const float4 *q4 = reinterpret_cast<const float4 *>(qv) + sub * DQ;
                        for (int base = j0; base < j1; base += 4 * (DS_NC / TPP)) {
                            float4 kk[4][DQ];
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                const int jj = min(base + pl + k * (DS_NC / TPP), j1 - 1);
                                const float4 *kg4 = jj < pos
                                    ? reinterpret_cast<const float4 *>(kcl + ((size_t)g * a.max_pos + jj) * HD)
                                    : reinterpret_cast<const float4 *>(knv[0]);
#pragma unroll
                                for (int e = 0; e < DQ; e++) kk[k][e] = kg4[sub * DQ + e];
                            }
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                float dot = 0.f;
#pragma unroll
                                for (int e = 0; e < DQ; e++) {
                                    const float4 qq = q4[e];
                                    dot = __fadd_rn(dot, __fmul_rn(qq.x, kk[k][e].x));
                                    dot = __fadd_rn(dot, __fmul_rn(qq.y, kk[k][e].y));
                                    dot = __fadd_rn(dot, __fmul_rn(qq.z, kk[k][e].z));
                                    dot = __fadd_rn(dot, __fmul_rn(qq.w, kk[k][e].w));
                                }
                                dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, 1));
                                dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, 2));
                                dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, 4));
                                const int jj = base + pl + k * (DS_NC / TPP);
                                if (sub == 0 && jj < j1) sc[jj - j0] = __fmul_rn(dot, a.scale);
                            }
                        }
                    }
                    cbar_sync();
                    float m = -INFINITY;
                    for (int jj = tid; jj < n; jj += DS_NC) m = fmaxf(m, sc[jj]);
                    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                    if (lane == 0) red[warp] = m;
                    cbar_sync();
                    float mx = red[0];
                    for (int w2 = 1; w2 < DS_NCW; w2++) mx = fmaxf(mx, red[w2]);
                    float sum = 0.f;
                    for (int jj = tid; jj < n; jj += DS_NC) {
                        const float e = (float)exp((double)__fsub_rn(sc[jj], mx));
                        sc[jj] = e;
                        sum = __fadd_rn(sum, e);
                    }
                    const float tot = ds_block_sum(sum, red);
                    if (nsp == 1)
                        for (int jj = tid; jj < n; jj += DS_NC) sc[jj] = __fdiv_rn(sc[jj], tot);
                    cbar_sync();
                    {   // P.V: thread = (dim quad, position group), 4 positions in flight
                        const int dq = tid % NQ, pg = tid / NQ;
                        const float4 *vg4 =
                            reinterpret_cast<const float4 *>(vcl + (size_t)g * a.max_pos * HD) + dq;
                        const float4 vnew = reinterpret_cast<const float4 *>(knv[1])[dq];
                        auto vrow = [&](int j) {
                            return j < pos ? __ldcg(vg4 + (size_t)j * NQ) : vnew;
                        };
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        int jj = pg;
                        for (; jj + 7 * NPG < n; jj += 8 * NPG) {
                            float4 vj[8];
#pragma unroll
                            for (int e = 0; e < 8; e++) vj[e] = vrow(j0 + jj + e * NPG);
#pragma unroll
                            for (int e = 0; e < 8; e++) {
                                const float pj = sc[jj + e * NPG];
                                acc.x = __fadd_rn(acc.x, __fmul_rn(pj, vj[e].x));
                                acc.y = __fadd_rn(acc.y, __fmul_rn(pj, vj[e].y));
                                acc.z = __fadd_rn(acc.z, __fmul_rn(pj, vj[e].z));
                                acc.w = __fadd_rn(acc.w, __fmul_rn(pj, vj[e].w));
                            }
                        }
                        for (; jj < n; jj += NPG) {
                            const float4 vj = vrow(j0 + jj);
                            const float pj = sc[jj];
                            acc.x = __fadd_rn(acc.x, __fmul_rn(pj, vj.x));
                            acc.y = __fadd_rn(acc.y, __fmul_rn(pj, vj.y));
                            acc.z = __fadd_rn(acc.z, __fmul_rn(pj, vj.z));
                            acc.w = __fadd_rn(acc.w, __fmul_rn(pj, vj.w));
                        }
                        reinterpret_cast<float4 *>(pctx[pg])[dq] = acc;
                    }
                    cbar_sync();
                    for (int d = tid; d < HD; d += DS_NC) {
                        float acc = pctx[0][d];
                        for (int i2 = 1; i2 < NPG; i2++) acc = __fadd_rn(acc, pctx[i2][d]);
                        if (nsp == 1) {
                            st_ll(a.ctx + hq * HD + d, acc, otag);
                        } else {
                            st_ll(a.att_part + (size_t)sp * a.qd + hq * HD + d, acc, otag);
                            if (d == 0) {
                                st_ll(a.att_ml + ((size_t)sp * a.nh + hq) * 2, mx, otag);
                                st_ll(a.att_ml + ((size_t)sp * a.nh + hq) * 2 + 1, tot, otag);
                            }
                        }
                    }
                }
                ph_ready();
                cbar_sync();   // qv, knv, sc and pctx are free again
                DS_STAMP(tid == 0, 4, globaltimer());
            }
            if (s_bad) break;
        }
    }
    ph_ready();   // no copy into shared memory outlives the CTA
}

}  // namespace kllm
