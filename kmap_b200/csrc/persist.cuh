// persist.cuh -- the persistent decode step: one cooperative launch runs a
// whole tape step of the compiler's LLaMA template.
//
// Grid = one CTA per SM (all co-resident: cooperative launch).  Each CTA has
// one producer warp and four consumer warps.  The step is a list of phases
// (per layer: QKV, attention, O, gate_up, down; then lm_head and argmax).
// Tasks of a phase are dealt round-robin to the CTAs.
//
// Producer: walks the CTA's GEMV tiles of every phase in order and streams
// their index boxes (16 KB each) through a ring of shared-memory stages with
// 2-D TMA tile loads (no multicast), loading each matrix's codebook into one
// of two shared-memory slots ahead of its tiles.  Weights do not depend on
// activations, so the stream runs ahead across phase boundaries, limited
// only by ring space.
//
// Consumers: for each phase, wait until every CTA has finished the previous
// one (a device-wide arrival counter, polled with a time limit), then do the
// CTA's tasks:
//   GEMV      x for the tile's chunk (plain vector, rmsnorm of the residual,
//             or silu(gate) * up from the gate_up partials), then the chunk's
//             rows in order -- acc = fl(acc + fl(x * cb[idx])), the
//             reference's serial chunk sum -- and the partial row to HBM
//   attention one head: ordered chunk sums of the QKV partials, RoPE, KV
//             append, softmax(q.K^T * scale).V
//   argmax    a slice of the vocabulary: logits = ordered chunk sums of the
//             lm_head partials, first maximum; the CTA that finishes last
//             picks the token and advances the step.
// Chunk partials are always added in chunk order (_tape_runner.c:646-662),
// so every TT-GEMV result is bit-identical to the reference's.
//
// Residual versions alternate between two HBM buffers: the phase that needs
// rmsnorm(h) rebuilds h = h_prev + sum_t part[t] in every CTA (shared
// memory) and CTA 0 stores it for later phases.
#pragma once

#include "common.cuh"
#include "sm100.cuh"
#include "tt_fused.cuh"

namespace kllm {

enum PhaseKind : int { PH_GEMV = 0, PH_ATT = 1, PH_ARGMAX = 2 };
enum PhaseX : int { PX_VEC = 0, PX_NORM_EMBED = 1, PX_NORM_RES = 2, PX_SWIGLU = 3 };

struct MKPhase {
    int kind, ntasks;
    // GEMV
    int mat, K, N, T, ncb, cpl, nsub, F, xmode;
    const float *x;        // PX_VEC: input; PX_NORM_RES: previous residual version
    const float *xpart;    // PX_NORM_RES / PX_SWIGLU: partial rows to reduce
    int xpart_T, xpart_N;
    const float *norm_w;
    float eps;
    float *h_out;          // norm phases: CTA 0 stores the new residual version
    float *part;           // output partial rows [T][N]
    // attention
    int layer;
};

struct MKArgs {
    const MKPhase *phases;
    int nphases;
    const CUtensorMap *maps;     // per matrix
    const float *const *cbp;     // per matrix (padded to a multiple of 4 floats)
    const int *ncodes;           // per matrix
    int *done;                   // per phase arrival counters (zeroed per step)
    int *status;
    int *abort;
    int stages, cb_cap, h_cap, xs_cap, sc_cap;
    int H;
    // step state and embedding
    StepState *st;
    const float *embed;
    const int *prompt;
    int *gen;
    volatile int *gen_host;
    int vocab, max_gen;
    // attention
    const float *qkv_part;
    int qkv_T, nq, nh, nkv, groups, max_pos;
    const float *rope_cos, *rope_sin;
    float *kc, *vc;              // [L][nkv][max_pos][hd]
    float scale;
    float *ctx;
    // argmax
    const float *lm_part;
    int lm_T;
    float *logits, *hist;
    int hist_rows;
    float *cand_v;
    int *cand_i;
};

constexpr int MK_NCW = 4;
constexpr int MK_NC = MK_NCW * 32;
constexpr int MK_THREADS = (MK_NCW + 1) * 32;
constexpr int MK_STAGE = 16384;   // bytes per ring stage (one box, or two half boxes)

__host__ __device__ inline int mk_box_rows(int cpl, int nsub) {
    return (cpl == 1 && nsub == 1) ? 64 : 32;   // 128 x 64 or 256 x 32 uint16
}

__device__ __forceinline__ int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *ctr >= target; false (abort raised) on timeout or abort.
__device__ __forceinline__ bool mk_wait_counter(const int *ctr, int target, int *status,
                                                int *abort) {
    if (ld_acquire(ctr) >= target) return true;
    const unsigned long long t0 = globaltimer();
    while (ld_acquire(ctr) < target) {
        if (ld_acquire(abort)) return false;
        if (globaltimer() - t0 > kWaitLimitNs) {
            atomicOr(status, ST_WAIT_TIMEOUT);
            atomicExch(abort, 1);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ void cbar_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(MK_NC) : "memory");
}

// Fixed-shape sum over the consumer threads (same result in every CTA).
__device__ __forceinline__ float mk_block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    cbar_sync();
    float r = 0.f;
    if (w == 0) {
        r = l < MK_NCW ? red[l] : 0.f;
        for (int o = 16; o; o >>= 1) r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, o));
        if (l == 0) red[MK_NCW] = r;
    }
    cbar_sync();
    return red[MK_NCW];
}

template <int HD>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_step(const __grid_constant__ MKArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[MK_NCW + 2];
    __shared__ float s_rsq;
    __shared__ int s_tok, s_last;
    __shared__ float qv[HD], kv[HD], vv[HD], pctx[MK_NC / HD > 0 ? MK_NC / HD : 1][HD];
    __shared__ int ri[MK_NCW];

    const int G = gridDim.x, cta = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    uint8_t *ring = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * MK_STAGE);
    uint64_t *empty = full + S;
    uint64_t *cbf = empty + S;
    uint64_t *cbe = cbf + 2;
    float *cbs = reinterpret_cast<float *>(cbe + 2);   // 2 slots x cb_cap
    float *hs = cbs + 2 * a.cb_cap;
    float *xs = hs + a.h_cap;
    float *sc = xs + a.xs_cap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MK_NCW);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&cbf[s], 1);
            mbar_init(&cbe[s], MK_NCW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // ================================================================ producer
    if (warp == MK_NCW) {
        if (lane != 0) return;
        int seq = 0, q = 0;
        for (int p = 0; p < a.nphases; p++) {
            const MKPhase &ph = a.phases[p];
            if (ph.kind != PH_GEMV || cta >= ph.ntasks) continue;
            if (ld_acquire(a.abort)) return;
            const int slot = q & 1;
            if (q >= 2 && !mbar_wait(&cbe[slot], ((q >> 1) - 1) & 1, a.status)) {
                atomicExch(a.abort, 1);
                return;
            }
            const uint32_t cbytes = (uint32_t)(((a.ncodes[ph.mat] + 3) & ~3) * 4);
            mbar_expect_tx(&cbf[slot], cbytes);
            float *dst = cbs + (size_t)slot * a.cb_cap;
            for (uint32_t off = 0; off < cbytes; off += 32768)
                bulk_load(reinterpret_cast<uint8_t *>(dst) + off,
                          reinterpret_cast<const uint8_t *>(a.cbp[ph.mat]) + off,
                          min(32768u, cbytes - off), &cbf[slot]);
            q++;
            const CUtensorMap *map = a.maps + ph.mat;
            prefetch_tmap(map);
            const int BN = 128 * ph.cpl, BR = mk_box_rows(ph.cpl, ph.nsub);
            const int BW = BN / ph.nsub;
            const int base = ph.K / ph.T, rem = ph.K % ph.T;
            for (int i = cta; i < ph.ntasks; i += G) {
                const int t = i / ph.ncb, j = i % ph.ncb;
                const int k0 = t * base + min(t, rem), len = base + (t < rem ? 1 : 0);
                const int nbox = (len + BR - 1) / BR;
                for (int b = 0; b < nbox; b++, seq++) {
                    const int s = seq % S;
                    if (seq >= S && !mbar_wait(&empty[s], ((seq / S) - 1) & 1, a.status)) {
                        atomicExch(a.abort, 1);
                        return;
                    }
                    mbar_expect_tx(&full[s], MK_STAGE);
                    uint8_t *d = ring + (size_t)s * MK_STAGE;
                    if (ph.nsub == 1) {
                        tma_load_2d(d, map, j * BN, k0 + b * BR, &full[s]);
                    } else {
                        tma_load_2d(d, map, j * BW, k0 + b * BR, &full[s]);
                        tma_load_2d(d + MK_STAGE / 2, map, ph.F + j * BW, k0 + b * BR, &full[s]);
                    }
                }
            }
        }
        return;
    }

    // =============================================================== consumers
    const int tid = threadIdx.x;
    int seq = 0, q = 0;
    bool ok = true;
    for (int p = 0; p < a.nphases; p++) {
        const MKPhase &ph = a.phases[p];
        if (p > 0) {
            if (tid == 0) s_last = mk_wait_counter(a.done + p - 1, G, a.status, a.abort) ? 1 : 0;
            cbar_sync();
            if (!s_last) {
                ok = false;
                break;
            }
        }
        if (ph.kind == PH_GEMV) {
            const bool mine = cta < ph.ntasks;
            // ---------------------------------------------- norm prologue
            if ((ph.xmode == PX_NORM_EMBED || ph.xmode == PX_NORM_RES) && (mine || cta == 0)) {
                const int H = ph.K;
                const float *src = nullptr;
                if (ph.xmode == PX_NORM_EMBED) {
                    if (tid == 0) {
                        const int pos = a.st->pos, P = a.st->prompt_len;
                        int tok = pos < P ? a.prompt[pos] : __ldcg(a.gen + pos - P);
                        if (tok < 0 || tok >= a.vocab) {
                            atomicOr(a.status, ST_BAD_TOKEN);
                            tok = 0;
                        }
                        s_tok = tok;
                    }
                    cbar_sync();
                    src = a.embed + (size_t)s_tok * H;
                }
                float ss = 0.f;
                for (int i0 = tid; i0 < H; i0 += 4 * MK_NC) {
                    float v[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int i = i0 + u * MK_NC;
                        if (i < H) {
                            if (src) {
                                v[u] = src[i];
                            } else {
                                float y = __ldcg(ph.xpart + i);
                                for (int tt = 1; tt < ph.xpart_T; tt++)
                                    y = __fadd_rn(y, __ldcg(ph.xpart + (size_t)tt * ph.xpart_N + i));
                                v[u] = __fadd_rn(__ldcg(ph.x + i), y);
                            }
                        } else {
                            v[u] = 0.f;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int i = i0 + u * MK_NC;
                        if (i < H) {
                            hs[i] = v[u];
                            ss = __fadd_rn(ss, __fmul_rn(v[u], v[u]));
                        }
                    }
                }
                const float tot = mk_block_sum(ss, red);
                if (tid == 0) {
                    const float add = __fadd_rn(__fmul_rn(tot, 1.0f / (float)H), ph.eps);
                    s_rsq = (float)(1.0 / sqrt((double)add));
                }
                if (cta == 0)
                    for (int i = tid; i < H; i += MK_NC) ph.h_out[i] = hs[i];
                cbar_sync();
            }
            if (mine) {
                // A wait that gives up raises the abort flag and marks this
                // thread bad: it skips the math but keeps every barrier and
                // stage arrival, so no warp is left waiting; the phase
                // boundary then ends the step uniformly.
                const int slot = q & 1;
                bool bad = !mbar_wait(&cbf[slot], (q >> 1) & 1, a.status);
                if (bad) atomicExch(a.abort, 1);
                const float *cb = cbs + (size_t)slot * a.cb_cap;
                const int BN = 128 * ph.cpl, BR = mk_box_rows(ph.cpl, ph.nsub);
                const int BW = BN / ph.nsub;
                const int base = ph.K / ph.T, rem = ph.K % ph.T;
                const float rsq = s_rsq;
                const int wps = MK_NCW / ph.nsub;
                const int qh = warp / wps;                       // half (nsub == 2)
                const int wcol = (warp % wps) * 32 * ph.cpl + lane * ph.cpl;
                const int rowstride = BW;
                for (int i = cta; i < ph.ntasks; i += G) {
                    const int t = i / ph.ncb, j = i % ph.ncb;
                    const int k0 = t * base + min(t, rem), len = base + (t < rem ? 1 : 0);
                    // x for the chunk's rows
                    if (ph.xmode == PX_VEC) {
                        for (int r = tid; r < len; r += MK_NC) xs[r] = __ldcg(ph.x + k0 + r);
                    } else if (ph.xmode == PX_SWIGLU) {
                        for (int r0 = tid; r0 < len; r0 += 2 * MK_NC) {
                            float g[2], u[2];
#pragma unroll
                            for (int e = 0; e < 2; e++) {
                                const int r = r0 + e * MK_NC;
                                g[e] = u[e] = 0.f;
                                if (r < len) {
                                    const float *pg = ph.xpart + k0 + r;
                                    g[e] = __ldcg(pg);
                                    u[e] = __ldcg(pg + ph.F);
                                    for (int tt = 1; tt < ph.xpart_T; tt++) {
                                        g[e] = __fadd_rn(g[e], __ldcg(pg + (size_t)tt * ph.xpart_N));
                                        u[e] = __fadd_rn(u[e], __ldcg(pg + (size_t)tt * ph.xpart_N + ph.F));
                                    }
                                }
                            }
#pragma unroll
                            for (int e = 0; e < 2; e++) {
                                const int r = r0 + e * MK_NC;
                                if (r < len) {
                                    const double d = (double)g[e];
                                    xs[r] = __fmul_rn((float)(d / (1.0 + exp(-d))), u[e]);
                                }
                            }
                        }
                    } else {
                        for (int r = tid; r < len; r += MK_NC)
                            xs[r] = __fmul_rn(__fmul_rn(hs[k0 + r], rsq), __ldg(ph.norm_w + k0 + r));
                    }
                    cbar_sync();
                    // the chunk's rows, in order
                    const int nbox = (len + BR - 1) / BR;
                    float acc0 = 0.f, acc1 = 0.f;
                    for (int b = 0; b < nbox; b++, seq++) {
                        const int s = seq % S;
                        if (!bad && !mbar_wait(&full[s], (seq / S) & 1, a.status)) {
                            bad = true;
                            atomicExch(a.abort, 1);
                        }
                        if (!bad) {
                            const uint16_t *tile =
                                reinterpret_cast<const uint16_t *>(
                                    ring + (size_t)s * MK_STAGE +
                                    (size_t)qh * (MK_STAGE / 2) * (ph.nsub - 1)) +
                                wcol;
                            const float *xb = xs + b * BR;
                            const int rows = min(BR, len - b * BR);
                            if (ph.cpl == 1) {
                                if (rows == 64) {
#pragma unroll 8
                                    for (int r = 0; r < 64; r++)
                                        acc0 = __fadd_rn(acc0, __fmul_rn(xb[r], cb[tile[r * rowstride]]));
                                } else {
                                    for (int r = 0; r < rows; r++)
                                        acc0 = __fadd_rn(acc0, __fmul_rn(xb[r], cb[tile[r * rowstride]]));
                                }
                            } else {
                                if (rows == 32) {
#pragma unroll 8
                                    for (int r = 0; r < 32; r++) {
                                        const uint32_t w =
                                            *reinterpret_cast<const uint32_t *>(tile + r * rowstride);
                                        const float xv = xb[r];
                                        acc0 = __fadd_rn(acc0, __fmul_rn(xv, cb[w & 0xffffu]));
                                        acc1 = __fadd_rn(acc1, __fmul_rn(xv, cb[w >> 16]));
                                    }
                                } else {
                                    for (int r = 0; r < rows; r++) {
                                        const uint32_t w =
                                            *reinterpret_cast<const uint32_t *>(tile + r * rowstride);
                                        const float xv = xb[r];
                                        acc0 = __fadd_rn(acc0, __fmul_rn(xv, cb[w & 0xffffu]));
                                        acc1 = __fadd_rn(acc1, __fmul_rn(xv, cb[w >> 16]));
                                    }
                                }
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);
                    }
                    // partial row of this chunk
                    int col;
                    bool valid0, valid1;
                    if (ph.nsub == 1) {
                        col = j * BN + wcol;
                        valid0 = col < ph.N;
                        valid1 = col + 1 < ph.N;
                    } else {
                        const int c = j * BW + wcol;
                        col = (qh == 0 ? 0 : ph.F) + c;
                        valid0 = c < ph.F;
                        valid1 = c + 1 < ph.F;
                    }
                    if (!bad) {
                        float *out = ph.part + (size_t)t * ph.N + col;
                        if (valid0) out[0] = acc0;
                        if (ph.cpl == 2 && valid1) out[1] = acc1;
                    }
                    cbar_sync();   // xs is rewritten by the next task
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&cbe[slot]);
                q++;
            }
        } else if (ph.kind == PH_ATT) {
            const int l = ph.layer, nkvh = a.nkv;
            float *kcl = a.kc + (size_t)l * nkvh * a.max_pos * HD;
            float *vcl = a.vc + (size_t)l * nkvh * a.max_pos * HD;
            const int pos = a.st->pos;
            const int qd = a.nh * HD, kvd = nkvh * HD;
            for (int hq = cta; hq < ph.ntasks; hq += G) {
                const int g = hq / a.groups;
                if (pos >= a.max_pos) break;
                for (int i = tid; i < 3 * HD; i += MK_NC) {
                    const int which = i / HD, d = i % HD;
                    const int col = which == 0 ? hq * HD + d
                                               : (which == 1 ? qd + g * HD + d : qd + kvd + g * HD + d);
                    float v = __ldcg(a.qkv_part + col);
                    for (int tt = 1; tt < a.qkv_T; tt++)
                        v = __fadd_rn(v, __ldcg(a.qkv_part + (size_t)tt * a.nq + col));
                    (which == 0 ? qv : which == 1 ? kv : vv)[d] = v;
                }
                cbar_sync();
                float qr = 0.f, kr = 0.f;
                for (int d = tid; d < HD; d += MK_NC) {
                    const float c = a.rope_cos[(size_t)pos * HD + d];
                    const float s = a.rope_sin[(size_t)pos * HD + d];
                    const int half = HD / 2;
                    const float rq = d < half ? -qv[d + half] : qv[d - half];
                    const float rk = d < half ? -kv[d + half] : kv[d - half];
                    qr = __fadd_rn(__fmul_rn(qv[d], c), __fmul_rn(rq, s));
                    kr = __fadd_rn(__fmul_rn(kv[d], c), __fmul_rn(rk, s));
                }
                cbar_sync();
                for (int d = tid; d < HD; d += MK_NC) {
                    qv[d] = qr;
                    kv[d] = kr;
                    if (hq % a.groups == 0) {
                        const size_t o = ((size_t)g * a.max_pos + pos) * HD + d;
                        kcl[o] = kr;
                        vcl[o] = vv[d];
                    }
                }
                cbar_sync();
                constexpr int DPL = HD / 32;
                float qreg[DPL];
#pragma unroll
                for (int e = 0; e < DPL; e++) qreg[e] = qv[lane + 32 * e];
                for (int jj = warp; jj <= pos; jj += MK_NCW) {
                    const float *kj = jj == pos ? kv : kcl + ((size_t)g * a.max_pos + jj) * HD;
                    float dot = __fmul_rn(qreg[0], jj == pos ? kj[lane] : __ldcg(kj + lane));
#pragma unroll
                    for (int e = 1; e < DPL; e++)
                        dot = __fadd_rn(dot, __fmul_rn(qreg[e], jj == pos ? kj[lane + 32 * e]
                                                                          : __ldcg(kj + lane + 32 * e)));
                    for (int o = 16; o; o >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
                    if (lane == 0) sc[jj] = __fmul_rn(dot, a.scale);
                }
                cbar_sync();
                float m = -INFINITY;
                for (int jj = tid; jj <= pos; jj += MK_NC) m = fmaxf(m, sc[jj]);
                for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (lane == 0) red[warp] = m;
                cbar_sync();
                float mx = red[0];
                for (int w2 = 1; w2 < MK_NCW; w2++) mx = fmaxf(mx, red[w2]);
                float sum = 0.f;
                for (int jj = tid; jj <= pos; jj += MK_NC) {
                    const float e = (float)exp((double)__fsub_rn(sc[jj], mx));
                    sc[jj] = e;
                    sum = __fadd_rn(sum, e);
                }
                cbar_sync();   // everyone has read red[] (max) before it is reused
                const float tot = mk_block_sum(sum, red);
                for (int jj = tid; jj <= pos; jj += MK_NC) sc[jj] = __fdiv_rn(sc[jj], tot);
                cbar_sync();
                constexpr int NG = MK_NC / HD > 0 ? MK_NC / HD : 1;
                for (int d0 = tid % HD; d0 < HD; d0 += MK_NC) {
                    const int grp = tid / HD;
                    float acc = 0.f;
                    for (int jj = grp; jj <= pos; jj += NG) {
                        const float vj = jj == pos ? vv[d0]
                                                   : __ldcg(vcl + ((size_t)g * a.max_pos + jj) * HD + d0);
                        acc = __fadd_rn(acc, __fmul_rn(sc[jj], vj));
                    }
                    if (grp < NG) pctx[grp][d0] = acc;
                }
                cbar_sync();
                for (int d = tid; d < HD; d += MK_NC) {
                    float acc = pctx[0][d];
                    for (int i = 1; i < NG; i++) acc = __fadd_rn(acc, pctx[i][d]);
                    a.ctx[hq * HD + d] = acc;
                }
                cbar_sync();
            }
        } else {   // PH_ARGMAX
            const int V = a.vocab;
            const int per = (V + ph.ntasks - 1) / ph.ntasks;
            const int pos = a.st->pos;
            for (int sl = cta; sl < ph.ntasks; sl += G) {
                const int v0 = sl * per, v1 = min(V, v0 + per);
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int v = v0 + tid; v < v1; v += MK_NC) {
                    float y = __ldcg(a.lm_part + v);
                    for (int tt = 1; tt < a.lm_T; tt++)
                        y = __fadd_rn(y, __ldcg(a.lm_part + (size_t)tt * V + v));
                    a.logits[v] = y;
                    if (a.hist && pos < a.hist_rows) a.hist[(size_t)pos * V + v] = y;
                    if (y > bv || bi == 0x7fffffff) {
                        bv = y;
                        bi = v;
                    }
                }
                for (int o = 16; o; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) {
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
                    for (int w2 = 1; w2 < MK_NCW; w2++)
                        if (red[w2] > bv || (red[w2] == bv && ri[w2] < bi)) {
                            bv = red[w2];
                            bi = ri[w2];
                        }
                    a.cand_v[sl] = bv;
                    a.cand_i[sl] = bi;
                }
                cbar_sync();
            }
        }
        // ------------------------------------------------------ arrival
        cbar_sync();
        if (tid == 0) {
            __threadfence();
            const int prev = atomicAdd(a.done + p, 1);
            if (ph.kind == PH_ARGMAX && prev == G - 1) {
                __threadfence();
                float best = __ldcg(a.cand_v);
                int bidx = __ldcg(a.cand_i);
                for (int j = 1; j < ph.ntasks; j++) {
                    const float cv = __ldcg(a.cand_v + j);
                    const int ci = __ldcg(a.cand_i + j);
                    if (cv > best || (cv == best && ci < bidx)) {
                        best = cv;
                        bidx = ci;
                    }
                }
                if (bidx < 0 || bidx >= a.vocab) bidx = 0;
                const int pos = a.st->pos, P0 = a.st->prompt_len;
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
            }
        }
    }
    if (!ok && tid == 0) atomicExch(a.abort, 1);
}

}  // namespace kllm
