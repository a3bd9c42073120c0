// tt_fused.cuh -- the TT-GEMV with fused prologues and epilogues.
//
// Core (unchanged arithmetic): one CTA owns (chunk t, BN columns); a
// producer warp streams the chunk's index rows through a ring of shared
// memory stages with 2-D TMA tile loads (no multicast); NCW consumer warps
// hold the codebook and the chunk's x in shared memory and walk the rows in
// order, each lane owning CPL columns:
//     acc[c] = fl(acc[c] + fl(x[k] * cb[idx[k][col_c]]))
// which is the reference's per-chunk serial sum (_tape_runner.c:517-545).
//
// Prologue (x source), after griddepcontrol.wait:
//   X_PLAIN  x from a vector
//   X_NORM   x = rmsnorm(h) * w for the chunk's rows, h = a residual vector
//            or (first layer) this step's embedding row; every CTA reduces
//            sum(h*h) itself with the same fixed tree, so all CTAs agree
//            (template ops MUL, MEAN, ADD eps, RSQRT in double, MUL, MUL:
//            kllm_compile.c:1143-1164)
// Epilogue: each CTA writes its chunk's partial row; the last of the T CTAs
// of a column block (arrival counter) adds the T partials in chunk order --
// exactly the reference's reduction (_tape_runner.c:646-662) -- and
//   E_Y       writes y
//   E_RESID   adds y into the residual vector: h = fl(h + y)
//   E_SWIGLU  (tiles hold gate columns n and up columns F + n side by side)
//             writes act[n] = fl(silu(gate[n]) * up[n]), SILU in double
//   E_ARGMAX  writes the logits, keeps the block's first maximum, and the
//             last block to finish publishes this step's greedy token
//             (first maximum wins, _tape_runner.c:1717-1727)
// then resets its counter for the next launch.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace kllm {

enum XMode : int { X_PLAIN = 0, X_NORM = 1 };
enum EMode : int { E_Y = 0, E_RESID = 1, E_SWIGLU = 2, E_ARGMAX = 3 };

struct StepState {
    int pos;          // position of the token fed this step
    int prompt_len;
    int n_gen;        // tokens generated so far
    int counter;      // block arrival counter of the argmax epilogue
};

struct TTArgs {
    const float *cb;
    int n_codes;
    int K, N, T, stages;
    int sub_cols;       // columns per TMA box (BN / nsub)
    int F;              // E_SWIGLU: gate/up split (up columns start at F)
    // x source
    int xmode;
    const float *x;     // X_PLAIN: x[K];  X_NORM: residual h[K]
    const float *norm_w;
    float eps, inv_k;
    const float *embed; // X_NORM from the step's embedding row (first layer)
    const StepState *st;
    const int *prompt, *gen;
    int vocab;
    float *h_init;      // X_NORM from embed: block 0 also stores h = embed row
    // epilogue
    int emode;
    float *part;        // [T][N] partial rows
    int *counters;      // [N / BN] arrival counters (zero between launches)
    float *y;           // E_Y: y[N]; E_RESID: h[N]; E_SWIGLU: act[F]
    // E_ARGMAX
    float *logits, *hist;
    int hist_rows;
    float *cand_v;
    int *cand_i;
    StepState *stw;
    int *gen_dev;
    volatile int *gen_host;
    int max_gen;
    int *status;
};

template <int NCW, int CPL, int BR, int NSUB>
struct TFGeom {
    static constexpr int BN = NCW * 32 * CPL;
    static constexpr int BW = BN / NSUB;              // columns per sub-box
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int STAGE_BYTES = BN * BR * 2;
};

template <int NCW, int CPL, int BR, int NSUB>
__host__ __device__ inline size_t tf_smem_bytes(int n_codes, int len, int ns) {
    using G = TFGeom<NCW, CPL, BR, NSUB>;
    size_t ncb4 = ((size_t)n_codes + 3) / 4;
    size_t len4 = ((size_t)len + 3) / 4;
    return (size_t)ns * G::STAGE_BYTES + 16 * (size_t)ns + 16 + ncb4 * 16 + len4 * 16 + 256;
}

// Block-wide sum with a fixed shape (same result in every CTA).
template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    asm volatile("bar.sync 1, %0;" ::"r"(NT) : "memory");
    float r = 0.f;
    if (w == 0) {
        r = l < NT / 32 ? red[l] : 0.f;
        for (int o = 16; o; o >>= 1) r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, o));
        if (l == 0) red[NT / 32] = r;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(NT) : "memory");
    return red[NT / 32];
}

template <int NCW, int CPL, int BR, int NSUB>
__global__ void __launch_bounds__(TFGeom<NCW, CPL, BR, NSUB>::THREADS)
k_tt_fused(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ TTArgs a) {
    using G = TFGeom<NCW, CPL, BR, NSUB>;
    constexpr int BN = G::BN, BW = G::BW, NC = NCW * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[NC / 32 + 1];
    __shared__ int s_last;
    pdl_launch_dependents();

    const int t = blockIdx.y, jb = blockIdx.x;
    const int K = a.K, T = a.T;
    const int base = K / T, rem = K % T;
    const int k0 = t * base + min(t, rem);
    const int len = base + (t < rem ? 1 : 0);
    const int nbox = (len + BR - 1) / BR;
    const int NS = min(a.stages, nbox);
    const int ncb4 = (a.n_codes + 3) / 4;
    const int cb_bulk = (a.n_codes & ~3) * 4;
    // first global column of each sub-box of this tile
    const int col0 = (a.emode == E_SWIGLU) ? jb * BW : jb * BN;

    uint16_t *stage = reinterpret_cast<uint16_t *>(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)NS * G::STAGE_BYTES);
    uint64_t *empty = full + NS;
    uint64_t *cbar = empty + NS;
    float *cbs = reinterpret_cast<float *>(cbar + 2);
    float *xs = cbs + 4 * ncb4;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_init(cbar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == NCW) {
        if (lane == 0) {
            prefetch_tmap(&tmap);
            mbar_expect_tx(cbar, (uint32_t)cb_bulk);
            for (int off = 0; off < cb_bulk; off += 32768)
                bulk_load(reinterpret_cast<uint8_t *>(cbs) + off,
                          reinterpret_cast<const uint8_t *>(a.cb) + off,
                          (uint32_t)min(32768, cb_bulk - off), cbar);
            int issued = 0;
            for (int b = 0; b < nbox; b++) {
                const int s = b % NS;
                if (b >= NS && !mbar_wait(&empty[s], ((b / NS) - 1) & 1, a.status)) break;
                mbar_expect_tx(&full[s], G::STAGE_BYTES);
                uint16_t *dst = stage + (size_t)s * BR * BN;
#pragma unroll
                for (int q = 0; q < NSUB; q++) {
                    const int cx = q == 0 ? col0 : a.F + col0;   // NSUB == 2: gate | up
                    tma_load_2d(dst + q * BR * BW, &tmap, cx, k0 + b * BR, &full[s]);
                }
                issued = b + 1;
            }
            // No copy may still be writing this CTA's shared memory when it
            // exits (after a wait that gave up, the consumers may leave
            // early): wait, bounded, for the codebook and the last tiles.
            mbar_wait(cbar, 0, a.status);
            for (int b = max(0, issued - NS); b < issued; b++)
                mbar_wait(&full[b % NS], (b / NS) & 1, a.status);
        }
        return;
    }

    // ---------------------------------------------------------- prologue --
    if ((int)threadIdx.x < (a.n_codes & 3)) {
        int i = (a.n_codes & ~3) + threadIdx.x;
        cbs[i] = __ldg(a.cb + i);
    }
    pdl_wait();
    if (a.xmode == X_PLAIN) {
        for (int r0 = threadIdx.x; r0 < len; r0 += 8 * NC) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = r0 + i * NC < len ? a.x[k0 + r0 + i * NC] : 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (r0 + i * NC < len) xs[r0 + i * NC] = v[i];
        }
    } else {
        const float *h = a.x;
        if (a.embed) {
            const int pos = a.st->pos, P = a.st->prompt_len;
            int tok = pos < P ? a.prompt[pos] : a.gen[pos - P];
            if (tok < 0 || tok >= a.vocab) {
                if (threadIdx.x == 0) atomicOr(a.status, ST_BAD_TOKEN);
                tok = 0;
            }
            h = a.embed + (size_t)tok * K;
            if (jb == 0 && t == 0)
                for (int i = threadIdx.x; i < K; i += NC) a.h_init[i] = h[i];
        }
        float ss = 0.f;
        for (int i0 = threadIdx.x; i0 < K; i0 += 8 * NC) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = i0 + i * NC < K ? h[i0 + i * NC] : 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        }
        const float tot = block_sum<NC>(ss, red);
        const float add = __fadd_rn(__fmul_rn(tot, a.inv_k), a.eps);
        const float rsq = (float)(1.0 / sqrt((double)add));
        for (int r = threadIdx.x; r < len; r += NC)
            xs[r] = __fmul_rn(__fmul_rn(h[k0 + r], rsq), a.norm_w[k0 + r]);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    // a wait that gives up (status flagged) skips the math but still passes
    // every barrier below, so no warp is left waiting at one
    bool ok = mbar_wait(cbar, 0, a.status);

    // -------------------------------------------------------------- core --
    constexpr int WPS = NCW / NSUB;                 // warps per sub-box
    const int q = warp / WPS;                       // this warp's sub-box
    const int wcol = (warp % WPS) * 32 * CPL + lane * CPL;   // column inside the sub-box
    float acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) acc[c] = 0.0f;

    for (int b = 0; ok && b < nbox; b++) {
        const int s = b % NS;
        if (!mbar_wait(&full[s], (b / NS) & 1, a.status)) {
            ok = false;
            break;
        }
        const uint16_t *tile = stage + (size_t)s * BR * BN + q * BR * BW + wcol;
        const float *xb = xs + b * BR;
        const int rows = min(BR, len - b * BR);
        if (rows == BR) {
#pragma unroll 8
            for (int r = 0; r < BR; r++) {
                const float xv = xb[r];
                if (CPL == 1) {
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(xv, cbs[tile[r * BW]]));
                } else if (CPL == 2) {
                    const uint32_t w = *reinterpret_cast<const uint32_t *>(tile + r * BW);
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(xv, cbs[w & 0xffffu]));
                    acc[CPL - 1] = __fadd_rn(acc[CPL - 1], __fmul_rn(xv, cbs[w >> 16]));
                } else {
                    const uint2 w = *reinterpret_cast<const uint2 *>(tile + r * BW);
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(xv, cbs[w.x & 0xffffu]));
                    acc[1 % CPL] = __fadd_rn(acc[1 % CPL], __fmul_rn(xv, cbs[w.x >> 16]));
                    acc[2 % CPL] = __fadd_rn(acc[2 % CPL], __fmul_rn(xv, cbs[w.y & 0xffffu]));
                    acc[3 % CPL] = __fadd_rn(acc[3 % CPL], __fmul_rn(xv, cbs[w.y >> 16]));
                }
            }
        } else {
            for (int r = 0; r < rows; r++) {
                const float xv = xb[r];
#pragma unroll
                for (int c = 0; c < CPL; c++)
                    acc[c] = __fadd_rn(acc[c], __fmul_rn(xv, cbs[tile[r * BW + c]]));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // A wait that gave up (ST_WAIT_TIMEOUT in *a.status) leaves this CTA's
    // chunk sums incomplete: publish NaN, so the affected columns of y are
    // NaN rather than plausible wrong numbers.
    if (!ok) {
#pragma unroll
        for (int c = 0; c < CPL; c++) acc[c] = __int_as_float(0x7fffffff);
    }

    // ---------------------------------------------------------- epilogue --
    const bool swig = a.emode == E_SWIGLU;
    const int gcol = (q == 0 ? col0 : a.F + col0) + wcol;   // global column of acc[0]
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        const bool ok = swig ? (col0 + wcol + c < a.F) : (gcol + c < a.N);
        if (ok) a.part[(size_t)t * a.N + gcol + c] = acc[c];
    }
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[jb], 1) == T - 1;
    asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
    if (!s_last) return;   // uniform across the CTA
    __threadfence();
    // the last CTA of this column block: ordered sum of the T partials
    const float *P = a.part;
    if (a.emode == E_SWIGLU) {
        for (int c = threadIdx.x; c < BW; c += NC) {
            const int n = col0 + c;
            if (n >= a.F) continue;
            const float g = sum_parts(P + n, a.N, T), u = sum_parts(P + a.F + n, a.N, T);
            const double d = (double)g;
            a.y[n] = __fmul_rn((float)(d / (1.0 + exp(-d))), u);
        }
    } else {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = threadIdx.x; c < BN; c += NC) {
            const int n = col0 + c;
            if (n >= a.N) continue;
            const float v = sum_parts(P + n, a.N, T);
            if (a.emode == E_Y) {
                a.y[n] = v;
            } else if (a.emode == E_RESID) {
                a.y[n] = __fadd_rn(a.y[n], v);
            } else {
                a.logits[n] = v;
                const int pos = a.st->pos;
                if (a.hist && pos < a.hist_rows) a.hist[(size_t)pos * a.N + n] = v;
                if (v > bv || bi == 0x7fffffff) {
                    bv = v;
                    bi = n;
                }
            }
        }
        if (a.emode == E_ARGMAX) {
            for (int o = 16; o; o >>= 1) {
                float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            float *rv = red;
            __shared__ int ri[NC / 32];
            if (lane == 0) {
                rv[warp] = bv;
                ri[warp] = bi;
            }
            asm volatile("bar.sync 1, %0;" ::"r"(NC) : "memory");
            if (threadIdx.x == 0) {
                for (int w = 1; w < NC / 32; w++)
                    if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) {
                        bv = rv[w];
                        bi = ri[w];
                    }
                a.cand_v[jb] = bv;
                a.cand_i[jb] = bi;
                __threadfence();
                const bool last_block = atomicAdd(&a.stw->counter, 1) == (int)gridDim.x - 1;
                if (last_block) {
                    __threadfence();
                    float best = __ldcg(a.cand_v);
                    int bidx = __ldcg(a.cand_i);
                    for (int j = 1; j < (int)gridDim.x; j++) {
                        float cv = __ldcg(a.cand_v + j);
                        int ci = __ldcg(a.cand_i + j);
                        if (cv > best || (cv == best && ci < bidx)) {
                            best = cv;
                            bidx = ci;
                        }
                    }
                    if (bidx < 0 || bidx >= a.N) bidx = 0;
                    const int pos = a.stw->pos, P0 = a.stw->prompt_len;
                    if (pos >= P0 - 1) {
                        const int gi = pos - (P0 - 1);
                        if (gi < a.max_gen) {
                            a.gen_dev[gi] = bidx;
                            a.gen_host[gi] = bidx;
                            __threadfence_system();
                        }
                        a.stw->n_gen = gi + 1;
                    }
                    a.stw->counter = 0;
                    a.stw->pos = pos + 1;
                }
            }
        }
    }
    if (threadIdx.x == 0) a.counters[jb] = 0;
}

// Launch geometry for one matrix.
struct TFConfig {
    int ncw = 4, cpl = 1, nsub = 1, stages = 2;
    int bn() const { return ncw * 32 * cpl; }
    int bw() const { return bn() / nsub; }
};

// Geometry for a K x N matrix used with epilogue `emode`.
TFConfig tf_config(int K, int N, int n_codes, int emode);
// Tensor-map box of a geometry: {bw() columns, 32 rows}.
bool make_idx_tmap(CUtensorMap *map, const uint16_t *idx, int K, int N, int box_cols,
                   int box_rows);
bool tf_tma_ok(const uint16_t *idx, const float *cb, int K, int N, int n_codes,
               const TFConfig &c);
// Column blocks (grid.x) of a launch; counters must have this many zeros.
int tf_blocks(const TFConfig &c, int N, int F, int emode);
bool launch_tt_fused(cudaStream_t s, const TFConfig &c, const CUtensorMap &map, TTArgs a,
                     bool pdl);

}  // namespace kllm
