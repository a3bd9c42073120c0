// batch.cuh -- the row kernels of batched greedy decode (plan.cu,
// plan_infer_batch): one row per sequence, every sequence at its own
// position with its own KV cache.  Around the projections (the few-row
// tensor-core GEMM, or the bit-exact TT-GEMM per row) each kernel does
// the whole stretch between two of them: it reads the previous GEMM's
// output as the sum of its K-range partial tiles (in range order), applies
// the tape's float arithmetic of that stretch (RMSNorm, RoPE + cache
// append, attention, residual add, SwiGLU), and writes the next GEMM's
// input directly -- fp32 rows, or the three bf16 terms of the exact split
// the tensor cores take.  Reductions run in a fixed order of their own, as
// in the prompt pass.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "prefill.cuh"

namespace kllm {

namespace cg = cooperative_groups;

// One element of a GEMM output: the sum of its nz K-range partial tiles,
// part[z * plane + i], in range order (nz = 1: the output itself).
__device__ __forceinline__ float bd_sum(const float *__restrict__ part, int nz, size_t plane,
                                        size_t i) {
    float a = part[i];
    for (int z = 1; z < nz; z++) a = __fadd_rn(a, part[(size_t)z * plane + i]);
    return a;
}

// One element of the next GEMM's input: fp32 (terms 0), or the bf16 terms
// hi = bf16(v), mid = bf16(v - hi), lo = bf16(v - hi - mid), term t at
// t * plane + i.
__device__ __forceinline__ void bd_emit(float v, size_t i, int terms, size_t plane,
                                        void *__restrict__ xs) {
    if (!terms) {
        reinterpret_cast<float *>(xs)[i] = v;
        return;
    }
    __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(xs);
    float r = v;
    for (int t = 0; t < terms; t++) {
        const __nv_bfloat16 b = __float2bfloat16_rn(r);
        o[(size_t)t * plane + i] = b;
        r = __fsub_rn(r, __bfloat162float(b));
    }
}

// Row r: x = res[r] + (the GEMM output's row, or nothing when part is
// null; with res null, the embedding row of tok[r]); hout[r] = x; then
// the tape's RMSNORM -- sum of squares, mean as sum * (1 / H) + eps, rsqrt
// in double, two rounded products -- into the next GEMM's input.  A
// cluster of BD_CL CTAs per row, each a contiguous slice of H: the slices'
// sums of squares (block sums of a fixed shape) are read from every CTA's
// shared memory and added in slice order, so all CTAs of the row agree.
// (grid: nseq * BD_CL blocks, PF_THREADS threads)
constexpr int BD_CL = 8;

__global__ void __cluster_dims__(BD_CL, 1, 1) __launch_bounds__(PF_THREADS)
k_bd_add_norm(const float *__restrict__ res, const float *__restrict__ embed,
              const int *__restrict__ tok, const float *__restrict__ part, int nz,
              const float *__restrict__ w, float eps, int H, float *__restrict__ hout, int terms,
              void *__restrict__ xs) {
    __shared__ float red[PF_THREADS / 32];
    __shared__ float css;
    cg::cluster_group cl = cg::this_cluster();
    const int r = blockIdx.x / BD_CL, c = (int)cl.block_rank();
    const size_t plane = (size_t)(gridDim.x / BD_CL) * H;
    const int per = (H + BD_CL - 1) / BD_CL, i0 = c * per, i1 = min(H, i0 + per);
    const float *src = res ? res + (size_t)r * H : embed + (size_t)tok[r] * H;
    float *hr = hout + (size_t)r * H;
    float ss = 0.f;
    for (int i = i0 + threadIdx.x; i < i1; i += PF_THREADS) {
        float v = src[i];
        if (part) v = __fadd_rn(v, bd_sum(part, nz, plane, (size_t)r * H + i));
        hr[i] = v;
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    const float mine = pf_block_sum(ss, red);
    if (threadIdx.x == 0) css = mine;
    cl.sync();
    float tot = *cl.map_shared_rank(&css, 0);
    for (int k = 1; k < BD_CL; k++) tot = __fadd_rn(tot, *cl.map_shared_rank(&css, k));
    cl.sync();   // every CTA has read every slice's sum before any leaves
    const float add = __fadd_rn(__fmul_rn(tot, 1.0f / (float)H), eps);
    const float rsq = (float)(1.0 / sqrt((double)add));
    for (int i = i0 + threadIdx.x; i < i1; i += PF_THREADS)   // this thread's own writes above
        bd_emit(__fmul_rn(__fmul_rn(hr[i], rsq), w[i]), (size_t)r * H + i, terms, plane, xs);
}

// act[r][n] = silu(gate) * up, gate = column n and up = column F + n of the
// gate_up GEMM's row r (silu in double as the tape's SILU), into the down
// GEMM's input.  (grid-stride over nseq * F)
__global__ void k_bd_swiglu(const float *__restrict__ part, int nz, int nseq, int F, int terms,
                            void *__restrict__ xs) {
    const long long rf = (long long)nseq * F;
    const size_t plane = (size_t)nseq * 2 * F;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rf;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / F, n = i % F;
        const double dg = (double)bd_sum(part, nz, plane, (size_t)(r * 2 * F + n));
        const float up = bd_sum(part, nz, plane, (size_t)(r * 2 * F + F + n));
        bd_emit(__fmul_rn((float)(dg / (1.0 + exp(-dg))), up), (size_t)i, terms, (size_t)rf, xs);
    }
}

// Row r of the QKV GEMM output at position pos[r]: rotate-half RoPE of q
// (to q_out[r]) and k, k and v appended to sequence r's cache (row pos[r]).
// Caches: [seq][layer][kv_head][max_pos][hd]; kc / vc point at this layer of
// sequence 0, seq_stride floats apart.  (grid: nseq x any number of
// blocks over the row's outputs)
__global__ void k_bd_rope_kv(const float *__restrict__ part, int nz, const int *__restrict__ pos,
                             int nq, int nh, int nkv, int hd, const float *__restrict__ rcos,
                             const float *__restrict__ rsin, int max_pos, size_t seq_stride,
                             float *__restrict__ q_out, float *__restrict__ kc,
                             float *__restrict__ vc) {
    const int r = blockIdx.x, p = pos[r];
    const int qd = nh * hd, kvd = nkv * hd;
    const size_t plane = (size_t)gridDim.x * nq, row = (size_t)r * nq;
    float *kr = kc + (size_t)r * seq_stride, *vr = vc + (size_t)r * seq_stride;
    for (int n = blockIdx.y * blockDim.x + threadIdx.x; n < qd + 2 * kvd;
         n += gridDim.y * blockDim.x) {
        const float y = bd_sum(part, nz, plane, row + n);
        if (n < qd + kvd) {
            const int head = n / hd, dim = n % hd, half = hd / 2;
            const float pk = dim < half ? -bd_sum(part, nz, plane, row + n + half)
                                        : bd_sum(part, nz, plane, row + n - half);
            const float v = __fadd_rn(__fmul_rn(y, rcos[(size_t)p * hd + dim]),
                                      __fmul_rn(pk, rsin[(size_t)p * hd + dim]));
            if (head < nh)
                q_out[(size_t)r * qd + n] = v;
            else
                kr[((size_t)(head - nh) * max_pos + p) * hd + dim] = v;
        } else {
            const int vi = n - qd - kvd;
            vr[((size_t)(vi / hd) * max_pos + p) * hd + vi % hd] = y;
        }
    }
}

// Attention of row r for the `groups` query heads of kv head g at once
// (each cached k / v row read once): grid nseq x nkv, BD_ATT_THREADS
// threads (8 warps, 8 rows of each in flight; two CTAs per SM).  Scores:
// warp w takes positions w, w + 8, ...; lane i holds
// dims [VEC i, VEC i + VEC) of the row; q.k is the lane's serial sum over
// its dims, then the xor-shuffle tree over the lanes, times the scale.
// Softmax of query head j by warp j: max, exp in double of the difference,
// the lanes' serial sums then the tree, division.  P.V: warp w sums its
// positions serially per dim, the warps' sums added in warp order, into
// the O GEMM's input.  Dynamic shared memory: bd_att_smem(groups, HD,
// max_pos) bytes.
constexpr int BD_ATT_THREADS = 256;

__host__ __device__ inline size_t bd_att_smem(int groups, int hd, int max_pos) {
    return ((size_t)groups * max_pos + (size_t)groups * hd +
            (size_t)(BD_ATT_THREADS / 32) * groups * hd) * 4;
}

template <int VEC>
__device__ __forceinline__ void bd_load(const float *p, float (&v)[VEC]) {
    if constexpr (VEC == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else if constexpr (VEC == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        v[0] = t.x, v[1] = t.y;
    } else {
        v[0] = *p;
    }
}

// Butterfly reduce-scatter over the warp: on return lane l holds the sum
// over all 32 lanes of v[l % P] (P - 1 shuffles for the low lane bits, one
// per higher bit), the additions in a fixed order.
template <int P>
__device__ __forceinline__ float bd_bfly(float (&v)[P], int lane) {
#pragma unroll
    for (int m = P / 2, L = P; m >= 1; m >>= 1, L >>= 1) {
        const bool up = lane & m;
#pragma unroll
        for (int i = 0; i < L / 2; i++) {
            const float send = up ? v[i] : v[i + L / 2];
            const float keep = up ? v[i + L / 2] : v[i];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
        }
    }
    float r = v[0];
#pragma unroll
    for (int m = 16; m >= P; m >>= 1) r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, m));
    return r;
}

// G: query heads per kv head when it is 1, 2, 4 or 8 (0: any, read at run
// time).  With G known, a warp takes U positions at once and all U x G dot
// products share one butterfly (lane l ends with product l: position l / G,
// head l % G); otherwise each product has its own xor tree.
template <int HD, int G>
__global__ void __launch_bounds__(BD_ATT_THREADS, 2)
k_bd_attn_group(const float *__restrict__ q, const float *__restrict__ kc,
                const float *__restrict__ vc, const int *__restrict__ pos, int nh, int groups,
                int max_pos, size_t seq_stride, float scale, int terms, void *__restrict__ xs) {
    constexpr int VEC = HD / 32, NW = BD_ATT_THREADS / 32, U = 8, GB = 8;
    extern __shared__ float bsm[];
    const int r = blockIdx.x, g = blockIdx.y, n = pos[r] + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *sc = bsm;                                   // [groups][max_pos]
    float *qs = sc + (size_t)groups * max_pos;         // [groups][HD]
    float *pv = qs + groups * HD;                      // [NW][groups][HD]
    const int qd = nh * HD;
    const float *qrow = q + (size_t)r * qd + (size_t)g * groups * HD;
    const float *kg = kc + (size_t)r * seq_stride + (size_t)g * max_pos * HD + VEC * lane;
    const float *vg = vc + (size_t)r * seq_stride + (size_t)g * max_pos * HD + VEC * lane;
    for (int i = threadIdx.x; i < groups * HD; i += BD_ATT_THREADS) qs[i] = qrow[i];
    __syncthreads();
    if constexpr (G > 0) {
        constexpr int UG = 32 / G < 32 / VEC ? 32 / G : 32 / VEC, P = UG * G;
        float qv[G][VEC];
#pragma unroll
        for (int hq = 0; hq < G; hq++)
#pragma unroll
            for (int e = 0; e < VEC; e++) qv[hq][e] = qs[hq * HD + VEC * lane + e];
        for (int j0 = warp; j0 < n; j0 += UG * NW) {
            float kv[UG][VEC];
#pragma unroll
            for (int u = 0; u < UG; u++) {
                const int j = j0 + u * NW;
                if (j < n) {
                    bd_load<VEC>(kg + (size_t)j * HD, kv[u]);
                } else {
#pragma unroll
                    for (int e = 0; e < VEC; e++) kv[u][e] = 0.f;
                }
            }
            float v[P];
#pragma unroll
            for (int u = 0; u < UG; u++)
#pragma unroll
                for (int hq = 0; hq < G; hq++) {
                    float d = 0.f;
#pragma unroll
                    for (int e = 0; e < VEC; e++) d = __fadd_rn(d, __fmul_rn(qv[hq][e], kv[u][e]));
                    v[u * G + hq] = d;
                }
            const float tot = bd_bfly<P>(v, lane);
            const int j = j0 + (lane / G) * NW;
            if (lane < P && j < n) sc[(size_t)(lane % G) * max_pos + j] = __fmul_rn(tot, scale);
        }
    } else
    // scores: U positions of this warp in flight at a time
    for (int j0 = warp; j0 < n; j0 += U * NW) {
        float kv[U][VEC];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * NW;
            if (j < n)
                bd_load<VEC>(kg + (size_t)j * HD, kv[u]);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * NW;
            if (j >= n) break;
            for (int hq = 0; hq < groups; hq++) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < VEC; e++)
                    d = __fadd_rn(d, __fmul_rn(qs[hq * HD + VEC * lane + e], kv[u][e]));
#pragma unroll
                for (int o = 16; o; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, o));
                if (lane == 0) sc[(size_t)hq * max_pos + j] = __fmul_rn(d, scale);
            }
        }
    }
    __syncthreads();
    for (int hq = warp; hq < groups; hq += NW) {
        float *row = sc + (size_t)hq * max_pos;
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, row[j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sum = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float e = (float)exp((double)__fsub_rn(row[j], m));
            row[j] = e;
            sum = __fadd_rn(sum, e);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        for (int j = lane; j < n; j += 32) row[j] = __fdiv_rn(row[j], sum);
    }
    __syncthreads();
    // P.V: each v row read once per block of GB query heads
    for (int h0 = 0; h0 < groups; h0 += GB) {
        float acc[GB][VEC];
#pragma unroll
        for (int hh = 0; hh < GB; hh++)
#pragma unroll
            for (int e = 0; e < VEC; e++) acc[hh][e] = 0.f;
        for (int j0 = warp; j0 < n; j0 += U * NW) {
            float vv[U][VEC];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = j0 + u * NW;
                if (j < n)
                    bd_load<VEC>(vg + (size_t)j * HD, vv[u]);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = j0 + u * NW;
                if (j >= n) break;
#pragma unroll
                for (int hh = 0; hh < GB; hh++) {
                    if (h0 + hh >= groups) break;
                    const float pj = sc[(size_t)(h0 + hh) * max_pos + j];
#pragma unroll
                    for (int e = 0; e < VEC; e++)
                        acc[hh][e] = __fadd_rn(acc[hh][e], __fmul_rn(pj, vv[u][e]));
                }
            }
        }
#pragma unroll
        for (int hh = 0; hh < GB; hh++) {
            if (h0 + hh >= groups) break;
#pragma unroll
            for (int e = 0; e < VEC; e++)
                pv[((size_t)warp * groups + h0 + hh) * HD + VEC * lane + e] = acc[hh][e];
        }
    }
    __syncthreads();
    const size_t plane = (size_t)gridDim.x * qd, o0 = (size_t)r * qd + (size_t)g * groups * HD;
    for (int i = threadIdx.x; i < groups * HD; i += BD_ATT_THREADS) {
        float o = pv[i];
        for (int w = 1; w < NW; w++) o = __fadd_rn(o, pv[(size_t)w * groups * HD + i]);
        bd_emit(o, o0 + i, terms, plane, xs);
    }
}

// Greedy pick of row r of the lm_head GEMM output, the reference's rule
// (best = logits[0], then strict > over the rest in index order: the first
// maximum; NaN never wins, a NaN at 0 keeps 0).  Stage 1, grid nseq x
// BD_AC blocks: the first maximum of each contiguous slice of the row
// (index -1 when the slice has none).
constexpr int BD_AC = 32;

__global__ void k_bd_argmax_part(const float *__restrict__ part, int nz, int V,
                                 float *__restrict__ cand_v, int *__restrict__ cand_i) {
    __shared__ float bv[PF_THREADS];
    __shared__ int bi[PF_THREADS];
    const int r = blockIdx.x, c = blockIdx.y;
    const size_t plane = (size_t)gridDim.x * V, row = (size_t)r * V;
    const int per = (V + BD_AC - 1) / BD_AC, v0 = c * per, v1 = min(V, v0 + per);
    float best = -INFINITY;
    int idx = -1;
    for (int v = v0 + threadIdx.x; v < v1; v += PF_THREADS) {
        const float x = bd_sum(part, nz, plane, row + v);
        if (x > best) {   // per thread: first maximum in index order
            best = x;
            idx = v;
        }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = -INFINITY;
        int k = -1;
        for (int t = 0; t < PF_THREADS; t++)
            if (bi[t] >= 0 && (k < 0 || bv[t] > b || (bv[t] == b && bi[t] < k))) {
                b = bv[t];
                k = bi[t];
            }
        cand_v[r * BD_AC + c] = b;
        cand_i[r * BD_AC + c] = k;
    }
}

// Stage 2, one thread per row: the slices' maxima in slice order from
// (logits[0], 0), strict >; written as the row's next token and as its
// generated token pos[r] - start[r]; the row's position advances.
__global__ void k_bd_argmax_pick(const float *__restrict__ part, int nz, int V, int nseq,
                                 const float *__restrict__ cand_v, const int *__restrict__ cand_i,
                                 const int *__restrict__ start, int max_new,
                                 int *__restrict__ tok, int *__restrict__ pos,
                                 int *__restrict__ gen) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= nseq) return;
    float b = bd_sum(part, nz, (size_t)nseq * V, (size_t)r * V);
    int k = 0;
    if (!(b != b))   // NaN at 0: the reference keeps index 0
        for (int c = 0; c < BD_AC; c++) {
            const int i = cand_i[r * BD_AC + c];
            if (i >= 0 && cand_v[r * BD_AC + c] > b) {
                b = cand_v[r * BD_AC + c];
                k = i;
            }
        }
    tok[r] = k;
    const int step = pos[r] - start[r];
    if (step >= 0 && step < max_new) gen[(size_t)r * max_new + step] = k;
    pos[r] = pos[r] + 1;
}

}  // namespace kllm
