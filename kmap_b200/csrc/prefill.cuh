// prefill.cuh -- the row kernels of the batched prompt pass (plan.cu,
// plan_prefill): R prompt positions go through every layer at once, the
// projections as TT-GEMMs (ttgemm.cu), these kernels around them.  Each
// element is the tape's float arithmetic for its position, the same
// operations the decode step applies to one position (reductions -- the
// RMSNorm sum of squares, attention dot products and softmax sums -- in a
// fixed order of their own).
#pragma once

#include "common.cuh"

namespace kllm {

constexpr int PF_THREADS = 256;

// Fixed-shape block sum (PF_THREADS threads): warp trees, then warps in order.
__device__ __forceinline__ float pf_block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < PF_THREADS / 32; i++) r = __fadd_rn(r, red[i]);
    return r;
}

__device__ __forceinline__ float pf_block_max(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < PF_THREADS / 32; i++) r = fmaxf(r, red[i]);
    return r;
}

// h[r][:] = embed[prompt[r]][:]   (grid: R blocks)
__global__ void k_pf_embed(const float *__restrict__ embed, const int *__restrict__ prompt,
                           int H, float *__restrict__ h) {
    const int r = blockIdx.x;
    const float *e = embed + (size_t)prompt[r] * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) h[(size_t)r * H + i] = e[i];
}

// out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w, the tape's RMSNORM
// arithmetic: mean as sum * (1 / H), rsqrt in double, two rounded products.
__global__ void k_pf_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, float eps,
                             int H, float *__restrict__ out) {
    __shared__ float red[PF_THREADS / 32];
    const int r = blockIdx.x;
    const float *xr = x + (size_t)r * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += PF_THREADS) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
    const float tot = pf_block_sum(ss, red);
    const float add = __fadd_rn(__fmul_rn(tot, 1.0f / (float)H), eps);
    const float rsq = (float)(1.0 / sqrt((double)add));
    for (int i = threadIdx.x; i < H; i += PF_THREADS)
        out[(size_t)r * H + i] = __fmul_rn(__fmul_rn(xr[i], rsq), w[i]);
}

// Rotate-half RoPE of row r (position r) of the fused QKV output, q to
// q_out[r][qd], rotated k and plain v into the layer's cache rows r:
// v' = y * cos[dim] + rot * sin[dim], rot = -y[dim + hd/2] in the first
// half of a head and +y[dim - hd/2] in the second.  (grid: R blocks)
__global__ void k_pf_rope_kv(const float *__restrict__ qkv, int nq, int nh, int nkv, int hd,
                             const float *__restrict__ rcos, const float *__restrict__ rsin,
                             int max_pos, float *__restrict__ q_out, float *__restrict__ kc,
                             float *__restrict__ vc) {
    const int r = blockIdx.x;
    const int qd = nh * hd, kvd = nkv * hd;
    const float *y = qkv + (size_t)r * nq;
    for (int n = threadIdx.x; n < qd + 2 * kvd; n += blockDim.x) {
        if (n < qd + kvd) {
            const int head = n / hd, dim = n % hd, half = hd / 2;
            const float pk = dim < half ? -y[n + half] : y[n - half];
            const float v = __fadd_rn(__fmul_rn(y[n], rcos[(size_t)r * hd + dim]),
                                      __fmul_rn(pk, rsin[(size_t)r * hd + dim]));
            if (head < nh)
                q_out[(size_t)r * qd + n] = v;
            else
                kc[((size_t)(head - nh) * max_pos + r) * hd + dim] = v;
        } else {
            const int vi = n - qd - kvd;
            vc[((size_t)(vi / hd) * max_pos + r) * hd + vi % hd] = y[n];
        }
    }
}

// Causal attention of row r (position r), head h: scores over positions
// 0..r of the head's kv group, softmax (exp in double), P.V.
// (grid: R x nh blocks, dynamic shared memory: (R + 1) floats)
__global__ void k_pf_attention(const float *__restrict__ q, const float *__restrict__ kc,
                               const float *__restrict__ vc, int nh, int groups, int hd,
                               int max_pos, float scale, float *__restrict__ ctx) {
    extern __shared__ float sc[];
    __shared__ float red[PF_THREADS / 32];
    const int r = blockIdx.x, h = blockIdx.y, g = h / groups;
    const int qd = nh * hd;
    const float *qr = q + (size_t)r * qd + h * hd;
    const float *kg = kc + (size_t)g * max_pos * hd;
    const float *vg = vc + (size_t)g * max_pos * hd;
    float m = -INFINITY;
    for (int j = threadIdx.x; j <= r; j += PF_THREADS) {
        float dot = 0.f;
        for (int d = 0; d < hd; d++) dot = __fadd_rn(dot, __fmul_rn(qr[d], kg[(size_t)j * hd + d]));
        const float s = __fmul_rn(dot, scale);
        sc[j] = s;
        m = fmaxf(m, s);
    }
    const float mx = pf_block_max(m, red);
    float sum = 0.f;
    for (int j = threadIdx.x; j <= r; j += PF_THREADS) {
        const float e = (float)exp((double)__fsub_rn(sc[j], mx));
        sc[j] = e;
        sum = __fadd_rn(sum, e);
    }
    const float tot = pf_block_sum(sum, red);
    for (int j = threadIdx.x; j <= r; j += PF_THREADS) sc[j] = __fdiv_rn(sc[j], tot);
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += PF_THREADS) {
        float acc = 0.f;
        for (int j = 0; j <= r; j++) acc = __fadd_rn(acc, __fmul_rn(sc[j], vg[(size_t)j * hd + d]));
        ctx[(size_t)r * qd + h * hd + d] = acc;
    }
}

// Causal attention of R prompt positions, tiled (flash-style): block =
// (64 queries, head h); key/value tiles of 64 positions of the head's kv
// group go through shared memory, scores with fused multiply-adds, an
// online softmax per query row (running max and sum, exp in float) and the
// P.V tile product.  A tolerance result like the row kernel above (whose
// exact-order sums it replaces at long prompts): the decode step and the
// reference sum in other orders.  (grid: ceil(R / 64) x nh blocks, 256
// threads, dynamic shared memory pf_flash_smem<HD>())
constexpr int PFA_BQ = 64, PFA_BK = 64;

template <int HD>
__host__ __device__ constexpr size_t pf_flash_smem() {
    return (size_t)4 * (PFA_BQ * (HD + 1) + PFA_BK * (HD + 1) + PFA_BK * HD + PFA_BQ * (PFA_BK + 1));
}

template <int HD>
__global__ void __launch_bounds__(256)
k_pf_flash(const float *__restrict__ q, const float *__restrict__ kc, const float *__restrict__ vc,
           int R, int nh, int groups, int max_pos, float scale, float *__restrict__ ctx) {
    constexpr int DQ = HD / 16;                 // output dims per thread (4 or 8)
    extern __shared__ float sm[];
    float *Qs = sm;                             // [BQ][HD + 1]
    float *Ks = Qs + PFA_BQ * (HD + 1);         // [BK][HD + 1]
    float *Vs = Ks + PFA_BK * (HD + 1);         // [BK][HD]
    float *Ps = Vs + PFA_BK * HD;               // [BQ][BK + 1]
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int qt = blockIdx.x, h = blockIdx.y, g = h / groups;
    const int q0 = qt * PFA_BQ, qd = nh * HD;
    const float *kg = kc + (size_t)g * max_pos * HD;
    const float *vg = vc + (size_t)g * max_pos * HD;
    for (int i = tid; i < PFA_BQ * HD; i += 256) {
        const int r = i / HD, d = i % HD;
        Qs[r * (HD + 1) + d] = q0 + r < R ? q[(size_t)(q0 + r) * qd + h * HD + d] : 0.f;
    }
    float m[4], l[4], o[4][DQ];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int d = 0; d < DQ; d++) o[i][d] = 0.f;
    }
    const int last_q = min(q0 + PFA_BQ, R) - 1;
    for (int k0 = 0; k0 <= last_q; k0 += PFA_BK) {
        __syncthreads();   // the previous tile's Ks, Vs, Ps are free
        for (int i = tid; i < PFA_BK * HD; i += 256) {
            const int r = i / HD, d = i % HD;
            const bool in = k0 + r <= last_q;
            Ks[r * (HD + 1) + d] = in ? kg[(size_t)(k0 + r) * HD + d] : 0.f;
            Vs[r * HD + d] = in ? vg[(size_t)(k0 + r) * HD + d] : 0.f;
        }
        __syncthreads();
        // scores: rows ty*4 + i, key columns tx + 16 j
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 8
        for (int d = 0; d < HD; d++) {
            float qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = Qs[(ty * 4 + i) * (HD + 1) + d];
#pragma unroll
            for (int j = 0; j < 4; j++) kv[j] = Ks[(tx + 16 * j) * (HD + 1) + d];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qi = q0 + ty * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int kj = k0 + tx + 16 * j;
                sc[i][j] = kj <= qi ? sc[i][j] * scale : -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float pj = sc[i][j] == -INFINITY ? 0.f : expf(sc[i][j] - mn);
                Ps[(ty * 4 + i) * (PFA_BK + 1) + tx + 16 * j] = pj;
                rs += pj;
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[i] = l[i] * corr + rs;
            m[i] = mn;
#pragma unroll
            for (int d = 0; d < DQ; d++) o[i][d] *= corr;
        }
        __syncthreads();
        // P.V: rows ty*4 + i, dims tx*DQ .. tx*DQ + DQ - 1
#pragma unroll 4
        for (int jj = 0; jj < PFA_BK; jj++) {
            float vv[DQ];
#pragma unroll
            for (int d = 0; d < DQ; d += 4) {
                const float4 v4 = *reinterpret_cast<const float4 *>(Vs + jj * HD + tx * DQ + d);
                vv[d] = v4.x;
                vv[d + 1] = v4.y;
                vv[d + 2] = v4.z;
                vv[d + 3] = v4.w;
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float pv = Ps[(ty * 4 + i) * (PFA_BK + 1) + jj];
#pragma unroll
                for (int d = 0; d < DQ; d++) o[i][d] = fmaf(pv, vv[d], o[i][d]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int qi = q0 + ty * 4 + i;
        if (qi >= R) continue;
        const float inv = 1.f / l[i];
#pragma unroll
        for (int d = 0; d < DQ; d++) ctx[(size_t)qi * qd + h * HD + tx * DQ + d] = o[i][d] * inv;
    }
}

// out = a + b, elementwise (the residual adds)
__global__ void k_pf_add(const float *__restrict__ a, const float *__restrict__ b, long long n,
                         float *__restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// act[r][n] = silu(gu[r][n]) * gu[r][F + n], silu in double as the tape's
// SILU: g / (1 + exp(-g)).  (grid-stride over R * F)
__global__ void k_pf_swiglu(const float *__restrict__ gu, int F, long long rf,
                            float *__restrict__ act) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rf;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / F, n = i % F;
        const double dg = (double)gu[r * 2 * F + n];
        act[i] = __fmul_rn((float)(dg / (1.0 + exp(-dg))), gu[r * 2 * F + F + n]);
    }
}

}  // namespace kllm
