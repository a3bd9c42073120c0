// batch.cuh -- the row kernels of batched greedy decode (plan.cu,
// plan_infer_batch): one row per sequence, every sequence at its own
// position with its own KV cache.  The projections around them are the
// prompt pass's GEMMs (bit-exact TT-GEMM per row, or the tensor cores);
// norms, residual adds and SwiGLU are the prompt pass's row kernels.  Each
// element is the tape's float arithmetic for its sequence (reductions in a
// fixed order of their own, as in the prompt pass).
#pragma once

#include "common.cuh"
#include "prefill.cuh"

namespace kllm {

// Row r of the fused QKV output at position pos[r]: rotate-half RoPE of q
// (to q_out[r]) and k, k and v appended to sequence r's cache (row pos[r]).
// Caches: [seq][layer][kv_head][max_pos][hd]; kc / vc point at this layer of
// sequence 0, seq_stride floats apart.  (grid: nseq blocks)
__global__ void k_bd_rope_kv(const float *__restrict__ qkv, const int *__restrict__ pos, int nq,
                             int nh, int nkv, int hd, const float *__restrict__ rcos,
                             const float *__restrict__ rsin, int max_pos, size_t seq_stride,
                             float *__restrict__ q_out, float *__restrict__ kc,
                             float *__restrict__ vc) {
    const int r = blockIdx.x, p = pos[r];
    const int qd = nh * hd, kvd = nkv * hd;
    const float *y = qkv + (size_t)r * nq;
    float *kr = kc + (size_t)r * seq_stride, *vr = vc + (size_t)r * seq_stride;
    for (int n = threadIdx.x; n < qd + 2 * kvd; n += blockDim.x) {
        if (n < qd + kvd) {
            const int head = n / hd, dim = n % hd, half = hd / 2;
            const float pk = dim < half ? -y[n + half] : y[n - half];
            const float v = __fadd_rn(__fmul_rn(y[n], rcos[(size_t)p * hd + dim]),
                                      __fmul_rn(pk, rsin[(size_t)p * hd + dim]));
            if (head < nh)
                q_out[(size_t)r * qd + n] = v;
            else
                kr[((size_t)(head - nh) * max_pos + p) * hd + dim] = v;
        } else {
            const int vi = n - qd - kvd;
            vr[((size_t)(vi / hd) * max_pos + p) * hd + vi % hd] = y[n];
        }
    }
}

// Attention of row r (position pos[r]), head h, over positions 0..pos[r]
// of sequence r's cache: scores q.k * scale, max-subtracted exp in double,
// sum, divide, P.V.  (grid: nseq x nh blocks, PF_THREADS threads, dynamic
// shared memory: max(max_pos, PF_THREADS) floats; hd divides PF_THREADS)
__global__ void k_bd_attention(const float *__restrict__ q, const float *__restrict__ kc,
                               const float *__restrict__ vc, const int *__restrict__ pos, int nh,
                               int groups, int hd, int max_pos, size_t seq_stride, float scale,
                               float *__restrict__ ctx) {
    extern __shared__ float sc[];
    __shared__ float red[PF_THREADS / 32];
    const int r = blockIdx.x, h = blockIdx.y, g = h / groups, n = pos[r] + 1;
    const int qd = nh * hd;
    const float *qr = q + (size_t)r * qd + h * hd;
    const float *kg = kc + (size_t)r * seq_stride + (size_t)g * max_pos * hd;
    const float *vg = vc + (size_t)r * seq_stride + (size_t)g * max_pos * hd;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < n; j += PF_THREADS) {
        float dot = 0.f;
        for (int d = 0; d < hd; d++) dot = __fadd_rn(dot, __fmul_rn(qr[d], kg[(size_t)j * hd + d]));
        const float s = __fmul_rn(dot, scale);
        sc[j] = s;
        m = fmaxf(m, s);
    }
    const float mx = pf_block_max(m, red);
    float sum = 0.f;
    for (int j = threadIdx.x; j < n; j += PF_THREADS) {
        const float e = (float)exp((double)__fsub_rn(sc[j], mx));
        sc[j] = e;
        sum = __fadd_rn(sum, e);
    }
    const float tot = pf_block_sum(sum, red);
    for (int j = threadIdx.x; j < n; j += PF_THREADS) sc[j] = __fdiv_rn(sc[j], tot);
    __syncthreads();
    // P.V: PF_THREADS / hd position groups per dim, summed in group order
    const int per = PF_THREADS / hd;   // hd divides PF_THREADS (32, 64, 128)
    const int d = threadIdx.x % hd, grp = threadIdx.x / hd;
    float acc = 0.f;
    for (int j = grp; j < n; j += per) acc = __fadd_rn(acc, __fmul_rn(sc[j], vg[(size_t)j * hd + d]));
    __syncthreads();
    sc[threadIdx.x] = acc;   // sc is free again (n >= 1 entries were read above)
    __syncthreads();
    if (grp == 0) {
        float o = sc[d];
        for (int i = 1; i < per; i++) o = __fadd_rn(o, sc[i * hd + d]);
        ctx[(size_t)r * qd + h * hd + d] = o;
    }
}

// Greedy pick of row r (the reference's: best = logits[0], then strict >
// over the rest in index order), written as the row's next token and as
// generated token `step`; the row's position advances.  (grid: nseq
// blocks, PF_THREADS threads)
__global__ void k_bd_argmax(const float *__restrict__ logits, int V, int step, int max_new,
                            int *__restrict__ tok, int *__restrict__ pos, int *__restrict__ gen) {
    __shared__ float bv[PF_THREADS];
    __shared__ int bi[PF_THREADS];
    const int r = blockIdx.x;
    const float *lg = logits + (size_t)r * V;
    float best = -INFINITY;
    int idx = -1;
    for (int v = threadIdx.x; v < V; v += PF_THREADS) {
        const float x = lg[v];
        if (x > best) {   // per thread: first maximum in index order (NaN never wins)
            best = x;
            idx = v;
        }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = lg[0];
        int k = 0;
        if (!(b != b)) {   // NaN at 0: the reference keeps index 0
            for (int t = 0; t < PF_THREADS; t++)
                if (bi[t] >= 0 && (bv[t] > b || (bv[t] == b && bi[t] < k))) {
                    b = bv[t];
                    k = bi[t];
                }
        }
        tok[r] = k;
        gen[(size_t)r * max_new + step] = k;
        pos[r] = pos[r] + 1;
    }
}

}  // namespace kllm
