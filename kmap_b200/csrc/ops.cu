// ops.cu -- one device kernel per tape opcode, for tapes (or parts of tapes)
// that the fused decode plan does not cover.  Each kernel computes exactly
// what the reference op computes (reference _tape_runner.c:98-300, 677-992):
//   * SILU / EXP / RSQRT / COS / SIN evaluate in double and round to float
//     (_tape_runner.c:98-123);
//   * ADD/SUB/MUL/DIV/MAX broadcast right-aligned (numpy rules,
//     _tape_runner.c:81-92, 132-161), MAX is `a > b ? a : b`;
//   * SUM / MEAN / MAX_RED / ARGMAX walk the reduced axis in order with a
//     float accumulator starting at 0.0f, MEAN multiplies by 1.0f/n, ARGMAX
//     keeps the first maximum (_tape_runner.c:163-239, 839-871);
//   * TRANSPOSE / REPEAT / SLICE / CONCAT move data with the same index
//     arithmetic (_tape_runner.c:241-300, 895-947).
// MATMUL is a plain dot product per output; the reference calls BLAS there,
// whose summation order is implementation-defined, so that op is only
// tolerance-equal.
#include "common.cuh"

namespace kllm {

static constexpr int kThreads = 256;

static inline int blocks_for(long long n) {
    long long b = (n + kThreads - 1) / kThreads;
    if (b < 1) b = 1;
    if (b > 148 * 32) b = 148 * 32;
    return (int)b;
}

#define GRID_STRIDE(i, n) \
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (n); \
         i += (long long)gridDim.x * blockDim.x)

template <int OP>
__global__ void k_unary(const float *__restrict__ x, float *__restrict__ y, long long n) {
    GRID_STRIDE(i, n) {
        float v = x[i];
        float r;
        if (OP == OP_SILU) {
            double d = (double)v;
            r = (float)(d / (1.0 + exp(-d)));
        } else if (OP == OP_EXP) {
            r = (float)exp((double)v);
        } else if (OP == OP_RSQRT) {
            r = (float)(1.0 / sqrt((double)v));
        } else if (OP == OP_COS) {
            r = (float)cos((double)v);
        } else if (OP == OP_SIN) {
            r = (float)sin((double)v);
        } else if (OP == OP_NEG) {
            r = __uint_as_float(__float_as_uint(v) ^ 0x80000000u);
        } else {  // SQUARE
            r = __fmul_rn(v, v);
        }
        y[i] = r;
    }
}

bool launch_unary(cudaStream_t s, int op, const float *x, float *y, long long n) {
    if (n <= 0) return true;
    int g = blocks_for(n);
    switch (op) {
    case OP_SILU: k_unary<OP_SILU><<<g, kThreads, 0, s>>>(x, y, n); break;
    case OP_EXP: k_unary<OP_EXP><<<g, kThreads, 0, s>>>(x, y, n); break;
    case OP_RSQRT: k_unary<OP_RSQRT><<<g, kThreads, 0, s>>>(x, y, n); break;
    case OP_COS: k_unary<OP_COS><<<g, kThreads, 0, s>>>(x, y, n); break;
    case OP_SIN: k_unary<OP_SIN><<<g, kThreads, 0, s>>>(x, y, n); break;
    case OP_NEG: k_unary<OP_NEG><<<g, kThreads, 0, s>>>(x, y, n); break;
    default: k_unary<OP_SQUARE><<<g, kThreads, 0, s>>>(x, y, n); break;
    }
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

template <int OP>
__device__ __forceinline__ float binop(float a, float b) {
    if (OP == OP_ADD) return __fadd_rn(a, b);
    if (OP == OP_SUB) return __fsub_rn(a, b);
    if (OP == OP_MUL) return __fmul_rn(a, b);
    if (OP == OP_DIV) return __fdiv_rn(a, b);
    return a > b ? a : b;
}

template <int OP>
__global__ void k_binop_same(const float *__restrict__ a, const float *__restrict__ b,
                             float *__restrict__ y, long long n) {
    GRID_STRIDE(i, n) y[i] = binop<OP>(a[i], b[i]);
}

// Broadcast strides: element stride of each output dimension in a / b,
// zero where the operand dimension is 1 or missing.
struct BStrides {
    int nd;
    long long ydim[MAX_DIMS];
    long long sa[MAX_DIMS];
    long long sb[MAX_DIMS];
};

template <int OP>
__global__ void k_binop_bcast(const float *__restrict__ a, const float *__restrict__ b,
                              float *__restrict__ y, long long n, BStrides bs) {
    GRID_STRIDE(i, n) {
        long long rem = i, ia = 0, ib = 0;
        for (int d = bs.nd - 1; d >= 0; d--) {
            long long q = rem % bs.ydim[d];
            rem /= bs.ydim[d];
            ia += q * bs.sa[d];
            ib += q * bs.sb[d];
        }
        y[i] = binop<OP>(a[ia], b[ib]);
    }
}

static void bstride(const Dims &in, const Dims &out, long long *st) {
    long long s[MAX_DIMS];
    long long acc = 1;
    for (int d = in.nd - 1; d >= 0; d--) {
        s[d] = acc;
        acc *= in.d[d];
    }
    int off = out.nd - in.nd;
    for (int d = 0; d < out.nd; d++) {
        int j = d - off;
        st[d] = (j < 0 || in.d[j] == 1) ? 0 : s[j];
    }
}

bool launch_binop(cudaStream_t s, int op, const float *a, const Dims &da, const float *b,
                  const Dims &db, float *y, const Dims &dy) {
    long long n = 1;
    for (int d = 0; d < dy.nd; d++) n *= dy.d[d];
    if (n <= 0) return true;
    bool same = da.nd == db.nd && da.nd == dy.nd;
    for (int d = 0; same && d < da.nd; d++) same = da.d[d] == db.d[d];
    int g = blocks_for(n);
    if (same) {
        switch (op) {
        case OP_ADD: k_binop_same<OP_ADD><<<g, kThreads, 0, s>>>(a, b, y, n); break;
        case OP_SUB: k_binop_same<OP_SUB><<<g, kThreads, 0, s>>>(a, b, y, n); break;
        case OP_MUL: k_binop_same<OP_MUL><<<g, kThreads, 0, s>>>(a, b, y, n); break;
        case OP_DIV: k_binop_same<OP_DIV><<<g, kThreads, 0, s>>>(a, b, y, n); break;
        default: k_binop_same<OP_MAX><<<g, kThreads, 0, s>>>(a, b, y, n); break;
        }
    } else {
        BStrides bs;
        bs.nd = dy.nd;
        for (int d = 0; d < dy.nd; d++) bs.ydim[d] = dy.d[d];
        bstride(da, dy, bs.sa);
        bstride(db, dy, bs.sb);
        switch (op) {
        case OP_ADD: k_binop_bcast<OP_ADD><<<g, kThreads, 0, s>>>(a, b, y, n, bs); break;
        case OP_SUB: k_binop_bcast<OP_SUB><<<g, kThreads, 0, s>>>(a, b, y, n, bs); break;
        case OP_MUL: k_binop_bcast<OP_MUL><<<g, kThreads, 0, s>>>(a, b, y, n, bs); break;
        case OP_DIV: k_binop_bcast<OP_DIV><<<g, kThreads, 0, s>>>(a, b, y, n, bs); break;
        default: k_binop_bcast<OP_MAX><<<g, kThreads, 0, s>>>(a, b, y, n, bs); break;
        }
    }
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

// One thread per output element walks the reduced axis in order.
template <int OP>
__global__ void k_reduce(const float *__restrict__ x, float *__restrict__ y, long long outer,
                         int axis_n, long long inner, float scale) {
    GRID_STRIDE(o, outer * inner) {
        long long oo = o / inner, ii = o % inner;
        const float *p = x + oo * axis_n * inner + ii;
        if (OP == OP_SUM || OP == OP_MEAN) {
            float acc = 0.0f;
            for (int a = 0; a < axis_n; a++) acc = __fadd_rn(acc, p[(long long)a * inner]);
            if (OP == OP_MEAN) acc = __fmul_rn(acc, scale);
            y[o] = acc;
        } else if (OP == OP_MAX_RED) {
            float m = p[0];
            for (int a = 1; a < axis_n; a++) {
                float v = p[(long long)a * inner];
                if (v > m) m = v;
            }
            y[o] = m;
        } else {  // ARGMAX
            float m = p[0];
            int mi = 0;
            for (int a = 1; a < axis_n; a++) {
                float v = p[(long long)a * inner];
                if (v > m) {
                    m = v;
                    mi = a;
                }
            }
            y[o] = (float)mi;
        }
    }
}

bool launch_reduce(cudaStream_t s, int op, const float *x, float *y, long long outer,
                   int axis_n, long long inner) {
    long long n = outer * inner;
    if (n <= 0) return true;
    int g = blocks_for(n);
    float scale = 1.0f / (float)axis_n;
    switch (op) {
    case OP_SUM: k_reduce<OP_SUM><<<g, kThreads, 0, s>>>(x, y, outer, axis_n, inner, scale); break;
    case OP_MEAN: k_reduce<OP_MEAN><<<g, kThreads, 0, s>>>(x, y, outer, axis_n, inner, scale); break;
    case OP_MAX_RED:
        k_reduce<OP_MAX_RED><<<g, kThreads, 0, s>>>(x, y, outer, axis_n, inner, scale);
        break;
    default: k_reduce<OP_ARGMAX><<<g, kThreads, 0, s>>>(x, y, outer, axis_n, inner, scale); break;
    }
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

// Generic gather: y[i] = x[src(i)], where the output index is decomposed
// over `odim` and mapped through per-dimension (div, stride, offset) rules.
struct Gather {
    int nd;
    long long odim[MAX_DIMS];   // output dims
    long long istride[MAX_DIMS];  // input element stride for each output dim
    long long ioff[MAX_DIMS];   // constant input offset per dim (slice start)
    long long idiv[MAX_DIMS];   // index divisor per dim (repeat)
};

__global__ void k_gather(const float *__restrict__ x, float *__restrict__ y, long long n,
                         Gather g) {
    GRID_STRIDE(i, n) {
        long long rem = i, src = 0;
        for (int d = g.nd - 1; d >= 0; d--) {
            long long q = rem % g.odim[d];
            rem /= g.odim[d];
            src += (q / g.idiv[d] + g.ioff[d]) * g.istride[d];
        }
        y[i] = x[src];
    }
}

static void in_strides(const Dims &din, long long *st) {
    long long acc = 1;
    for (int d = din.nd - 1; d >= 0; d--) {
        st[d] = acc;
        acc *= din.d[d];
    }
}

static bool run_gather(cudaStream_t s, const float *x, float *y, const Gather &g) {
    long long n = 1;
    for (int d = 0; d < g.nd; d++) n *= g.odim[d];
    if (n <= 0) return true;
    k_gather<<<blocks_for(n), kThreads, 0, s>>>(x, y, n, g);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool launch_transpose(cudaStream_t s, const float *x, const Dims &din, const int *axes,
                      float *y) {
    long long st[MAX_DIMS];
    in_strides(din, st);
    Gather g;
    g.nd = din.nd;
    for (int d = 0; d < din.nd; d++) {
        g.odim[d] = din.d[axes[d]];
        g.istride[d] = st[axes[d]];
        g.ioff[d] = 0;
        g.idiv[d] = 1;
    }
    return run_gather(s, x, y, g);
}

bool launch_repeat(cudaStream_t s, const float *x, const Dims &din, int reps, int axis,
                   float *y) {
    long long st[MAX_DIMS];
    in_strides(din, st);
    Gather g;
    g.nd = din.nd;
    for (int d = 0; d < din.nd; d++) {
        g.odim[d] = din.d[d] * (d == axis ? reps : 1);
        g.istride[d] = st[d];
        g.ioff[d] = 0;
        g.idiv[d] = d == axis ? reps : 1;
    }
    return run_gather(s, x, y, g);
}

bool launch_slice(cudaStream_t s, const float *x, const Dims &din, const int *starts,
                  const int *steps, const Dims &dout, float *y) {
    long long st[MAX_DIMS];
    in_strides(din, st);
    Gather g;
    g.nd = din.nd;
    for (int d = 0; d < din.nd; d++) {
        g.odim[d] = dout.d[d];
        g.istride[d] = st[d] * steps[d];
        g.ioff[d] = 0;
        g.idiv[d] = 1;
    }
    // fold the starts into a base offset
    long long base = 0;
    for (int d = 0; d < din.nd; d++) base += (long long)starts[d] * st[d];
    return run_gather(s, x + base, y, g);
}

struct ConcatArgs {
    const float *x[MAX_CONCAT_INPUTS];
    long long chunk[MAX_CONCAT_INPUTS];
    long long prefix[MAX_CONCAT_INPUTS + 1];
    int n;
};

// out[o][prefix[ci] + j] = x_ci[o][j] for each outer row o.
__global__ void k_concat(float *__restrict__ y, long long outer, ConcatArgs a) {
    long long row = a.prefix[a.n];
    GRID_STRIDE(i, outer * row) {
        long long o = i / row, j = i % row;
        int ci = 0;
        while (ci + 1 < a.n && j >= a.prefix[ci + 1]) ci++;
        y[i] = a.x[ci][o * a.chunk[ci] + (j - a.prefix[ci])];
    }
}

bool launch_concat(cudaStream_t s, const float *const *xs, const long long *chunk, int n,
                   long long outer, float *y) {
    ConcatArgs a;
    a.n = n;
    a.prefix[0] = 0;
    for (int i = 0; i < n; i++) {
        a.x[i] = xs[i];
        a.chunk[i] = chunk[i];
        a.prefix[i + 1] = a.prefix[i] + chunk[i];
    }
    long long tot = outer * a.prefix[n];
    if (tot <= 0) return true;
    k_concat<<<blocks_for(tot), kThreads, 0, s>>>(y, outer, a);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

// y[b][i][j] = sum_k a[b][i][k] * b[b][k][j], k ascending.
__global__ void k_matmul(const float *__restrict__ a, const float *__restrict__ b,
                         float *__restrict__ y, int batch, int m, int k, int n) {
    GRID_STRIDE(o, (long long)batch * m * n) {
        long long bi = o / ((long long)m * n);
        long long r = o % ((long long)m * n);
        int i = (int)(r / n), j = (int)(r % n);
        const float *pa = a + (bi * m + i) * (long long)k;
        const float *pb = b + bi * (long long)k * n + j;
        float acc = 0.f;
        for (int kk = 0; kk < k; kk++) acc = fmaf(pa[kk], pb[(long long)kk * n], acc);
        y[o] = acc;
    }
}

bool launch_matmul(cudaStream_t s, const float *a, const float *b, float *y, int batch, int m,
                   int k, int n) {
    long long tot = (long long)batch * m * n;
    if (tot <= 0) return true;
    k_matmul<<<blocks_for(tot), kThreads, 0, s>>>(a, b, y, batch, m, k, n);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

__global__ void k_fill(float *y, long long n, float v) {
    GRID_STRIDE(i, n) y[i] = v;
}

bool launch_fill(cudaStream_t s, float *y, long long n, float v) {
    if (n <= 0) return true;
    k_fill<<<blocks_for(n), kThreads, 0, s>>>(y, n, v);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

}  // namespace kllm
