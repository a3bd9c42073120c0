// ttgemm.cu -- the TT-GEMM: many rows of x against one truth-table matrix
// (prefill: every prompt position through the same MATMUL_TT), each row
// bit-identical to the TT-GEMV of that row (_tape_runner.c:474-663).
//
// y[r][n] = sum over chunks t (in order) of the chunk's serial sum
// fl(acc + fl(x[r][k] * codebook[idx[k][n]])) for k in the chunk, with the
// reference's chunking of K (T = min(8, ceil(K / 128)) chunks, the first
// K % T one row longer).  A block owns a 64 x 128 tile of y; its 256
// threads own 4 x 8 outputs each.  The K loop runs over 16-row slices of x
// and of the decoded weights, double-buffered in shared memory; every
// accumulator restarts at each chunk boundary of K and is folded into the
// output in chunk order ((p0 + p1) + p2 ...), the same arithmetic as the
// TT-GEMV's chunk reduction.  Weight reuse is 64 rows per decoded tile, so
// the kernel is bound by the FP32 pipes (separate multiply and add: a fused
// multiply-add would round differently), not by the 2-byte index stream.
// No scratch memory: partial sums live in registers.
#include "common.cuh"

namespace kllm {

constexpr int GM = 64;    // rows of y per block
constexpr int GN = 128;   // columns of y per block
constexpr int GK = 16;    // rows of K per slice
constexpr int GT = 256;   // threads: 16 column groups of 8 x 16 row groups of 4

__global__ void __launch_bounds__(GT, 2)
k_tt_gemm(const float *__restrict__ x, int rows, const float *__restrict__ cb,
          const uint16_t *__restrict__ idx, int K, int N, int T, float *__restrict__ y) {
    // x slice, k-major; rows padded to 68 floats so the transposing stores
    // spread over the banks (float4 reads stay 16-byte aligned)
    __shared__ __align__(16) float xs[2][GK][GM + 4];
    __shared__ __align__(16) float ws[2][GK][GN];   // decoded weights
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int r0 = blockIdx.y * GM, n0 = blockIdx.x * GN;
    const int base = K / T, rem = K % T;

    float xr[GM * GK / GT], wr[GN * GK / GT];       // the next slice, global -> registers
    auto gload = [&](int k0) {
#pragma unroll
        for (int i = 0; i < GM * GK / GT; i++) {
            const int e = tid + i * GT, m = e / GK, kk = e % GK;
            const int r = r0 + m, k = k0 + kk;
            xr[i] = (r < rows && k < K) ? __ldg(x + (size_t)r * K + k) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < GN * GK / GT; i++) {
            const int e = tid + i * GT, kk = e / GN, n = e % GN;
            const int k = k0 + kk, nn = n0 + n;
            wr[i] = (k < K && nn < N) ? __ldg(cb + __ldg(idx + (size_t)k * N + nn)) : 0.f;
        }
    };
    auto sstore = [&](int b) {
#pragma unroll
        for (int i = 0; i < GM * GK / GT; i++) {
            const int e = tid + i * GT;
            xs[b][e % GK][e / GK] = xr[i];
        }
#pragma unroll
        for (int i = 0; i < GN * GK / GT; i++) {
            const int e = tid + i * GT;
            ws[b][e / GN][e % GN] = wr[i];
        }
    };

    float acc[4][8], out[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = out[i][j] = 0.f;
    int t = 0;                                   // current chunk
    int kend = base + (rem > 0 ? 1 : 0);         // first row past chunk t
    // the finished chunk's sums into the output, in chunk order
    auto fold = [&]() {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                out[i][j] = t == 0 ? acc[i][j] : __fadd_rn(out[i][j], acc[i][j]);
                acc[i][j] = 0.f;
            }
    };

    const int nk = (K + GK - 1) / GK;
    gload(0);
    sstore(0);
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        const int b = kt & 1;
        if (kt + 1 < nk) gload((kt + 1) * GK);
#pragma unroll
        for (int kk = 0; kk < GK; kk++) {
            const int k = kt * GK + kk;
            if (k < K) {   // uniform across the block
                if (k == kend) {
                    fold();
                    t++;
                    kend += base + (t < rem ? 1 : 0);
                }
                const float4 a = *reinterpret_cast<const float4 *>(&xs[b][kk][ty * 4]);
                // columns tx*4 .. +3 and 64 + tx*4 .. +3: 16 lanes read 256
                // contiguous bytes per half, without bank conflicts
                const float4 w0 = *reinterpret_cast<const float4 *>(&ws[b][kk][tx * 4]);
                const float4 w1 = *reinterpret_cast<const float4 *>(&ws[b][kk][GN / 2 + tx * 4]);
                const float av[4] = {a.x, a.y, a.z, a.w};
                const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], wv[j]));
            }
        }
        if (kt + 1 < nk) sstore(b ^ 1);   // buffer b ^ 1 was last read before the previous barrier
        __syncthreads();
    }
    fold();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = r0 + ty * 4 + i;
        if (r >= rows) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int n = n0 + (j < 4 ? tx * 4 + j : GN / 2 + tx * 4 + (j - 4));
            if (n < N) y[(size_t)r * N + n] = out[i][j];
        }
    }
}

}  // namespace kllm

using namespace kllm;

extern "C" int kllm_tt_gemm(const float *x, int rows, const float *codebook, int n_codes,
                            const uint16_t *idx, int K, int N, float *y, void *stream) {
    if (rows < 0 || K < 0 || N < 0 || n_codes <= 0 || !codebook || !idx || !x || !y) {
        set_error("kllm_tt_gemm: invalid arguments");
        return -1;
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (rows == 0 || N == 0) return 0;
    if (K == 0) return launch_fill(s, y, (long long)rows * N, 0.f) ? 0 : -1;
    const long long gy = (rows + GM - 1) / GM;
    if (gy > 65535) {
        set_error("kllm_tt_gemm: %d rows (at most %d)", rows, 65535 * GM);
        return -1;
    }
    dim3 grid((N + GN - 1) / GN, (unsigned)gy);
    k_tt_gemm<<<grid, GT, 0, s>>>(x, rows, codebook, idx, K, N, tt_chunks(K), y);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError()) ? 0 : -1;
}
