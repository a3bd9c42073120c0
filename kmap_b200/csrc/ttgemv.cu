// ttgemv.cu -- truth-table GEMV: y[r][n] = sum_k fl(x[r][k] * cb[idx[k][n]]).
//
// Accumulation order is the reference's (tt_gemv_mt / tt_gemv_thread,
// _tape_runner.c:495-663), so results are bit-identical for every input:
//   * K is cut into T = min(8, ceil(K/128)) chunks; chunk t has K/T rows,
//     plus one for t < K%T (_tape_runner.c:599-629);
//   * inside a chunk each column is summed row by row from 0.0f, each term
//     being the float product x[k]*cb[i] rounded before the add
//     (_tape_runner.c:517-545: the LUT holds rounded products);
//   * the chunk sums are added in chunk order (_tape_runner.c:646-662).
// Every (column, chunk) chain is an independent serial sum, so the device
// parallelises over columns x chunks and writes T partial rows; a second
// pass adds them in order.  __fmul_rn/__fadd_rn keep the compiler from
// contracting the product and the add into one FMA.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace kllm {

int tt_chunks(int K) {
    // _tape_runner.c:599-603 with TT_NUM_THREADS 8, TT_THREAD_THRESHOLD 128
    int t = 8;
    if (K < 128 * t) t = (K + 127) / 128;
    if (t < 1) t = 1;
    if (t > 8) t = 8;
    return t;
}

void tt_chunk_range(int K, int T, int t, int *k0, int *len) {
    int base = K / T, rem = K % T;
    *k0 = t * base + std::min(t, rem);
    *len = base + (t < rem ? 1 : 0);
}

// ------------------------------------------------------ simple kernel ----
// One thread per (column, chunk); indices read straight from HBM (columns
// are contiguous across the warp), codebook through the read-only cache.
__global__ void k_tt_gemv_simple(const float *__restrict__ x, int rows,
                                 const float *__restrict__ cb,
                                 const uint16_t *__restrict__ idx, int K, int N, int T,
                                 float *__restrict__ part) {
    int n = blockIdx.x * blockDim.x + threadIdx.x;
    int t = blockIdx.y;
    if (n >= N) return;
    int base = K / T, rem = K % T;
    int k0 = t * base + min(t, rem);
    int len = base + (t < rem ? 1 : 0);
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (size_t)r * K;
        float acc = 0.0f;
        const uint16_t *col = idx + (size_t)k0 * N + n;
#pragma unroll 8
        for (int k = 0; k < len; k++) {
            float p = __fmul_rn(__ldg(xr + k0 + k), __ldg(cb + __ldg(col + (size_t)k * N)));
            acc = __fadd_rn(acc, p);
        }
        part[((size_t)t * rows + r) * N + n] = acc;
    }
}

bool tt_gemv_partials(cudaStream_t s, const float *x, int rows, const float *cb, int n_codes,
                      const uint16_t *idx, int K, int N, float *part) {
    (void)n_codes;
    int T = tt_chunks(K);
    dim3 grid((N + 127) / 128, T);
    k_tt_gemv_simple<<<grid, 128, 0, s>>>(x, rows, cb, idx, K, N, T, part);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

// y = ((p0 + p1) + p2) + ...  (memcpy of chunk 0, then in-order adds)
__global__ void k_tt_reduce(const float *__restrict__ part, int T, long long rn,
                            float *__restrict__ y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rn;
         i += (long long)gridDim.x * blockDim.x) {
        float acc = part[i];
        for (int t = 1; t < T; t++) acc = __fadd_rn(acc, part[(size_t)t * rn + i]);
        y[i] = acc;
    }
}

bool tt_reduce_partials(cudaStream_t s, const float *part, int T, int rows, int N, float *y) {
    long long rn = (long long)rows * N;
    if (rn <= 0) return true;
    long long b = std::min<long long>((rn + 255) / 256, 148 * 16);
    k_tt_reduce<<<(int)b, 256, 0, s>>>(part, T, rn, y);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------- raw C ABI ----
// Per-device scratch for the chunk partials of kllm_tt_gemv.
struct GemvScratch {
    float *part = nullptr;
    size_t cap = 0;
};
static std::mutex g_scratch_mu;
static GemvScratch g_scratch[64];

static float *scratch_for(int dev, size_t floats) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    GemvScratch &s = g_scratch[dev & 63];
    if (s.cap < floats) {
        if (s.part) cudaFree(s.part);
        s.part = nullptr;
        s.cap = 0;
        if (!KLLM_CUDA(cudaMalloc((void **)&s.part, floats * sizeof(float)))) return nullptr;
        s.cap = floats;
    }
    return s.part;
}

}  // namespace kllm

using namespace kllm;

extern "C" int kllm_tt_gemv(const float *x, int rows, const float *codebook, int n_codes,
                            const uint16_t *idx, int K, int N, float *y, void *stream) {
    if (rows < 0 || K < 0 || N < 0 || n_codes <= 0 || !codebook || !idx || !x || !y) {
        set_error("kllm_tt_gemv: invalid arguments");
        return -1;
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (rows == 0 || N == 0) return 0;
    if (K == 0) {
        return launch_fill(s, y, (long long)rows * N, 0.f) ? 0 : -1;
    }
    int dev = 0;
    if (!KLLM_CUDA(cudaGetDevice(&dev))) return -1;
    int T = tt_chunks(K);
    float *part = scratch_for(dev, (size_t)T * rows * N);
    if (!part) return -1;
    if (!tt_gemv_partials(s, x, rows, codebook, n_codes, idx, K, N, part)) return -1;
    if (!tt_reduce_partials(s, part, T, rows, N, y)) return -1;
    return 0;
}

extern "C" int kllm_tt_gemv_host(const float *x, int rows, const float *codebook, int n_codes,
                                 const uint16_t *idx, int K, int N, float *y) {
    if (rows < 0 || K < 0 || N < 0 || n_codes <= 0) {
        set_error("kllm_tt_gemv_host: invalid arguments");
        return -1;
    }
    if (rows == 0 || N == 0) return 0;
    size_t nx = (size_t)rows * K, ni = (size_t)K * N, ny = (size_t)rows * N;
    size_t ncb = ((size_t)n_codes + 3) & ~(size_t)3;
    float *dx = nullptr, *dcb = nullptr, *dy = nullptr;
    uint16_t *di = nullptr;
    int rc = -1;
    cudaStream_t s = nullptr;
    if (!KLLM_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking))) return -1;
    if (KLLM_CUDA(cudaMallocAsync((void **)&dx, std::max<size_t>(nx, 1) * 4, s)) &&
        KLLM_CUDA(cudaMallocAsync((void **)&dcb, ncb * 4, s)) &&
        KLLM_CUDA(cudaMallocAsync((void **)&di, std::max<size_t>(ni, 8) * 2, s)) &&
        KLLM_CUDA(cudaMallocAsync((void **)&dy, ny * 4, s)) &&
        KLLM_CUDA(cudaMemsetAsync(dcb, 0, ncb * 4, s)) &&
        (nx == 0 || KLLM_CUDA(cudaMemcpyAsync(dx, x, nx * 4, cudaMemcpyHostToDevice, s))) &&
        KLLM_CUDA(cudaMemcpyAsync(dcb, codebook, (size_t)n_codes * 4, cudaMemcpyHostToDevice, s)) &&
        (ni == 0 || KLLM_CUDA(cudaMemcpyAsync(di, idx, ni * 2, cudaMemcpyHostToDevice, s))) &&
        kllm_tt_gemv(dx, rows, dcb, n_codes, di, K, N, dy, s) == 0 &&
        KLLM_CUDA(cudaMemcpyAsync(y, dy, ny * 4, cudaMemcpyDeviceToHost, s)) &&
        KLLM_CUDA(cudaStreamSynchronize(s)))
        rc = 0;
    if (dx) cudaFreeAsync(dx, s);
    if (dcb) cudaFreeAsync(dcb, s);
    if (di) cudaFreeAsync(di, s);
    if (dy) cudaFreeAsync(dy, s);
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    return rc;
}
