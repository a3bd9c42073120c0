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
// pass (or the consuming kernel) adds them in order.  __fmul_rn/__fadd_rn
// keep the compiler from contracting the product and the add into one FMA.
//
// Two kernels: the TMA-staged one (tt_kernels.cuh) for 16-byte aligned
// matrices with N % 8 == 0 and codebooks up to 16384 entries, and a simple
// one (indices straight from HBM, codebook through the read-only cache) for
// everything else.
#include <cudaTypedefs.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "tt_fused.cuh"

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

bool make_idx_tmap(CUtensorMap *map, const uint16_t *idx, int K, int N, int box_cols,
                   int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    });
    if (!encode) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)N * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (void *)idx, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for a %dx%d index matrix", (int)r, K, N);
        return false;
    }
    return true;
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

// ------------------------------------------------------ fused kernel ----

static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return v && *v ? atoi(v) : dflt;
}

// Geometry heuristic.  Every (column, chunk) chain is serial, so a matrix
// with few columns has few chains: it gets one column per lane and four
// consumer warps per 128 columns (many warps to hide the gather latency).
// Wide matrices are bound by shared-memory wavefronts instead: two or four
// columns per lane halve the index reads.  KLLM_TT_CPL / KLLM_TT_STAGES
// override for tuning.
TFConfig tf_config(int K, int N, int n_codes, int emode) {
    (void)K;
    (void)n_codes;
    TFConfig c;
    c.ncw = 4;
    c.nsub = emode == E_SWIGLU ? 2 : 1;
    long long cols = emode == E_SWIGLU ? N / 2 : N;
    c.cpl = cols >= 8192 ? 2 : 1;
    // Ring depth: a grid that fits in one wave keeps its whole chunk in
    // flight (one DRAM round trip); larger grids leave room for more CTAs
    // per SM instead.
    const int T = tt_chunks(K);
    const long long ctas = (long long)((cols + c.bw() - 1) / c.bw()) * T;
    const int nbox = ((K + T - 1) / T + 31) / 32;
    const int per_sm = (int)std::max<long long>(1, (ctas + 147) / 148);
    const size_t fixed = (size_t)n_codes * 4 + 4096;
    const size_t budget = per_sm <= 1 ? 200 * 1024 : (size_t)(220 * 1024) / per_sm;
    const size_t stage_bytes = (size_t)c.bn() * 32 * 2;
    int st = budget > fixed ? (int)((budget - fixed) / stage_bytes) : 2;
    c.stages = std::max(2, std::min(std::min(st, nbox), 12));
    int e = env_int("KLLM_TT_CPL", 0);
    if (e == 1 || e == 2) c.cpl = e;
    e = env_int("KLLM_TT_STAGES", 0);
    if (e >= 1 && e <= 16) c.stages = e;
    return c;
}

int tf_blocks(const TFConfig &c, int N, int F, int emode) {
    return emode == E_SWIGLU ? (F + c.bw() - 1) / c.bw() : (N + c.bn() - 1) / c.bn();
}

bool tf_tma_ok(const uint16_t *idx, const float *cb, int K, int N, int n_codes,
               const TFConfig &c) {
    return K > 0 && N >= 8 && (N % 8) == 0 && ((uintptr_t)idx % 16) == 0 &&
           ((uintptr_t)cb % 16) == 0 && n_codes <= 16384 && c.bw() % 8 == 0 && c.bw() <= 256;
}

template <int NCW, int CPL, int NSUB>
static bool launch_g(cudaStream_t s, const TFConfig &c, const CUtensorMap &map, TTArgs a,
                     bool pdl) {
    constexpr int BR = 32;
    using G = TFGeom<NCW, CPL, BR, NSUB>;
    int maxlen = (a.K + a.T - 1) / a.T;
    int nbox = (maxlen + BR - 1) / BR;
    a.stages = std::max(1, std::min(c.stages, nbox));
    size_t smem = tf_smem_bytes<NCW, CPL, BR, NSUB>(a.n_codes, maxlen, a.stages);
    auto kern = k_tt_fused<NCW, CPL, BR, NSUB>;
    // per device and instance; concurrent first calls may both set it
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    if (!KLLM_CUDA(cudaGetDevice(&dev))) return false;
    if (!attr_set[dev & 63].load(std::memory_order_acquire)) {
        if (!KLLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024)))
            return false;
        attr_set[dev & 63].store(true, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tf_blocks(c, a.N, a.F, a.emode), a.T);
    cfg.blockDim = dim3(G::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    g_launches++;
    return KLLM_CUDA(cudaLaunchKernelEx(&cfg, kern, map, a));
}

bool launch_tt_fused(cudaStream_t s, const TFConfig &c, const CUtensorMap &map, TTArgs a,
                     bool pdl) {
    if (c.ncw != 4) {
        set_error("unsupported TT-GEMV geometry");
        return false;
    }
    if (c.nsub == 1) {
        if (c.cpl == 1) return launch_g<4, 1, 1>(s, c, map, a, pdl);
        if (c.cpl == 2) return launch_g<4, 2, 1>(s, c, map, a, pdl);
        if (c.cpl == 4) return launch_g<4, 4, 1>(s, c, map, a, pdl);
    } else if (c.nsub == 2) {
        if (c.cpl == 1) return launch_g<4, 1, 2>(s, c, map, a, pdl);
        if (c.cpl == 2) return launch_g<4, 2, 2>(s, c, map, a, pdl);
    }
    set_error("unsupported TT-GEMV geometry");
    return false;
}

bool tt_gemv_partials(cudaStream_t s, const float *x, int rows, const float *cb, int n_codes,
                      const uint16_t *idx, int K, int N, float *part) {
    int T = tt_chunks(K);
    dim3 grid((N + 127) / 128, T);
    k_tt_gemv_simple<<<grid, 128, 0, s>>>(x, rows, cb, idx, K, N, T, part);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool tt_fused_applies(const uint16_t *idx, const float *cb, int K, int N, int n_codes) {
    return tf_tma_ok(idx, cb, K, N, n_codes, tf_config(K, N, n_codes, E_Y));
}

// Single-row TT-GEMV with the reduction fused (the fast path of the tape's
// MATMUL_TT and of kllm_tt_gemv): part holds T*N floats, counters
// tf_blocks() zeros (left zero again).
bool tt_gemv_fused_y(cudaStream_t s, const float *x, const float *cb, int n_codes,
                     const uint16_t *idx, int K, int N, float *part, int *counters, float *y,
                     int *status) {
    TFConfig c = tf_config(K, N, n_codes, E_Y);
    if (!tf_tma_ok(idx, cb, K, N, n_codes, c)) return false;
    CUtensorMap map;
    if (!make_idx_tmap(&map, idx, K, N, c.bw(), 32)) return false;
    TTArgs a = {};
    a.cb = cb;
    a.n_codes = n_codes;
    a.K = K;
    a.N = N;
    a.T = tt_chunks(K);
    a.xmode = X_PLAIN;
    a.x = x;
    a.emode = E_Y;
    a.part = part;
    a.counters = counters;
    a.y = y;
    a.status = status;
    return launch_tt_fused(s, c, map, a, false);
}

// y = ((p0 + p1) + p2) + ...  (memcpy of chunk 0, then in-order adds)
__global__ void k_tt_reduce(const float *__restrict__ part, int T, long long rn,
                            float *__restrict__ y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rn;
         i += (long long)gridDim.x * blockDim.x) {
        y[i] = sum_parts(part + i, (size_t)rn, T);
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
// Per-device scratch of kllm_tt_gemv: chunk partials and the column-block
// arrival counters of the fused reduction (kept zero between calls).
struct GemvScratch {
    float *part = nullptr;
    size_t cap = 0;
    int *counters = nullptr;
    size_t ccap = 0;
    int *status = nullptr;          // device alias of status_host (the kernel's status word)
    int *status_host = nullptr;     // mapped pinned word: the kernel flags a wait that
                                    // gave up here directly (no copy after each launch)
};
static std::mutex g_scratch_mu;
static GemvScratch g_scratch[64];

static bool scratch_for(int dev, size_t floats, size_t ncount, float **part, int **counters,
                        int **status, int **status_host) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    GemvScratch &s = g_scratch[dev & 63];
    if (!s.status) {
        if (!KLLM_CUDA(cudaHostAlloc((void **)&s.status_host, sizeof(int),
                                     cudaHostAllocMapped | cudaHostAllocPortable)))
            return false;
        *s.status_host = 0;
        if (!KLLM_CUDA(cudaHostGetDevicePointer((void **)&s.status, s.status_host, 0))) {
            cudaFreeHost(s.status_host);
            s.status_host = nullptr;
            return false;
        }
    }
    *status = s.status;
    *status_host = s.status_host;
    if (s.cap < floats) {
        if (s.part) cudaFree(s.part);
        s.part = nullptr;
        s.cap = 0;
        if (!KLLM_CUDA(cudaMalloc((void **)&s.part, floats * sizeof(float)))) return false;
        s.cap = floats;
    }
    if (s.ccap < ncount) {
        if (s.counters) cudaFree(s.counters);
        s.counters = nullptr;
        s.ccap = 0;
        size_t n = std::max<size_t>(ncount, 1024);
        if (!KLLM_CUDA(cudaMalloc((void **)&s.counters, n * sizeof(int))) ||
            !KLLM_CUDA(cudaMemset(s.counters, 0, n * sizeof(int))))
            return false;
        s.ccap = n;
    }
    *part = s.part;
    *counters = s.counters;
    return true;
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
    float *part = nullptr;
    int *counters = nullptr, *status = nullptr, *status_host = nullptr;
    if (!scratch_for(dev, (size_t)T * rows * N, (size_t)N / 64 + 1, &part, &counters, &status,
                     &status_host))
        return -1;
    // A wait of an earlier call's kernel that gave up (its y columns are
    // NaN) is reported here, once: the kernel writes the mapped pinned
    // status word itself.
    if (const int st = *reinterpret_cast<volatile int *>(status_host)) {
        *reinterpret_cast<volatile int *>(status_host) = 0;
        set_error("kllm_tt_gemv: an earlier call's kernel reported status 0x%x (a wait timed "
                  "out; its y holds NaN)", st);
        return -1;
    }
    if (rows == 1 && tf_tma_ok(idx, codebook, K, N, n_codes, tf_config(K, N, n_codes, E_Y)))
        return tt_gemv_fused_y(s, x, codebook, n_codes, idx, K, N, part, counters, y, status)
                   ? 0
                   : -1;
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
    if (!idx || !codebook || !x || !y) {
        set_error("kllm_tt_gemv_host: NULL argument");
        return -1;
    }
    if (n_codes < 65536) {
        for (size_t i = 0; i < ni; i++)
            if (idx[i] >= n_codes) {
                set_error("kllm_tt_gemv_host: index %u at %zu outside the codebook of %d",
                          (unsigned)idx[i], i, n_codes);
                return -1;
            }
    }
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
