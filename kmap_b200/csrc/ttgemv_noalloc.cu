// ttgemv_noalloc.cu -- kllm_tt_gemv_noalloc: the single-row TT-GEMV of
// kllm_tt_gemv, for callers that must not allocate device memory.
//
// Some hosts cannot tolerate a library calling cudaMalloc: code that runs
// while a CUDA graph is being captured (cudaMalloc is not allowed there),
// plugins inside a framework that owns the whole device memory budget
// through its own pool, and real-time or embedded hosts that fix their
// memory footprint up front.  kllm_tt_gemv grows a per-device scratch
// buffer with cudaMalloc on demand; this entry point instead keeps its
// scratch -- the chunk partial rows and the column-block arrival counters of
// the exact reduction -- in a fixed array that is part of the library's
// device image, so it never allocates.
//
// The array is sized for N <= kNoAllocMaxCols columns (8 partial rows of
// 65536 floats = 2 MiB, plus 4 KiB of counters).  Every GPU that loads the
// library holds it until the process exits.  All calls on a device share it:
// calls whose kernels overlap on the GPU (different streams, no ordering
// between them) race on it and give wrong results.  The counters are
// cleared on the caller's stream at every call; the partial rows are fully
// rewritten before they are read.
//
// Host code may not pass the array's name to a kernel: on the host that
// name is only a stand-in for the symbol, not a device address.  The first
// call on a device therefore looks the address up with cudaGetSymbolAddress
// (with that device current) and keeps it for the life of the process; make
// that first call before any stream capture starts, and do not call
// cudaDeviceReset between calls (the kept address would then be stale).
//
// A device wait of the kernel that gives up (it should never: the waits only
// end copies that never land) sets a status word kept beside the counters
// and leaves NaN in the affected columns of y, so the failure shows in the
// output without a host synchronisation.
#include <mutex>

#include "common.cuh"
#include "tt_fused.cuh"

namespace kllm {
namespace {

constexpr int kNoAllocMaxCols = 65536;
constexpr int kNoAllocChunks = 8;                    // tt_chunks() never exceeds 8
constexpr int kNoAllocCounters = kNoAllocMaxCols / 64 + 64;

static __device__ __align__(256) float g_noalloc_part[kNoAllocChunks * kNoAllocMaxCols];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];
static __device__ int g_noalloc_status;

struct NoAllocScratch {
    float *part = nullptr;
    int *counters = nullptr;
    int *status = nullptr;
    bool ready = false;
};

std::mutex g_mu;
NoAllocScratch g_dev[64];

// Device addresses of the scratch array on `dev` (the current device).
bool scratch_addresses(int dev, NoAllocScratch *out) {
    if (dev < 0 || dev >= 64) {
        set_error("kllm_tt_gemv_noalloc: device ordinal %d beyond 63", dev);
        return false;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    NoAllocScratch &s = g_dev[dev];
    if (!s.ready) {
        void *p = nullptr, *q = nullptr, *r = nullptr;
        if (!KLLM_CUDA(cudaGetSymbolAddress(&p, g_noalloc_part))) return false;
        if (!KLLM_CUDA(cudaGetSymbolAddress(&q, g_noalloc_counters))) return false;
        if (!KLLM_CUDA(cudaGetSymbolAddress(&r, g_noalloc_status))) return false;
        s.part = static_cast<float *>(p);
        s.counters = static_cast<int *>(q);
        s.status = static_cast<int *>(r);
        s.ready = true;
    }
    *out = s;
    return true;
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" int kllm_tt_gemv_noalloc(const float *x, const float *codebook, int n_codes,
                                    const uint16_t *idx, int K, int N, float *y, void *stream) {
    if (K < 0 || N < 0 || n_codes <= 0 || !codebook || !idx || !x || !y) {
        set_error("kllm_tt_gemv_noalloc: invalid arguments");
        return -1;
    }
    if (N > kNoAllocMaxCols) {
        set_error("kllm_tt_gemv_noalloc: N = %d exceeds its fixed scratch limit of %d columns "
                  "(use kllm_tt_gemv)", N, kNoAllocMaxCols);
        return -1;
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (N == 0) return 0;
    if (K == 0) return launch_fill(s, y, N, 0.f) ? 0 : -1;
    int dev = 0;
    if (!KLLM_CUDA(cudaGetDevice(&dev))) return -1;
    NoAllocScratch sc;
    if (!scratch_addresses(dev, &sc)) return -1;
    // counters must start at zero; an earlier call that was cut short could
    // have left some set
    if (!KLLM_CUDA(cudaMemsetAsync(sc.counters, 0, sizeof(int) * kNoAllocCounters, s)) ||
        !KLLM_CUDA(cudaMemsetAsync(sc.status, 0, sizeof(int), s)))
        return -1;
    if (tt_fused_applies(idx, codebook, K, N, n_codes))
        return tt_gemv_fused_y(s, x, codebook, n_codes, idx, K, N, sc.part, sc.counters, y,
                               sc.status)
                   ? 0
                   : -1;
    const int T = tt_chunks(K);
    if (!tt_gemv_partials(s, x, 1, codebook, n_codes, idx, K, N, sc.part)) return -1;
    return tt_reduce_partials(s, sc.part, T, 1, N, y) ? 0 : -1;
}
