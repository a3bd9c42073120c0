// common.cuh -- internal declarations shared by the libkllm_cuda sources.
//
// A TapeCtx handed to callers is the first member of CtxImpl, so the public
// struct layout (include/tape_runner.h) is unchanged while each context also
// owns its device state: one CUDA stream, a device buffer per slot, the
// truth-table matrices in HBM, GEMV scratch, and the fused decode plan.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string>
#include <vector>

#include "tape_runner.h"
#include "kllm_cuda.h"

namespace kllm {

// ------------------------------------------------------------ opcodes ----
// Tape opcodes of the chip format (reference _tape_runner.c:29-54).
enum Op {
    OP_SILU = 0, OP_EXP = 1, OP_RSQRT = 2, OP_COS = 3, OP_SIN = 4,
    OP_ADD = 5, OP_SUB = 6, OP_MUL = 7, OP_DIV = 8, OP_MAX = 9,
    OP_NEG = 10, OP_SQUARE = 11, OP_MATMUL = 12, OP_MATMUL_TT = 13,
    OP_SUM = 14, OP_MAX_RED = 15, OP_MEAN = 16, OP_ARGMAX = 17,
    OP_RESHAPE = 18, OP_TRANSPOSE = 19, OP_CONCAT = 20, OP_REPEAT = 21,
    OP_SLICE = 22, OP_COPY = 23, OP_COUNT = 24
};

// ------------------------------------------------------------- errors ----
// Records the first failure of the calling thread; the public void
// functions report through this instead of aborting.
void set_error(const char *fmt, ...);
bool cuda_ok(cudaError_t e, const char *what, const char *file, int line);
#define KLLM_CUDA(call) ::kllm::cuda_ok((call), #call, __FILE__, __LINE__)

// -------------------------------------------------------------- shapes ---
struct Dims {
    int nd;
    int d[MAX_DIMS];
};

static inline long long dims_size(const int *shape, int nd) {
    long long s = 1;
    for (int i = 0; i < nd; i++) s *= shape[i];
    return s;
}

// ------------------------------------------------------ device slots -----
// Device mirror of one Slot.  The host Slot keeps the reference's shape and
// size bookkeeping; this holds the data in HBM.
struct DevSlot {
    float *d = nullptr;          // device data
    size_t cap = 0;              // capacity of d in floats
    size_t host_cap = 0;         // capacity of Slot.data when owned
    bool host_dirty = false;     // host copy newer (upload before use)
    bool dev_newer = false;      // device copy newer (download on read)
    bool zero_pending = false;   // tape_slot_alloc: device starts as zeros
    // truth-table matrix
    uint16_t *d_idx = nullptr;
    float *d_cb = nullptr;       // codebook padded to a multiple of 4 floats
    const void *tt_src_idx = nullptr;
    const void *tt_src_cb = nullptr;
    int tt_K = 0, tt_N = 0, tt_codes = 0;
    bool tt_ready = false;
};

struct DecodePlan;   // decode.cu

struct CtxImpl {
    TapeCtx base;                // must stay first
    int device = 0;
    cudaStream_t stream = nullptr;
    std::vector<DevSlot> ds;
    // GEMV scratch: ordered partial sums [T][rows][N]
    float *d_part = nullptr;
    size_t part_cap = 0;
    int *d_counters = nullptr;   // fused TT-GEMV arrival counters (zero at rest)
    // fused decode path
    DecodePlan *plan = nullptr;
    kllm_infer_opts opts;
    kllm_infer_stats stats;
    long long launches = 0;      // kernels this context launched
    int shard_rank = 0, shard_world = 1;   // column shard of the fused decode
};

static inline CtxImpl *impl(TapeCtx *c) { return reinterpret_cast<CtxImpl *>(c); }

// runtime.cu
bool ensure_device(CtxImpl *c, int slot, size_t need);
bool sync_inputs(CtxImpl *c);
bool upload_tt(CtxImpl *c, int slot);
bool ensure_part(CtxImpl *c, size_t floats);
bool run_generic(CtxImpl *c);
bool select_device(CtxImpl *c);
void plan_destroy(CtxImpl *c);   // plan.cu

// ops.cu -- generic kernels (one launch per tape instruction)
bool launch_unary(cudaStream_t s, int op, const float *x, float *y, long long n);
bool launch_binop(cudaStream_t s, int op, const float *a, const Dims &da,
                  const float *b, const Dims &db, float *y, const Dims &dy);
bool launch_reduce(cudaStream_t s, int op, const float *x, float *y,
                   long long outer, int axis_n, long long inner);
bool launch_transpose(cudaStream_t s, const float *x, const Dims &din,
                      const int *axes, float *y);
bool launch_repeat(cudaStream_t s, const float *x, const Dims &din, int reps,
                   int axis, float *y);
bool launch_slice(cudaStream_t s, const float *x, const Dims &din,
                  const int *starts, const int *steps, const Dims &dout, float *y);
bool launch_concat(cudaStream_t s, const float *const *xs, const long long *chunk,
                   int n, long long outer, float *y);
bool launch_matmul(cudaStream_t s, const float *a, const float *b, float *y,
                   int batch, int m, int k, int n);
bool launch_fill(cudaStream_t s, float *y, long long n, float v);

// ttgemv.cu -- truth-table GEMV in the reference accumulation order
int tt_chunks(int K);
void tt_chunk_range(int K, int T, int t, int *k0, int *len);
bool tt_gemv_partials(cudaStream_t s, const float *x, int rows, const float *cb,
                      int n_codes, const uint16_t *idx, int K, int N, float *part);
bool tt_reduce_partials(cudaStream_t s, const float *part, int T, int rows, int N,
                        float *y);
// One-row TT-GEMV with the ordered reduction fused; false (no error) when
// the matrix does not meet the TMA rules.  A device wait that gives up sets
// ST_WAIT_TIMEOUT in *status (when not null) and leaves NaN in the columns
// it could not finish.
bool tt_gemv_fused_y(cudaStream_t s, const float *x, const float *cb, int n_codes,
                     const uint16_t *idx, int K, int N, float *part, int *counters, float *y,
                     int *status);
bool tt_fused_applies(const uint16_t *idx, const float *cb, int K, int N, int n_codes);

extern long long g_launches;   // kernels launched by this process

}  // namespace kllm
