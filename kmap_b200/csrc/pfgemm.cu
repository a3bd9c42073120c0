// pfgemm.cu -- the prefill TT-GEMM on the tensor cores (tcgen05, TMEM, TMA).
//
// Y[R][N] = X[R][K] . W[K][N] for many prompt positions R against one
// MATMUL_TT weight (_tape_runner.c:776-813 with m > 1, the per-row loop of
// :804-811), when every codebook entry of the matrix is a bf16 number (the
// compiler's codebook holds the distinct values of a bf16 checkpoint, so
// this is the usual case).  Then each weight is exact in bf16, and the fp32
// activation row splits exactly-enough into bf16 terms:
//     x = hi + mid + lo,  hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (each difference is exact in fp32; hi + mid + lo carries 24 significand
// bits, all of x for normal values).  Every product term * w is exact in
// the tensor core's fp32 accumulation, so Y = sum over terms of Xt . W
// differs from the reference's serial fp32 sums only in summation order and
// the accumulator's internal rounding: a tolerance result, not bit-exact.
// The exact FP32 TT-GEMM (ttgemm.cu) stays for matrices whose codebooks are
// not bf16.
//
// Layout:  Xs[TERMS][R][K] bf16 (row-major: K-major for the MMA's A),
//          Wt[N][K] bf16 (the weight transposed: K-major B), built once
//          per plan from the index matrix and codebook (k_pf_wt);
//          Y[R][N] fp32.
// Kernel (k_pf_gemm_tc): one CTA per 128 x BN tile of Y, 192 threads:
//   warp 0 lane 0   TMA producer: per 64-wide K block, the TERMS A boxes
//                   (128 x 64) and the B box (BN x 64), 128-byte swizzle,
//                   into a ring of STAGES stages (mbarrier complete_tx);
//   warp 1          allocates BN TMEM columns; lane 0 issues
//                   tcgen05.mma.cta_group::1.kind::f16 (bf16 in, fp32
//                   accumulate in TMEM), 4 K-steps x TERMS per stage, and
//                   tcgen05.commit frees the stage / signals the epilogue;
//   warps 2..5      epilogue: tcgen05.ld of their 32 TMEM lanes (rows),
//                   fp32 rows to Y.
// TMA boxes start at K coordinates that are multiples of 64 (128 bytes)
// and cover only this GPU's memory; no multicast.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <string.h>

#include <algorithm>
#include <cmath>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "pfgemm.cuh"
#include "sm100.cuh"

namespace kllm {

// ------------------------------------------------------------ helpers ----

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
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
    return encode;
}

// bf16 tensor map of `rank` dims (innermost first), box {64, box_rows, 1},
// 128-byte swizzle (64 bf16 = one 128-byte swizzle row).
static bool bf16_tmap(CUtensorMap *map, const void *base, int rank, const cuuint64_t *dims,
                      const cuuint64_t *strides_bytes, uint32_t box_rows) {
    auto encode = tmap_encoder();
    if (!encode) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    cuuint32_t box[3] = {64, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base),
                        dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for a bf16 operand", (int)r);
        return false;
    }
    return true;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// UMMA shared-memory descriptor of a K-major operand tile in the canonical
// 128-byte-swizzle layout TMA writes: rows of 128 bytes (64 bf16), groups of
// 8 rows 1024 bytes apart (stride byte offset), base 1024-byte aligned.
// Bits: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused
// for swizzled K-major: 1), stride byte offset >> 4 [32,46), version 1
// [46,48), layout type [61,64) = 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3fff);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits [4,6) = 1), A
// and B bf16 ([7,10) = 1, [10,13) = 1), both K-major (bits 15, 16 = 0),
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
        ::"r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 TMEM columns of this warp's 32 lanes: lane i of the warp gets row
// (32 * (warp % 4) + i), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------- kernel ----

template <int TERMS, int BN, int STAGES>
struct PFGeom {
    static constexpr int BM = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK * 2;          // one term's box
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = TERMS * A_BYTES + B_BYTES;
    static constexpr int THREADS = 192;
    // stages (1024-byte aligned), then the mbarriers and the TMEM address
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int TERMS, int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
k_pf_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
             int R, int K, int N, float *__restrict__ y, int *status) {
    using G = PFGeom<TERMS, BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * G::STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *done = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * G::BM, n0 = blockIdx.x * BN;
    const int nk = K / G::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1) {   // TMEM accumulator: BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(BN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {   // ------------------------------------ producer
            prefetch_tmap(&amap);
            prefetch_tmap(&bmap);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % STAGES;
                if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, status))
                    break;
                uint8_t *st = smem + s * G::STAGE_BYTES;
                mbar_expect_tx(&full[s], G::STAGE_BYTES);
#pragma unroll
                for (int t = 0; t < TERMS; t++)
                    tma_load_3d(st + t * G::A_BYTES, &amap, kb * G::BK, m0, t, &full[s]);
                tma_load_2d(st + TERMS * G::A_BYTES, &bmap, kb * G::BK, n0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // ------------------------------------ MMA issue
            constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
            bool ok = true;
            for (int kb = 0; kb < nk && ok; kb++) {
                const int s = kb % STAGES;
                if (!mbar_wait(&full[s], (kb / STAGES) & 1, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * G::STAGE_BYTES);
                const uint32_t sb = sa + TERMS * G::A_BYTES;
#pragma unroll
                for (int kk = 0; kk < G::BK / 16; kk++)   // 16 bf16 = 32 bytes per MMA step
#pragma unroll
                    for (int t = 0; t < TERMS; t++)
                        umma_bf16(tmem, umma_desc_sw128(sa + t * G::A_BYTES + 32 * kk),
                                  umma_desc_sw128(sb + 32 * kk), idesc,
                                  (kb | kk | t) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);   // the stage is free once these MMAs read it
            }
            umma_commit(done);
        }
    } else {   // ---------------------------------------------- epilogue
        const int q = warp & 3;                  // TMEM lane quarter of this warp
        const int row = m0 + 32 * q + lane;
        const bool ok = mbar_wait(done, 0, status);
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
            if (!ok || row >= R) continue;
            float4 *dst = reinterpret_cast<float4 *>(y + (size_t)row * N + n0 + c0);
#pragma unroll
            for (int i = 0; i < 8; i++)
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN)
                     : "memory");
    }
}

// ------------------------------------------------- skinny (few rows) ----
//
// Decode of many sequences at once (one row per sequence, R <= 128): the
// operands swap roles so the weight fills the MMA's 128-row side.  A CTA
// owns 128 columns of Y (the rows of Wt, A) against all R rows of x (B, the
// MMA's N = RN, R rounded up; rows past R read zeros) over one range of K
// blocks (split K: gridDim.y ranges, their partial tiles summed in range
// order by k_bd_ksum).  TMEM holds the 128 x RN fp32 tile: lane = column of
// Y, TMEM column = row of x.  Stages of 16 KB of weight + TERMS x RN x 128
// bytes of x; two CTAs per SM keep 2 x STAGES weight boxes in flight.

template <int TERMS, int RN>
struct BDGeom {
    static constexpr int BM = 128, BK = 64;
    static constexpr int A_BYTES = BM * BK * 2;      // weight box (128 columns of Y)
    static constexpr int B_BYTES = RN * BK * 2;      // one term's box of x
    static constexpr int STAGE_BYTES = A_BYTES + TERMS * B_BYTES;
    static constexpr int THREADS = 192;
    // as many stages as fit two CTAs in an SM's 228 KB (at least 2)
    static constexpr int FIT = (113 * 1024 - 1280) / STAGE_BYTES;
    static constexpr int STAGES = FIT < 2 ? 2 : FIT > 8 ? 8 : FIT;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

template <int TERMS, int RN>
__global__ void __launch_bounds__(192, 2)
k_bd_gemm_tc(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
             int R, int K, int N, int kb_per, float *__restrict__ out, int *status) {
    using G = BDGeom<TERMS, RN>;
    constexpr int STAGES = G::STAGES;
    static_assert(RN % 32 == 0 && RN <= 128, "x rows per tile: 32, 64 or 128");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * G::STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *done = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * G::BM;
    const int nk = K / G::BK;
    const int kb0 = blockIdx.y * kb_per, kb1 = min(nk, kb0 + kb_per), nkb = kb1 - kb0;
    out += (size_t)blockIdx.y * R * N;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        mbar_fence_init();
    }
    if (warp == 1) {   // TMEM accumulator: RN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(RN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {   // ------------------------------------ producer
            prefetch_tmap(&wmap);
            prefetch_tmap(&xmap);
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, status)) break;
                uint8_t *st = smem + s * G::STAGE_BYTES;
                const int kx = (kb0 + i) * G::BK;
                mbar_expect_tx(&full[s], G::STAGE_BYTES);
                tma_load_2d(st, &wmap, kx, n0, &full[s]);
#pragma unroll
                for (int t = 0; t < TERMS; t++)
                    tma_load_3d(st + G::A_BYTES + t * G::B_BYTES, &xmap, kx, 0, t, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // ------------------------------------ MMA issue
            constexpr uint32_t idesc = umma_idesc_bf16(128, RN);
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (!mbar_wait(&full[s], (i / STAGES) & 1, status)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * G::STAGE_BYTES);
                const uint32_t sb = sa + G::A_BYTES;
#pragma unroll
                for (int kk = 0; kk < G::BK / 16; kk++)
#pragma unroll
                    for (int t = 0; t < TERMS; t++)
                        umma_bf16(tmem, umma_desc_sw128(sa + 32 * kk),
                                  umma_desc_sw128(sb + t * G::B_BYTES + 32 * kk), idesc,
                                  (i | kk | t) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(done);
        }
    } else {   // ---------------------------------------------- epilogue
        const int q = warp & 3;                  // TMEM lane quarter: columns 32q .. 32q + 31
        const int n = n0 + 32 * q + lane;
        const bool ok = mbar_wait(done, 0, status) && nkb > 0;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < RN; c0 += 32) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
            if (!ok) continue;
#pragma unroll
            for (int i = 0; i < 32; i++)   // lanes write 32 consecutive columns of row c0 + i
                if (c0 + i < R) out[(size_t)(c0 + i) * N + n] = v[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(RN)
                     : "memory");
    }
}

// y[i] = part[0][i] + part[1][i] + ... (the K ranges in order)
__global__ void k_bd_ksum(const float *__restrict__ part, int ks, long long n,
                          float *__restrict__ y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float a = part[i];
        for (int z = 1; z < ks; z++) a = __fadd_rn(a, part[(size_t)z * n + i]);
        y[i] = a;
    }
}

// x -> TERMS bf16 planes: hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (round to nearest even; each difference exact in fp32).
template <int TERMS>
__global__ void k_pf_split(const float *__restrict__ x, long long n, __nv_bfloat16 *__restrict__ xs) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float r = x[i];
#pragma unroll
        for (int t = 0; t < TERMS; t++) {
            const __nv_bfloat16 b = __float2bfloat16_rn(r);
            xs[t * n + i] = b;
            r = __fsub_rn(r, __bfloat162float(b));
        }
    }
}

// Wt[n][k] = bf16(codebook[idx[k][n]]): the weight, transposed, exact (the
// caller checked that every codebook entry is a bf16 number).  32 x 32
// tiles through shared memory.
__global__ void k_pf_wt(const uint16_t *__restrict__ idx, const float *__restrict__ cb, int K,
                        int N, __nv_bfloat16 *__restrict__ wt) {
    __shared__ float tile[32][33];
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int k = k0 + i, n = n0 + threadIdx.x;
        tile[i][threadIdx.x] = (k < K && n < N) ? cb[idx[(size_t)k * N + n]] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int n = n0 + i, k = k0 + threadIdx.x;
        if (n < N && k < K) wt[(size_t)n * K + k] = __float2bfloat16_rn(tile[threadIdx.x][i]);
    }
}

// ------------------------------------------------------------ host side --

template <int TERMS, int BN, int STAGES>
static bool launch_pf(cudaStream_t s, const CUtensorMap &am, const CUtensorMap &bm, int R, int K,
                      int N, float *y, int *status) {
    using G = PFGeom<TERMS, BN, STAGES>;
    auto kern = k_pf_gemm_tc<TERMS, BN, STAGES>;
    static std::atomic<bool> attr[64] = {};
    int dev = 0;
    if (!KLLM_CUDA(cudaGetDevice(&dev))) return false;
    if (!attr[dev & 63].load()) {
        if (!KLLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            G::SMEM)))
            return false;
        attr[dev & 63].store(true);
    }
    dim3 grid(N / BN, (R + G::BM - 1) / G::BM);
    kern<<<grid, G::THREADS, G::SMEM, s>>>(am, bm, R, K, N, y, status);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool pf_gemm_applies(int K, int N) { return K > 0 && N > 0 && K % 64 == 0 && N % 128 == 0; }

bool pf_build_wt(cudaStream_t s, const uint16_t *idx, const float *cb, int K, int N,
                 void *wt_bf16) {
    dim3 grid((N + 31) / 32, (K + 31) / 32), block(32, 8);
    k_pf_wt<<<grid, block, 0, s>>>(idx, cb, K, N, reinterpret_cast<__nv_bfloat16 *>(wt_bf16));
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool pf_split(cudaStream_t s, const float *x, long long n, int terms, void *xs_bf16) {
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 16);
    auto *o = reinterpret_cast<__nv_bfloat16 *>(xs_bf16);
    if (terms == 2)
        k_pf_split<2><<<blocks, 256, 0, s>>>(x, n, o);
    else if (terms == 3)
        k_pf_split<3><<<blocks, 256, 0, s>>>(x, n, o);
    else {
        set_error("pf_split: %d terms", terms);
        return false;
    }
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool pf_gemm_tc(cudaStream_t s, const void *xs_bf16, int terms, int R, int K, const void *wt_bf16,
                int N, float *y, int *status) {
    if (!pf_gemm_applies(K, N) || R <= 0 || (terms != 2 && terms != 3) ||
        (reinterpret_cast<uintptr_t>(xs_bf16) & 15) || (reinterpret_cast<uintptr_t>(wt_bf16) & 15)) {
        set_error("pf_gemm_tc: unsupported shape or alignment (R %d, K %d, N %d)", R, K, N);
        return false;
    }
    CUtensorMap am, bm;
    const cuuint64_t adims[3] = {(cuuint64_t)K, (cuuint64_t)R, (cuuint64_t)terms};
    const cuuint64_t astr[2] = {(cuuint64_t)K * 2, (cuuint64_t)R * K * 2};
    const cuuint64_t bdims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t bstr[1] = {(cuuint64_t)K * 2};
    const bool wide = N % 256 == 0;
    if (!bf16_tmap(&am, xs_bf16, 3, adims, astr, 128) ||
        !bf16_tmap(&bm, wt_bf16, 2, bdims, bstr, wide ? 256 : 128))
        return false;
    if (terms == 3)
        return wide ? launch_pf<3, 256, 2>(s, am, bm, R, K, N, y, status)
                    : launch_pf<3, 128, 3>(s, am, bm, R, K, N, y, status);
    return wide ? launch_pf<2, 256, 3>(s, am, bm, R, K, N, y, status)
                : launch_pf<2, 128, 4>(s, am, bm, R, K, N, y, status);
}

// K ranges of the skinny kernel for a 128-column-tile count: the smallest
// split whose CTAs fill the 148 SMs (two CTAs each) to at least 85 %, every
// range at least 4 K blocks.
int bd_gemm_splits(int K, int N) {
    const int nk = K / 64, tiles = N / 128;
    int best = 1;
    double best_eff = 0;
    for (int ks = 1; ks <= 16 && nk / ks >= 4; ks++) {
        const int per = (nk + ks - 1) / ks, real = (nk + per - 1) / per;
        const double waves = (double)tiles * real / (2 * 148);
        const double eff = waves / std::ceil(waves);
        if (eff > best_eff + 1e-9) {
            best = real;
            best_eff = eff;
        }
        if (eff >= 0.85) break;
    }
    return best;
}

template <int TERMS, int RN>
static bool bd_attr(int dev) {
    static std::atomic<bool> attr[64] = {};
    if (attr[dev & 63].load()) return true;
    if (!KLLM_CUDA(cudaFuncSetAttribute(k_bd_gemm_tc<TERMS, RN>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BDGeom<TERMS, RN>::SMEM)))
        return false;
    attr[dev & 63].store(true);
    return true;
}

bool bd_gemm_prepare() {
    int dev = 0;
    return KLLM_CUDA(cudaGetDevice(&dev)) && bd_attr<3, 32>(dev) && bd_attr<3, 64>(dev) &&
           bd_attr<3, 128>(dev) && bd_attr<2, 32>(dev) && bd_attr<2, 64>(dev) &&
           bd_attr<2, 128>(dev);
}

template <int TERMS, int RN>
static bool launch_bd(cudaStream_t s, const CUtensorMap &wm, const CUtensorMap &xm, int R, int K,
                      int N, int per, int nz, float *out, int *status) {
    using G = BDGeom<TERMS, RN>;
    auto kern = k_bd_gemm_tc<TERMS, RN>;
    int dev = 0;
    if (!KLLM_CUDA(cudaGetDevice(&dev)) || !bd_attr<TERMS, RN>(dev)) return false;
    dim3 grid(N / 128, nz);
    kern<<<grid, G::THREADS, G::SMEM, s>>>(wm, xm, R, K, N, per, out, status);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

bool bd_gemm_tc(cudaStream_t s, const void *xs_bf16, int terms, int R, int K, const void *wt_bf16,
                int N, float *y, float *part, int *status, int *nz_out) {
    if (!pf_gemm_applies(K, N) || R <= 0 || R > 128 || (terms != 2 && terms != 3) ||
        (reinterpret_cast<uintptr_t>(xs_bf16) & 15) || (reinterpret_cast<uintptr_t>(wt_bf16) & 15)) {
        set_error("bd_gemm_tc: unsupported shape or alignment (R %d, K %d, N %d)", R, K, N);
        return false;
    }
    const int ks = bd_gemm_splits(K, N);
    if (ks > 1 && !part) {
        set_error("bd_gemm_tc: %d K ranges need a partial-sum buffer", ks);
        return false;
    }
    CUtensorMap wm, xm;
    const int RN = R <= 32 ? 32 : R <= 64 ? 64 : 128;
    const cuuint64_t wdims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t wstr[1] = {(cuuint64_t)K * 2};
    const cuuint64_t xdims[3] = {(cuuint64_t)K, (cuuint64_t)R, (cuuint64_t)terms};
    const cuuint64_t xstr[2] = {(cuuint64_t)K * 2, (cuuint64_t)R * K * 2};
    if (!bf16_tmap(&wm, wt_bf16, 2, wdims, wstr, 128) ||
        !bf16_tmap(&xm, xs_bf16, 3, xdims, xstr, RN))
        return false;
    // ranges of `per` K blocks; nz <= ks of them (the partial buffer's count)
    const int nk = K / 64, per = (nk + ks - 1) / ks, nz = (nk + per - 1) / per;
    float *out = nz > 1 ? part : y;
    bool ok;
    if (terms == 3)
        ok = RN == 32 ? launch_bd<3, 32>(s, wm, xm, R, K, N, per, nz, out, status)
           : RN == 64 ? launch_bd<3, 64>(s, wm, xm, R, K, N, per, nz, out, status)
                      : launch_bd<3, 128>(s, wm, xm, R, K, N, per, nz, out, status);
    else
        ok = RN == 32 ? launch_bd<2, 32>(s, wm, xm, R, K, N, per, nz, out, status)
           : RN == 64 ? launch_bd<2, 64>(s, wm, xm, R, K, N, per, nz, out, status)
                      : launch_bd<2, 128>(s, wm, xm, R, K, N, per, nz, out, status);
    if (nz_out) *nz_out = nz;
    if (!ok || nz == 1 || nz_out) return ok;   // nz_out: the caller sums the partial tiles
    const long long n = (long long)R * N;
    k_bd_ksum<<<(int)std::min<long long>((n + 255) / 256, 148 * 8), 256, 0, s>>>(part, nz, n, y);
    g_launches++;
    return KLLM_CUDA(cudaGetLastError());
}

}  // namespace kllm

using namespace kllm;

extern "C" int kllm_tt_gemm_tc(const float *x, int rows, const float *codebook, int n_codes,
                               const uint16_t *idx, int K, int N, float *y, int terms,
                               void *stream) {
    if (rows < 0 || K < 0 || N < 0 || n_codes <= 0 || !codebook || !idx || !x || !y ||
        (terms != 2 && terms != 3)) {
        set_error("kllm_tt_gemm_tc: invalid arguments");
        return -1;
    }
    if (rows == 0 || N == 0) return 0;
    if (!pf_gemm_applies(K, N)) {
        set_error("kllm_tt_gemm_tc: K = %d must be a multiple of 64 and N = %d of 128", K, N);
        return -1;
    }
    cudaStream_t s = (cudaStream_t)stream;
    std::vector<float> cb(n_codes);
    if (!KLLM_CUDA(cudaMemcpyAsync(cb.data(), codebook, (size_t)n_codes * 4,
                                   cudaMemcpyDeviceToHost, s)) ||
        !KLLM_CUDA(cudaStreamSynchronize(s)))
        return -1;
    for (int i = 0; i < n_codes; i++) {
        uint32_t b;
        memcpy(&b, &cb[i], 4);
        if (b & 0xffffu) {
            set_error("kllm_tt_gemm_tc: codebook entry %d is not a bf16 number", i);
            return -1;
        }
    }
    // few rows: the weight on the MMA's 128-row side, K split over ranges
    const bool skinny = rows <= 64;
    const int ks = skinny ? bd_gemm_splits(K, N) : 1;
    void *xs = nullptr, *wt = nullptr;
    float *part = nullptr;
    int *st = nullptr;
    bool ok = KLLM_CUDA(cudaMallocAsync(&xs, (size_t)terms * rows * K * 2, s)) &&
              KLLM_CUDA(cudaMallocAsync(&wt, (size_t)N * K * 2, s)) &&
              KLLM_CUDA(cudaMallocAsync((void **)&st, 4, s)) &&
              (ks == 1 || KLLM_CUDA(cudaMallocAsync((void **)&part, (size_t)ks * rows * N * 4, s))) &&
              KLLM_CUDA(cudaMemsetAsync(st, 0, 4, s)) &&
              pf_build_wt(s, idx, codebook, K, N, wt) &&
              pf_split(s, x, (long long)rows * K, terms, xs) &&
              (skinny ? bd_gemm_tc(s, xs, terms, rows, K, wt, N, y, part, st)
                      : pf_gemm_tc(s, xs, terms, rows, K, wt, N, y, st));
    int status = 0;
    if (ok) ok = KLLM_CUDA(cudaMemcpyAsync(&status, st, 4, cudaMemcpyDeviceToHost, s)) &&
                 KLLM_CUDA(cudaStreamSynchronize(s));
    if (xs) cudaFreeAsync(xs, s);
    if (wt) cudaFreeAsync(wt, s);
    if (st) cudaFreeAsync(st, s);
    if (part) cudaFreeAsync(part, s);
    if (ok && status) {
        set_error("kllm_tt_gemm_tc: kernel reported status 0x%x (a wait timed out)", status);
        ok = false;
    }
    return ok ? 0 : -1;
}
