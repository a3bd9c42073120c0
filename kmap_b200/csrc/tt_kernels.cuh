// tt_kernels.cuh -- TMA-staged truth-table GEMV for sm_100a.
//
// One CTA owns (chunk t, BN columns).  A producer warp streams the chunk's
// index rows [k0, k0+len) x [n0, n0+BN) from HBM into a ring of shared
// memory stages with 2-D TMA tile loads (no multicast); NCW consumer warps
// hold the codebook (fp32) and the chunk's slice of x in shared memory and
// walk the rows in order, each lane owning CPL adjacent columns:
//     acc[c] = fl(acc[c] + fl(x[k] * cb[idx[k][n0 + c]]))
// which is the reference's per-chunk serial sum (_tape_runner.c:517-545),
// so the T partial rows it writes, added in chunk order, give the
// reference's result bit for bit.
//
// The weight stream and the codebook do not depend on earlier kernels, so
// they start before griddepcontrol.wait: under programmatic dependent
// launch the tiles are already in flight while the previous kernel runs.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace kllm {

// ---------------------------------------------------------- x sources ---
// x[k] of the GEMV input, evaluated for the CTA's chunk after pdl_wait().
struct XPlain {
    const float *x;
    __device__ __forceinline__ float load(int k) const { return x[k]; }
};

// x[k] = silu(gate[k]) * up[k] with gate/up the ordered chunk sums of the
// gate_up projection's partials [T][2F] (the MLP tail of the compiler's
// template: SLICE, SLICE, SILU in double, MUL; kllm_compile.c:1364-1384).
struct XSwiGLU {
    const float *part;
    int T, F;
    long long stride;   // floats between partial rows (= 2F)
    __device__ __forceinline__ float load(int k) const {
        float g = part[k], u = part[F + k];
        for (int t = 1; t < T; t++) {
            g = __fadd_rn(g, part[t * stride + k]);
            u = __fadd_rn(u, part[t * stride + F + k]);
        }
        double d = (double)g;
        float a = (float)(d / (1.0 + exp(-d)));
        return __fmul_rn(a, u);
    }
};

template <int NCW, int CPL, int BR>
struct TTGeom {
    static constexpr int BN = NCW * 32 * CPL;
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int BOX_BYTES = BN * BR * 2;
};

// Shared memory bytes for one CTA.
template <int NCW, int CPL, int BR>
__host__ __device__ inline size_t tt_smem_bytes(int n_codes, int len, int ns) {
    using G = TTGeom<NCW, CPL, BR>;
    size_t ncb4 = ((size_t)n_codes + 3) / 4;
    size_t len4 = ((size_t)len + 3) / 4;
    return (size_t)ns * G::BOX_BYTES + 16 * (size_t)ns + ncb4 * 16 + len4 * 16;
}

template <int NCW, int CPL, int BR, class XS>
__global__ void __launch_bounds__(TTGeom<NCW, CPL, BR>::THREADS)
k_ttgemv_tma(const __grid_constant__ CUtensorMap tmap, const float *__restrict__ cb,
             int n_codes, XS xsrc, int K, int N, int T, int nstages, float *__restrict__ part,
             int *status) {
    using G = TTGeom<NCW, CPL, BR>;
    constexpr int BN = G::BN;
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_launch_dependents();

    const int t = blockIdx.y;
    const int n0 = blockIdx.x * BN;
    const int base = K / T, rem = K % T;
    const int k0 = t * base + min(t, rem);
    const int len = base + (t < rem ? 1 : 0);
    const int nbox = (len + BR - 1) / BR;
    const int NS = min(nstages, nbox);
    const int ncb4 = (n_codes + 3) / 4;

    uint16_t *stage = reinterpret_cast<uint16_t *>(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)NS * G::BOX_BYTES);
    uint64_t *empty = full + NS;
    float *cbs = reinterpret_cast<float *>(empty + NS);
    float *xs = cbs + 4 * ncb4;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == NCW) {
        // producer: stream the chunk's index tiles through the stage ring
        if (lane == 0) {
            prefetch_tmap(&tmap);
            for (int b = 0; b < nbox; b++) {
                const int s = b % NS;
                if (b >= NS && !mbar_wait(&empty[s], ((b / NS) - 1) & 1, status)) break;
                mbar_expect_tx(&full[s], G::BOX_BYTES);
                tma_load_2d(stage + (size_t)s * BR * BN, &tmap, n0, k0 + b * BR, &full[s]);
            }
        }
        return;
    }

    // consumers: codebook first (static data), then the dependent input
    const float4 *cb4 = reinterpret_cast<const float4 *>(cb);
    for (int i = threadIdx.x; i < ncb4; i += NCW * 32)
        reinterpret_cast<float4 *>(cbs)[i] = __ldg(cb4 + i);
    pdl_wait();
    for (int r = threadIdx.x; r < len; r += NCW * 32) xs[r] = xsrc.load(k0 + r);
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");

    const int cofs = warp * 32 * CPL + lane * CPL;
    float acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) acc[c] = 0.0f;

    for (int b = 0; b < nbox; b++) {
        const int s = b % NS;
        if (!mbar_wait(&full[s], (b / NS) & 1, status)) return;
        const uint16_t *tile = stage + (size_t)s * BR * BN + cofs;
        const float *xb = xs + b * BR;
        const int rows = min(BR, len - b * BR);
        if (rows == BR) {
#pragma unroll 8
            for (int r = 0; r < BR; r++) {
                const float xv = xb[r];
                if (CPL == 2) {
                    const uint32_t w = *reinterpret_cast<const uint32_t *>(tile + r * BN);
                    const float c0 = cbs[w & 0xffffu], c1 = cbs[w >> 16];
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(xv, c0));
                    acc[CPL - 1] = __fadd_rn(acc[CPL - 1], __fmul_rn(xv, c1));
                } else {
                    acc[0] = __fadd_rn(acc[0], __fmul_rn(xv, cbs[tile[r * BN]]));
                }
            }
        } else {
            for (int r = 0; r < rows; r++) {
                const float xv = xb[r];
#pragma unroll
                for (int c = 0; c < CPL; c++)
                    acc[c] = __fadd_rn(acc[c], __fmul_rn(xv, cbs[tile[r * BN + c]]));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    float *out = part + (size_t)t * N + n0 + cofs;
#pragma unroll
    for (int c = 0; c < CPL; c++)
        if (n0 + cofs + c < N) out[c] = acc[c];
}

// Tensor map of a [K][N] uint16 index matrix with a (BR rows x BN cols) box.
bool make_idx_tmap(CUtensorMap *map, const uint16_t *idx, int K, int N, int box_cols,
                   int box_rows);

// Whether the TMA kernel applies to this matrix (alignment rules of TMA).
inline bool tt_tma_ok(const uint16_t *idx, int K, int N, int n_codes) {
    return K > 0 && N >= 8 && (N % 8) == 0 && ((uintptr_t)idx % 16) == 0 &&
           n_codes <= 16384;
}

}  // namespace kllm
