// ttx.cuh -- the decode step kernel's device layout of a TT weight matrix.
//
// A MATMUL_TT weight is a uint16 index matrix idx[K][N] into a float32
// codebook (_tape_runner.c:474-663).  The reference splits K into
// T = min(8, ceil(K/128)) chunks (the first K % T one row longer), sums each
// chunk serially per column and adds the chunk sums in order.  The decode
// step kernel gives one warp a group of 8 columns and all T chunks:
// lane = 8 * pair + chunk, each lane two adjacent columns of its chunk, so
// the chunk sums meet inside the warp and are added in order there.  The
// device copy of a matrix is laid out for that warp, still 2 bytes a weight:
//
//  * Stream.  Group g is one contiguous run of NS = ceil(len_max / 8) steps
//    of 1 KB; step s holds rows 8s..8s+7 of every lane's chunk: first the
//    32 lanes' 16 bytes for their first column, then for their second, so
//    each lane reads a step with two conflict-free 128-bit loads.
//  * Bank-spread codebook.  The codebook is stored R times (R <= 4) in a
//    table of R x npad floats; copy r keeps entry e at row e >> 5 of the
//    copy, bank (e & 31) ^ h(e >> 5, r).  The stream holds table slots (the
//    byte offset of the chosen copy's word, so R * npad * 4 <= 64 KB), not
//    codes: for every warp-wide gather (one row, one column of each lane)
//    the upload picks the copy of each code so that the most-loaded bank
//    holds as few distinct words as possible (an exact bipartite
//    assignment with bank capacities).  The values read are the codebook
//    entries themselves, so products and sums are unchanged bit for bit.
//  * Value streams.  When every codebook entry is a bf16 (or fp16) number --
//    the usual case: the compiler's codebook is the sorted distinct values
//    of a bf16 (fp16) checkpoint -- the stream holds each weight's 16-bit
//    pattern instead of a table slot, still 2 bytes a weight.  Converting
//    the pattern to float gives the codebook entry exactly, so products and
//    sums are unchanged bit for bit, and no table or gather is needed.
//  * Split groups (decode's fast order).  With W > 1 a group's K is cut into
//    8W equal chunks instead of the reference's T: sub-task w of the group
//    (its own NS steps, lane chunk 8w + lane % 8) goes to its own warp, and
//    the W partial sums are added in w order.  Same bytes, W times the
//    warps; the sums are no longer the reference's bit for bit.
//  * Column shards.  A rank of a multi-GPU decode stores only its groups:
//    group i of its stream is group i * world + rank of the matrix.
//  * Column groups.  Plain matrices take 8 consecutive columns.  gate_up
//    (N = 2F) takes gate columns 4g..4g+3 and the matching up columns, so a
//    group holds both inputs of its SwiGLU.  QKV with RoPE takes, inside one
//    q or k head, dims d..d+3 and d+hd/2..d+hd/2+3 (the rotate-half pairs),
//    and 8 consecutive v dims.
#pragma once

#include "common.cuh"

namespace kllm {

constexpr int TTX_STEP = 1024;   // bytes per step of a column group
constexpr int TTX_GCOLS = 8;     // columns per group

enum TTXCols : int { TTX_IDENT = 0, TTX_GATE_UP = 1, TTX_ROPE = 2 };
// What a stream holds per weight: a table slot, or the value's bf16 / fp16
// pattern (exact codebooks only).
enum TTXVals : int { TTX_VSLOT = 0, TTX_VBF16 = 1, TTX_VF16 = 2 };

struct TTXDesc {
    int K, N, n_codes;
    int T, base, rem;     // the chunking of K (the reference's when W == 1)
    int W;                // sub-tasks (warps) per group
    int ns;               // steps per group (8 rows of every chunk per step)
    int ngroups;          // groups stored here (a column shard: every gstride-th)
    int gstride, goff;    // stored group i is group i * gstride + goff of the matrix
    int R, npad;          // codebook copies, entries per copy (multiple of 32); R = 0
                          // for value streams (no table)
    int colmode;
    int vmode;            // TTXVals
    int F;                // TTX_GATE_UP: N == 2F
    int hd, rope_heads;   // TTX_ROPE: head dim, q + k heads (rotated)
    __host__ __device__ size_t stream_bytes() const {
        return (size_t)ngroups * W * ns * TTX_STEP;
    }
    __host__ __device__ size_t table_elems() const { return (size_t)R * npad; }
    __host__ __device__ int chunk_start(int t) const { return t * base + (t < rem ? t : rem); }
    __host__ __device__ int chunk_len(int t) const {
        return t < T ? base + (t < rem ? 1 : 0) : 0;
    }
};

// Bank-spreading permutation of copy r inside each row of 32 entries.
__host__ __device__ inline int ttx_swz(int e, int r) {
    const int h = r == 0 ? 0 : (((e >> 5) * (2 * r + 1) * 7 + 13 * r) & 31);
    return (e & ~31) | ((e & 31) ^ h);
}

// Logical column of slot c (0..7) of group g, or -1 for padding.
__host__ __device__ inline int ttx_col(const TTXDesc &d, int g, int c) {
    if (d.colmode == TTX_GATE_UP) {
        const int n = 4 * g + (c & 3);
        if (n >= d.F) return -1;
        return c < 4 ? n : d.F + n;
    }
    if (d.colmode == TTX_ROPE) {
        const int per_head = d.hd / 8;
        const int rg = d.rope_heads * per_head;
        if (g < rg) {
            const int head = g / per_head, d0 = (g % per_head) * 4;
            const int dim = c < 4 ? d0 + c : d0 + d.hd / 2 + (c - 4);
            return head * d.hd + dim;
        }
        const int n = rg * 8 + (g - rg) * 8 + c;
        return n < d.N ? n : -1;
    }
    const int n = g * TTX_GCOLS + c;
    return n < d.N ? n : -1;
}

// Fill in the layout of a K x N matrix with n_codes codes.  For slot
// streams R is the largest of 4, 2, 1 (at most max_r) whose table fits
// max_table_bytes and whose slots fit 16 bits.  TTX_ROPE needs hd (a
// multiple of 8) and the number of rotated heads.  split_w = 1 keeps the
// reference's chunks; 2, 4 or 8 splits each group into that many sub-tasks
// (fast order).
bool ttx_describe(int K, int N, int n_codes, int colmode, int vmode, int hd, int rope_heads,
                  int max_table_bytes, int max_r, int split_w, TTXDesc *d);
// The value streams a codebook allows: bit TTX_VBF16 set when every entry
// is a bf16 number, bit TTX_VF16 when every entry is an fp16 number (bit
// patterns compared, so -0.0 and NaN payloads must survive the round trip).
unsigned ttx_value_modes(const float *cb, int n_codes);
// Restrict d to the column groups of one rank (group g with g % world == rank).
void ttx_shard(TTXDesc *d, int rank, int world);
// Build the stream and (slot streams, table != nullptr) the replicated
// table on the device.
bool ttx_build(cudaStream_t s, const uint16_t *idx, const float *cb, const TTXDesc &d,
               uint8_t *stream, float *table);

}  // namespace kllm
