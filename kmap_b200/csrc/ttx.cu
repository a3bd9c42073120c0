// ttx.cu -- builds the decode step kernel's layout of a TT weight matrix
// (column-group slot stream + bank-spread replicated codebook); see ttx.cuh.
#include "ttx.cuh"

#include <cuda_fp16.h>
#include <string.h>

namespace kllm {

unsigned ttx_value_modes(const float *cb, int n_codes) {
    bool bf = true, hf = true;
    for (int i = 0; i < n_codes && (bf || hf); i++) {
        uint32_t u;
        memcpy(&u, cb + i, 4);
        if (u & 0xffffu) bf = false;
        if (hf) {
            const float back = __half2float(__float2half_rn(cb[i]));
            uint32_t v;
            memcpy(&v, &back, 4);
            if (v != u) hf = false;
        }
    }
    return (bf ? 1u << TTX_VBF16 : 0u) | (hf ? 1u << TTX_VF16 : 0u);
}

bool ttx_describe(int K, int N, int n_codes, int colmode, int vmode, int hd, int rope_heads,
                  int max_table_bytes, int max_r, int split_w, TTXDesc *d) {
    if (K <= 0 || N <= 0 || n_codes <= 0) return false;
    if (vmode != TTX_VSLOT && vmode != TTX_VBF16 && vmode != TTX_VF16) return false;
    if (split_w != 1 && split_w != 2 && split_w != 4 && split_w != 8) return false;
    TTXDesc t = {};
    t.K = K;
    t.N = N;
    t.n_codes = n_codes;
    t.W = split_w;
    t.T = split_w == 1 ? tt_chunks(K) : 8 * split_w;
    if ((split_w == 1 && t.T > 8) || t.T > K) return false;
    t.base = K / t.T;
    t.rem = K % t.T;
    const int len_max = t.base + (t.rem > 0 ? 1 : 0);
    t.ns = (len_max + 7) / 8;
    t.colmode = colmode;
    if (colmode == TTX_GATE_UP) {
        if (N % 2) return false;
        t.F = N / 2;
        t.ngroups = (t.F + 3) / 4;
    } else if (colmode == TTX_ROPE) {
        if (hd <= 0 || hd % 8 || rope_heads * hd > N) return false;
        t.hd = hd;
        t.rope_heads = rope_heads;
        const int rest = N - rope_heads * hd;
        t.ngroups = rope_heads * (hd / 8) + (rest + 7) / 8;
    } else {
        t.ngroups = (N + TTX_GCOLS - 1) / TTX_GCOLS;
    }
    t.gstride = 1;
    t.goff = 0;
    t.vmode = vmode;
    t.npad = (n_codes + 31) & ~31;
    if (vmode != TTX_VSLOT) {   // values in the stream: no table
        t.R = 0;
        *d = t;
        return true;
    }
    // slots are byte offsets into the table: R * npad * 4 must fit 16 bits
    int r = 4;
    while (r > max_r || (r > 1 && ((size_t)r * t.npad * 4 > (size_t)max_table_bytes ||
                                   (size_t)r * t.npad * 4 > 65536)))
        r >>= 1;
    if ((size_t)t.npad * 4 > (size_t)max_table_bytes || (size_t)t.npad * 4 > 65536) return false;
    t.R = r;
    *d = t;
    return true;
}

void ttx_shard(TTXDesc *d, int rank, int world) {
    d->ngroups = rank < d->ngroups ? (d->ngroups - rank + world - 1) / world : 0;
    d->gstride = world;
    d->goff = rank;
}

// One thread per warp-wide gather of the decode kernel: group g, sub-task w,
// step s, column half k, row e -- lane l = 8 * pair + c reads column
// 2 * pair + k, row 8s + e of chunk 8w + c.  Value streams store the code's
// bf16 / fp16 pattern.  Slot streams choose a codebook copy for every
// distinct code so that the bank holding the most distinct words holds as
// few as possible.  Exact: for cap = 1, 2, ... every code is inserted with a
// breadth-first augmenting path over banks (a bank may hold cap words).
__global__ void k_ttx_build(const uint16_t *__restrict__ idx, const float *__restrict__ cb,
                            const TTXDesc d, uint8_t *__restrict__ out, long long ngather) {
    const long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (gid >= ngather) return;
    const int e = (int)(gid & 7), k = (int)((gid >> 3) & 1);
    const long long gs = gid >> 4;
    const int s = (int)(gs % d.ns);
    const long long gw = gs / d.ns;          // i * W + w, i a stored group
    const int g = (int)(gw / d.W) * d.gstride + d.goff, w = (int)(gw % d.W);

    uint16_t *step = reinterpret_cast<uint16_t *>(out + ((size_t)gw * d.ns + s) * TTX_STEP);
    if (d.vmode != TTX_VSLOT) {
        for (int l = 0; l < 32; l++) {
            const int t = 8 * w + (l & 7), pair = l >> 3;
            const int row = 8 * s + e;
            const int n = ttx_col(d, g, 2 * pair + k);
            uint16_t v = 0;   // rows past the chunk and padding columns are never used
            if (row < d.chunk_len(t) && n >= 0) {
                int c = idx[((size_t)d.chunk_start(t) + row) * d.N + n];
                if (c >= d.n_codes) c = 0;   // indices are validated at upload
                v = d.vmode == TTX_VBF16 ? (uint16_t)(__float_as_uint(cb[c]) >> 16)
                                         : __half_as_ushort(__float2half_rn(cb[c]));
            }
            step[k * 256 + l * 8 + e] = v;
        }
        return;
    }
    int code[32];   // distinct codes
    int lane_u[32];
    int nu = 0;
    for (int l = 0; l < 32; l++) {
        lane_u[l] = -1;
        const int t = 8 * w + (l & 7), pair = l >> 3;
        const int row = 8 * s + e;
        if (row >= d.chunk_len(t)) continue;
        const int n = ttx_col(d, g, 2 * pair + k);
        if (n < 0) continue;
        int c = idx[((size_t)d.chunk_start(t) + row) * d.N + n];
        if (c >= d.n_codes) c = 0;   // indices are validated at upload
        int u = 0;
        while (u < nu && code[u] != c) u++;
        if (u == nu) code[nu++] = c;
        lane_u[l] = u;
    }
    int copy[32], bank_of[32], load[32];
    int pball[32], pcopy[32], pbank[32], q[32];
    for (int u = 0; u < nu; u++) copy[u] = 0;
    for (int cap = 1; cap <= 32; cap++) {
        for (int i = 0; i < 32; i++) load[i] = 0;
        for (int u = 0; u < nu; u++) bank_of[u] = -1;
        bool ok = true;
        for (int u = 0; u < nu && ok; u++) {
            unsigned vis = 0;
            int qh = 0, qt = 0;
            for (int c = 0; c < d.R; c++) {
                const int bk = ttx_swz(code[u], c) & 31;
                if (vis >> bk & 1u) continue;
                vis |= 1u << bk;
                pball[bk] = u;
                pcopy[bk] = c;
                pbank[bk] = -1;
                q[qt++] = bk;
            }
            bool found = false;
            while (qh < qt && !found) {
                const int bk = q[qh++];
                if (load[bk] < cap) {
                    int cur = bk;
                    for (;;) {   // shift the path: every code on it moves one bank
                        const int ball = pball[cur], pb = pbank[cur];
                        copy[ball] = pcopy[cur];
                        bank_of[ball] = cur;
                        load[cur]++;
                        if (pb < 0) break;
                        load[pb]--;
                        cur = pb;
                    }
                    found = true;
                    break;
                }
                for (int v = 0; v < nu; v++) {
                    if (bank_of[v] != bk) continue;
                    for (int c = 0; c < d.R; c++) {
                        const int nb = ttx_swz(code[v], c) & 31;
                        if (vis >> nb & 1u) continue;
                        vis |= 1u << nb;
                        pball[nb] = v;
                        pcopy[nb] = c;
                        pbank[nb] = bk;
                        q[qt++] = nb;
                    }
                }
            }
            ok = found;
        }
        if (ok) break;
    }
    // lanes without a code read the first lane's word (no extra bank load)
    int fill = 0;
    for (int l = 0; l < 32; l++)
        if (lane_u[l] >= 0) {
            const int u = lane_u[l];
            fill = 4 * (copy[u] * d.npad + ttx_swz(code[u], copy[u]));
            break;
        }
    for (int l = 0; l < 32; l++) {
        const int u = lane_u[l];
        const int slot = u >= 0 ? 4 * (copy[u] * d.npad + ttx_swz(code[u], copy[u])) : fill;
        step[k * 256 + l * 8 + e] = (uint16_t)slot;
    }
}

__global__ void k_ttx_table(const float *__restrict__ cb, const TTXDesc d, float *__restrict__ tab) {
    const int total = d.R * d.npad;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int c = i / d.npad, e = i % d.npad;
        tab[c * d.npad + ttx_swz(e, c)] = e < d.n_codes ? cb[e] : 0.f;
    }
}

bool ttx_build(cudaStream_t s, const uint16_t *idx, const float *cb, const TTXDesc &d,
               uint8_t *stream, float *table) {
    const long long ngather = (long long)d.ngroups * d.W * d.ns * 16;
    if (ngather < 0) return false;
    if (ngather == 0) return true;   // a rank without groups of this matrix
    const int bs = 128;
    k_ttx_build<<<(unsigned)((ngather + bs - 1) / bs), bs, 0, s>>>(idx, cb, d, stream, ngather);
    if (!KLLM_CUDA(cudaGetLastError())) return false;
    if (!table || d.table_elems() == 0) return true;
    k_ttx_table<<<64, 256, 0, s>>>(cb, d, table);
    return KLLM_CUDA(cudaGetLastError());
}

}  // namespace kllm
