/*
 * kllm_cuda.h -- extensions of the kllm C ABI that the B200 executor adds
 * next to the drop-in surface of tape_runner.h.
 *
 * None of these exists in the reference runtime (csrc/tape_runner.h); each
 * comment says which reference behaviour it complements.  All functions are
 * plain C: pointers and sizes only.
 */
#ifndef KLLM_CUDA_H
#define KLLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#include "tape_runner.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- errors --
 * The reference has no error reporting (void functions, exit(1) in the
 * loaders, processor_infer* always return 0: _tape_runner.c:1587,1762).
 * Here every failure is recorded per thread and the call returns. */

/* Message of the first error recorded on this thread since the last clear,
 * or NULL when there is none. */
const char *kllm_last_error(void);
void kllm_clear_error(void);

/* Version string of this library. */
const char *kllm_version(void);

/* Number of CUDA devices visible to this process (0 without a GPU). */
int kllm_device_count(void);

/* Device used by contexts created afterwards on this thread (default: the
 * CUDA current device).  Returns 0, or -1 for an invalid ordinal. */
int kllm_set_device(int device);

/* tape_run with a status: 0 on success, non-zero on error
 * (complements _tape_runner.c:665, which cannot fail). */
int kllm_tape_run(TapeCtx *ctx);

/* Kernels launched by this process so far (all contexts). */
long long kllm_launch_count(void);

/* --------------------------------------------------- inference options --
 * processor_infer / processor_infer_bytes keep the reference signatures;
 * these settings ride on the context. */
enum {
    KLLM_MODE_AUTO = 0,     /* fused decode plan when the tape matches the
                               compiler's LLaMA template, else per-op */
    KLLM_MODE_GENERIC = 1,  /* per-op device execution of every instruction
                               (same loop structure as the reference) */
    KLLM_MODE_FUSED = 2     /* fused plan or an error */
};

/* Summation order of the fused decode step's TT-GEMVs. */
enum {
    KLLM_ORDER_EXACT = 0,   /* the reference's chunked order: every MATMUL_TT
                               result is bit-identical to _tape_runner.c's */
    KLLM_ORDER_FAST = 1     /* K split finer across warps (decode only): same
                               tokens and logits within the decode tolerance,
                               more parallelism in the narrow projections; one
                               GPU only (a column-sharded context builds the
                               exact order) */
};

typedef struct {
    int mode;                /* KLLM_MODE_* */
    float *logits_out;       /* optional host buffer: the logits row after
                                every tape step, [logits_rows][vocab] */
    int logits_rows;         /* capacity of logits_out in rows */
    int use_graphs;          /* replay each step as a CUDA graph (fused) */
    int order;               /* KLLM_ORDER_*, fused decode step */
    int prefill;             /* 1: the prompt's positions but the last run as one
                                batched pass (TT-GEMMs, kllm_tt_gemm) instead of
                                one tape step each (persistent plan, one GPU, no
                                logits_out); 0: the default, step by step */
    int reserved[6];
} kllm_infer_opts;

typedef struct {
    int fused;               /* 1 when the fused plan ran */
    int steps;               /* tape steps run (prompt + generated) */
    double prefill_ms;       /* device time of the prompt steps */
    double decode_ms;        /* device time of the generation steps */
    double total_ms;         /* wall time inside the call */
    long long launches;      /* kernels launched inside the call */
    int step_kernel;         /* fused: 1 = one persistent kernel per tape step,
                                0 = the per-kernel plan */
    int stream_values;       /* persistent step: what the weight streams hold,
                                0 = codebook table slots, 1 = bf16 values,
                                2 = fp16 values (exact codebooks only) */
    int reserved[6];
} kllm_infer_stats;

void kllm_default_infer_opts(kllm_infer_opts *o);
int kllm_set_infer_opts(TapeCtx *ctx, const kllm_infer_opts *o);
int kllm_get_infer_stats(TapeCtx *ctx, kllm_infer_stats *s);

/* Whether processor_infer takes the fused decode plan for this tape: 1
 * when the tape is the kllm compiler's LLaMA decode template
 * (kllm_compile.c:1143-1385) for these dimensions and slot maps, 0 when not
 * (the first mismatch is written to why), -1 on bad arguments.  Host only;
 * needs no GPU. */
int kllm_plan_match(TapeCtx *ctx, int vocab_size, int hidden_dim, int head_dim,
                    int token_embed_slot, int rope_cos_slot, int rope_sin_slot,
                    const int *kv_in_slots, const int *kv_out_slots, int logits_slot,
                    int n_layers, int num_kv_heads, char *why, int why_len);

/* Build the fused decode plan now (weights to the device layout, buffers)
 * for contexts of up to max_pos positions, instead of at the first
 * processor_infer call.  Same model arguments as processor_infer.  0 on
 * success, -1 (kllm_last_error) when the tape does not match the template. */
int kllm_plan_prepare(TapeCtx *ctx, const float *embed_table, int vocab_size, int hidden_dim,
                      const float *rope_cos, const float *rope_sin, int head_dim,
                      int token_embed_slot, int rope_cos_slot, int rope_sin_slot,
                      const int *kv_in_slots, const int *kv_out_slots, int logits_slot,
                      int n_layers, int num_kv_heads, int max_pos);

/* ----------------------------------------------- column-sharded decode -----
 * One process per GPU.  Rank r of `world` stores and multiplies every
 * world-th column group of each TT matrix (N is sharded, K and the
 * codebooks are not), and stores its results into every rank's copy of the
 * activations over NVLink peer memory inside the decode kernel; each output
 * column's arithmetic is unchanged, so results equal the 1-GPU run.
 * Sequence: kllm_shard_set (before the plan exists), kllm_plan_prepare,
 * kllm_shard_export on every rank, exchange the blocks (any transport,
 * e.g. torch.distributed), kllm_shard_connect with all blocks in rank
 * order, then processor_infer on every rank with the same arguments.  The
 * reference has no multi-GPU path. */
int kllm_shard_set(TapeCtx *ctx, int rank, int world);
/* This rank's block (CUDA IPC handles); *len gets its size. */
int kllm_shard_export(TapeCtx *ctx, void *out, size_t cap, size_t *len);
/* world blocks of per_rank bytes each, in rank order. */
int kllm_shard_connect(TapeCtx *ctx, const void *all, size_t per_rank);

/* ----------------------------------------------------------- TT-GEMV -----
 * y[r][n] = sum_k fl(x[r][k] * codebook[idx[k][n]]) in the accumulation
 * order of the reference TT-GEMV (_tape_runner.c:495-663): K is cut into
 * T = min(8, ceil(K/128)) chunks (the first K%T chunks one row longer),
 * each chunk is summed row by row from 0.0f, and the chunk sums are added
 * in chunk order.  Results are bit-identical to the reference for every
 * input.  idx is uint16 row-major [K][N]; codebook has n_codes floats.
 *
 * Device-pointer form: all pointers are device memory of the calling
 * thread's device; stream is a cudaStream_t (NULL = default stream).  Every
 * index must be < n_codes (not checked here: the caller owns the data).
 * Uses a per-device scratch buffer for the chunk partials, grown on demand
 * with cudaMalloc.  Returns 0 or non-zero on error (see kllm_last_error). */
int kllm_tt_gemv(const float *x, int rows, const float *codebook, int n_codes,
                 const uint16_t *idx, int K, int N, float *y, void *stream);

/* Host-buffer form of the same product: checks every index against
 * n_codes, copies x, codebook and idx to the device, runs, copies y back
 * (synchronous). */
int kllm_tt_gemv_host(const float *x, int rows, const float *codebook,
                      int n_codes, const uint16_t *idx, int K, int N, float *y);

/* TT-GEMM: the same product for many rows at once (prefill: every prompt
 * position against one MATMUL_TT weight), each row bit-identical to
 * kllm_tt_gemv of that row (the reference order of _tape_runner.c:474-663 per
 * row).  x is [rows][K] and y [rows][N], device memory; the decoded weight
 * tile is reused across 64 rows, so this form is bound by the FP32 pipes
 * rather than by the index stream.  Allocates nothing.  Every index must be
 * < n_codes; rows <= 4194240.  Returns 0 or non-zero (kllm_last_error). */
int kllm_tt_gemm(const float *x, int rows, const float *codebook, int n_codes,
                 const uint16_t *idx, int K, int N, float *y, void *stream);

/* TT-GEMM on the tensor cores (the same product as kllm_tt_gemm, replacing
 * the per-row MATMUL_TT loop of _tape_runner.c:804-811 for prefill), for
 * matrices whose codebook entries are all bf16 numbers: x is split into
 * `terms` (2 or 3) bf16 terms (hi, mid, lo; 3 terms carry all 24 significand
 * bits of a normal fp32), each weight is exact in bf16, and the products
 * accumulate in fp32 in tensor memory.  Results agree with kllm_tt_gemm to
 * fp32 rounding in a different summation order, not bit for bit.  K must be
 * a multiple of 64 and N of 128; the codebook is checked (a device-to-host
 * copy) and a codebook with any non-bf16 entry is an error.  Allocates and
 * frees its bf16 operands on the stream.  Returns 0 or non-zero
 * (kllm_last_error). */
int kllm_tt_gemm_tc(const float *x, int rows, const float *codebook, int n_codes,
                    const uint16_t *idx, int K, int N, float *y, int terms, void *stream);

/* Allocation-free form of kllm_tt_gemv for one row (x is [K], y is [N]).
 * No counterpart in the reference runtime.  For callers that may not
 * allocate device memory -- code running during CUDA graph capture, plugins
 * whose host framework owns the device memory pool, fixed-footprint
 * real-time hosts -- it keeps its scratch in a fixed array inside the
 * library's device image instead of growing one with cudaMalloc: N is at
 * most 65536 (2 MiB of partial rows per device, held until exit); larger N
 * is rejected with an error.  The first call on a device looks up the
 * array's device address and should come before any stream capture.  Calls
 * whose kernels overlap on the GPU share the array and race.  Same result,
 * bit for bit, as kllm_tt_gemv; every index must be < n_codes. */
int kllm_tt_gemv_noalloc(const float *x, const float *codebook, int n_codes,
                         const uint16_t *idx, int K, int N, float *y, void *stream);

/* ------------------------------------------------------------- chips -----
 * Chip directory loader: the same files, read the same way, as the
 * reference CLI's static chip_load (csrc/kllm.c:152-388): processor.json,
 * tables/<name>.bin, bpe/<files>, circuit/tape.bin + slots.bin + const_<slot>*.bin.
 * The loader validates what the reference trusts (file sizes against
 * slots.bin, the 276-byte record size, slot ids in processor.json) and
 * returns NULL with kllm_last_error() set instead of exiting. */
typedef struct kllm_chip kllm_chip;

kllm_chip *kllm_chip_open(const char *chip_dir);
void kllm_chip_close(kllm_chip *chip);
TapeCtx *kllm_chip_ctx(kllm_chip *chip);

/* info[0..17] = vocab_size, hidden_dim, num_layers, num_kv_heads, head_dim,
 * max_seq_len, eos_token_id, logits_slot, token_embed_slot, rope_cos_slot,
 * rope_sin_slot, n_slots, n_instrs, bos_token_id, hash table_size,
 * max_piece_len, num_merges, num_special. */
int kllm_chip_info(kllm_chip *chip, int *info);

/* processor_infer with the chip's tables and slot maps (what kllm.c passes,
 * csrc/kllm.c:566-584, minus the BPE). */
int kllm_chip_infer(kllm_chip *chip, const int *prompt, int prompt_len, int max_new,
                    int eos_token_id, int *out_tokens, int *out_len);

/* Batched greedy decode of nseq independent sequences on one GPU -- the
 * reference has no counterpart: its processor_infer (_tape_runner.c:
 * 1602-1763) runs one sequence; this runs that loop for all of them at
 * once, each with its own KV cache and position.  prompts holds the
 * sequences' token IDs back to back (prompt_lens[i] each); out receives
 * nseq x max_new tokens (row i: sequence i's greedy tokens, computed for all
 * max_new steps), out_lens[i] the number before sequence i's first `eos`
 * (the reference would stop there; pass -1 for none).  Prompts go through
 * the batched prompt pass, then each step is one GEMM per projection over
 * the nseq rows: on the tensor cores when every codebook entry is a bf16
 * number and nseq <= 128 (a tolerance result), else -- or with
 * KLLM_BATCH_TC=0 in the environment -- the exact TT-GEMM, each row
 * bit-identical to the TT-GEMV.  The context must not be column-sharded.
 * Returns 0 or non-zero (kllm_last_error); kllm_get_infer_stats gives the
 * prompt and decode device times. */
int kllm_infer_batch(TapeCtx *ctx, const int *prompts, const int *prompt_lens, int nseq,
                     int max_new, int eos, int *out, int *out_lens);
/* The same on a loaded chip (prepares its fused plan first). */
int kllm_chip_infer_batch(kllm_chip *chip, const int *prompts, const int *prompt_lens, int nseq,
                          int max_new, int eos, int *out, int *out_lens);

/* kllm_plan_prepare with the chip's tables, for its max_seq_len. */
int kllm_chip_plan_prepare(kllm_chip *chip);

/* processor_infer_bytes with the chip's ROMs, as `kllm infer` calls it
 * (csrc/kllm.c:566-584); max_seq_tokens <= 0 means the chip's max_seq_len. */
int kllm_chip_infer_bytes(kllm_chip *chip, const uint8_t *input, int input_len, int max_new,
                          int max_seq_tokens, token_callback_fn cb, void *user_data,
                          int *total_generated);

/* bpe_encode / bpe_decode with the chip's ROMs. */
int kllm_chip_encode(kllm_chip *chip, const uint8_t *bytes, int len, int max_tokens,
                     int32_t *out_ids);
int kllm_chip_decode(kllm_chip *chip, const int32_t *ids, int n, int max_bytes,
                     int skip_leading_space, uint8_t *out_bytes);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_CUDA_H */
