/*
 * tape_runner.h -- drop-in C ABI of the kllm tape runtime, implemented on
 * NVIDIA B200 (sm_100a) by libkllm_cuda.so.
 *
 * Every declaration below replaces the declaration of the same name in the
 * reference runtime header csrc/tape_runner.h (line numbers cited per item);
 * names, argument meaning, struct layouts and ownership rules are unchanged,
 * so the reference CLI (csrc/kllm.c) links against this library as-is.
 *
 * Layout is ABI: the reference CLI's chip loader memcpy's tape.bin records
 * straight into ctx->tape (csrc/kllm.c:317), and tape.bin stores 276-byte
 * TapeInstr records (checked at csrc/kllm.c:312-316).
 *
 * Device behaviour (what changes behind the same signatures):
 *   - slot data lives in HBM; host pointers handed in through
 *     tape_slot_set_external / tape_slot_set_truth_table are copied to the
 *     device at the next tape_run (ownership stays with the caller, exactly
 *     as csrc/_tape_runner.c:335-375);
 *   - tape_slot_read stages a device->host copy of the slot and returns a
 *     host pointer owned by the context (valid until the next tape_run or
 *     tape_ctx_destroy);
 *   - processor_infer / processor_infer_bytes keep the KV cache, the
 *     embedding lookup and the greedy argmax on the device and replay one
 *     CUDA graph per decode step;
 *   - errors never abort the process: the void functions record the error
 *     (kllm_last_error() in kllm_cuda.h) and the int functions return
 *     non-zero.  There is no CPU fallback: without a usable GPU every call
 *     fails with an error.
 */
#ifndef TAPE_RUNNER_H
#define TAPE_RUNNER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MAX_DIMS 8
#define MAX_CONCAT_INPUTS 8

/* Replaces csrc/tape_runner.h:17-28 (same fields, same order). */
typedef struct {
    float    *data;
    int       shape[MAX_DIMS];
    int       ndim;
    int       size;
    int       owns_data;
    float    *codebook;
    uint16_t *w_indices;
    int       n_codes;
    int       tt_K;
    int       tt_N;
} Slot;

/* Replaces csrc/tape_runner.h:30-49 (69 x int32 = 276 bytes). */
typedef struct {
    int tag;
    int out_slot;
    int in0, in1, in2;
    int axis;
    int keepdims;
    int repeats;
    int out_shape[MAX_DIMS];
    int out_ndim;
    int out_size;
    int axes[MAX_DIMS];
    int starts[MAX_DIMS];
    int stops[MAX_DIMS];
    int steps[MAX_DIMS];
    int slice_out_shape[MAX_DIMS];
    int slice_out_ndim;
    int concat_inputs[MAX_CONCAT_INPUTS];
    int concat_n_inputs;
    int tt_weight_slot;
} TapeInstr;

/* Replaces csrc/tape_runner.h:51-56.  The device state of a context lives
 * in a private block allocated together with this struct. */
typedef struct {
    Slot      *slots;
    int        n_slots;
    TapeInstr *tape;
    int        n_instrs;
} TapeCtx;

/* Context API: replaces csrc/tape_runner.h:62-65 (_tape_runner.c:306-325,
 * :423-430). */
TapeCtx *tape_ctx_create(int n_slots, int n_instrs);
void tape_ctx_destroy(TapeCtx *ctx);
int tape_ctx_n_instrs(TapeCtx *ctx);
int tape_ctx_n_slots(TapeCtx *ctx);

/* Slot API: replaces csrc/tape_runner.h:71-84 (_tape_runner.c:328-420). */
void tape_slot_alloc(TapeCtx *ctx, int slot_idx,
                     const int *shape, int ndim);
void tape_slot_set_external(TapeCtx *ctx, int slot_idx,
                            float *data, const int *shape, int ndim);
void tape_slot_set_truth_table(TapeCtx *ctx, int slot_idx,
                               float *codebook, int n_codes,
                               uint16_t *w_indices, int K, int N);
void tape_slot_write(TapeCtx *ctx, int slot_idx,
                     const float *data, int n);
void tape_slot_set_shape(TapeCtx *ctx, int slot_idx,
                         const int *shape, int ndim);
const float *tape_slot_read(TapeCtx *ctx, int slot_idx, int *out_size);
int tape_slot_read_shape(TapeCtx *ctx, int slot_idx, int *out_shape);
TapeInstr *tape_get_instr(TapeCtx *ctx, int instr_idx);

/* One step of the tape: replaces csrc/tape_runner.h:90 (_tape_runner.c:665). */
void tape_run(TapeCtx *ctx);

/* Replaces csrc/tape_runner.h:96-97 (_tape_runner.c:1412-1416): return
 * non-zero to stop generation. */
typedef int (*token_callback_fn)(
    const uint8_t *bytes, int byte_len, void *user_data);

/* Token IDs in, token IDs out: replaces csrc/tape_runner.h:99-108
 * (_tape_runner.c:1602-1763). Returns 0 on success, non-zero on error. */
int processor_infer(
    TapeCtx *ctx,
    const float *embed_table, int vocab_size, int hidden_dim,
    const float *rope_cos, const float *rope_sin, int head_dim,
    int token_embed_slot, int rope_cos_slot, int rope_sin_slot,
    const int *kv_in_slots, const int *kv_out_slots,
    int logits_slot, int n_layers, int num_kv_heads,
    const int *prompt_tokens, int prompt_len,
    int max_new_tokens, int eos_token_id,
    int *output_tokens, int *output_len);

/* Bytes in, streamed bytes out: replaces csrc/tape_runner.h:110-130
 * (_tape_runner.c:1418-1588). Returns 0 on success, non-zero on error. */
int processor_infer_bytes(
    TapeCtx *ctx,
    const uint8_t *hash_keys, const int32_t *hash_vals,
    const int32_t *hash_lens,
    int table_size, int max_piece_len,
    const int32_t *merge_a, const int32_t *merge_b,
    const int32_t *merge_result, int num_merges,
    const uint8_t *id_to_bytes_rom, const int32_t *id_to_offsets,
    const int32_t *special_ids, int num_special,
    int bos_token_id,
    const float *embed_table, int vocab_size, int hidden_dim,
    const float *rope_cos, const float *rope_sin, int head_dim,
    int token_embed_slot, int rope_cos_slot, int rope_sin_slot,
    const int *kv_in_slots, const int *kv_out_slots,
    int logits_slot, int n_layers, int num_kv_heads,
    const uint8_t *input_bytes, int input_len,
    int max_new_tokens, int eos_token_id,
    int max_seq_tokens, int max_bpe_bytes,
    token_callback_fn callback, void *user_data,
    int *total_generated);

/* Host BPE: replaces csrc/tape_runner.h:132-142 (_tape_runner.c:1208). */
int bpe_encode(
    const uint8_t *raw_bytes, int raw_len,
    const uint8_t *hash_keys, const int32_t *hash_vals,
    const int32_t *hash_lens,
    int table_size, int max_piece_len,
    const int32_t *merge_a, const int32_t *merge_b,
    const int32_t *merge_result, int num_merges,
    int bos_token_id, int max_tokens,
    const uint8_t *id_to_bytes, const int32_t *id_to_offsets,
    const int32_t *special_ids, int num_special, int vocab_size,
    int32_t *out_ids);

/* Host BPE: replaces csrc/tape_runner.h:144-150 (_tape_runner.c:1309). */
int bpe_decode(
    const int32_t *token_ids, int num_tokens,
    const uint8_t *id_to_bytes, const int32_t *id_to_offsets,
    int vocab_size,
    const int32_t *special_ids, int num_special,
    int max_bytes, int skip_leading_space,
    uint8_t *out_bytes);

#ifdef __cplusplus
}
#endif

#endif /* TAPE_RUNNER_H */
