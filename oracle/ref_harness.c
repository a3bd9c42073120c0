/*
 * ref_harness.c -- ctypes-friendly entry points around the UNMODIFIED
 * reference runtime (kllm.c + _tape_runner.c), compiled from the sources
 * where they lie by oracle/Makefile into oracle/_ref/libkllm_ref.so.
 *
 * Test infrastructure only: the product never links or loads this file.
 *
 * The reference keeps its chip loader `chip_load` static inside kllm.c
 * (kllm.c:152-388), so this file includes kllm.c textually with its `main`
 * renamed; everything below only calls the reference's own functions:
 *   chip_load / chip_destroy      kllm.c:152, kllm.c:391
 *   processor_infer               _tape_runner.c:1602
 *   processor_infer_bytes         _tape_runner.c:1418
 *   bpe_encode / bpe_decode       _tape_runner.c:1208, :1309
 *   tape_run + slot API           _tape_runner.c:665, :306-435
 *   compile_chip (exported)       kllm_compile.c:1392
 */
#define main kllm_reference_cli_main
#include "kllm.c"
#undef main

/* Machine description of a loaded chip, in a fixed order. */
void refh_chip_info(void *h, int *info)
{
    ChipCtx *c = (ChipCtx *)h;
    info[0] = c->vocab_size;
    info[1] = c->hidden_dim;
    info[2] = c->num_layers;
    info[3] = c->num_kv_heads;
    info[4] = c->head_dim;
    info[5] = c->max_seq_len;
    info[6] = c->eos_token_id;
    info[7] = c->logits_slot;
    info[8] = c->token_embed_slot;
    info[9] = c->rope_cos_slot;
    info[10] = c->rope_sin_slot;
    info[11] = c->ctx->n_slots;
    info[12] = c->ctx->n_instrs;
    info[13] = c->bos_token_id;
    info[14] = c->table_size;
    info[15] = c->max_piece_len;
    info[16] = c->num_merges;
    info[17] = c->num_special;
}

void *refh_chip_load(const char *dir) { return chip_load(dir); }
void refh_chip_destroy(void *h) { chip_destroy((ChipCtx *)h); }
void *refh_chip_tape(void *h) { return ((ChipCtx *)h)->ctx; }
const int *refh_chip_kv_in(void *h) { return ((ChipCtx *)h)->kv_in_slots; }
const int *refh_chip_kv_out(void *h) { return ((ChipCtx *)h)->kv_out_slots; }

/* The reference's own token-ID driver (_tape_runner.c:1602). */
int refh_processor_infer(void *h, const int *prompt, int prompt_len,
                         int max_new, int eos, int *out, int *out_len)
{
    ChipCtx *c = (ChipCtx *)h;
    return processor_infer(c->ctx, c->embed_table, c->vocab_size, c->hidden_dim,
                           c->rope_cos, c->rope_sin, c->head_dim,
                           c->token_embed_slot, c->rope_cos_slot, c->rope_sin_slot,
                           c->kv_in_slots, c->kv_out_slots, c->logits_slot,
                           c->num_layers, c->num_kv_heads, prompt, prompt_len,
                           max_new, eos, out, out_len);
}

/*
 * Greedy loop with per-step logits capture.  It drives the reference tape
 * through its public slot API exactly the way FEED_TOKEN does
 * (_tape_runner.c:1658-1708) and picks tokens with the same first-max argmax
 * (_tape_runner.c:1717-1727).  Token IDs from this loop are checked against
 * refh_processor_infer in the tests, which pins the loop to the reference.
 * logits: [prompt_len + max_new][vocab] rows, one per tape_run.
 */
int refh_greedy_logits(void *h, const int *prompt, int prompt_len, int max_new,
                       int *out, float *logits)
{
    ChipCtx *c = (ChipCtx *)h;
    TapeCtx *ctx = c->ctx;
    int L = c->num_layers, nkv = c->num_kv_heads, hd = c->head_dim;
    int H = c->hidden_dim, V = c->vocab_size;
    int total = prompt_len + max_new;
    size_t kvcap = (size_t)nkv * hd * (total > 64 ? total : 64);
    float **kb = calloc(L, sizeof(float *)), **vb = calloc(L, sizeof(float *));
    for (int l = 0; l < L; l++) {
        kb[l] = calloc(kvcap, sizeof(float));
        vb[l] = calloc(kvcap, sizeof(float));
    }
    int es[2] = {1, H}, rs[2] = {1, hd};
    int tok = prompt_len > 0 ? prompt[0] : 0;
    for (int step = 0; step < total; step++) {
        if (step < prompt_len) tok = prompt[step];
        tape_slot_write(ctx, c->token_embed_slot, c->embed_table + (size_t)tok * H, H);
        tape_slot_set_shape(ctx, c->token_embed_slot, es, 2);
        tape_slot_write(ctx, c->rope_cos_slot, c->rope_cos + (size_t)step * hd, hd);
        tape_slot_set_shape(ctx, c->rope_cos_slot, rs, 2);
        tape_slot_write(ctx, c->rope_sin_slot, c->rope_sin + (size_t)step * hd, hd);
        tape_slot_set_shape(ctx, c->rope_sin_slot, rs, 2);
        for (int l = 0; l < L; l++) {
            int ks[3] = {nkv, step, hd};
            tape_slot_set_external(ctx, c->kv_in_slots[2 * l], kb[l], ks, 3);
            tape_slot_set_external(ctx, c->kv_in_slots[2 * l + 1], vb[l], ks, 3);
        }
        tape_run(ctx);
        for (int l = 0; l < L; l++) {
            int sz;
            size_t n = (size_t)nkv * (step + 1) * hd;
            memcpy(kb[l], tape_slot_read(ctx, c->kv_out_slots[2 * l], &sz), n * 4);
            memcpy(vb[l], tape_slot_read(ctx, c->kv_out_slots[2 * l + 1], &sz), n * 4);
        }
        int lsz;
        const float *lg = tape_slot_read(ctx, c->logits_slot, &lsz);
        const float *row = lg + (lsz - V > 0 ? lsz - V : 0);
        memcpy(logits + (size_t)step * V, row, (size_t)V * 4);
        if (step >= prompt_len - 1) {
            int gi = step - (prompt_len - 1);
            if (gi < max_new) {
                float best = row[0];
                int bi = 0;
                for (int v = 1; v < V; v++)
                    if (row[v] > best) { best = row[v]; bi = v; }
                out[gi] = bi;
                tok = bi;
            }
        }
    }
    for (int l = 0; l < L; l++) { free(kb[l]); free(vb[l]); }
    free(kb);
    free(vb);
    return 0;
}

typedef struct { uint8_t *buf; int cap; int len; } RefhBuf;

static int refh_buf_cb(const uint8_t *bytes, int n, void *ud)
{
    RefhBuf *b = (RefhBuf *)ud;
    if (b->len + n <= b->cap) {
        memcpy(b->buf + b->len, bytes, n);
        b->len += n;
    }
    return 0;
}

/* The reference's bytes-in/bytes-out driver (_tape_runner.c:1418). */
int refh_infer_bytes(void *h, const uint8_t *in, int in_len, int max_new,
                     int max_seq_tokens, uint8_t *out, int out_cap,
                     int *out_len, int *generated)
{
    ChipCtx *c = (ChipCtx *)h;
    RefhBuf b = {out, out_cap, 0};
    processor_infer_bytes(c->ctx, c->hash_keys, c->hash_vals, c->hash_lens,
                          c->table_size, c->max_piece_len, c->merge_a, c->merge_b,
                          c->merge_result, c->num_merges, c->id_to_bytes,
                          c->id_to_offsets, c->special_ids, c->num_special,
                          c->bos_token_id, c->embed_table, c->vocab_size,
                          c->hidden_dim, c->rope_cos, c->rope_sin, c->head_dim,
                          c->token_embed_slot, c->rope_cos_slot, c->rope_sin_slot,
                          c->kv_in_slots, c->kv_out_slots, c->logits_slot,
                          c->num_layers, c->num_kv_heads, in, in_len, max_new,
                          c->eos_token_id, max_seq_tokens, 8192, refh_buf_cb, &b,
                          generated);
    *out_len = b.len;
    return 0;
}

int refh_bpe_encode(void *h, const uint8_t *in, int in_len, int max_tokens, int32_t *out)
{
    ChipCtx *c = (ChipCtx *)h;
    return bpe_encode(in, in_len, c->hash_keys, c->hash_vals, c->hash_lens,
                      c->table_size, c->max_piece_len, c->merge_a, c->merge_b,
                      c->merge_result, c->num_merges, c->bos_token_id, max_tokens,
                      c->id_to_bytes, c->id_to_offsets, c->special_ids,
                      c->num_special, c->vocab_size, out);
}

int refh_bpe_decode(void *h, const int32_t *ids, int n, int max_bytes,
                    int skip_leading_space, uint8_t *out)
{
    ChipCtx *c = (ChipCtx *)h;
    return bpe_decode(ids, n, c->id_to_bytes, c->id_to_offsets, c->vocab_size,
                      c->special_ids, c->num_special, max_bytes,
                      skip_leading_space, out);
}

/*
 * A resumable greedy session over the reference tape: the loop of
 * refh_greedy_logits (FEED_TOKEN, _tape_runner.c:1658-1708, and the
 * first-max pick, :1717-1727) cut into calls of a few positions each, so a
 * benchmark can time the whole prompt + generation workload in bounded
 * windows.  A session holds the prompt, the KV buffers of every layer and
 * the position reached; refh_session_run advances it by up to n positions
 * and returns how many it ran (0 once the workload is complete).
 */
typedef struct {
    ChipCtx *c;
    int *prompt;
    int prompt_len, max_new, total, step, tok;
    int *out;
    float **kb, **vb;
} RefhSession;

void *refh_session_create(void *h, const int *prompt, int prompt_len, int max_new)
{
    ChipCtx *c = (ChipCtx *)h;
    RefhSession *s = calloc(1, sizeof *s);
    s->c = c;
    s->prompt_len = prompt_len;
    s->max_new = max_new;
    s->total = prompt_len + max_new;
    s->prompt = malloc(sizeof(int) * (prompt_len > 0 ? prompt_len : 1));
    memcpy(s->prompt, prompt, sizeof(int) * prompt_len);
    s->out = calloc(max_new > 0 ? max_new : 1, sizeof(int));
    s->tok = prompt_len > 0 ? prompt[0] : 0;
    int L = c->num_layers;
    size_t kvcap = (size_t)c->num_kv_heads * c->head_dim * (s->total > 64 ? s->total : 64);
    s->kb = calloc(L, sizeof(float *));
    s->vb = calloc(L, sizeof(float *));
    for (int l = 0; l < L; l++) {
        s->kb[l] = calloc(kvcap, sizeof(float));
        s->vb[l] = calloc(kvcap, sizeof(float));
    }
    return s;
}

/* Run up to n more positions; logits (optional): [n][vocab] rows. */
int refh_session_run(void *sp, int n, float *logits)
{
    RefhSession *s = (RefhSession *)sp;
    ChipCtx *c = s->c;
    TapeCtx *ctx = c->ctx;
    int L = c->num_layers, nkv = c->num_kv_heads, hd = c->head_dim;
    int H = c->hidden_dim, V = c->vocab_size;
    int es[2] = {1, H}, rs[2] = {1, hd};
    int ran = 0;
    for (; ran < n && s->step < s->total; ran++, s->step++) {
        int step = s->step;
        if (step < s->prompt_len) s->tok = s->prompt[step];
        tape_slot_write(ctx, c->token_embed_slot, c->embed_table + (size_t)s->tok * H, H);
        tape_slot_set_shape(ctx, c->token_embed_slot, es, 2);
        tape_slot_write(ctx, c->rope_cos_slot, c->rope_cos + (size_t)step * hd, hd);
        tape_slot_set_shape(ctx, c->rope_cos_slot, rs, 2);
        tape_slot_write(ctx, c->rope_sin_slot, c->rope_sin + (size_t)step * hd, hd);
        tape_slot_set_shape(ctx, c->rope_sin_slot, rs, 2);
        for (int l = 0; l < L; l++) {
            int ks[3] = {nkv, step, hd};
            tape_slot_set_external(ctx, c->kv_in_slots[2 * l], s->kb[l], ks, 3);
            tape_slot_set_external(ctx, c->kv_in_slots[2 * l + 1], s->vb[l], ks, 3);
        }
        tape_run(ctx);
        for (int l = 0; l < L; l++) {
            int sz;
            size_t m = (size_t)nkv * (step + 1) * hd;
            memcpy(s->kb[l], tape_slot_read(ctx, c->kv_out_slots[2 * l], &sz), m * 4);
            memcpy(s->vb[l], tape_slot_read(ctx, c->kv_out_slots[2 * l + 1], &sz), m * 4);
        }
        int lsz;
        const float *lg = tape_slot_read(ctx, c->logits_slot, &lsz);
        const float *row = lg + (lsz - V > 0 ? lsz - V : 0);
        if (logits) memcpy(logits + (size_t)ran * V, row, (size_t)V * 4);
        if (step >= s->prompt_len - 1) {
            int gi = step - (s->prompt_len - 1);
            if (gi < s->max_new) {
                float best = row[0];
                int bi = 0;
                for (int v = 1; v < V; v++)
                    if (row[v] > best) { best = row[v]; bi = v; }
                s->out[gi] = bi;
                s->tok = bi;
            }
        }
    }
    return ran;
}

/* Generated tokens so far (returns their count). */
int refh_session_tokens(void *sp, int *out, int cap)
{
    RefhSession *s = (RefhSession *)sp;
    int n = s->step - (s->prompt_len - 1);
    if (n < 0) n = 0;
    if (n > s->max_new) n = s->max_new;
    if (n > cap) n = cap;
    memcpy(out, s->out, sizeof(int) * n);
    return n;
}

void refh_session_destroy(void *sp)
{
    RefhSession *s = (RefhSession *)sp;
    if (!s) return;
    for (int l = 0; l < s->c->num_layers; l++) { free(s->kb[l]); free(s->vb[l]); }
    free(s->kb);
    free(s->vb);
    free(s->prompt);
    free(s->out);
    free(s);
}
