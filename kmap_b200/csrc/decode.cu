// decode.cu -- processor_infer / processor_infer_bytes.
//
// Token loop of the reference drivers (_tape_runner.c:1418-1588 and
// :1602-1763): prefill one prompt token per tape step, then greedy decode
// with a first-maximum argmax over the last logits row, stop at EOS.
//
// Two executors sit behind the same loop:
//   * the fused plan (plan.cu) when the tape is the compiler's LLaMA decode
//     template: device KV cache, fused kernels, one CUDA graph per step;
//   * the generic executor otherwise: every instruction is a device kernel
//     and the KV buffers round-trip through the slot API exactly as the
//     reference's FEED_TOKEN does.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <vector>

#include "common.cuh"
#include "plan.cuh"

namespace kllm {

struct InferArgs {
    const float *embed;
    int vocab, hidden;
    const float *rope_cos, *rope_sin;
    int head_dim;
    int embed_slot, cos_slot, sin_slot;
    const int *kv_in, *kv_out;
    int logits_slot, n_layers, n_kv;
    int eos;
};

// Host-side generation state shared by both drivers.
struct TokenSink {
    virtual ~TokenSink() {}
    // called for every generated token; return false to stop
    virtual bool emit(int token, int index) = 0;
};

static int argmax_first(const float *row, int n) {
    float best = row[0];
    int bi = 0;
    for (int v = 1; v < n; v++)
        if (row[v] > best) {
            best = row[v];
            bi = v;
        }
    return bi;
}

// Generic executor: the reference loop with every tape step on the device.
static bool infer_generic(CtxImpl *c, const InferArgs &a, const int *prompt, int prompt_len,
                          int max_new, int max_pos, TokenSink *sink, int *generated) {
    TapeCtx *ctx = &c->base;
    int L = a.n_layers, kvd = a.n_kv * a.head_dim;
    int total_cap = std::max(max_pos, 64);
    std::vector<std::vector<float>> kb(L), vb(L);
    for (int l = 0; l < L; l++) {
        kb[l].assign((size_t)kvd * total_cap, 0.f);
        vb[l].assign((size_t)kvd * total_cap, 0.f);
    }
    std::vector<int> seq(L, 0);
    int es[2] = {1, a.hidden}, rs[2] = {1, a.head_dim};
    float *lrows = c->opts.logits_out;
    int lcap = lrows ? c->opts.logits_rows : 0;
    int steps = 0;
    auto feed = [&](int tok, int pos) -> bool {
        if (tok < 0 || tok >= a.vocab) {
            set_error("token id %d outside the vocabulary of %d", tok, a.vocab);
            return false;
        }
        tape_slot_write(ctx, a.embed_slot, a.embed + (size_t)tok * a.hidden, a.hidden);
        tape_slot_set_shape(ctx, a.embed_slot, es, 2);
        tape_slot_write(ctx, a.cos_slot, a.rope_cos + (size_t)pos * a.head_dim, a.head_dim);
        tape_slot_set_shape(ctx, a.cos_slot, rs, 2);
        tape_slot_write(ctx, a.sin_slot, a.rope_sin + (size_t)pos * a.head_dim, a.head_dim);
        tape_slot_set_shape(ctx, a.sin_slot, rs, 2);
        for (int l = 0; l < L; l++) {
            int ks[3] = {a.n_kv, seq[l], a.head_dim};
            tape_slot_set_external(ctx, a.kv_in[2 * l], kb[l].data(), ks, 3);
            tape_slot_set_external(ctx, a.kv_in[2 * l + 1], vb[l].data(), ks, 3);
        }
        if (kllm_tape_run(ctx) != 0) return false;
        for (int l = 0; l < L; l++) {
            int sz = 0;
            int ns = seq[l] + 1;
            size_t tot = (size_t)a.n_kv * ns * a.head_dim;
            if (tot > kb[l].size()) {
                kb[l].resize(tot * 2);
                vb[l].resize(tot * 2);
            }
            const float *nk = tape_slot_read(ctx, a.kv_out[2 * l], &sz);
            if (!nk) return false;
            memcpy(kb[l].data(), nk, tot * 4);
            const float *nv = tape_slot_read(ctx, a.kv_out[2 * l + 1], &sz);
            if (!nv) return false;
            memcpy(vb[l].data(), nv, tot * 4);
            seq[l] = ns;
        }
        if (lrows && steps < lcap) {
            int lsz = 0;
            const float *lg = tape_slot_read(ctx, a.logits_slot, &lsz);
            if (!lg) return false;
            int off = std::max(lsz - a.vocab, 0);
            memcpy(lrows + (size_t)steps * a.vocab, lg + off, (size_t)a.vocab * 4);
        }
        steps++;
        return true;
    };
    int pos = 0;
    for (int i = 0; i < prompt_len; i++) {
        if (!feed(prompt[i], pos)) return false;
        pos++;
    }
    int gen = 0;
    for (int step = 0; step < max_new; step++) {
        if (pos >= max_pos) break;
        int lsz = 0;
        const float *lg = tape_slot_read(ctx, a.logits_slot, &lsz);
        if (!lg) return false;
        int off = std::max(lsz - a.vocab, 0);
        int best = argmax_first(lg + off, a.vocab);
        if (best == a.eos) break;
        gen++;
        if (!sink->emit(best, gen - 1)) break;
        if (!feed(best, pos)) return false;
        pos++;
    }
    *generated = gen;
    c->stats.steps = steps;
    return true;
}

static bool infer_dispatch(CtxImpl *c, const InferArgs &a, const int *prompt, int prompt_len,
                           int max_new, int max_pos, TokenSink *sink, int *generated) {
    auto t0 = std::chrono::steady_clock::now();
    memset(&c->stats, 0, sizeof c->stats);
    long long l0 = g_launches;
    bool ok;
    if (!select_device(c)) return false;
    if (prompt_len < 1) {
        set_error("processor_infer: empty prompt");
        return false;
    }
    if (max_pos > 0 && prompt_len > max_pos) {
        set_error("processor_infer: prompt of %d tokens exceeds the position limit %d",
                  prompt_len, max_pos);
        return false;
    }
    int mode = c->opts.mode;
    bool fused = false;
    if (mode != KLLM_MODE_GENERIC) {
        PlanDesc pd;
        pd.embed = a.embed;
        pd.vocab = a.vocab;
        pd.hidden = a.hidden;
        pd.rope_cos = a.rope_cos;
        pd.rope_sin = a.rope_sin;
        pd.head_dim = a.head_dim;
        pd.embed_slot = a.embed_slot;
        pd.cos_slot = a.cos_slot;
        pd.sin_slot = a.sin_slot;
        pd.kv_in = a.kv_in;
        pd.kv_out = a.kv_out;
        pd.logits_slot = a.logits_slot;
        pd.n_layers = a.n_layers;
        pd.n_kv = a.n_kv;
        std::string why;
        fused = plan_prepare(c, pd, max_pos, &why);
        if (!fused && mode == KLLM_MODE_AUTO && !why.empty() && getenv("KLLM_VERBOSE") &&
            atoi(getenv("KLLM_VERBOSE")))
            fprintf(stderr, "kllm: fused decode plan unavailable: %s\n", why.c_str());
        if (!fused && mode == KLLM_MODE_FUSED) {
            set_error("fused decode plan unavailable: %s", why.c_str());
            return false;
        }
    }
    if (fused) {
        ok = plan_infer(c, prompt, prompt_len, max_new, max_pos, a.eos,
                        [&](int tok, int i) { return sink->emit(tok, i); }, generated);
    } else {
        ok = infer_generic(c, a, prompt, prompt_len, max_new, max_pos, sink, generated);
    }
    c->stats.fused = fused ? 1 : 0;
    c->stats.step_kernel = 0;
    c->stats.stream_values = 0;
    if (fused) plan_kind(c, &c->stats.step_kernel, &c->stats.stream_values);
    c->stats.launches = g_launches - l0;
    c->stats.total_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ok;
}

}  // namespace kllm

using namespace kllm;

namespace {
struct IdSink : TokenSink {
    int *out;
    bool emit(int tok, int i) override {
        out[i] = tok;
        return true;
    }
};

struct ByteSink : TokenSink {
    const uint8_t *id_to_bytes;
    const int32_t *id_to_offsets;
    int vocab;
    const int32_t *special;
    int n_special;
    int max_bpe;
    std::vector<uint8_t> buf;
    token_callback_fn cb;
    void *ud;
    bool emit(int tok, int i) override {
        if (!cb) return true;
        int32_t t = tok;
        int n = bpe_decode(&t, 1, id_to_bytes, id_to_offsets, vocab, special, n_special,
                           max_bpe, i == 0 ? 1 : 0, buf.data());
        return cb(buf.data(), n, ud) == 0;
    }
};
}  // namespace

extern "C" int kllm_infer_batch(TapeCtx *ctx, const int *prompts, const int *prompt_lens,
                                int nseq, int max_new, int eos, int *out, int *out_lens) {
    if (!ctx || !prompts || !prompt_lens || !out || !out_lens || nseq < 1 || max_new < 1) {
        set_error("kllm_infer_batch: bad argument");
        return -1;
    }
    CtxImpl *c = impl(ctx);
    if (!select_device(c)) return -1;
    auto t0 = std::chrono::steady_clock::now();
    memset(&c->stats, 0, sizeof c->stats);
    const long long l0 = g_launches;
    double pre = 0, dec = 0;
    const bool ok = plan_infer_batch(c, prompts, prompt_lens, nseq, max_new, eos, out, out_lens,
                                     &pre, &dec);
    c->stats.fused = 1;
    c->stats.steps = max_new;
    c->stats.prefill_ms = pre;
    c->stats.decode_ms = dec;
    c->stats.launches = g_launches - l0;
    c->stats.total_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return ok ? 0 : -1;
}

extern "C" int kllm_plan_prepare(TapeCtx *ctx, const float *embed_table, int vocab_size,
                                 int hidden_dim, const float *rope_cos, const float *rope_sin,
                                 int head_dim, int token_embed_slot, int rope_cos_slot,
                                 int rope_sin_slot, const int *kv_in_slots,
                                 const int *kv_out_slots, int logits_slot, int n_layers,
                                 int num_kv_heads, int max_pos) {
    if (!ctx || !embed_table || !rope_cos || !rope_sin || !kv_in_slots || !kv_out_slots ||
        max_pos < 1) {
        set_error("kllm_plan_prepare: bad argument");
        return -1;
    }
    CtxImpl *c = impl(ctx);
    if (!select_device(c)) return -1;
    PlanDesc pd;
    pd.embed = embed_table;
    pd.vocab = vocab_size;
    pd.hidden = hidden_dim;
    pd.rope_cos = rope_cos;
    pd.rope_sin = rope_sin;
    pd.head_dim = head_dim;
    pd.embed_slot = token_embed_slot;
    pd.cos_slot = rope_cos_slot;
    pd.sin_slot = rope_sin_slot;
    pd.kv_in = kv_in_slots;
    pd.kv_out = kv_out_slots;
    pd.logits_slot = logits_slot;
    pd.n_layers = n_layers;
    pd.n_kv = num_kv_heads;
    std::string why;
    if (!plan_prepare(c, pd, max_pos, &why)) {
        if (!why.empty()) set_error("fused decode plan unavailable: %s", why.c_str());
        return -1;
    }
    return 0;
}

extern "C" int kllm_shard_set(TapeCtx *ctx, int rank, int world) {
    if (!ctx || world < 1 || rank < 0 || rank >= world) {
        set_error("kllm_shard_set: rank %d of %d", rank, world);
        return -1;
    }
    CtxImpl *c = impl(ctx);
    if (c->shard_rank != rank || c->shard_world != world) plan_destroy(c);
    c->shard_rank = rank;
    c->shard_world = world;
    return 0;
}

extern "C" int kllm_shard_export(TapeCtx *ctx, void *out, size_t cap, size_t *len) {
    if (!ctx) return -1;
    return plan_shard_export(impl(ctx), out, cap, len) ? 0 : -1;
}

extern "C" int kllm_shard_connect(TapeCtx *ctx, const void *all, size_t per_rank) {
    if (!ctx) return -1;
    return plan_shard_connect(impl(ctx), all, per_rank) ? 0 : -1;
}

extern "C" int processor_infer(TapeCtx *ctx, const float *embed_table, int vocab_size,
                               int hidden_dim, const float *rope_cos, const float *rope_sin,
                               int head_dim, int token_embed_slot, int rope_cos_slot,
                               int rope_sin_slot, const int *kv_in_slots,
                               const int *kv_out_slots, int logits_slot, int n_layers,
                               int num_kv_heads, const int *prompt_tokens, int prompt_len,
                               int max_new_tokens, int eos_token_id, int *output_tokens,
                               int *output_len) {
    if (output_len) *output_len = 0;
    if (!ctx || !embed_table || !rope_cos || !rope_sin || !kv_in_slots || !kv_out_slots ||
        !prompt_tokens || (max_new_tokens > 0 && !output_tokens) || !output_len) {
        set_error("processor_infer: NULL argument");
        return -1;
    }
    InferArgs a{embed_table, vocab_size, hidden_dim, rope_cos, rope_sin, head_dim,
                token_embed_slot, rope_cos_slot, rope_sin_slot, kv_in_slots, kv_out_slots,
                logits_slot, n_layers, num_kv_heads, eos_token_id};
    IdSink sink;
    sink.out = output_tokens;
    int gen = 0;
    // the reference sizes its KV for prompt + generation (_tape_runner.c:1633)
    int max_pos = prompt_len + std::max(max_new_tokens, 0);
    bool ok = infer_dispatch(impl(ctx), a, prompt_tokens, prompt_len, max_new_tokens, max_pos,
                             &sink, &gen);
    *output_len = gen;
    return ok ? 0 : -1;
}

extern "C" int processor_infer_bytes(
    TapeCtx *ctx, const uint8_t *hash_keys, const int32_t *hash_vals, const int32_t *hash_lens,
    int table_size, int max_piece_len, const int32_t *merge_a, const int32_t *merge_b,
    const int32_t *merge_result, int num_merges, const uint8_t *id_to_bytes_rom,
    const int32_t *id_to_offsets, const int32_t *special_ids, int num_special, int bos_token_id,
    const float *embed_table, int vocab_size, int hidden_dim, const float *rope_cos,
    const float *rope_sin, int head_dim, int token_embed_slot, int rope_cos_slot,
    int rope_sin_slot, const int *kv_in_slots, const int *kv_out_slots, int logits_slot,
    int n_layers, int num_kv_heads, const uint8_t *input_bytes, int input_len,
    int max_new_tokens, int eos_token_id, int max_seq_tokens, int max_bpe_bytes,
    token_callback_fn callback, void *user_data, int *total_generated) {
    if (total_generated) *total_generated = 0;
    if (!ctx || !embed_table || !rope_cos || !rope_sin || !kv_in_slots || !kv_out_slots ||
        !total_generated || max_seq_tokens <= 0 || max_bpe_bytes <= 0) {
        set_error("processor_infer_bytes: invalid argument");
        return -1;
    }
    // Phase 1: BPE encode (_tape_runner.c:1442-1452)
    std::vector<int32_t> prompt((size_t)max_seq_tokens);
    int plen = bpe_encode(input_bytes, input_len, hash_keys, hash_vals, hash_lens, table_size,
                          max_piece_len, merge_a, merge_b, merge_result, num_merges,
                          bos_token_id, max_seq_tokens, id_to_bytes_rom, id_to_offsets,
                          special_ids, num_special, vocab_size, prompt.data());
    InferArgs a{embed_table, vocab_size, hidden_dim, rope_cos, rope_sin, head_dim,
                token_embed_slot, rope_cos_slot, rope_sin_slot, kv_in_slots, kv_out_slots,
                logits_slot, n_layers, num_kv_heads, eos_token_id};
    ByteSink sink;
    sink.id_to_bytes = id_to_bytes_rom;
    sink.id_to_offsets = id_to_offsets;
    sink.vocab = vocab_size;
    sink.special = special_ids;
    sink.n_special = num_special;
    sink.max_bpe = max_bpe_bytes;
    sink.buf.assign((size_t)max_bpe_bytes + 256, 0);
    sink.cb = callback;
    sink.ud = user_data;
    int gen = 0;
    // the reference stops decoding at max_seq_tokens positions (:1537)
    bool ok = infer_dispatch(impl(ctx), a, prompt.data(), plen, max_new_tokens, max_seq_tokens,
                             &sink, &gen);
    *total_generated = gen;
    return ok ? 0 : -1;
}

extern "C" int kllm_plan_match(TapeCtx *ctx, int vocab_size, int hidden_dim, int head_dim,
                               int token_embed_slot, int rope_cos_slot, int rope_sin_slot,
                               const int *kv_in_slots, const int *kv_out_slots, int logits_slot,
                               int n_layers, int num_kv_heads, char *why, int why_len) {
    if (!ctx || !kv_in_slots || !kv_out_slots) {
        set_error("kllm_plan_match: NULL argument");
        return -1;
    }
    PlanDesc pd;
    pd.vocab = vocab_size;
    pd.hidden = hidden_dim;
    pd.head_dim = head_dim;
    pd.embed_slot = token_embed_slot;
    pd.cos_slot = rope_cos_slot;
    pd.sin_slot = rope_sin_slot;
    pd.kv_in = kv_in_slots;
    pd.kv_out = kv_out_slots;
    pd.logits_slot = logits_slot;
    pd.n_layers = n_layers;
    pd.n_kv = num_kv_heads;
    std::string w;
    bool ok = plan_match(ctx, pd, &w);
    if (why && why_len > 0) {
        snprintf(why, (size_t)why_len, "%s", ok ? "" : w.c_str());
    }
    return ok ? 1 : 0;
}
