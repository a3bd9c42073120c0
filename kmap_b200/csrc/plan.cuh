// plan.cuh -- fused decode plan for the compiler's LLaMA decode template.
#pragma once

#include <functional>
#include <string>

#include "common.cuh"

namespace kllm {

// What processor_infer knows about the chip (its arguments).
struct PlanDesc {
    const float *embed = nullptr;
    int vocab = 0, hidden = 0;
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    int head_dim = 0;
    int embed_slot = -1, cos_slot = -1, sin_slot = -1;
    const int *kv_in = nullptr, *kv_out = nullptr;
    int logits_slot = -1, n_layers = 0, n_kv = 0;
};

// Whether the tape is the compiler's template (no device work).
bool plan_match(const TapeCtx *ctx, const PlanDesc &d, std::string *why);

// Match the tape against the template and stage the plan's device state
// (weights, KV cache for max_pos positions, graphs).  Returns false with a
// reason when the tape is not the template; no error is recorded then.
bool plan_prepare(CtxImpl *c, const PlanDesc &d, int max_pos, std::string *why);
// Column-sharded decode: export this rank's shared buffers, map the others'.
bool plan_shard_export(CtxImpl *c, void *out, size_t cap, size_t *len);
bool plan_shard_connect(CtxImpl *c, const void *all, size_t per_rank);

// Which step kernel the plan runs (persistent: 1) and what its weight
// streams hold (TTXVals); zeros without a plan.
void plan_kind(const CtxImpl *c, int *persist, int *values);

// Prefill + greedy decode on the plan.  emit(token, i) is called for every
// generated token in order and returns false to stop.
bool plan_infer(CtxImpl *c, const int *prompt, int prompt_len, int max_new, int max_pos,
                int eos, const std::function<bool(int, int)> &emit, int *generated);

// Batched greedy decode of nseq sequences (prompts concatenated, lens[i]
// tokens each): out[i * max_new + j] is sequence i's token j, out_lens[i]
// the count before its first EOS.  One GPU, persistent plan prepared;
// prefill_ms / decode_ms: device time of the prompt passes and the steps.
bool plan_infer_batch(CtxImpl *c, const int *prompts, const int *lens, int nseq, int max_new,
                      int eos, int *out, int *out_lens, double *prefill_ms, double *decode_ms);

}  // namespace kllm
