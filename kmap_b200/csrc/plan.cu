// plan.cu -- fused decode plan (placeholder: the template is not matched
// yet, so processor_infer runs the generic executor).
#include "plan.cuh"

namespace kllm {

struct DecodePlan {};

bool plan_prepare(CtxImpl *c, const PlanDesc &d, int max_pos, std::string *why) {
    (void)c;
    (void)d;
    (void)max_pos;
    *why = "fused plan not built";
    return false;
}

bool plan_infer(CtxImpl *c, const int *prompt, int prompt_len, int max_new, int max_pos,
                int eos, const std::function<bool(int, int)> &emit, int *generated) {
    (void)c; (void)prompt; (void)prompt_len; (void)max_new; (void)max_pos; (void)eos;
    (void)emit; (void)generated;
    set_error("fused plan not built");
    return false;
}

void plan_destroy(CtxImpl *c) {
    delete c->plan;
    c->plan = nullptr;
}

}  // namespace kllm
