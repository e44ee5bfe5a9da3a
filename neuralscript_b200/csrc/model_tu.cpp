// Per-model translation unit: the ns_runtime.h C-ABI for one network.
//
// This is what a B200 emitter for NeuralScript produces in place of the
// reference's generated CUDA driver (src/codegen/codegen.cpp:916-1126): the
// model's spec baked in as a string, every ns_runtime.h entry point mapped
// onto libns_b200.so. Build one library per model:
//   g++ -shared -fPIC -DNSB_SPEC_FILE='"c2.inc"' model_tu.cpp -lns_b200
// where c2.inc is the spec text as a comma-separated byte list (the
// Makefile makes it with od), or define NSB_SPEC_TEXT as a string literal.
// or define NSB_SPEC_TEXT directly.
#include "../../include/ns_b200.h"

#ifndef NSB_SPEC_TEXT
#ifndef NSB_SPEC_FILE
#error "define NSB_SPEC_TEXT or NSB_SPEC_FILE"
#endif
static const char kSpec[] = {
#include NSB_SPEC_FILE
    0};
#else
static const char kSpec[] = NSB_SPEC_TEXT;
#endif

extern "C" {

ns_model* ns_runtime_init(const float* weights, size_t num_floats) {
    return nsb_runtime_init(kSpec, weights, num_floats);
}
int ns_eval_infer(ns_model* m, const float* input, float* output, size_t input_numel) {
    return nsb_eval_infer(m, input, output, input_numel);
}
size_t ns_model_output_numel(const ns_model* m, size_t input_numel) {
    return nsb_model_output_numel(m, input_numel);
}
size_t ns_model_weight_count(const ns_model* m) { return m ? nsb_model_weight_count(m) : nsb_spec_weight_count(kSpec); }
size_t ns_weight_count_static(void) { return nsb_spec_weight_count(kSpec); }
int ns_model_get_weights(const ns_model* m, float* out, size_t n) { return nsb_model_get_weights(m, out, n); }
const ns_weight_layout* ns_model_layout(const ns_model* m) {
    (void)m;
    return nsb_spec_layout(kSpec);
}
void ns_free(ns_model* m) { nsb_free(m); }
int ns_save_checkpoint(const ns_model* m, const char* path) { return nsb_save_checkpoint(m, path); }
int ns_load_checkpoint(ns_model* m, const char* path) { return nsb_load_checkpoint(m, path); }
size_t ns_expert_count(const ns_model* m) { return nsb_expert_count(m); }
size_t ns_expert_birth(ns_model* m, int n) { return nsb_expert_birth(m, n); }
size_t ns_expert_merge(ns_model* m, int a, int b) { return nsb_expert_merge(m, a, b); }
size_t ns_expert_kill(ns_model* m, int k) { return nsb_expert_kill(m, k); }
int ns_runtime_train_step(ns_model* m, const float* input, const float* labels, size_t input_numel, float* loss_out,
                          float lr) {
    return nsb_runtime_train_step(m, input, labels, input_numel, loss_out, lr);
}
int ns_objective_loss(ns_model* m, const float* input, const float* labels, size_t input_numel, float* loss_out) {
    return nsb_objective_loss(m, input, labels, input_numel, loss_out);
}

}  // extern "C"
