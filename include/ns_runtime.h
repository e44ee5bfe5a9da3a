/* NeuralScript AOT runtime C-ABI, as implemented by the B200 backend.
 *
 * These are exactly the entry points a NeuralScript model translation unit
 * exports (reference: include/ns/runtime/ns_runtime.h:48-129, version 1.2.0).
 * The declarations must stay identical so a host application, or a binding
 * written against the reference, links against a B200 model library
 * unchanged. Every function here is provided by a per-model library built
 * from neuralscript_b200/csrc/model_tu.cpp with the model's spec baked in;
 * all of them forward to the nsb_* functions of ns_b200.h.
 *
 * Weights are one contiguous host-owned fp32 blob, the concatenation of the
 * layer weights in definition order (ns_model_layout). Inputs and outputs are
 * host pointers; device memory is owned by the model.
 * Return codes: 0 success, -1 error.
 */
#ifndef NS_RUNTIME_H
#define NS_RUNTIME_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NS_RUNTIME_VERSION_MAJOR 1
#define NS_RUNTIME_VERSION_MINOR 2
#define NS_RUNTIME_VERSION_PATCH 0
#define NS_RUNTIME_VERSION "1.2.0"

typedef struct ns_model ns_model;

/* One trainable parameter in the blob (reference ns_runtime.h:31-35). */
typedef struct ns_weight_desc {
    const char* name;
    size_t offset;
    size_t count;
} ns_weight_desc;

/* reference ns_runtime.h:38-41 */
typedef struct ns_weight_layout {
    size_t num_weights;
    const ns_weight_desc* desc;
} ns_weight_layout;

/* Copies the blob; NULL if num_floats != ns_weight_count_static() or on
 * allocation failure. (reference ns_runtime.h:48) */
ns_model* ns_runtime_init(const float* weights, size_t num_floats);

/* Rows = input_numel / input columns (1 for token-id inputs); writes
 * rows * output columns floats. (reference ns_runtime.h:54) */
int ns_eval_infer(ns_model* m, const float* input, float* output, size_t input_numel);

/* reference ns_runtime.h:57 */
size_t ns_model_output_numel(const ns_model* m, size_t input_numel);
/* reference ns_runtime.h:60 */
size_t ns_model_weight_count(const ns_model* m);
/* reference ns_runtime.h:65 */
size_t ns_weight_count_static(void);
/* -1 if m/out is NULL or n != ns_model_weight_count(m). (reference ns_runtime.h:69) */
int ns_model_get_weights(const ns_model* m, float* out, size_t n);
/* reference ns_runtime.h:72 */
const ns_weight_layout* ns_model_layout(const ns_model* m);
/* reference ns_runtime.h:75 */
void ns_free(ns_model* m);

/* NSM2 file: u32 magic 0x4E534D32, size_t float count, the floats, then for
 * MoE models u32 n_layers (1), size_t capacity, capacity mask bytes. Loading
 * accepts NSM1 (weights only, every expert live) and NSM2.
 * (reference ns_runtime.h:81, :86) */
int ns_save_checkpoint(const ns_model* m, const char* path);
int ns_load_checkpoint(ns_model* m, const char* path);

/* MoE expert lifecycle (reference ns_runtime.h:106-109). */
size_t ns_expert_count(const ns_model* m);
size_t ns_expert_birth(ns_model* m, int n);
size_t ns_expert_merge(ns_model* m, int a, int b);
size_t ns_expert_kill(ns_model* m, int k);

/* One forward + backward + optimizer step; labels are one-hot
 * [rows, output columns] fp32; loss_out receives the mean loss; lr is scaled
 * by the compiled schedule. (reference ns_runtime.h:123) */
int ns_runtime_train_step(ns_model* m, const float* input, const float* labels, size_t input_numel,
                          float* loss_out, float lr);

/* Forward-only mean loss, weights untouched. (reference ns_runtime.h:128) */
int ns_objective_loss(ns_model* m, const float* input, const float* labels, size_t input_numel, float* loss_out);

#ifdef __cplusplus
}
#endif

#endif /* NS_RUNTIME_H */
