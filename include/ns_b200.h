/* B200 backend library (libns_b200.so): the engine behind ns_runtime.h.
 *
 * A NeuralScript model is described by a spec string (the facts the
 * reference compiler bakes into its emitted translation unit:
 * src/codegen/codegen.cpp:552-558, 916-1126). The per-model translation unit
 * (neuralscript_b200/csrc/model_tu.cpp) embeds the spec and maps every
 * ns_runtime.h entry point onto the nsb_* function of the same name below.
 * The nsb_* functions take the same arguments and return the same codes as
 * their ns_* counterparts, except that the initialisers also take the spec.
 *
 * Extensions beyond the reference ABI are marked EXT.
 */
#ifndef NS_B200_H
#define NS_B200_H

#include <stddef.h>

#include "ns_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- the ns_runtime.h entry points, spec-parameterised ------------------ */

/* ns_runtime_init (reference ns_runtime.h:48) for the model `spec`. */
ns_model* nsb_runtime_init(const char* spec, const float* weights, size_t num_floats);
/* reference ns_runtime.h:54 */
int nsb_eval_infer(ns_model* m, const float* input, float* output, size_t input_numel);
/* reference ns_runtime.h:57 */
size_t nsb_model_output_numel(const ns_model* m, size_t input_numel);
/* reference ns_runtime.h:60 */
size_t nsb_model_weight_count(const ns_model* m);
/* reference ns_runtime.h:65, for a spec instead of the compiled-in model */
size_t nsb_spec_weight_count(const char* spec);
/* reference ns_runtime.h:69 */
int nsb_model_get_weights(const ns_model* m, float* out, size_t n);
/* reference ns_runtime.h:72; the table is owned by the library and lives
 * until process exit. */
const ns_weight_layout* nsb_spec_layout(const char* spec);
/* reference ns_runtime.h:75 */
void nsb_free(ns_model* m);
/* reference ns_runtime.h:81, :86 */
int nsb_save_checkpoint(const ns_model* m, const char* path);
int nsb_load_checkpoint(ns_model* m, const char* path);
/* reference ns_runtime.h:106-109 */
size_t nsb_expert_count(const ns_model* m);
size_t nsb_expert_birth(ns_model* m, int n);
size_t nsb_expert_merge(ns_model* m, int a, int b);
size_t nsb_expert_kill(ns_model* m, int k);
/* reference ns_runtime.h:123 */
int nsb_runtime_train_step(ns_model* m, const float* input, const float* labels, size_t input_numel,
                           float* loss_out, float lr);
/* reference ns_runtime.h:128 */
int nsb_objective_loss(ns_model* m, const float* input, const float* labels, size_t input_numel,
                       float* loss_out);

/* ---- EXT: precision, device-resident and index-label fast paths -------- */

/* Precision of the contractions: 0 = pure fp32 SIMT (parity mode),
 * 1 = TF32 tensor cores, 2 = bf16 tensor cores (fp32 accumulate; fp32
 * master weights, statistics, losses and optimizer state in every mode).
 * The spec's `precision` line, then the NS_B200_PRECISION environment
 * variable (fp32|tf32|bf16), set the initial mode. */
int nsb_set_precision(ns_model* m, int mode);
int nsb_get_precision(const ns_model* m);

/* Train step with int32 class targets [rows] instead of dense one-hot labels
 * (the one-hot ABI moves rows x classes floats per step). */
int nsb_runtime_train_step_idx(ns_model* m, const float* input, const int* targets, size_t input_numel,
                               float* loss_out, float lr);

/* Device-resident variants: pointers are device memory, `stream` the
 * caller's cudaStream_t (NULL = the legacy default stream). The work is
 * ordered after prior work on `stream`, and later work on `stream` sees the
 * outputs; neither call blocks the host on the GPU, except that a train step
 * given a non-NULL loss_out waits for the step to finish and returns the
 * loss. Device-side errors of a non-blocking call (a timed-out pipeline
 * wait, a failed collective) are reported by the next call that waits. */
int nsb_eval_infer_device(ns_model* m, const float* d_input, float* d_output, size_t input_numel, void* stream);
int nsb_train_step_device(ns_model* m, const float* d_input, const float* d_labels, const int* d_targets,
                          size_t input_numel, float* loss_out, float lr, void* stream);

/* Gradient blob of the last train step (same layout as the weights; summed
 * over ranks when data-parallel), copied to host `out` of n floats. */
int nsb_model_get_gradients(const ns_model* m, float* out, size_t n);

/* Gradient of the loss with respect to the network input of the last train
 * step (rows x input width floats, this rank's rows), for specs with a
 * `grad input` statement. The reference forms it inside ns_moe_grad_x /
 * ns_matmul_grad_a (src/codegen/codegen.cpp:1318-1326, 1388-1443) but keeps
 * it internal; here it can be read back, e.g. by a caller chaining layers. */
int nsb_model_get_input_gradient(const ns_model* m, float* out, size_t n);

/* Per-region timing: CUDA events recorded on the model's stream around every
 * forward op (attention split into qkv / core / out), every backward op,
 * the loss, the all-reduce and the optimizer. enable != 0 switches it on and
 * resets the totals (also on at init when NS_B200_REGION_TIMING is set).
 * nsb_region_count synchronises and folds pending events into the totals;
 * nsb_region_get returns region i's label, total milliseconds and count. */
int nsb_region_timing(ns_model* m, int enable);
int nsb_region_count(ns_model* m);
int nsb_region_get(const ns_model* m, int i, const char** label, double* total_ms, long long* count);

/* Number of kernel launches issued by the last public call on this model. */
long long nsb_last_launch_count(const ns_model* m);

/* ---- EXT: data parallelism over NCCL ---------------------------------- */

/* Writes a 128-byte NCCL unique id (call on rank 0, share it out of band). */
int nsb_dist_unique_id(void* id128);
/* Joins `world` ranks (one process per GPU, the model's current device).
 * Afterwards each train step all-reduces gradients (sum, over NVLink) and
 * scales the loss seed by the global row count; `timeout_ms` bounds every
 * collective wait (0 = 60 s). */
int nsb_dist_init(ns_model* m, int rank, int world, const void* id128, int timeout_ms);

/* ---- EXT: diagnostics --------------------------------------------------- */

/* Last error message of the calling thread (empty string if none). */
const char* nsb_last_error(void);
/* Library version string. */
const char* nsb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NS_B200_H */
