/* Kernel-level C-ABI of libns_b200.so: the hot-path kernels on caller-owned
 * DEVICE pointers, one call per kernel family, for tests, benchmarks and
 * integrators that drive their own buffers. Each entry names the reference
 * computation it replaces (file:line in MrModelOS/NeuralScript). `stream` is
 * a cudaStream_t (NULL = legacy default stream). Returns 0 on success, a
 * negative value on a bad argument or launch failure. Nothing here
 * allocates device memory: scratch, where a kernel needs it, is passed in
 * and its size is given by the matching *_scratch_bytes query.
 */
#ifndef NS_B200_OPS_H
#define NS_B200_OPS_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define NSB_F32 0
#define NSB_BF16 1

/* engine codes */
#define NSB_ENGINE_AUTO 0   /* tcgen05 when operands allow, else SIMT */
#define NSB_ENGINE_SIMT 1   /* exact fp32 FMA, sequential in k */
#define NSB_ENGINE_TENSOR 2 /* tcgen05 only (error if not possible) */

/* C[M,N] = act(alpha * A[M,K] B[N,K]^T + add) with
 *   A element (i,k) at A[i*lda + k] (a_mn = 0) or A[k*lda + i] (a_mn = 1),
 *   B element (n,k) at B[n*ldb + k] (b_mn = 0) or B[k*ldb + n] (b_mn = 1).
 * Replaces ns_gemm_kernel / ns_grad_a_kernel / ns_grad_w_kernel
 * (src/codegen/cuda_backend.cpp:58-79, 446-467) and ns_matmul /
 * ns_matmul_grad_a / ns_matmul_grad_w (src/codegen/codegen.cpp:1257-1337).
 * act: 0 identity .. 6 GELU (codegen.cpp:1244-1255). add (fp32, ld_add) may be
 * NULL. c32 / c16 outputs (either may be NULL). workspace: fp32 scratch of
 * nsb_op_gemm_workspace_floats(...) floats (may be NULL when that is 0). */
int nsb_op_gemm(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn, const void* B, int b_dtype,
                long long ldb, int b_mn, float alpha, const float* add, long long ld_add, int act, float* c32,
                long long ldc32, void* c16, long long ldc16, int engine, float* workspace, size_t workspace_floats,
                int* dev_err, void* stream);
size_t nsb_op_gemm_workspace_floats(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn,
                                    const void* B, int b_dtype, long long ldb, int b_mn, int engine);
/* 1 when nsb_op_gemm would run on tcgen05 tensor cores for these operands. */
int nsb_op_gemm_uses_tensor_cores(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn,
                                  const void* B, int b_dtype, long long ldb, int b_mn, int engine);

/* out = W[(int)ids[r]] (ids fp32; out-of-range -> row 0).
 * Replaces ns_embedding_kernel (cuda_backend.cpp:172-181), ns_embedding
 * (codegen.cpp:1711-1718). */
int nsb_op_embedding_fwd(const float* W, const float* ids, int M, int V, int D, float* out32, void* out16,
                         void* stream);
/* dW = deterministic sort-then-segment scatter-add of dout rows by id
 * (rows in increasing order; out-of-range ids skipped). Replaces
 * ns_embedding_grad_w_kernel (cuda_backend.cpp:500-512) and
 * ns_embedding_grad_w (codegen.cpp:1374-1383). */
size_t nsb_op_embedding_bwd_scratch_bytes(int M, int V);
int nsb_op_embedding_bwd(const float* dout, const float* ids, int M, int V, int D, float* dW, void* scratch,
                         void* stream);

/* Allocation-free variant of nsb_op_embedding_bwd (same result, bit for
 * bit). No counterpart in the reference: it exists for callers that cannot
 * allocate device memory when they need this gradient - code running inside
 * a memory-pool or allocator callback, hosts that have given all device
 * memory to their own pool, runtimes that forbid cudaMalloc after start-up.
 * Its sort scratch is a fixed array in the library's device memory, so it
 * calls no cudaMalloc, cudaFree or allocating library routine.
 * Limits: M <= 262144 rows and V <= 65536 vocabulary rows; larger sizes
 * return -2 without launching anything. The work runs on the current device:
 * a non-NULL `stream` must belong to it (otherwise -4, nothing launched).
 * Every GPU that loads the library
 * holds the 1.75 MB array until the process exits. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress, once per
 * device, with that device current); make that first call before any CUDA
 * stream capture. All calls share the one array: calls that overlap on the
 * same GPU (for example on two streams) race on it, so serialise them on one
 * stream. Counters are cleared by every call. */
int nsb_op_embedding_bwd_noalloc(const float* dout, const float* ids, int M, int V, int D, float* dW, void* stream);

/* LayerNorm, no affine, eps 1e-5. Replaces ns_layernorm_kernel /
 * ns_layernorm_grad_kernel (cuda_backend.cpp:420-431, 473-499),
 * ns_layernorm / ns_layernorm_grad (codegen.cpp:1280-1291, 1346-1371). */
int nsb_op_layernorm_fwd(const float* x, int M, int D, float* out32, void* out16, void* stream);
int nsb_op_layernorm_bwd(const float* dy, const float* x, const float* add, int M, int D, float* dx32, void* dx16,
                         void* stream);

/* Attention core on qkv [B*S, ld_qkv] (Q | K | V column blocks, heads
 * concatenated) -> ctx [B*S, ld_ctx]; lse [B*H*S] saved for the backward.
 * Replaces ns_attention_core_kernel / ns_attention_grad_kernel
 * (cuda_backend.cpp:186-366) and the per-head core of ns_attention_fwd /
 * ns_attention_bwd (codegen.cpp:1724-1907). dvec: [B*H*S] fp32 scratch. */
int nsb_op_attention_fwd(int B, int S, int H, int D, int dtype, const void* qkv, long long ld_qkv, void* ctx,
                         long long ld_ctx, float* lse, void* stream);
int nsb_op_attention_bwd(int B, int S, int H, int D, int dtype, const void* qkv, long long ld_qkv, const void* ctx,
                         long long ld_ctx, const float* lse, const void* dctx, long long ld_dctx, void* dqkv,
                         long long ld_dqkv, float* dvec, void* stream);

/* Softmax cross-entropy forward + seed gradient: row_loss[r] and
 * d = (softmax - y) / denom. labels one-hot [M,C] fp32, or targets int32 [M]
 * when labels is NULL. Replaces ns_ce_row_kernel + ns_loss_grad_kernel
 * (cuda_backend.cpp:690-719), ns_cross_entropy / ns_loss_grad
 * (codegen.cpp:1582-1613). */
int nsb_op_cross_entropy(const float* logits, const float* labels, const int* targets, int M, int C, float denom,
                         float* row_loss, float* d32, void* d16, void* stream);
/* Second half of the fused head loss: logits16 holds fp16 logits [M,C]
 * (16-byte aligned, C % 8 == 0) as the head GEMM writes them, tlogit the
 * fp32 target logit of each row; writes row_loss[r] = lse - tlogit[r] (0 for
 * a target outside [0,C)) and overwrites the row in place with the bf16 seed
 * (softmax - onehot) / denom. Same arithmetic as nsb_op_cross_entropy with
 * targets (ns_ce_row_kernel + ns_loss_grad_kernel, cuda_backend.cpp:690-719). */
int nsb_op_cross_entropy_finish(void* logits16, int M, int C, const int* targets, const float* tlogit, float denom,
                                float* row_loss, void* stream);
/* out[0] = scale * sum(x[0..n)), fixed reduction order. */
int nsb_op_reduce_sum(const float* x, int n, float scale, float* out, void* stream);

/* One AdamW step of one tensor (step counter t >= 1). Replaces
 * ns_adamw_kernel (cuda_backend.cpp:720-733) / codegen.cpp:3108-3120. */
int nsb_op_adamw(float* w, const float* g, float* m, float* v, long long n, long long t, float lr, float beta1,
                 float beta2, float one_minus_beta1, float one_minus_beta2, float eps, float decay, void* stream);
/* Modified Gram-Schmidt in place on an r x c matrix (columns if r >= c, rows
 * otherwise). Replaces ns_orthonom_kernel (cuda_backend.cpp:747-773) /
 * ns_orthonom (codegen.cpp:1617-1633). */
int nsb_op_mgs(float* G, int r, int c, void* stream);

/* Top-1 MoE router: logits x.Wg accumulated with fmaf in increasing k (the
 * reference's scalar order, so the logits are bit-identical to its CPU emit),
 * softmax over live experts (active[e] != 0; NULL = all live), best = first
 * maximum of the exp'd logits (-1 if none live), pb = its probability, probs
 * [M,E] (may be NULL) the live softmax. Replaces the routing of ns_moe_kernel
 * (cuda_backend.cpp:371-407) and ns_moe_fwd (codegen.cpp:1915-1931). */
int nsb_op_moe_route(const float* x, const float* Wg, const unsigned char* active, int M, int D, int E, int* best,
                     float* pb, float* probs, void* stream);

/* Activation forward / derivative product. Replaces ns_act_kernel /
 * ns_act_grad_kernel (cuda_backend.cpp:80-84, 468-472). */
int nsb_op_act_fwd(const float* x, size_t n, int act, float* out32, void* out16, void* stream);
int nsb_op_act_bwd(const float* dy, const float* z, int act, size_t n, float* out32, void* stream);

/* Y[M,512] = LayerNorm(alpha * A[M,K] B[K,512] + add) row by row (no affine,
 * eps 1e-5), the LayerNorm in the GEMM's epilogue: a 128 x 512 tile holds
 * whole rows. A K-major (element (i,k) at A[i*lda + k]), B row-major
 * [K, 512] (B[k*ldb + n]), both bf16 or both fp32 (TF32); add fp32 (may be
 * NULL); c32 / c16 receive Y (either may be NULL), rstd[M] the rows'
 * 1 / sqrt(var + eps). Replaces a Dense / attention output GEMM, the
 * residual ns_binop and ns_layernorm_kernel in sequence
 * (cuda_backend.cpp:58-79, 408-431). */
int nsb_op_gemm_layernorm(int M, int K, const void* A, int dtype, long long lda, const void* B, long long ldb,
                          float alpha, const float* add, long long ld_add, float* c32, long long ldc32, void* c16,
                          long long ldc16, float* rstd, int* dev_err, void* stream);

/* y = 2^x for x <= 0 by the FMA-pipe exponential the attention softmax and
 * the loss pass use for part of their exponentials (Cody-Waite reduction and
 * a fitted cubic; relative error <= 7.5e-5; x below -125 gives 2^-125).
 * No reference counterpart: exposed so its error bound can be tested. */
int nsb_op_exp2_poly3(const float* x, float* y, size_t n, void* stream);

/* Row softmax (max-subtracted, exp, normalised). Replaces ns_softmax_kernel
 * (cuda_backend.cpp:432-441) / ns_softmax (codegen.cpp CPU helper). */
int nsb_op_softmax(const float* x, int M, int C, float* out32, void* out16, void* stream);

/* out = a (op) b over n elements, code 0 + 1 - 2 * 3 /, full-size b.
 * Replaces ns_binop_kernel (cuda_backend.cpp:408-419) / ns_binop
 * (codegen.cpp:1267-1278). The backward (no reference counterpart: the
 * reference has no binop gradient) writes da and/or db (either may be NULL). */
int nsb_op_binop(const float* a, const float* b, size_t n, int code, float* out32, void* out16, void* stream);
int nsb_op_binop_bwd(const float* dout, const float* a, const float* b, size_t n, int code, float* da, float* db,
                     void* stream);

/* Inverted dropout with a counter-based mask: element i keeps its value with
 * probability 1 - rate (scaled by 1/(1 - rate)), decided by Philox4x32-10 of
 * (i, step, site) under key (key0, key1); the backward regenerates the same
 * mask. Replaces ns_dropout_fwd_kernel / ns_dropout_mul_kernel
 * (cuda_backend.cpp:778-793), whose curand mask (and the CPU emit's
 * std::mt19937 mask, codegen.cpp:2874-2893) it does not reproduce. */
int nsb_op_dropout_fwd(const float* x, size_t n, float rate, unsigned key0, unsigned key1, unsigned step,
                       unsigned site, float* out32, void* out16, void* stream);
int nsb_op_dropout_bwd(const float* dy, size_t n, float rate, unsigned key0, unsigned key1, unsigned step,
                       unsigned site, float* dx, void* stream);

/* Data movement on row-major fp32 tensors. axis 1: column forms on [rows,
 * cols]; axis 0: row forms. Indices are int64. A scatter keeps the last
 * update of a repeated index (the reference CPU helpers' order); an index
 * outside the source reads 0. Replace ns_transpose2d_kernel,
 * ns_concat2/0_kernel, ns_slice2/slicerows_kernel, ns_index/indexrows_kernel
 * and ns_scatter/scatterrows_kernel (cuda_backend.cpp:93-171). */
int nsb_op_transpose(const float* in, int R, int C, float* out, void* stream);
int nsb_op_concat(const float* a, const float* b, int axis, int rows_a, int rows_b, int ca, int cb, float* out,
                  void* stream);
int nsb_op_slice(const float* in, int axis, int rows, int cols, int start, int end, float* out, void* stream);
int nsb_op_index(const float* in, int axis, int rows, int cols, const long long* idx, int L, float* out,
                 void* stream);
int nsb_op_scatter(const float* in, int axis, int rows, int cols, const long long* idx, int L, const float* upd,
                   float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NS_B200_OPS_H */
