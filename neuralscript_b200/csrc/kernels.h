// Memory-bound kernels of the hot path (launchers). All take device
// pointers and the stream to run on; all are deterministic (fixed reduction
// orders, no float atomics).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsb {

// out[r,:] = W[(int)ids[r], :] (ids fp32, truncated toward zero; ids outside
// [0,V) read row 0). Writes fp32 and/or bf16 outputs.
int embedding_fwd(const float* W, const float* ids, int M, int V, int D, float* out32, __nv_bfloat16* out16,
                  cudaStream_t s);

// dW[v,:] = sum over rows r with (int)ids[r] == v, in increasing r, of
// dout[r,:]; ids outside [0,V) are skipped; untouched rows are zero.
// scratch: at least embedding_bwd_scratch_bytes(M, V) bytes of device memory.
size_t embedding_bwd_scratch_bytes(int M, int V);
// embedding_bwd = embedding_bwd_sort (depends on the ids only) followed by
// embedding_bwd_sum on the same scratch.
int embedding_bwd_sort(const float* ids, int M, int V, void* scratch, cudaStream_t s);
int embedding_bwd_sum(const float* dout, int M, int V, int D, float* dW, const void* scratch, cudaStream_t s);
int embedding_bwd(const float* dout, const float* ids, int M, int V, int D, float* dW, void* scratch,
                  cudaStream_t s);

// Row-wise LayerNorm without affine, eps 1e-5, biased variance.
int layernorm_fwd(const float* x, int M, int D, float* out32, __nv_bfloat16* out16, cudaStream_t s);
// dx = (dy - mean(dy) - xc * mean(xc*dy)) * rstd, statistics from x; then
// dx += add (if given). Writes fp32 and/or bf16.
int layernorm_bwd(const float* dy, const float* x, const float* add, int M, int D, float* dx32, __nv_bfloat16* dx16,
                  cudaStream_t s);
// The same gradient from the LayerNorm's output y and the row's rstd =
// 1 / sqrt(var + eps) (a LayerNorm fused into its producer's GEMM): the
// centred input x - mean(x) is y / rstd. D a multiple of 128, at most 1024.
int layernorm_bwd_from_output(const float* dy, const float* y, const float* rstd, const float* add, int M, int D,
                              float* dx32, __nv_bfloat16* dx16, cudaStream_t s);

// Fused softmax cross-entropy forward + seed gradient, one row per CTA:
//   loss_r = sum_{j: y_j > 0} -log softmax(x)_j      (one-hot labels [M,C])
//   d_rj   = (softmax(x)_j - y_j) / denom
// targets (int32 [M]) replaces labels when labels == nullptr.
int cross_entropy_fwd_bwd(const float* logits, const float* labels, const int* targets, int M, int C, float denom,
                          float* row_loss, float* d32, __nv_bfloat16* d16, cudaStream_t s);

// Completes the head GEMM + cross-entropy fusion: g16 holds the fp16
// logits [M, C] and tlogit the fp32 target logits. Writes row_loss =
// log-sum-exp - logit[target] and overwrites g16 in place with the bf16
// seed (softmax - onehot) / denom. C a multiple of 8, g16 16-byte aligned.
int cross_entropy_finish(void* g16, int M, int C, const int* targets, const float* tlogit, float denom,
                         float* row_loss, cudaStream_t s);

// Mean squared error (sum of squares per row) and seed d = 2 (p - y) / denom.
int mse_fwd_bwd(const float* p, const float* y, int M, int C, float denom, float* row_loss, float* d32,
                __nv_bfloat16* d16, cudaStream_t s);

// out = sum(x[0..n)) in a fixed tree order (single CTA), times scale.
int reduce_sum(const float* x, int n, float scale, float* out, cudaStream_t s);

// Elementwise: out = a + b (fp32 and/or bf16 outputs).
int add_f32(const float* a, const float* b, size_t n, float* out32, __nv_bfloat16* out16, cudaStream_t s);
// out = act(x); optionally bf16 copy.
int act_fwd_f32(const float* x, size_t n, int act, float* out32, __nv_bfloat16* out16, cudaStream_t s);
// out = dy * act'(z) (+ add); z fp32 or bf16.
int act_bwd(const float* dy, const void* z, int z_dtype, int act, const float* add, size_t n, float* out32,
            __nv_bfloat16* out16, cudaStream_t s);
int f32_to_bf16(const float* x, size_t n, __nv_bfloat16* out, cudaStream_t s);
int softmax_rows(const float* x, int M, int C, float* out32, __nv_bfloat16* out16, cudaStream_t s);

// Working copy of a weight: dst[r * ld_dst + col_off + c] = src[r * cols + c]
// for an [rows, cols] fp32 source; dst fp32 or bf16.
int pack_weight(const float* src, int rows, int cols, void* dst, int dst_dtype, long long ld_dst, int col_off,
                cudaStream_t s);

// ---- optimizers -------------------------------------------------------------
struct AdamTensor {
    float* w;
    const float* g;
    float* m;
    float* v;
    long long n;
    float b1t;  // 1 - beta1^t
    float b2t;  // 1 - beta2^t
    // optional working copy refreshed from the updated weight in the same
    // pass: element i = (r, c) of a [n / wk_cols, wk_cols] view goes to
    // wk[r * wk_ld + wk_off + c] (bf16 when wk_bf16, else fp32)
    void* wk = nullptr;
    long long wk_ld = 0;
    int wk_cols = 0;
    int wk_off = 0;
    int wk_bf16 = 0;
    int vec4 = 0;  // all streams 16-byte aligned, n and the copy layout multiples of 4
};
struct AdamHyper {
    float lr, beta1, beta2, one_minus_beta1, one_minus_beta2, eps, decay;
};
// Sets t.vec4 from the pointers and layout.
void adamw_prepare(AdamTensor& t);
// One tensor, descriptor passed by value.
int adamw_single(AdamTensor t, AdamHyper h, cudaStream_t s);
// All tensors in launches of up to kAdamBatch descriptors passed as kernel
// parameters (no staging copy, no host synchronisation).
constexpr int kAdamBatch = 40;
int adamw_multi(const AdamTensor* host_tensors, int count, AdamHyper h, cudaStream_t s);

// m = momentum * m + g
int muon_momentum(float* m, const float* g, long long n, float momentum, cudaStream_t s);
// Modified Gram-Schmidt on an r x c matrix in place (columns if r >= c,
// rows otherwise), one CTA per matrix.
int mgs_orthonormalize(float* G, int r, int c, cudaStream_t s);
// w -= le * o + (decay * lr) * w ; then (if zero_m) m = 0; w16 (optional)
// receives the updated weights in bf16 (a flat working copy)
int muon_apply(float* w, const float* o, float* m, long long n, float le, float decay_lr, int zero_m,
               cudaStream_t s, __nv_bfloat16* w16 = nullptr);
// X /= (||X||_F + eps) as a two-kernel deterministic reduction; scratch >= 1024 floats.
// out = x / (||x||_F + eps); out16 (optional) receives the same values in bf16
int frob_normalize(const float* x, long long n, float eps, float* out, float* scratch, cudaStream_t s,
                   __nv_bfloat16* out16 = nullptr);

}  // namespace nsb
