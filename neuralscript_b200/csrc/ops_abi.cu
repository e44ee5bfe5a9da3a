// Kernel-level C-ABI (include/ns_b200_ops.h): thin argument marshalling onto
// the launchers in gemm.cu, kernels.cu and attention.cu.
#include <cuda_bf16.h>
#include <math.h>

#include "../../include/ns_b200_ops.h"
#include "attention.h"
#include "elementwise.h"
#include "engine.h"
#include "gemm.h"
#include "kernels.h"
#include "moe.h"

using namespace nsb;

static GemmDesc make_desc(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn, const void* B,
                          int b_dtype, long long ldb, int b_mn, int engine) {
    GemmDesc d;
    d.M = M;
    d.N = N;
    d.K = K;
    d.a.ptr = A;
    d.a.dtype = a_dtype;
    d.a.ld = lda;
    d.a.mn_major = a_mn != 0;
    d.b.ptr = B;
    d.b.dtype = b_dtype;
    d.b.ld = ldb;
    d.b.mn_major = b_mn != 0;
    d.engine = engine;
    return d;
}

namespace {
__global__ void exp2_poly3_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = exp2_poly3(x[i]);
}

}  // namespace

extern "C" {

int nsb_op_gemm(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn, const void* B, int b_dtype,
                long long ldb, int b_mn, float alpha, const float* add, long long ld_add, int act, float* c32,
                long long ldc32, void* c16, long long ldc16, int engine, float* workspace, size_t workspace_floats,
                int* dev_err, void* stream) {
    if (M < 0 || N < 0 || K <= 0 || !A || !B) return -1;
    GemmDesc d = make_desc(M, N, K, A, a_dtype, lda, a_mn, B, b_dtype, ldb, b_mn, engine);
    d.ep.alpha = alpha;
    d.ep.add = add;
    d.ep.ld_add = (int)ld_add;
    d.ep.act = act;
    d.ep.c32 = c32;
    d.ep.ld_c32 = (int)ldc32;
    d.ep.c16 = reinterpret_cast<__nv_bfloat16*>(c16);
    d.ep.ld_c16 = (int)ldc16;
    d.workspace = workspace;
    d.workspace_floats = workspace_floats;
    launch_counter() += 1;
    return gemm(d, (cudaStream_t)stream, dev_err);
}

size_t nsb_op_gemm_workspace_floats(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn,
                                    const void* B, int b_dtype, long long ldb, int b_mn, int engine) {
    GemmDesc d = make_desc(M, N, K, A, a_dtype, lda, a_mn, B, b_dtype, ldb, b_mn, engine);
    return gemm_workspace_floats(d);
}

int nsb_op_gemm_uses_tensor_cores(int M, int N, int K, const void* A, int a_dtype, long long lda, int a_mn,
                                  const void* B, int b_dtype, long long ldb, int b_mn, int engine) {
    GemmDesc d = make_desc(M, N, K, A, a_dtype, lda, a_mn, B, b_dtype, ldb, b_mn, engine);
    return gemm_uses_tensor_cores(d) ? 1 : 0;
}

int nsb_op_embedding_fwd(const float* W, const float* ids, int M, int V, int D, float* out32, void* out16,
                         void* stream) {
    return embedding_fwd(W, ids, M, V, D, out32, reinterpret_cast<__nv_bfloat16*>(out16), (cudaStream_t)stream);
}

size_t nsb_op_embedding_bwd_scratch_bytes(int M, int V) { return embedding_bwd_scratch_bytes(M, V); }

int nsb_op_embedding_bwd(const float* dout, const float* ids, int M, int V, int D, float* dW, void* scratch,
                         void* stream) {
    if (!scratch) return -1;
    return embedding_bwd(dout, ids, M, V, D, dW, scratch, (cudaStream_t)stream);
}

int nsb_op_layernorm_fwd(const float* x, int M, int D, float* out32, void* out16, void* stream) {
    return layernorm_fwd(x, M, D, out32, reinterpret_cast<__nv_bfloat16*>(out16), (cudaStream_t)stream);
}

int nsb_op_layernorm_bwd(const float* dy, const float* x, const float* add, int M, int D, float* dx32, void* dx16,
                         void* stream) {
    return layernorm_bwd(dy, x, add, M, D, dx32, reinterpret_cast<__nv_bfloat16*>(dx16), (cudaStream_t)stream);
}

static AttnArgs attn_args(int B, int S, int H, int D, int dtype) {
    AttnArgs a;
    a.B = B;
    a.S = S;
    a.H = H;
    a.D = D;
    a.dh = H > 0 ? D / H : 0;
    a.scale = a.dh > 0 ? 1.0f / sqrtf((float)a.dh) : 1.f;
    a.dtype = dtype;
    return a;
}

int nsb_op_attention_fwd(int B, int S, int H, int D, int dtype, const void* qkv, long long ld_qkv, void* ctx,
                         long long ld_ctx, float* lse, void* stream) {
    if (H <= 0 || D % H) return -1;
    AttnArgs a = attn_args(B, S, H, D, dtype);
    a.qkv = qkv;
    a.ld_qkv = ld_qkv;
    a.ctx = ctx;
    a.ld_ctx = ld_ctx;
    a.lse = lse;
    return attention_fwd(a, (cudaStream_t)stream);
}

int nsb_op_attention_bwd(int B, int S, int H, int D, int dtype, const void* qkv, long long ld_qkv, const void* ctx,
                         long long ld_ctx, const float* lse, const void* dctx, long long ld_dctx, void* dqkv,
                         long long ld_dqkv, float* dvec, void* stream) {
    if (H <= 0 || D % H || !lse || !dvec) return -1;
    AttnArgs a = attn_args(B, S, H, D, dtype);
    a.qkv = qkv;
    a.ld_qkv = ld_qkv;
    a.ctx = const_cast<void*>(ctx);
    a.ld_ctx = ld_ctx;
    a.lse = const_cast<float*>(lse);
    a.dctx = dctx;
    a.ld_dctx = ld_dctx;
    a.dqkv = dqkv;
    a.ld_dqkv = ld_dqkv;
    a.dvec = dvec;
    return attention_bwd(a, (cudaStream_t)stream);
}

int nsb_op_cross_entropy(const float* logits, const float* labels, const int* targets, int M, int C, float denom,
                         float* row_loss, float* d32, void* d16, void* stream) {
    if (!labels && !targets) return -1;
    return cross_entropy_fwd_bwd(logits, labels, targets, M, C, denom, row_loss, d32,
                                 reinterpret_cast<__nv_bfloat16*>(d16), (cudaStream_t)stream);
}

int nsb_op_cross_entropy_finish(void* logits16, int M, int C, const int* targets, const float* tlogit, float denom,
                                float* row_loss, void* stream) {
    if (!logits16 || !targets || !tlogit || !row_loss || M < 0 || C <= 0) return -1;
    launch_counter() += 1;
    return cross_entropy_finish(logits16, M, C, targets, tlogit, denom, row_loss, (cudaStream_t)stream);
}

int nsb_op_reduce_sum(const float* x, int n, float scale, float* out, void* stream) {
    return reduce_sum(x, n, scale, out, (cudaStream_t)stream);
}

int nsb_op_adamw(float* w, const float* g, float* m, float* v, long long n, long long t, float lr, float beta1,
                 float beta2, float one_minus_beta1, float one_minus_beta2, float eps, float decay, void* stream) {
    if (t < 1 || n < 0) return -1;
    AdamTensor a;
    a.w = w;
    a.g = g;
    a.m = m;
    a.v = v;
    a.n = n;
    a.b1t = 1.f - powf(beta1, (float)t);
    a.b2t = 1.f - powf(beta2, (float)t);
    AdamHyper h{lr, beta1, beta2, one_minus_beta1, one_minus_beta2, eps, decay};
    return adamw_single(a, h, (cudaStream_t)stream);
}

int nsb_op_mgs(float* G, int r, int c, void* stream) { return mgs_orthonormalize(G, r, c, (cudaStream_t)stream); }

int nsb_op_moe_route(const float* x, const float* Wg, const unsigned char* active, int M, int D, int E, int* best,
                     float* pb, float* probs, void* stream) {
    if (E <= 0 || E > 64 || D <= 0) return -1;
    return moe_route(x, Wg, active, M, D, E, best, pb, probs, (cudaStream_t)stream);
}

int nsb_op_act_fwd(const float* x, size_t n, int act, float* out32, void* out16, void* stream) {
    return act_fwd_f32(x, n, act, out32, reinterpret_cast<__nv_bfloat16*>(out16), (cudaStream_t)stream);
}

int nsb_op_act_bwd(const float* dy, const float* z, int act, size_t n, float* out32, void* stream) {
    return act_bwd(dy, z, kF32, act, nullptr, n, out32, nullptr, (cudaStream_t)stream);
}


int nsb_op_exp2_poly3(const float* x, float* y, size_t n, void* stream) {
    if (!x || !y) return -1;
    if (n == 0) return 0;
    launch_counter() += 1;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    exp2_poly3_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(x, y, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int nsb_op_softmax(const float* x, int M, int C, float* out32, void* out16, void* stream) {
    if (!x || M < 0 || C <= 0) return -1;
    launch_counter() += 1;
    return softmax_rows(x, M, C, out32, reinterpret_cast<__nv_bfloat16*>(out16), (cudaStream_t)stream);
}

int nsb_op_binop(const float* a, const float* b, size_t n, int code, float* out32, void* out16, void* stream) {
    launch_counter() += 1;
    return binop_fwd(a, b, n, code, out32, reinterpret_cast<__nv_bfloat16*>(out16), (cudaStream_t)stream);
}

int nsb_op_binop_bwd(const float* dout, const float* a, const float* b, size_t n, int code, float* da, float* db,
                     void* stream) {
    launch_counter() += 1;
    return binop_bwd(dout, a, b, n, code, nullptr, da, nullptr, db, (cudaStream_t)stream);
}

static DropoutSite site_of(float rate, unsigned key0, unsigned key1, unsigned step, unsigned site) {
    DropoutSite d;
    d.rate = rate;
    d.key0 = key0;
    d.key1 = key1;
    d.step = step;
    d.site = site;
    return d;
}

int nsb_op_dropout_fwd(const float* x, size_t n, float rate, unsigned key0, unsigned key1, unsigned step,
                       unsigned site, float* out32, void* out16, void* stream) {
    launch_counter() += 1;
    return dropout_fwd(x, n, site_of(rate, key0, key1, step, site), out32, reinterpret_cast<__nv_bfloat16*>(out16),
                       (cudaStream_t)stream);
}

int nsb_op_dropout_bwd(const float* dy, size_t n, float rate, unsigned key0, unsigned key1, unsigned step,
                       unsigned site, float* dx, void* stream) {
    launch_counter() += 1;
    return dropout_bwd(dy, n, site_of(rate, key0, key1, step, site), nullptr, dx, (cudaStream_t)stream);
}

int nsb_op_transpose(const float* in, int R, int C, float* out, void* stream) {
    launch_counter() += 1;
    return transpose2d(in, R, C, out, (cudaStream_t)stream);
}

int nsb_op_concat(const float* a, const float* b, int axis, int rows_a, int rows_b, int ca, int cb, float* out,
                  void* stream) {
    launch_counter() += 1;
    if (axis == 0) {
        if (ca != cb) return -1;
        return concat_rows(a, rows_a, b, rows_b, ca, out, (cudaStream_t)stream);
    }
    if (rows_a != rows_b) return -1;
    return concat_cols(a, ca, b, cb, rows_a, out, nullptr, (cudaStream_t)stream);
}

int nsb_op_slice(const float* in, int axis, int rows, int cols, int start, int end, float* out, void* stream) {
    launch_counter() += 1;
    if (axis == 0) {
        if (start < 0 || end > rows) return -1;
        return slice_rows(in, cols, start, end, out, (cudaStream_t)stream);
    }
    return slice_cols(in, rows, cols, start, end, out, nullptr, (cudaStream_t)stream);
}

int nsb_op_index(const float* in, int axis, int rows, int cols, const long long* idx, int L, float* out,
                 void* stream) {
    launch_counter() += 1;
    const int64_t* ix = reinterpret_cast<const int64_t*>(idx);
    if (axis == 0) return index_rows(in, rows, cols, ix, L, out, (cudaStream_t)stream);
    return index_cols(in, rows, cols, ix, L, out, nullptr, (cudaStream_t)stream);
}

int nsb_op_scatter(const float* in, int axis, int rows, int cols, const long long* idx, int L, const float* upd,
                   float* out, void* stream) {
    launch_counter() += 1;
    const int64_t* ix = reinterpret_cast<const int64_t*>(idx);
    if (axis == 0) return scatter_rows(in, rows, cols, ix, L, upd, out, (cudaStream_t)stream);
    return scatter_cols(in, rows, cols, ix, L, upd, out, nullptr, (cudaStream_t)stream);
}

int nsb_op_gemm_layernorm(int M, int K, const void* A, int dtype, long long lda, const void* B, long long ldb,
                          float alpha, const float* add, long long ld_add, float* c32, long long ldc32, void* c16,
                          long long ldc16, float* rstd, int* dev_err, void* stream) {
    if (M < 0 || K <= 0 || !A || !B || !rstd || (!c32 && !c16)) return -1;
    GemmDesc d = make_desc(M, 512, K, A, dtype, lda, 0, B, dtype, ldb, 1, kEngineTensor);
    d.ep.alpha = alpha;
    d.ep.add = add;
    d.ep.ld_add = (int)ld_add;
    d.ep.c32 = c32;
    d.ep.ld_c32 = (int)ldc32;
    d.ep.c16 = reinterpret_cast<__nv_bfloat16*>(c16);
    d.ep.ld_c16 = (int)ldc16;
    d.ep.ln_rstd = rstd;
    launch_counter() += 1;
    return gemm(d, (cudaStream_t)stream, dev_err);
}

}  // extern "C"
