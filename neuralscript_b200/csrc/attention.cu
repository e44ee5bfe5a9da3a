// Multi-head attention core, per (sequence, head): softmax(Q K^T * scale) V,
// non-causal, with scale = 1/sqrt(dh) applied to the finished dot product as
// the reference does (src/codegen/codegen.cpp:1757-1767).
//
// Layout: qkv [M, ld] with Q at column 0, K at column D, V at column 2D,
// head h at columns h*dh .. h*dh+dh-1 of each block (the output of one
// fused x . [Wq|Wk|Wv] GEMM); ctx [M, D] with heads concatenated, exactly the
// reference's out[(b*S+i)*D + h*Dk + d]. Sequences are consecutive runs of S
// rows.
//
// This is the SIMT path: one group of TPR = DHP/32 threads per query (or
// key) row, each owning 32 head dimensions; K/V (or Q/dO) tiles staged in
// shared memory and read as broadcasts; online softmax per 64-key tile; the
// forward saves the row log-sum-exp so the backward recomputes P without
// storing it (dQ pass over keys, dK/dV pass over queries; no atomics).
#include <cuda_bf16.h>
#include <math.h>

#include "attention.h"
#include "common.cuh"

namespace nsb {

namespace {

template <typename T>
__device__ __forceinline__ float ldv(const T* p, size_t i);
template <>
__device__ __forceinline__ float ldv<float>(const float* p, size_t i) {
    return p[i];
}
template <>
__device__ __forceinline__ float ldv<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
    return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void stv(T* p, size_t i, float v);
template <>
__device__ __forceinline__ void stv<float>(float* p, size_t i, float v) {
    p[i] = v;
}
template <>
__device__ __forceinline__ void stv<__nv_bfloat16>(__nv_bfloat16* p, size_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
}

template <int TPR>
__device__ __forceinline__ float group_sum(float v) {
    if (TPR >= 2) v += __shfl_xor_sync(0xffffffffu, v, 1);
    if (TPR >= 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

constexpr int ROWS = 64;  // query (or key) rows per CTA
// keys (or queries) per shared-memory tile; two fp32 tiles stay under the
// 48 KB static shared-memory limit
template <int DHP>
struct Tile {
    static constexpr int KT = DHP > 64 ? 32 : 64;
};

}  // namespace

// grid (ceil(S/ROWS), H, B), block ROWS*TPR threads.
template <typename T, int DHP>
__global__ void __launch_bounds__(ROWS*(DHP / 32)) attn_fwd_kernel(const T* __restrict__ qkv, long long ld, int D,
                                                                  int S, int dh, float scale, T* __restrict__ ctx,
                                                                  long long ld_ctx, float* __restrict__ lse) {
    constexpr int TPR = DHP / 32;
    constexpr int KT = Tile<DHP>::KT;
    __shared__ float Ks[KT][DHP + 1];
    __shared__ float Vs[KT][DHP + 1];
    const int b = blockIdx.z, h = blockIdx.y;
    const int tid = threadIdx.x;
    const int lr = tid / TPR, part = tid % TPR;
    const int i = blockIdx.x * ROWS + lr;
    const bool valid = i < S;
    const size_t row = (size_t)b * S + (valid ? i : 0);
    const int d0 = part * 32;
    float q[32], o[32];
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        q[d] = (valid && dd < dh) ? ldv(qkv, row * ld + h * dh + dd) : 0.f;
        o[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j0 = 0; j0 < S; j0 += KT) {
        __syncthreads();
        for (int e = tid; e < KT * DHP; e += blockDim.x) {
            int jj = e / DHP, dd = e % DHP;
            int j = j0 + jj;
            float kv = 0.f, vv = 0.f;
            if (j < S && dd < dh) {
                size_t r = ((size_t)b * S + j) * ld;
                kv = ldv(qkv, r + D + h * dh + dd);
                vv = ldv(qkv, r + 2 * D + h * dh + dd);
            }
            Ks[jj][dd] = kv;
            Vs[jj][dd] = vv;
        }
        __syncthreads();
        const int kn = min(KT, S - j0);
        float s[KT];
        float tmax = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < KT; jj++) {
            float a = 0.f;
#pragma unroll
            for (int d = 0; d < 32; d++) a += q[d] * Ks[jj][d0 + d];
            a = group_sum<TPR>(a) * scale;
            s[jj] = jj < kn ? a : -INFINITY;
            tmax = fmaxf(tmax, s[jj]);
        }
        const float mnew = fmaxf(m, tmax);
        const float corr = expf(m - mnew);
        l *= corr;
#pragma unroll
        for (int d = 0; d < 32; d++) o[d] *= corr;
#pragma unroll
        for (int jj = 0; jj < KT; jj++) {
            const float p = jj < kn ? expf(s[jj] - mnew) : 0.f;
            l += p;
#pragma unroll
            for (int d = 0; d < 32; d++) o[d] += p * Vs[jj][d0 + d];
        }
        m = mnew;
    }
    if (!valid) return;
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        if (dd < dh) stv(ctx, row * ld_ctx + h * dh + dd, o[d] * inv);
    }
    if (lse && part == 0) lse[((size_t)b * gridDim.y + h) * S + i] = m + logf(l);
}

// dQ pass: one query row per thread group. Also stores Dv[i] = dO_i . O_i.
template <typename T, int DHP>
__global__ void __launch_bounds__(ROWS*(DHP / 32)) attn_bwd_dq_kernel(
    const T* __restrict__ qkv, long long ld, int D, int S, int dh, float scale, const T* __restrict__ ctx,
    long long ld_ctx, const T* __restrict__ dctx, long long ld_dctx, const float* __restrict__ lse,
    float* __restrict__ Dv, T* __restrict__ dqkv, long long ld_dqkv) {
    constexpr int TPR = DHP / 32;
    constexpr int KT = Tile<DHP>::KT;
    __shared__ float Ks[KT][DHP + 1];
    __shared__ float Vs[KT][DHP + 1];
    const int b = blockIdx.z, h = blockIdx.y, H = gridDim.y;
    const int tid = threadIdx.x;
    const int lr = tid / TPR, part = tid % TPR;
    const int i = blockIdx.x * ROWS + lr;
    const bool valid = i < S;
    const size_t row = (size_t)b * S + (valid ? i : 0);
    const int d0 = part * 32;
    float q[32], g[32], dq[32];
    float dd_dot = 0.f;
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        bool in = valid && dd < dh;
        q[d] = in ? ldv(qkv, row * ld + h * dh + dd) : 0.f;
        g[d] = in ? ldv(dctx, row * ld_dctx + h * dh + dd) : 0.f;
        float ov = in ? ldv(ctx, row * ld_ctx + h * dh + dd) : 0.f;
        dd_dot += g[d] * ov;
        dq[d] = 0.f;
    }
    const float Di = group_sum<TPR>(dd_dot);
    const float L = valid ? lse[((size_t)b * H + h) * S + i] : 0.f;
    for (int j0 = 0; j0 < S; j0 += KT) {
        __syncthreads();
        for (int e = tid; e < KT * DHP; e += blockDim.x) {
            int jj = e / DHP, dd = e % DHP;
            int j = j0 + jj;
            float kv = 0.f, vv = 0.f;
            if (j < S && dd < dh) {
                size_t r = ((size_t)b * S + j) * ld;
                kv = ldv(qkv, r + D + h * dh + dd);
                vv = ldv(qkv, r + 2 * D + h * dh + dd);
            }
            Ks[jj][dd] = kv;
            Vs[jj][dd] = vv;
        }
        __syncthreads();
        const int kn = min(KT, S - j0);
        for (int jj = 0; jj < kn; jj++) {
            float a = 0.f, bp = 0.f;
#pragma unroll
            for (int d = 0; d < 32; d++) {
                a += q[d] * Ks[jj][d0 + d];
                bp += g[d] * Vs[jj][d0 + d];
            }
            a = group_sum<TPR>(a) * scale;
            bp = group_sum<TPR>(bp);
            const float p = expf(a - L);
            const float ds = p * (bp - Di);
#pragma unroll
            for (int d = 0; d < 32; d++) dq[d] += ds * Ks[jj][d0 + d];
        }
    }
    if (!valid) return;
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        if (dd < dh) stv(dqkv, row * ld_dqkv + h * dh + dd, dq[d] * scale);
    }
    if (part == 0) Dv[((size_t)b * H + h) * S + i] = Di;
}

// dK/dV pass: one key row per thread group, looping over query tiles.
template <typename T, int DHP>
__global__ void __launch_bounds__(ROWS*(DHP / 32)) attn_bwd_dkv_kernel(
    const T* __restrict__ qkv, long long ld, int D, int S, int dh, float scale, const T* __restrict__ dctx,
    long long ld_dctx, const float* __restrict__ lse, const float* __restrict__ Dv, T* __restrict__ dqkv,
    long long ld_dqkv) {
    constexpr int TPR = DHP / 32;
    constexpr int KT = Tile<DHP>::KT;
    __shared__ float Qs[KT][DHP + 1];
    __shared__ float Gs[KT][DHP + 1];
    __shared__ float Ls[KT], Ds[KT];
    const int b = blockIdx.z, h = blockIdx.y, H = gridDim.y;
    const int tid = threadIdx.x;
    const int lr = tid / TPR, part = tid % TPR;
    const int j = blockIdx.x * ROWS + lr;
    const bool valid = j < S;
    const size_t row = (size_t)b * S + (valid ? j : 0);
    const int d0 = part * 32;
    float k[32], v[32], dk[32], dv[32];
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        bool in = valid && dd < dh;
        k[d] = in ? ldv(qkv, row * ld + D + h * dh + dd) : 0.f;
        v[d] = in ? ldv(qkv, row * ld + 2 * D + h * dh + dd) : 0.f;
        dk[d] = 0.f;
        dv[d] = 0.f;
    }
    for (int i0 = 0; i0 < S; i0 += KT) {
        __syncthreads();
        for (int e = tid; e < KT * DHP; e += blockDim.x) {
            int ii = e / DHP, dd = e % DHP;
            int i = i0 + ii;
            float qv = 0.f, gv = 0.f;
            if (i < S && dd < dh) {
                size_t r = (size_t)b * S + i;
                qv = ldv(qkv, r * ld + h * dh + dd);
                gv = ldv(dctx, r * ld_dctx + h * dh + dd);
            }
            Qs[ii][dd] = qv;
            Gs[ii][dd] = gv;
        }
        for (int e = tid; e < KT; e += blockDim.x) {
            int i = i0 + e;
            Ls[e] = i < S ? lse[((size_t)b * H + h) * S + i] : 0.f;
            Ds[e] = i < S ? Dv[((size_t)b * H + h) * S + i] : 0.f;
        }
        __syncthreads();
        const int qn = min(KT, S - i0);
        for (int ii = 0; ii < qn; ii++) {
            float a = 0.f, bp = 0.f;
#pragma unroll
            for (int d = 0; d < 32; d++) {
                a += Qs[ii][d0 + d] * k[d];
                bp += Gs[ii][d0 + d] * v[d];
            }
            a = group_sum<TPR>(a) * scale;
            bp = group_sum<TPR>(bp);
            const float p = expf(a - Ls[ii]);
            const float ds = p * (bp - Ds[ii]);
#pragma unroll
            for (int d = 0; d < 32; d++) {
                dv[d] += p * Gs[ii][d0 + d];
                dk[d] += ds * Qs[ii][d0 + d];
            }
        }
    }
    if (!valid) return;
#pragma unroll
    for (int d = 0; d < 32; d++) {
        int dd = d0 + d;
        if (dd < dh) {
            stv(dqkv, row * ld_dqkv + D + h * dh + dd, dk[d] * scale);
            stv(dqkv, row * ld_dqkv + 2 * D + h * dh + dd, dv[d]);
        }
    }
}

template <typename T, int DHP>
static int fwd_launch(const AttnArgs& a, cudaStream_t s) {
    dim3 grid((a.S + ROWS - 1) / ROWS, a.H, a.B);
    attn_fwd_kernel<T, DHP><<<grid, ROWS * (DHP / 32), 0, s>>>(
        reinterpret_cast<const T*>(a.qkv), a.ld_qkv, a.D, a.S, a.dh, a.scale, reinterpret_cast<T*>(a.ctx), a.ld_ctx,
        a.lse);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

template <typename T, int DHP>
static int bwd_launch(const AttnArgs& a, cudaStream_t s) {
    dim3 grid((a.S + ROWS - 1) / ROWS, a.H, a.B);
    attn_bwd_dq_kernel<T, DHP><<<grid, ROWS * (DHP / 32), 0, s>>>(
        reinterpret_cast<const T*>(a.qkv), a.ld_qkv, a.D, a.S, a.dh, a.scale, reinterpret_cast<const T*>(a.ctx),
        a.ld_ctx, reinterpret_cast<const T*>(a.dctx), a.ld_dctx, a.lse, a.dvec, reinterpret_cast<T*>(a.dqkv),
        a.ld_dqkv);
    attn_bwd_dkv_kernel<T, DHP><<<grid, ROWS * (DHP / 32), 0, s>>>(
        reinterpret_cast<const T*>(a.qkv), a.ld_qkv, a.D, a.S, a.dh, a.scale, reinterpret_cast<const T*>(a.dctx),
        a.ld_dctx, a.lse, a.dvec, reinterpret_cast<T*>(a.dqkv), a.ld_dqkv);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int attention_fwd(const AttnArgs& a, cudaStream_t s) {
    if (a.B <= 0 || a.S <= 0) return 0;
    if (a.dh > 128) return -1;
    if (attention_tc_supported(a)) return attention_tc_fwd(a, s, a.err);
    const bool bf = a.dtype == kBF16;
    if (a.dh <= 32) return bf ? fwd_launch<__nv_bfloat16, 32>(a, s) : fwd_launch<float, 32>(a, s);
    if (a.dh <= 64) return bf ? fwd_launch<__nv_bfloat16, 64>(a, s) : fwd_launch<float, 64>(a, s);
    return bf ? fwd_launch<__nv_bfloat16, 128>(a, s) : fwd_launch<float, 128>(a, s);
}

int attention_bwd_launches(const AttnArgs& a) { return attention_tc_bwd_supported(a) ? 1 : 2; }

int attention_bwd(const AttnArgs& a, cudaStream_t s) {
    if (a.B <= 0 || a.S <= 0) return 0;
    if (a.dh > 128) return -1;
    if (attention_tc_bwd_supported(a)) return attention_tc_bwd(a, s, a.err);
    const bool bf = a.dtype == kBF16;
    if (a.dh <= 32) return bf ? bwd_launch<__nv_bfloat16, 32>(a, s) : bwd_launch<float, 32>(a, s);
    if (a.dh <= 64) return bf ? bwd_launch<__nv_bfloat16, 64>(a, s) : bwd_launch<float, 64>(a, s);
    return bf ? bwd_launch<__nv_bfloat16, 128>(a, s) : bwd_launch<float, 128>(a, s);
}

}  // namespace nsb
