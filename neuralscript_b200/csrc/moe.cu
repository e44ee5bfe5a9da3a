// Top-1 mixture-of-experts layer (reference ns_moe_fwd and
// ns_moe_grad_{x,wg,we1,we2}, src/codegen/codegen.cpp:1388-1579, 1915-1945;
// CUDA ns_moe_kernel and grads, src/codegen/cuda_backend.cpp:371-689).
//
// Forward:
//   1. router: fp32 logits x . Wg accumulated with fmaf in increasing k (the
//      reference's scalar loop order, so logits are bit-identical), max over
//      live experts, exp weights, top-1 = first maximum of the exp'd
//      weights, softmax over live experts;
//   2. dispatch: stable counting sort of tokens by expert (per-chunk
//      histograms, exclusive scan, warp-ballot ranks), each expert segment
//      padded to a multiple of 128 rows;
//   3. gather x rows into expert order; grouped GEMM GELU(x We1[e]); grouped
//      GEMM (. We2[e]) with the routing weight as a row scale, scattered back
//      to token order in the epilogue.
// Backward recomputes nothing the forward kept (routing, gathered rows,
// hidden activations) and reduces every weight gradient with grouped GEMMs
// over each expert's rows in token order, so results are deterministic
// (the reference accumulates with float atomics).
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"
#include "engine.h"
#include "gemm.h"
#include "kernels.h"
#include "moe.h"

namespace nsb {

struct MoeScratch {
    int D = 0, E = 0, H = 0, mpad = 0, chunks = 0;
    bool linear = false;
    int* best = nullptr;
    float* pb = nullptr;
    float* probs = nullptr;
    int* perm = nullptr;
    int* pos = nullptr;
    int* seg = nullptr;      // [E + 1]
    int* seg_end = nullptr;  // [E]
    int* hist = nullptr;     // [chunks, E]
    void* xs = nullptr;
    float* pbs = nullptr;
    void* hs = nullptr;
    void* hpre = nullptr;
    float* ys = nullptr;
    // backward
    void* dys = nullptr;
    float* dpre2 = nullptr;
    float* dpb = nullptr;
    void* dH = nullptr;
    void* hp = nullptr;
    float* dg = nullptr;
    float* t1 = nullptr;
    float* wg_part = nullptr;  // [ceil(rows / kWgTokens), D, E] partial gate-weight gradients
};

namespace {
constexpr int kRouteTokens = 128;
constexpr int kRouteRegE = 8;  // expert count whose logits the router keeps in registers
constexpr int kChunk = 256;  // tokens per dispatch chunk (one warp each)
constexpr int kWgTokens = 128;  // tokens per partial gate-weight-gradient block
constexpr int kWgMaxE = 8;      // experts handled by the two-pass gate-weight gradient

inline int launch_ok() { return cudaGetLastError() == cudaSuccess ? 0 : -5; }
}  // namespace

// One thread per token; x and Wg staged through shared memory 32 k at a time.
__global__ void __launch_bounds__(kRouteTokens) moe_router_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ Wg,
                                                                  const uint8_t* __restrict__ active, int M, int D,
                                                                  int E, int* __restrict__ best,
                                                                  float* __restrict__ pb,
                                                                  float* __restrict__ probs) {
    extern __shared__ float sh[];
    float* xt = sh;                              // [kRouteTokens][33]
    float* wt = xt + kRouteTokens * 33;          // [32][E]
    float* acc = wt + 32 * E;                    // [kRouteTokens][E]
    const int t0 = blockIdx.x * kRouteTokens;
    const int t = threadIdx.x;
    for (int e = 0; e < E; e++) acc[t * E + e] = 0.f;
    for (int k0 = 0; k0 < D; k0 += 32) {
        __syncthreads();
        for (int i = t; i < kRouteTokens * 32; i += kRouteTokens) {
            int r = i / 32, kk = i % 32;
            int tok = t0 + r, k = k0 + kk;
            xt[r * 33 + kk] = (tok < M && k < D) ? x[(size_t)tok * D + k] : 0.f;
        }
        for (int i = t; i < 32 * E; i += kRouteTokens) {
            int kk = i / E, e = i % E;
            wt[i] = (k0 + kk < D) ? Wg[(size_t)(k0 + kk) * E + e] : 0.f;
        }
        __syncthreads();
        const int kn = min(32, D - k0);
        if (E == kRouteRegE && kn == 32) {
            // the usual case: logits in registers, x read once per k, Wg
            // broadcast; each logit still accumulates in increasing k
            float a[kRouteRegE];
#pragma unroll
            for (int e = 0; e < kRouteRegE; e++) a[e] = acc[t * kRouteRegE + e];
#pragma unroll 8
            for (int kk = 0; kk < 32; kk++) {
                const float xv = xt[t * 33 + kk];
#pragma unroll
                for (int e = 0; e < kRouteRegE; e++) a[e] = fmaf(xv, wt[kk * kRouteRegE + e], a[e]);
            }
#pragma unroll
            for (int e = 0; e < kRouteRegE; e++) acc[t * kRouteRegE + e] = a[e];
        } else {
            for (int e = 0; e < E; e++) {
                float a = acc[t * E + e];
                for (int kk = 0; kk < kn; kk++) a = fmaf(xt[t * 33 + kk], wt[kk * E + e], a);
                acc[t * E + e] = a;
            }
        }
    }
    const int tok = t0 + t;
    if (tok >= M) return;
    float mx = -1.0e30f;
    for (int e = 0; e < E; e++) {
        float a = acc[t * E + e];
        if ((!active || active[e]) && a > mx) mx = a;
    }
    float sum = 0.f;
    int b = -1;
    float wb = 0.f;
    for (int e = 0; e < E; e++) {
        if (active && !active[e]) {
            acc[t * E + e] = 0.f;
            continue;
        }
        // exp in double then rounded: the correctly rounded fp32 value (the
        // reference's glibc expf is within 0.502 ulp of it), so exp-ties that
        // decide the top-1 rule break the same way
        float w = (float)exp((double)(acc[t * E + e] - mx));
        acc[t * E + e] = w;
        sum += w;
        if (b < 0 || w > wb) {
            b = e;
            wb = w;
        }
    }
    best[tok] = b;
    pb[tok] = (sum > 0.f && b >= 0) ? wb / sum : 0.f;
    if (probs)
        for (int e = 0; e < E; e++)
            probs[(size_t)tok * E + e] = ((!active || active[e]) && sum > 0.f) ? acc[t * E + e] / sum : 0.f;
}

// Softmax over live experts and the first-max top-1 rule of the reference
// router (codegen.cpp:1915-1945) from fp32 logits a[0..E).
__device__ __forceinline__ void route_finish(float* a, const uint8_t* __restrict__ active, int E, int tok,
                                             int* __restrict__ best, float* __restrict__ pb,
                                             float* __restrict__ probs) {
    float mx = -1.0e30f;
    for (int e = 0; e < E; e++)
        if ((!active || active[e]) && a[e] > mx) mx = a[e];
    float sum = 0.f;
    int b = -1;
    float wb = 0.f;
    for (int e = 0; e < E; e++) {
        if (active && !active[e]) {
            a[e] = 0.f;
            continue;
        }
        // exp in double then rounded (see moe_router_kernel)
        const float w = (float)exp((double)(a[e] - mx));
        a[e] = w;
        sum += w;
        if (b < 0 || w > wb) {
            b = e;
            wb = w;
        }
    }
    best[tok] = b;
    pb[tok] = (sum > 0.f && b >= 0) ? wb / sum : 0.f;
    if (probs)
        for (int e = 0; e < E; e++)
            probs[(size_t)tok * E + e] = ((!active || active[e]) && sum > 0.f) ? a[e] / sum : 0.f;
}

// Router for 8 experts: a block of 128 threads owns 64 tokens, two
// adjacent threads per token, each accumulating 4 of the logits over all k
// in increasing order with fmaf (the same chain as moe_router_kernel, so
// logits are bit-identical). x streams through shared memory in
// [64 tokens x 128 k] stages, double-buffered with cp.async (coalesced
// 16-byte copies, the next stage in flight while this one is used); Wg
// sits in shared memory as two float4 per k.
constexpr int kR8Tok = 64, kR8K = 128, kR8Ld = kR8K + 4;  // row stride 528 B (16-byte aligned)

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

__global__ void __launch_bounds__(2 * kR8Tok) moe_router8_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ Wg,
                                                                  const uint8_t* __restrict__ active, int M, int D,
                                                                  int* __restrict__ best, float* __restrict__ pb,
                                                                  float* __restrict__ probs) {
    extern __shared__ float4 w4[];  // [D][2], then two x stages [kR8Tok][kR8Ld]
    float* xs = reinterpret_cast<float*>(w4 + 2 * D);
    const int t0 = blockIdx.x * kR8Tok;
    const int nt = min(kR8Tok, M - t0);
    const int nst = D / kR8K;
    auto stage = [&](int s) {
        float* dst = xs + (s & 1) * kR8Tok * kR8Ld;
        // 64 rows x 32 16-byte pieces; rows past M are not copied (their
        // tokens are never finished)
        for (int i = threadIdx.x; i < kR8Tok * (kR8K / 4); i += blockDim.x) {
            const int r = i / (kR8K / 4), q = i % (kR8K / 4);
            if (r < nt) cp_async16(dst + r * kR8Ld + 4 * q, x + (size_t)(t0 + r) * D + s * kR8K + 4 * q);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0);
    for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
        const float* w = Wg + (size_t)(i >> 1) * 8 + (i & 1) * 4;
        w4[i] = make_float4(w[0], w[1], w[2], w[3]);
    }
    const int tok = threadIdx.x >> 1, half = threadIdx.x & 1;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int s = 0; s < nst; s++) {
        if (s + 1 < nst) {
            stage(s + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float4* xr = reinterpret_cast<const float4*>(xs + (s & 1) * kR8Tok * kR8Ld + tok * kR8Ld);
        const float4* wp = w4 + (size_t)s * kR8K * 2 + half;
#pragma unroll 8
        for (int k4 = 0; k4 < kR8K / 4; k4++) {
            const float4 xv = xr[k4];
            const float xk[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float4 w = wp[(4 * k4 + j) * 2];
                a0 = fmaf(xk[j], w.x, a0);
                a1 = fmaf(xk[j], w.y, a1);
                a2 = fmaf(xk[j], w.z, a2);
                a3 = fmaf(xk[j], w.w, a3);
            }
        }
        __syncthreads();  // this stage's buffer is refilled two stages on
    }
    // both halves of the pair gather all 8 logits; the even thread finishes
    const float o0 = __shfl_xor_sync(0xffffffffu, a0, 1), o1 = __shfl_xor_sync(0xffffffffu, a1, 1);
    const float o2 = __shfl_xor_sync(0xffffffffu, a2, 1), o3 = __shfl_xor_sync(0xffffffffu, a3, 1);
    if (tok >= nt || half) return;
    float a[8] = {a0, a1, a2, a3, o0, o1, o2, o3};
    route_finish(a, active, 8, t0 + tok, best, pb, probs);
}

int moe_route(const float* x, const float* Wg, const uint8_t* active, int M, int D, int E, int* best, float* pb,
              float* probs, cudaStream_t s) {
    if (M <= 0) return 0;
    const size_t smem8 = (size_t)D * 32 + 2 * sizeof(float) * kR8Tok * kR8Ld;
    if (E == 8 && D % kR8K == 0 && !(reinterpret_cast<uintptr_t>(x) & 15) && smem8 <= 200 * 1024) {
        if (smem8 > 48 * 1024)
            cudaFuncSetAttribute(moe_router8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem8);
        moe_router8_kernel<<<(unsigned)((M + kR8Tok - 1) / kR8Tok), 2 * kR8Tok, smem8, s>>>(x, Wg, active, M, D, best,
                                                                                          pb, probs);
        return launch_ok();
    }
    size_t smem = sizeof(float) * ((size_t)kRouteTokens * 33 + 32 * E + (size_t)kRouteTokens * E);
    if (smem > 48 * 1024) cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    moe_router_kernel<<<(M + kRouteTokens - 1) / kRouteTokens, kRouteTokens, smem, s>>>(x, Wg, active, M, D, E, best,
                                                                                         pb, probs);
    return launch_ok();
}

// per-chunk expert histogram (one warp per chunk)
__global__ void moe_hist_kernel(const int* __restrict__ best, int M, int E, int* __restrict__ hist) {
    extern __shared__ int cnt[];
    const int c = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += 32) cnt[e] = 0;
    __syncwarp();
    for (int i = threadIdx.x; i < kChunk; i += 32) {
        int t = c * kChunk + i;
        if (t < M) {
            int b = best[t];
            if (b >= 0) atomicAdd(&cnt[b], 1);  // integer counts: order-independent
        }
    }
    __syncwarp();
    for (int e = threadIdx.x; e < E; e += 32) hist[(size_t)c * E + e] = cnt[e];
}

// Segment starts (each padded to 128 rows) and per-chunk bases: hist[c][e]
// (tokens of chunk c routed to expert e) becomes the position of chunk c's
// first such token. One warp per expert column scans the chunks 32 at a
// time with shuffles; the segment starts then follow from the expert
// totals in expert order.
__global__ void moe_scan_kernel(int* __restrict__ hist, int chunks, int E, int* __restrict__ seg,
                                int* __restrict__ seg_end) {
    extern __shared__ int tot[];  // [E] totals, then [E] segment starts
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = warp; e < E; e += nw) {
        int carry = 0;
        for (int c0 = 0; c0 < chunks; c0 += 32) {
            const int c = c0 + lane;
            const int v = c < chunks ? hist[(size_t)c * E + e] : 0;
            int inc = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += n;
            }
            if (c < chunks) hist[(size_t)c * E + e] = carry + inc - v;  // exclusive
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) tot[e] = carry;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int start = 0;
        for (int e = 0; e < E; e++) {
            tot[E + e] = start;
            seg[e] = start;
            seg_end[e] = start + tot[e];
            start += (tot[e] + 127) / 128 * 128;
        }
        seg[E] = start;
    }
    __syncthreads();
    for (int e = warp; e < E; e += nw) {
        const int base = tot[E + e];
        for (int c = lane; c < chunks; c += 32) hist[(size_t)c * E + e] += base;
    }
}

// stable placement: chunk c's tokens in token order, ranks from warp matches
__global__ void moe_place_kernel(const int* __restrict__ best, int M, int E, const int* __restrict__ base,
                                 int* __restrict__ perm, int* __restrict__ pos) {
    extern __shared__ int run[];
    const int c = blockIdx.x, lane = threadIdx.x;
    for (int e = lane; e < E; e += 32) run[e] = base[(size_t)c * E + e];
    __syncwarp();
    for (int i0 = 0; i0 < kChunk; i0 += 32) {
        int t = c * kChunk + i0 + lane;
        int b = t < M ? best[t] : -1;
        unsigned peers = __match_any_sync(0xffffffffu, b);
        int rank = __popc(peers & ((1u << lane) - 1u));
        int p = -1;
        if (b >= 0) p = run[b] + rank;
        __syncwarp();
        if (b >= 0 && rank == __popc(peers) - 1) run[b] += __popc(peers);
        __syncwarp();
        if (t < M) {
            pos[t] = p;
            if (p >= 0) perm[p] = t;
        }
    }
}

__global__ void fill_int_kernel(int* p, int n, int v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

// dst[p] = scale_p * src[perm[p]] (0 for padding rows); also pbs[p].
// perm == nullptr: identity (row p of src), used to scale rows in place order.
template <typename TS, typename TD>
__global__ void moe_gather_kernel(const TS* __restrict__ src, const int* __restrict__ perm, int mpad, int D,
                                  const float* __restrict__ rowscale, TD* __restrict__ dst,
                                  const float* __restrict__ pb, float* __restrict__ pbs) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < mpad; p += gridDim.x * warps) {
        const int t = perm ? perm[p] : p;
        const float sc = (t >= 0 && rowscale) ? rowscale[p] : 1.f;
        for (int c = lane; c < D; c += 32) {
            float v = t >= 0 ? (float)src[(size_t)t * D + c] * sc : 0.f;
            if constexpr (sizeof(TD) == 2) dst[(size_t)p * D + c] = __float2bfloat16_rn(v);
            else dst[(size_t)p * D + c] = v;
        }
        if (pbs && lane == 0) pbs[p] = (t >= 0 && perm) ? pb[t] : 0.f;
    }
}

__device__ __forceinline__ float tof(float v) { return v; }
__device__ __forceinline__ float tof(__nv_bfloat16 v) { return __bfloat162float(v); }

// per sorted row: dpb = sum_a h*dpre2 ; dH = dpre2 * pb * gelu'(hpre) ; hp = h * pb
template <typename T>
__global__ void moe_hidden_grad_kernel(const T* __restrict__ hs, const T* __restrict__ hpre,
                                       const float* __restrict__ dpre2, const float* __restrict__ pbs,
                                       const int* __restrict__ perm, int mpad, int H, float* __restrict__ dpb,
                                       T* __restrict__ dH, T* __restrict__ hp) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < mpad; p += gridDim.x * warps) {
        const bool real = perm[p] >= 0;
        const float pbv = pbs[p];
        float acc = 0.f;
        for (int a = lane; a < H; a += 32) {
            size_t i = (size_t)p * H + a;
            float h = real ? tof(hs[i]) : 0.f;
            float d = real ? dpre2[i] : 0.f;
            acc += h * d;
            float g = real ? d * pbv * act_deriv(tof(hpre[i]), kGeluMoe) : 0.f;
            if constexpr (sizeof(T) == 2) {
                dH[i] = __float2bfloat16_rn(g);
                hp[i] = __float2bfloat16_rn(h * pbv);
            } else {
                dH[i] = g;
                hp[i] = h * pbv;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) dpb[p] = acc;
    }
}

// bf16 form of the above for H a multiple of 256: lane l handles 8
// consecutive columns of every 256-column step (16-byte loads and stores).
__global__ void moe_hidden_grad_bf16x8_kernel(const __nv_bfloat16* __restrict__ hs,
                                              const __nv_bfloat16* __restrict__ hpre,
                                              const float* __restrict__ dpre2, const float* __restrict__ pbs,
                                              const int* __restrict__ perm, int mpad, int H,
                                              float* __restrict__ dpb, __nv_bfloat16* __restrict__ dH,
                                              __nv_bfloat16* __restrict__ hp) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < mpad; p += gridDim.x * warps) {
        const bool real = perm[p] >= 0;
        const float pbv = pbs[p];
        float acc = 0.f;
        for (int a0 = 8 * lane; a0 < H; a0 += 256) {
            const size_t i = (size_t)p * H + a0;
            uint4 go = make_uint4(0, 0, 0, 0), ho = make_uint4(0, 0, 0, 0);
            if (real) {
                const uint4 hv = *reinterpret_cast<const uint4*>(hs + i);
                const uint4 zv = *reinterpret_cast<const uint4*>(hpre + i);
                const float4 d0 = *reinterpret_cast<const float4*>(dpre2 + i);
                const float4 d1 = *reinterpret_cast<const float4*>(dpre2 + i + 4);
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&hv);
                const __nv_bfloat16* z = reinterpret_cast<const __nv_bfloat16*>(&zv);
                const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
                __nv_bfloat16* g16 = reinterpret_cast<__nv_bfloat16*>(&go);
                __nv_bfloat16* h16 = reinterpret_cast<__nv_bfloat16*>(&ho);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float hf = __bfloat162float(h[j]);
                    acc += hf * d[j];
                    g16[j] = __float2bfloat16_rn(d[j] * pbv * act_deriv(__bfloat162float(z[j]), kGeluMoe));
                    h16[j] = __float2bfloat16_rn(hf * pbv);
                }
            }
            *reinterpret_cast<uint4*>(dH + i) = go;
            *reinterpret_cast<uint4*>(hp + i) = ho;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) dpb[p] = acc;
    }
}

// linear experts: dpb = sum_j ys * dys (fp32), per sorted row
__global__ void moe_rowdot_kernel(const float* __restrict__ a, const float* __restrict__ b, int mpad, int D,
                                  float* __restrict__ out) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < mpad; p += gridDim.x * warps) {
        float acc = 0.f;
        for (int c = lane; c < D; c += 32) acc += a[(size_t)p * D + c] * b[(size_t)p * D + c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) out[p] = acc;
    }
}

// out[perm[p]] = pbs[p] * ys[p] (fp32 and/or bf16)
__global__ void moe_scale_scatter_kernel(const float* __restrict__ ys, const float* __restrict__ pbs,
                                         const int* __restrict__ perm, int mpad, int D, float* __restrict__ o32,
                                         __nv_bfloat16* __restrict__ o16) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < mpad; p += gridDim.x * warps) {
        const int t = perm[p];
        if (t < 0) continue;
        for (int c = lane; c < D; c += 32) {
            float v = pbs[p] * ys[(size_t)p * D + c];
            if (o32) o32[(size_t)t * D + c] = v;
            if (o16) o16[(size_t)t * D + c] = __float2bfloat16_rn(v);
        }
    }
}

// dg[i,e] = p[i,e] * ((e == best ? dpb : 0) - dpb * pb)   (token order)
__global__ void moe_gate_grad_kernel(const float* __restrict__ probs, const int* __restrict__ best,
                                     const float* __restrict__ pb, const int* __restrict__ pos,
                                     const float* __restrict__ dpb, int M, int E, float* __restrict__ dg) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M; i += gridDim.x * blockDim.x) {
        const int b = best[i];
        const float d = (b >= 0 && pos[i] >= 0) ? dpb[pos[i]] : 0.f;
        const float sd = d * pb[i];
        for (int e = 0; e < E; e++) dg[(size_t)i * E + e] = probs[(size_t)i * E + e] * ((e == b ? d : 0.f) - sd);
    }
}

// ---------------------------------------------------------------------------
// engine hooks
// ---------------------------------------------------------------------------
static unsigned rows_grid(int rows) {
    int g = (rows + 7) / 8;
    int cap = num_sms() * 16;
    return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

void moe_release(Op& op) {
    delete op.moe;
    op.moe = nullptr;
}

// Gate-weight gradient dWg[D, E] = x^T dg over all tokens, in two passes
// with a fixed summation order (deterministic, no atomics): block (c, y)
// sums tokens [c * kWgTokens, +kWgTokens) in ascending order for 4
// consecutive columns d per thread and every expert; the reduce kernel then
// adds the chunks in ascending order. x is read once, coalesced (a token row
// is 4 KB across the block at D = 1024).
__global__ void __launch_bounds__(256) moe_wg_partial_kernel(const float* __restrict__ x,
                                                             const float* __restrict__ dg, int M, int D, int E,
                                                             float* __restrict__ part) {
    __shared__ float sdg[kWgTokens * kWgMaxE];
    const int c = blockIdx.x;
    const int t0 = c * kWgTokens;
    const int nt = min(kWgTokens, M - t0);
    for (int i = threadIdx.x; i < nt * E; i += blockDim.x) sdg[(i / E) * kWgMaxE + i % E] = dg[(size_t)t0 * E + i];
    __syncthreads();
    const int d = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
    if (d >= D) return;
    float acc[4][kWgMaxE];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int e = 0; e < kWgMaxE; e++) acc[i][e] = 0.f;
    const float* xp = x + (size_t)t0 * D + d;
#pragma unroll 4
    for (int t = 0; t < nt; t++) {
        const float4 xv = *reinterpret_cast<const float4*>(xp + (size_t)t * D);
        const float* g = sdg + t * kWgMaxE;
#pragma unroll
        for (int e = 0; e < kWgMaxE; e++) {
            acc[0][e] = fmaf(xv.x, g[e], acc[0][e]);
            acc[1][e] = fmaf(xv.y, g[e], acc[1][e]);
            acc[2][e] = fmaf(xv.z, g[e], acc[2][e]);
            acc[3][e] = fmaf(xv.w, g[e], acc[3][e]);
        }
    }
    float* out = part + ((size_t)c * D + d) * E;
#pragma unroll
    for (int i = 0; i < 4; i++)
        for (int e = 0; e < E; e++) out[i * E + e] = acc[i][e];
}

__global__ void moe_wg_reduce_kernel(const float* __restrict__ part, int chunks, int n, float* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = 0.f;
#pragma unroll 8
    for (int c = 0; c < chunks; c++) s += part[(size_t)c * n + i];
    out[i] = s;
}

int moe_plan(ns_model* m, Op& op, int mmax, bool train) {
    const LayerSpec& l = m->spec.layers[op.layer];
    MoeScratch* s = new MoeScratch();
    op.moe = s;
    s->D = (int)l.geti("dim", 1);
    s->E = (int)l.geti("experts", 1);
    s->linear = l.gets("expert", "ffn") == "linear";
    s->H = s->linear ? s->D : (int)l.geti("ffn", 4LL * s->D);
    s->mpad = mmax + s->E * 128;
    s->chunks = (mmax + kChunk - 1) / kChunk;
    const size_t es = m->wdt == kBF16 ? 2 : 4;
    const size_t R = mmax, P = s->mpad;
    auto A = [&](size_t b) { return plan_alloc(m, b); };
    s->best = (int*)A(R * 4);
    s->pb = (float*)A(R * 4);
    s->probs = (float*)A(R * s->E * 4);
    s->perm = (int*)A(P * 4);
    s->pos = (int*)A(R * 4);
    s->seg = (int*)A((s->E + 1) * 4);
    s->seg_end = (int*)A(s->E * 4);
    s->hist = (int*)A((size_t)s->chunks * s->E * 4);
    s->xs = A(P * s->D * es);
    s->pbs = (float*)A(P * 4);
    if (s->linear) {
        s->ys = (float*)A(P * s->D * 4);
    } else {
        s->hs = A(P * s->H * es);
        if (train) s->hpre = A(P * s->H * es);
    }
    if (train) {
        s->dys = A(P * s->D * (s->linear ? 4 : es));
        s->dpb = (float*)A(P * 4);
        s->dg = (float*)A(R * s->E * 4);
        s->t1 = (float*)A(R * s->D * 4);
        if (s->E <= kWgMaxE && s->D % 4 == 0)
            s->wg_part = (float*)A((R + kWgTokens - 1) / kWgTokens * (size_t)s->D * s->E * 4);
        if (s->linear) {
            s->dH = A(P * s->D * es);  // pb-scaled dY in the GEMM dtype
        } else {
            s->dpre2 = (float*)A(P * s->H * 4);
            s->dH = A(P * s->H * es);
            s->hp = A(P * s->H * es);
        }
    }
    return 0;
}

static int gemm_run(ns_model* m, GemmDesc& d) {
    if (m->precision == 0) d.engine = kEngineSimt;
    launch_counter() += 1;
    int r = gemm(d, m->stream, m->d_err);
    return r ? -1 : 0;
}

static GemmOperand op_of(const void* p, int dt, long long ld, bool mn) {
    GemmOperand o;
    o.ptr = p;
    o.dtype = dt;
    o.ld = ld;
    o.mn_major = mn;
    return o;
}

int moe_forward(ns_model* m, Op& op, int M, bool train) {
    MoeScratch* s = op.moe;
    const Spec& sp = m->spec;
    Val& in = m->vals[op.in];
    Val& out = m->vals[op.out];
    const int D = s->D, E = s->E, H = s->H, dt = m->wdt;
    const WeightInfo& wg = sp.weights[op.widx];
    cudaStream_t st = m->stream;
    if (m->moe_active_count == 0) {
        if (out.f32) cudaMemsetAsync(out.f32, 0, sizeof(float) * (size_t)M * D, st);
        if (out.h16) cudaMemsetAsync(out.h16, 0, 2 * (size_t)M * D, st);
        return 0;
    }
    const std::string lname = sp.layers[op.layer].name;
    int reg = region_open(m, "fwd:" + lname + ".route");
    launch_counter() += 1;
    if (moe_route(in.f32, m->d_w + wg.off, m->d_active, M, D, E, s->best, s->pb, s->probs, st)) return -1;
    const int chunks = (M + kChunk - 1) / kChunk;
    const int mpad = M + E * 128;
    launch_counter() += 4;
    moe_hist_kernel<<<chunks, 32, sizeof(int) * E, st>>>(s->best, M, E, s->hist);
    moe_scan_kernel<<<1, 32 * (E < 32 ? E : 32), sizeof(int) * 2 * E, st>>>(s->hist, chunks, E, s->seg, s->seg_end);
    fill_int_kernel<<<(mpad + 255) / 256, 256, 0, st>>>(s->perm, mpad, -1);
    moe_place_kernel<<<chunks, 32, sizeof(int) * E, st>>>(s->best, M, E, s->hist, s->perm, s->pos);
    launch_counter() += 1;
    if (dt == kBF16)
        moe_gather_kernel<__nv_bfloat16, __nv_bfloat16><<<rows_grid(mpad), 256, 0, st>>>(
            in.h16, s->perm, mpad, D, nullptr, (__nv_bfloat16*)s->xs, s->pb, s->pbs);
    else
        moe_gather_kernel<float, float><<<rows_grid(mpad), 256, 0, st>>>(in.f32, s->perm, mpad, D, nullptr,
                                                                          (float*)s->xs, s->pb, s->pbs);
    region_close(m, reg);
    if (launch_ok()) return -1;
    reg = region_open(m, "fwd:" + lname + ".experts");
    const WeightInfo& w1 = sp.weights[op.widx + 1];
    if (s->linear) {
        GemmDesc g;  // ys = xs We[e]   (unscaled; scaled + scattered below)
        g.M = mpad;
        g.N = D;
        g.K = D;
        g.a = op_of(s->xs, dt, D, false);
        g.b = op_of(m->wk[op.widx + 1], dt, D, true);
        g.groups = E;
        g.seg = s->seg;
        g.seg_end = s->seg_end;
        g.b_group_stride = (long long)D * D;
        g.ep.c32 = s->ys;
        g.ep.ld_c32 = D;
        if (gemm_run(m, g)) return -1;
        launch_counter() += 1;
        moe_scale_scatter_kernel<<<rows_grid(mpad), 256, 0, st>>>(s->ys, s->pbs, s->perm, mpad, D, out.f32, out.h16);
        region_close(m, reg);
        (void)w1;
        return launch_ok();
    }
    GemmDesc g1;  // hs = GELU(xs We1[e])
    g1.M = mpad;
    g1.N = H;
    g1.K = D;
    g1.a = op_of(s->xs, dt, D, false);
    g1.b = op_of(m->wk[op.widx + 1], dt, H, true);
    g1.groups = E;
    g1.seg = s->seg;
    g1.seg_end = s->seg_end;
    g1.b_group_stride = (long long)D * H;
    g1.ep.act = kGeluMoe;
    if (train) {
        g1.ep.z = s->hpre;
        g1.ep.z_dtype = dt;
        g1.ep.ld_z = H;
    }
    if (dt == kBF16) {
        g1.ep.c16 = (__nv_bfloat16*)s->hs;
        g1.ep.ld_c16 = H;
    } else {
        g1.ep.c32 = (float*)s->hs;
        g1.ep.ld_c32 = H;
    }
    if (gemm_run(m, g1)) return -1;
    GemmDesc g2;  // out[perm] = pb * (hs We2[e])
    g2.M = mpad;
    g2.N = D;
    g2.K = H;
    g2.a = op_of(s->hs, dt, H, false);
    g2.b = op_of(m->wk[op.widx + 2], dt, D, true);
    g2.groups = E;
    g2.seg = s->seg;
    g2.seg_end = s->seg_end;
    g2.b_group_stride = (long long)H * D;
    g2.ep.row_scale = s->pbs;
    g2.ep.out_rows = s->perm;
    g2.ep.c32 = out.f32;
    g2.ep.ld_c32 = D;
    g2.ep.c16 = out.h16;
    g2.ep.ld_c16 = D;
    const int rc = gemm_run(m, g2);
    region_close(m, reg);
    return rc;
}

int moe_backward(ns_model* m, Op& op, int M) {
    MoeScratch* s = op.moe;
    const Spec& sp = m->spec;
    Val& in = m->vals[op.in];
    Val& out = m->vals[op.out];
    const int D = s->D, E = s->E, H = s->H, dt = m->wdt;
    const int mpad = M + E * 128;
    cudaStream_t st = m->stream;
    const WeightInfo& wg = sp.weights[op.widx];
    const WeightInfo& w1 = sp.weights[op.widx + 1];
    if (m->moe_active_count == 0) {
        cudaMemsetAsync(m->d_g + wg.off, 0, sizeof(float) * wg.count, st);
        cudaMemsetAsync(m->d_g + w1.off, 0, sizeof(float) * w1.count, st);
        if (!s->linear) cudaMemsetAsync(m->d_g + sp.weights[op.widx + 2].off, 0, sizeof(float) * w1.count, st);
        return 0;
    }
    const float* dY = out.gcur;
    const std::string lname = sp.layers[op.layer].name;
    int reg = region_open(m, "bwd:" + lname + ".experts");
    launch_counter() += 1;
    if (s->linear) {
        moe_gather_kernel<float, float><<<rows_grid(mpad), 256, 0, st>>>(dY, s->perm, mpad, D, nullptr,
                                                                          (float*)s->dys, nullptr, nullptr);
        launch_counter() += 2;
        moe_rowdot_kernel<<<rows_grid(mpad), 256, 0, st>>>(s->ys, (float*)s->dys, mpad, D, s->dpb);
        if (dt == kBF16)
            moe_gather_kernel<float, __nv_bfloat16><<<rows_grid(mpad), 256, 0, st>>>(
                (float*)s->dys, nullptr, mpad, D, s->pbs, (__nv_bfloat16*)s->dH, nullptr, nullptr);
        else
            moe_gather_kernel<float, float><<<rows_grid(mpad), 256, 0, st>>>((float*)s->dys, nullptr, mpad, D, s->pbs,
                                                                             (float*)s->dH, nullptr, nullptr);
    } else {
        if (dt == kBF16)
            moe_gather_kernel<float, __nv_bfloat16><<<rows_grid(mpad), 256, 0, st>>>(
                dY, s->perm, mpad, D, nullptr, (__nv_bfloat16*)s->dys, nullptr, nullptr);
        else
            moe_gather_kernel<float, float><<<rows_grid(mpad), 256, 0, st>>>(dY, s->perm, mpad, D, nullptr,
                                                                             (float*)s->dys, nullptr, nullptr);
        GemmDesc g;  // dpre2 = dys We2[e]^T
        g.M = mpad;
        g.N = H;
        g.K = D;
        g.a = op_of(s->dys, dt, D, false);
        g.b = op_of(m->wk[op.widx + 2], dt, D, false);
        g.groups = E;
        g.seg = s->seg;
        g.seg_end = s->seg_end;
        g.b_group_stride = (long long)H * D;
        g.ep.c32 = s->dpre2;
        g.ep.ld_c32 = H;
        if (gemm_run(m, g)) return -1;
        launch_counter() += 1;
        if (dt == kBF16 && H % 256 == 0)
            moe_hidden_grad_bf16x8_kernel<<<rows_grid(mpad), 256, 0, st>>>(
                (const __nv_bfloat16*)s->hs, (const __nv_bfloat16*)s->hpre, s->dpre2, s->pbs, s->perm, mpad, H,
                s->dpb, (__nv_bfloat16*)s->dH, (__nv_bfloat16*)s->hp);
        else if (dt == kBF16)
            moe_hidden_grad_kernel<__nv_bfloat16><<<rows_grid(mpad), 256, 0, st>>>(
                (const __nv_bfloat16*)s->hs, (const __nv_bfloat16*)s->hpre, s->dpre2, s->pbs, s->perm, mpad, H,
                s->dpb, (__nv_bfloat16*)s->dH, (__nv_bfloat16*)s->hp);
        else
            moe_hidden_grad_kernel<float><<<rows_grid(mpad), 256, 0, st>>>(
                (const float*)s->hs, (const float*)s->hpre, s->dpre2, s->pbs, s->perm, mpad, H, s->dpb,
                (float*)s->dH, (float*)s->hp);
        const WeightInfo& w2 = sp.weights[op.widx + 2];
        GemmDesc gw2;  // dWe2[e] = (h pb)^T dys over the expert's rows
        gw2.M = H;
        gw2.N = D;
        gw2.K = mpad;
        gw2.a = op_of(s->hp, dt, H, true);
        gw2.b = op_of(s->dys, dt, D, true);
        gw2.groups = E;
        gw2.seg = s->seg;
        gw2.seg_end = s->seg_end;
        gw2.group_k = true;
        gw2.c_group_stride = (long long)H * D;
        gw2.ep.c32 = m->d_g + w2.off;
        gw2.ep.ld_c32 = D;
        if (gemm_run(m, gw2)) return -1;
    }
    if (launch_ok()) return -1;
    // dWe1[e] = xs^T dH  (linear: dWe = xs^T (pb dY))
    GemmDesc gw1;
    gw1.M = D;
    gw1.N = H;
    gw1.K = mpad;
    gw1.a = op_of(s->xs, dt, D, true);
    gw1.b = op_of(s->dH, dt, H, true);
    gw1.groups = E;
    gw1.seg = s->seg;
    gw1.seg_end = s->seg_end;
    gw1.group_k = true;
    gw1.c_group_stride = (long long)D * H;
    gw1.ep.c32 = m->d_g + w1.off;
    gw1.ep.ld_c32 = H;
    if (gemm_run(m, gw1)) return -1;
    region_close(m, reg);
    reg = region_open(m, "bwd:" + lname + ".gate");
    // gate path
    launch_counter() += 1;
    moe_gate_grad_kernel<<<(M + 255) / 256, 256, 0, st>>>(s->probs, s->best, s->pb, s->pos, s->dpb, M, E, s->dg);
    if (s->wg_part && m->precision != 0 && !(reinterpret_cast<uintptr_t>(in.f32) & 15)) {
        // dWg = x^T dg: two fixed-order passes over the tokens
        const int chunks = (M + kWgTokens - 1) / kWgTokens;
        launch_counter() += 2;
        moe_wg_partial_kernel<<<dim3(chunks, (D / 4 + 255) / 256), 256, 0, st>>>(in.f32, s->dg, M, D, E, s->wg_part);
        moe_wg_reduce_kernel<<<(D * E + 255) / 256, 256, 0, st>>>(s->wg_part, chunks, D * E, m->d_g + wg.off);
        if (launch_ok()) return -1;
    } else {
        GemmDesc gg;  // dWg = x^T dg (fp32 parity mode: k-sequential FMA order)
        gg.M = D;
        gg.N = E;
        gg.K = M;
        gg.a = op_of(in.f32, kF32, D, true);
        gg.b = op_of(s->dg, kF32, E, true);
        gg.engine = kEngineSimt;
        gg.ep.c32 = m->d_g + wg.off;
        gg.ep.ld_c32 = E;
        if (gemm_run(m, gg)) return -1;
    }
    region_close(m, reg);
    if (!in.gbuf) return 0;
    GemmDesc gx;  // t1 = dH We1[e]^T scattered to tokens (+ running total)
    gx.M = mpad;
    gx.N = D;
    gx.K = H;
    gx.a = op_of(s->dH, dt, H, false);
    gx.b = op_of(m->wk[op.widx + 1], dt, H, false);
    gx.groups = E;
    gx.seg = s->seg;
    gx.seg_end = s->seg_end;
    gx.b_group_stride = (long long)D * H;
    gx.ep.out_rows = s->perm;
    gx.ep.c32 = s->t1;
    gx.ep.ld_c32 = D;
    if (gemm_run(m, gx)) return -1;
    GemmDesc gd;  // dx = dg Wg^T + t1 (+ running total)
    gd.M = M;
    gd.N = D;
    gd.K = E;
    gd.a = op_of(s->dg, kF32, E, false);
    gd.b = op_of(m->d_w + wg.off, kF32, E, false);
    gd.engine = kEngineSimt;
    gd.ep.add = s->t1;
    gd.ep.ld_add = D;
    gd.ep.c32 = in.gbuf;
    gd.ep.ld_c32 = D;
    if (gemm_run(m, gd)) return -1;
    if (in.gcur) {
        launch_counter() += 1;
        if (add_f32(in.gbuf, in.gcur, (size_t)M * D, in.gbuf, nullptr, st)) return -1;
    }
    in.gcur = in.gbuf;
    return 0;
}

// ---------------------------------------------------------------------------
// Expert lifecycle on the device (merge / birth), grid-stride over the gate
// column and the expert matrices; the arithmetic is the reference's, element
// for element: 0.5f * (a + b) and src + noise in fp32.
// ---------------------------------------------------------------------------
__global__ void expert_merge_kernel(float* w, ExpertGeom g, int a, int b) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (size_t k = t0; k < g.dim; k += stride) {
        float* pa = w + g.off_g + k * g.cap + a;
        *pa = 0.5f * (*pa + w[g.off_g + k * g.cap + b]);
    }
    for (size_t q = t0; q < g.n1; q += stride) {
        float* pa = w + g.off_e1 + (size_t)a * g.n1 + q;
        *pa = 0.5f * (*pa + w[g.off_e1 + (size_t)b * g.n1 + q]);
        if (!g.linear) {
            float* p2 = w + g.off_e2 + (size_t)a * g.n1 + q;
            *p2 = 0.5f * (*p2 + w[g.off_e2 + (size_t)b * g.n1 + q]);
        }
    }
}

__global__ void expert_birth_kernel(float* w, ExpertGeom g, int src, int e, const float* __restrict__ noise) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (size_t k = t0; k < g.dim; k += stride)
        w[g.off_g + k * g.cap + e] = w[g.off_g + k * g.cap + src] + noise[k];
    for (size_t q = t0; q < g.n1; q += stride) {
        w[g.off_e1 + (size_t)e * g.n1 + q] = w[g.off_e1 + (size_t)src * g.n1 + q] + noise[g.dim + q];
        if (!g.linear) w[g.off_e2 + (size_t)e * g.n1 + q] = w[g.off_e2 + (size_t)src * g.n1 + q] + noise[g.dim + g.n1 + q];
    }
}

static unsigned lifecycle_blocks(const ExpertGeom& g) {
    const size_t n = g.n1 > g.dim ? g.n1 : g.dim;
    size_t b = (n + 255) / 256;
    return (unsigned)(b > 148 * 8 ? 148 * 8 : (b ? b : 1));
}

int expert_merge_device(float* w, const ExpertGeom& g, int a, int b, cudaStream_t s) {
    expert_merge_kernel<<<lifecycle_blocks(g), 256, 0, s>>>(w, g, a, b);
    return launch_ok();
}

int expert_birth_device(float* w, const ExpertGeom& g, int src, int e, const float* noise, cudaStream_t s) {
    expert_birth_kernel<<<lifecycle_blocks(g), 256, 0, s>>>(w, g, src, e, noise);
    return launch_ok();
}

}  // namespace nsb
