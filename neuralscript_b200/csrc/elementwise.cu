// Elementwise and data-movement kernels (see elementwise.h).
//
// Reference computations replaced (MrModelOS/NeuralScript):
//   ns_binop_kernel                src/codegen/cuda_backend.cpp:408-419
//   ns_dropout_fwd/mul_kernel      src/codegen/cuda_backend.cpp:778-793
//   data-movement kernels          src/codegen/cuda_backend.cpp:93-171
// Memory-bound: each launch is a grid-stride loop sized to a few waves of
// 148 SMs, 16-byte loads and stores where the pointers and counts allow.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "elementwise.h"

namespace nsb {

namespace {

constexpr int kEwThreads = 256;

unsigned ew_blocks(size_t work) {
    size_t b = (work + kEwThreads - 1) / kEwThreads;
    const size_t cap = 148 * 16;  // a few waves of resident blocks, then grid-stride
    if (b > cap) b = cap;
    return (unsigned)(b ? b : 1);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float binop1(float a, float b, int code) {
    switch (code) {
        case kBinAdd: return a + b;
        case kBinSub: return a - b;
        case kBinMul: return a * b;
        default: return a / b;
    }
}

__device__ __forceinline__ void store4(float* o32, __nv_bfloat16* o16, size_t i, float4 v) {
    if (o32) *reinterpret_cast<float4*>(o32 + i) = v;
    if (o16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&lo);
        u.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(o16 + i) = u;
    }
}

__global__ void binop_fwd_kernel(const float* __restrict__ a, const float* __restrict__ b, size_t n, int code,
                                 float* __restrict__ o32, __nv_bfloat16* __restrict__ o16, int vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        for (size_t q = t; 4 * q < n; q += stride) {
            const float4 x = reinterpret_cast<const float4*>(a)[q], y = reinterpret_cast<const float4*>(b)[q];
            store4(o32, o16, 4 * q,
                   make_float4(binop1(x.x, y.x, code), binop1(x.y, y.y, code), binop1(x.z, y.z, code),
                               binop1(x.w, y.w, code)));
        }
        return;
    }
    for (size_t i = t; i < n; i += stride) {
        const float v = binop1(a[i], b[i], code);
        if (o32) o32[i] = v;
        if (o16) o16[i] = __float2bfloat16_rn(v);
    }
}

// d(a op b)/da and /db times dout, plus the running totals.
__global__ void binop_bwd_kernel(const float* __restrict__ d, const float* __restrict__ a, const float* __restrict__ b,
                                 size_t n, int code, const float* acc_a, float* da, const float* acc_b, float* db) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float g = d[i];
        float ga, gb;
        switch (code) {
            case kBinAdd: ga = g; gb = g; break;
            case kBinSub: ga = g; gb = -g; break;
            case kBinMul: ga = g * b[i]; gb = g * a[i]; break;
            default: {
                const float bv = b[i];
                ga = g / bv;
                gb = -g * a[i] / (bv * bv);
            }
        }
        if (da) da[i] = acc_a ? acc_a[i] + ga : ga;
        if (db) db[i] = acc_b ? acc_b[i] + gb : gb;
    }
}

// Multipliers of the local elements 4 q .. 4 q + 3 (batch elements base +
// 4 q ..): one Philox block when base is a multiple of 4, else two.
__device__ __forceinline__ void local_mask4(const DropoutSite& d, size_t q, float m[4]) {
    const unsigned long long g0 = d.base + 4ull * q;
    if ((g0 & 3ull) == 0) {
        dropout_mask4(d, g0 >> 2, m);
        return;
    }
    float a[4], b[4];
    dropout_mask4(d, g0 >> 2, a);
    dropout_mask4(d, (g0 >> 2) + 1, b);
    const int sh = (int)(g0 & 3ull);
#pragma unroll
    for (int j = 0; j < 4; j++) m[j] = j + sh < 4 ? a[j + sh] : b[j + sh - 4];
}

__global__ void dropout_fwd_kernel(const float* __restrict__ x, size_t n, DropoutSite d, float* __restrict__ o32,
                                   __nv_bfloat16* __restrict__ o16, int vec) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x; 4 * q < n; q += stride) {
        float m[4];
        local_mask4(d, q, m);
        if (vec) {
            const float4 v = reinterpret_cast<const float4*>(x)[q];
            store4(o32, o16, 4 * q, make_float4(v.x * m[0], v.y * m[1], v.z * m[2], v.w * m[3]));
        } else {
            for (int j = 0; j < 4 && 4 * q + j < n; j++) {
                const float v = x[4 * q + j] * m[j];
                if (o32) o32[4 * q + j] = v;
                if (o16) o16[4 * q + j] = __float2bfloat16_rn(v);
            }
        }
    }
}

__global__ void dropout_bwd_kernel(const float* __restrict__ dy, size_t n, DropoutSite d, const float* acc,
                                   float* dx) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x; 4 * q < n; q += stride) {
        float m[4];
        local_mask4(d, q, m);
        for (int j = 0; j < 4 && 4 * q + j < n; j++) {
            const size_t i = 4 * q + j;
            const float g = dy[i] * m[j];
            dx[i] = acc ? acc[i] + g : g;
        }
    }
}

// ---- data movement ----------------------------------------------------------
__device__ __forceinline__ void put(float* o32, __nv_bfloat16* o16, size_t i, float v) {
    if (o32) o32[i] = v;
    if (o16) o16[i] = __float2bfloat16_rn(v);
}

__global__ void concat_cols_kernel(const float* __restrict__ a, int ca, const float* __restrict__ b, int cb, int M,
                                   float* o32, __nv_bfloat16* o16) {
    const int co = ca + cb;
    const size_t n = (size_t)M * co, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / co;
        const int c = (int)(i - r * co);
        put(o32, o16, i, c < ca ? a[r * ca + c] : b[r * cb + (c - ca)]);
    }
}

__global__ void slice_cols_kernel(const float* __restrict__ in, int M, int C, int cs, int ow, float* o32,
                                  __nv_bfloat16* o16) {
    const size_t n = (size_t)M * ow, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / ow;
        put(o32, o16, i, in[r * C + cs + (i - r * ow)]);
    }
}

__global__ void index_cols_kernel(const float* __restrict__ in, int M, int C, const int64_t* __restrict__ idx, int L,
                                  float* o32, __nv_bfloat16* o16) {
    const size_t n = (size_t)M * L, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / L;
        const int64_t j = idx[i - r * L];
        put(o32, o16, i, (j >= 0 && j < C) ? in[r * C + j] : 0.f);
    }
}

// last k with idx[k] == c, or -1: the reference's CPU scatter writes the
// updates in increasing k, so a repeated index keeps its last update
// (src/codegen/codegen.cpp ns_scatter2 / ns_scatterrows helpers)
__device__ __forceinline__ int last_match(const int64_t* idx, int L, int c) {
    for (int k = L - 1; k >= 0; k--)
        if (idx[k] == c) return k;
    return -1;
}

__global__ void scatter_cols_kernel(const float* __restrict__ in, int M, int C, const int64_t* __restrict__ idx, int L,
                                    const float* __restrict__ upd, float* o32, __nv_bfloat16* o16) {
    const size_t n = (size_t)M * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / C;
        const int k = last_match(idx, L, (int)(i - r * C));
        put(o32, o16, i, k >= 0 ? upd[r * L + k] : in[i]);
    }
}

__global__ void concat_rows_kernel(const float* __restrict__ a, size_t na_el, const float* __restrict__ b,
                                   size_t n, float* out) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = i < na_el ? a[i] : b[i - na_el];
}

__global__ void index_rows_kernel(const float* __restrict__ in, int R, int C, const int64_t* __restrict__ idx, int L,
                                  float* out) {
    const size_t n = (size_t)L * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t k = i / C;
        const int64_t r = idx[k];
        out[i] = (r >= 0 && r < R) ? in[(size_t)r * C + (i - k * C)] : 0.f;
    }
}

__global__ void scatter_rows_kernel(const float* __restrict__ in, int R, int C, const int64_t* __restrict__ idx, int L,
                                    const float* __restrict__ upd, float* out) {
    const size_t n = (size_t)R * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / C;
        const int k = last_match(idx, L, (int)r);
        out[i] = k >= 0 ? upd[(size_t)k * C + (i - r * C)] : in[i];
    }
}

// 32 x 32 tiles through shared memory (padded against bank conflicts):
// coalesced reads of `in` rows and coalesced writes of `out` rows.
__global__ void transpose_kernel(const float* __restrict__ in, int R, int C, float* __restrict__ out) {
    __shared__ float t[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int r = r0 + y, c = c0 + threadIdx.x;
        if (r < R && c < C) t[y][threadIdx.x] = in[(size_t)r * C + c];
    }
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int c = c0 + y, r = r0 + threadIdx.x;
        if (c < C && r < R) out[(size_t)c * R + r] = t[threadIdx.x][y];
    }
}

__global__ void concat_cols_bwd_kernel(const float* __restrict__ d, int ca, int cb, int M, const float* acc_a,
                                       float* da, const float* acc_b, float* db) {
    const int co = ca + cb;
    const size_t n = (size_t)M * co, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / co;
        const int c = (int)(i - r * co);
        if (c < ca) {
            const size_t j = r * ca + c;
            if (da) da[j] = acc_a ? acc_a[j] + d[i] : d[i];
        } else {
            const size_t j = r * cb + (c - ca);
            if (db) db[j] = acc_b ? acc_b[j] + d[i] : d[i];
        }
    }
}

__global__ void slice_cols_bwd_kernel(const float* __restrict__ d, int M, int C, int cs, int ce, const float* acc,
                                      float* din) {
    const int ow = ce - cs;
    const size_t n = (size_t)M * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / C;
        const int c = (int)(i - r * C);
        const float g = (c >= cs && c < ce) ? d[r * ow + (c - cs)] : 0.f;
        din[i] = acc ? acc[i] + g : g;
    }
}

// din[r, c] = sum over k (increasing) with idx[k] == c of dout[r, k]
__global__ void index_cols_bwd_kernel(const float* __restrict__ d, int M, int C, const int64_t* __restrict__ idx,
                                      int L, const float* acc, float* din) {
    const size_t n = (size_t)M * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / C;
        const int c = (int)(i - r * C);
        float g = 0.f;
        for (int k = 0; k < L; k++)
            if (idx[k] == c) g += d[r * L + k];
        din[i] = acc ? acc[i] + g : g;
    }
}

__global__ void scatter_cols_bwd_kernel(const float* __restrict__ d, int M, int C, const int64_t* __restrict__ idx,
                                        int L, const float* acc_in, float* din, const float* acc_upd, float* dupd) {
    const size_t n = (size_t)M * C, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / C;
        const int c = (int)(i - r * C);
        const int k = last_match(idx, L, c);
        const float g = d[i];
        if (din) din[i] = (acc_in ? acc_in[i] : 0.f) + (k >= 0 ? 0.f : g);
        if (dupd && k >= 0) dupd[r * L + k] = acc_upd ? acc_upd[r * L + k] + g : g;
    }
}

// upd columns that no output column reads (a duplicate index after its first
// occurrence) get a zero gradient
__global__ void scatter_cols_bwd_unused_kernel(int M, int C, const int64_t* __restrict__ idx, int L,
                                               const float* acc_upd, float* dupd) {
    const size_t n = (size_t)M * L, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t r = i / L;
        const int k = (int)(i - r * L);
        const int64_t c = idx[k];
        if (c < 0 || c >= C || last_match(idx, L, (int)c) != k) dupd[r * L + k] = acc_upd ? acc_upd[i] : 0.f;
    }
}

int launched() { return cudaGetLastError() == cudaSuccess ? 0 : -5; }

}  // namespace

int binop_fwd(const float* a, const float* b, size_t n, int code, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (!n) return 0;
    if (!a || !b || (!out32 && !out16) || code < 0 || code > 3) return -1;
    const int vec = n % 4 == 0 && al16(a) && al16(b) && (!out32 || al16(out32)) &&
                    (!out16 || (reinterpret_cast<uintptr_t>(out16) & 7) == 0);
    binop_fwd_kernel<<<ew_blocks(vec ? n / 4 : n), kEwThreads, 0, s>>>(a, b, n, code, out32, out16, vec);
    return launched();
}

int binop_bwd(const float* dout, const float* a, const float* b, size_t n, int code, const float* acc_a, float* da,
              const float* acc_b, float* db, cudaStream_t s) {
    if (!n) return 0;
    if (!dout || code < 0 || code > 3) return -1;
    if (code >= kBinMul && (!a || !b)) return -1;
    binop_bwd_kernel<<<ew_blocks(n), kEwThreads, 0, s>>>(dout, a, b, n, code, acc_a, da, acc_b, db);
    return launched();
}

int dropout_fwd(const float* x, size_t n, const DropoutSite& d, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (!n) return 0;
    if (!x || (!out32 && !out16) || !(d.rate >= 0.f && d.rate < 1.f)) return -1;
    const int vec = n % 4 == 0 && al16(x) && (!out32 || al16(out32)) &&
                    (!out16 || (reinterpret_cast<uintptr_t>(out16) & 7) == 0);
    dropout_fwd_kernel<<<ew_blocks((n + 3) / 4), kEwThreads, 0, s>>>(x, n, d, out32, out16, vec);
    return launched();
}

int dropout_bwd(const float* dy, size_t n, const DropoutSite& d, const float* acc, float* dx, cudaStream_t s) {
    if (!n) return 0;
    if (!dy || !dx || !(d.rate >= 0.f && d.rate < 1.f)) return -1;
    dropout_bwd_kernel<<<ew_blocks((n + 3) / 4), kEwThreads, 0, s>>>(dy, n, d, acc, dx);
    return launched();
}

int concat_cols(const float* a, int ca, const float* b, int cb, int M, float* out32, __nv_bfloat16* out16,
                cudaStream_t s) {
    if (M <= 0) return 0;
    if (!a || !b || ca <= 0 || cb <= 0 || (!out32 && !out16)) return -1;
    concat_cols_kernel<<<ew_blocks((size_t)M * (ca + cb)), kEwThreads, 0, s>>>(a, ca, b, cb, M, out32, out16);
    return launched();
}

int slice_cols(const float* in, int M, int C, int cs, int ce, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!in || cs < 0 || ce > C || ce <= cs || (!out32 && !out16)) return -1;
    slice_cols_kernel<<<ew_blocks((size_t)M * (ce - cs)), kEwThreads, 0, s>>>(in, M, C, cs, ce - cs, out32, out16);
    return launched();
}

int index_cols(const float* in, int M, int C, const int64_t* idx, int L, float* out32, __nv_bfloat16* out16,
               cudaStream_t s) {
    if (M <= 0) return 0;
    if (!in || !idx || L <= 0 || C <= 0 || (!out32 && !out16)) return -1;
    index_cols_kernel<<<ew_blocks((size_t)M * L), kEwThreads, 0, s>>>(in, M, C, idx, L, out32, out16);
    return launched();
}

int scatter_cols(const float* in, int M, int C, const int64_t* idx, int L, const float* upd, float* out32,
                 __nv_bfloat16* out16, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!in || !idx || !upd || L <= 0 || C <= 0 || (!out32 && !out16)) return -1;
    scatter_cols_kernel<<<ew_blocks((size_t)M * C), kEwThreads, 0, s>>>(in, M, C, idx, L, upd, out32, out16);
    return launched();
}

int concat_rows(const float* a, int na, const float* b, int nb, int D, float* out, cudaStream_t s) {
    if (!a || !b || !out || na < 0 || nb < 0 || D <= 0) return -1;
    const size_t n = (size_t)(na + nb) * D;
    if (!n) return 0;
    concat_rows_kernel<<<ew_blocks(n), kEwThreads, 0, s>>>(a, (size_t)na * D, b, n, out);
    return launched();
}

int slice_rows(const float* in, int C, int rs, int re, float* out, cudaStream_t s) {
    if (!in || !out || rs < 0 || re < rs || C <= 0) return -1;
    const size_t n = (size_t)(re - rs) * C;
    if (!n) return 0;
    return cudaMemcpyAsync(out, in + (size_t)rs * C, n * sizeof(float), cudaMemcpyDeviceToDevice, s) == cudaSuccess
               ? 0
               : -5;
}

int index_rows(const float* in, int R, int C, const int64_t* idx, int L, float* out, cudaStream_t s) {
    if (!in || !idx || !out || L < 0 || C <= 0 || R < 0) return -1;
    if (!L) return 0;
    index_rows_kernel<<<ew_blocks((size_t)L * C), kEwThreads, 0, s>>>(in, R, C, idx, L, out);
    return launched();
}

int scatter_rows(const float* in, int R, int C, const int64_t* idx, int L, const float* upd, float* out,
                 cudaStream_t s) {
    if (!in || !idx || !upd || !out || R < 0 || C <= 0 || L < 0) return -1;
    if (!R) return 0;
    scatter_rows_kernel<<<ew_blocks((size_t)R * C), kEwThreads, 0, s>>>(in, R, C, idx, L, upd, out);
    return launched();
}

int transpose2d(const float* in, int R, int C, float* out, cudaStream_t s) {
    if (!in || !out || R < 0 || C < 0) return -1;
    if (!R || !C) return 0;
    dim3 grid((C + 31) / 32, (R + 31) / 32), block(32, 8);
    transpose_kernel<<<grid, block, 0, s>>>(in, R, C, out);
    return launched();
}

int concat_cols_bwd(const float* dout, int ca, int cb, int M, const float* acc_a, float* da, const float* acc_b,
                    float* db, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!dout || ca <= 0 || cb <= 0) return -1;
    concat_cols_bwd_kernel<<<ew_blocks((size_t)M * (ca + cb)), kEwThreads, 0, s>>>(dout, ca, cb, M, acc_a, da, acc_b,
                                                                                   db);
    return launched();
}

int slice_cols_bwd(const float* dout, int M, int C, int cs, int ce, const float* acc, float* din, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!dout || !din || cs < 0 || ce > C || ce <= cs) return -1;
    slice_cols_bwd_kernel<<<ew_blocks((size_t)M * C), kEwThreads, 0, s>>>(dout, M, C, cs, ce, acc, din);
    return launched();
}

int index_cols_bwd(const float* dout, int M, int C, const int64_t* idx, int L, const float* acc, float* din,
                   cudaStream_t s) {
    if (M <= 0) return 0;
    if (!dout || !idx || !din || L <= 0 || C <= 0) return -1;
    index_cols_bwd_kernel<<<ew_blocks((size_t)M * C), kEwThreads, 0, s>>>(dout, M, C, idx, L, acc, din);
    return launched();
}

int scatter_cols_bwd(const float* dout, int M, int C, const int64_t* idx, int L, const float* acc_in, float* din,
                     const float* acc_upd, float* dupd, cudaStream_t s) {
    if (M <= 0) return 0;
    if (!dout || !idx || L <= 0 || C <= 0) return -1;
    scatter_cols_bwd_kernel<<<ew_blocks((size_t)M * C), kEwThreads, 0, s>>>(dout, M, C, idx, L, acc_in, din, acc_upd,
                                                                            dupd);
    if (dupd)
        scatter_cols_bwd_unused_kernel<<<ew_blocks((size_t)M * L), kEwThreads, 0, s>>>(M, C, idx, L, acc_upd, dupd);
    return launched();
}

}  // namespace nsb
