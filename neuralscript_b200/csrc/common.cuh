// Shared definitions for the NeuralScript B200 kernels: error codes,
// activation functions (the reference formulas), bf16 helpers and the GEMM
// epilogue description shared by the tensor-core and SIMT GEMMs.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsb {

// Device error codes written into the per-context error word.
enum DevErr : int {
    kErrNone = 0,
    kErrTimeoutProducer = 101,
    kErrTimeoutMma = 102,
    kErrTimeoutEpilogue = 103,
    kErrTimeoutAttn = 104,
    kErrBadShape = 110,
};

// Operand element types.
enum DType : int { kF32 = 0, kBF16 = 1 };

// Activation codes (reference ns_act2, src/codegen/codegen.cpp:1244-1255).
enum Act : int { kIdentity = 0, kRelu = 1, kLeaky = 2, kSigmoid = 3, kTanh = 4, kSilu = 5, kGelu = 6, kGeluMoe = 7 };
// kGeluMoe is the exact-erf GELU as written in the reference's MoE helpers
// (src/codegen/codegen.cpp:1938, 1430-1431): multiplies by 0.7071067811865476f
// where ns_act2 divides by 1.41421356f.

__host__ __device__ __forceinline__ float act_fwd(float x, int code) {
    switch (code) {
        case kRelu: return x > 0.f ? x : 0.f;
        case kLeaky: return x > 0.f ? x : 0.01f * x;
        case kSigmoid: return 1.f / (1.f + expf(-x));
        case kTanh: return tanhf(x);
        case kSilu: return x / (1.f + expf(-x));
        case kGelu: return 0.5f * x * (1.f + erff(x / 1.41421356f));
        case kGeluMoe: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
        default: return x;
    }
}

// Reference ns_act_deriv (src/codegen/codegen.cpp:1305-1315).
__host__ __device__ __forceinline__ float act_deriv(float x, int code) {
    switch (code) {
        case kRelu: return x > 0.f ? 1.f : 0.f;
        case kLeaky: return x > 0.f ? 1.f : 0.01f;
        case kSigmoid: {
            float s = 1.f / (1.f + expf(-x));
            return s * (1.f - s);
        }
        case kTanh: {
            float t = tanhf(x);
            return 1.f - t * t;
        }
        case kSilu: {
            float s = x / (1.f + expf(-x));
            return s + x * (1.f - s);
        }
        case kGelu: {
            float u = x / 1.41421356f;
            float p = 0.5f * (1.f + erff(u));
            return p + x * expf(-u * u) / 2.50662827f;
        }
        case kGeluMoe:
            return 0.5f * (1.f + erff(x * 0.7071067811865476f)) + x * expf(-x * x * 0.5f) * 0.3989422804014327f;
        default: return 1.f;
    }
}

// GELU for the bf16 tensor-core path, from the rational approximation of
// erf in Abramowitz & Stegun, Handbook of Mathematical Functions, 7.1.26
// (|error| <= 1.5e-7):  for a >= 0,
//   erfc(a) ~= t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-a^2),  t = 1 / (1 + p a),
// with p = 0.3275911, a1..a5 = 0.254829592, -0.284496736, 1.421413741,
// -1.453152027, 1.061405429. With a = |x| / sqrt(2), Phi(x) = 1 - erfc(a)/2
// for x >= 0 and erfc(a)/2 for x < 0; GELU(x) = x Phi(x) and
// GELU'(x) = Phi(x) + x exp(-x^2/2) / sqrt(2 pi). exp and the reciprocal use
// the hardware approximations. Its error (~1e-7 absolute in Phi) is far below
// bf16 resolution; the fp32 and TF32 modes keep the exact erff form.
__device__ __forceinline__ float as_phi(float x, float& g) {
    const float a = fabsf(x) * 0.70710678f;
    const float t = __fdividef(1.f, fmaf(0.3275911f, a, 1.f));
    g = __expf(-a * a);  // exp(-x^2 / 2)
    const float poly =
        t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
    const float q = 0.5f * poly * g;
    return x >= 0.f ? 1.f - q : q;
}
__device__ __forceinline__ float gelu_fast(float x) {
    float g;
    return x * as_phi(x, g);
}
__device__ __forceinline__ float gelu_fast_deriv(float x) {
    float g;
    const float phi = as_phi(x, g);
    return fmaf(x * g, 0.39894228f, phi);
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

// GEMM epilogue, applied per output element (row r, col c) of
//   acc = sum_k A[r,k] * B[c,k]
// in this order:
//   v = alpha * acc
//   v += add_scale * Add[r,c]                 (residual / beta*C / partial-gradient sum)
//   v *= row_scale[r]                         (MoE routing weight)
//   v *= act'(DZ[r,c])                        (fused activation gradient)
//   Z[r,c] = v                                (pre-activation for a later backward)
//   v = act(v)
//   C32[r,c] = v ; C16[r,c] = bf16(v)
// Output row r is written at out_rows[r] when out_rows is given (MoE combine).
// Rows >= row_limit (per tile, from seg_end when given) are not written.
struct Epilogue {
    float alpha = 1.f;
    const float* add = nullptr;  // fp32 [M, ld_add]
    int ld_add = 0;
    float add_scale = 1.f;
    const float* row_scale = nullptr;
    const void* dz = nullptr;  // activation input for act'(.), fp32 or bf16
    int dz_dtype = kF32;
    int ld_dz = 0;
    int dz_act = 0;
    void* z = nullptr;  // pre-activation store
    int z_dtype = kF32;
    int ld_z = 0;
    int act = 0;
    float* c32 = nullptr;
    int ld_c32 = 0;
    __nv_bfloat16* c16 = nullptr;
    int ld_c16 = 0;
    const int* out_rows = nullptr;
    // c32 split in column blocks: output column c goes to block c / col_block
    // at c32 + block * col_block_stride, column c % col_block (0 = off)
    int col_block = 0;
    long long col_block_stride = 0;
};

__device__ __forceinline__ float ld_any(const void* p, int dtype, size_t idx) {
    return dtype == kBF16 ? bf2f(reinterpret_cast<const __nv_bfloat16*>(p)[idx]) : reinterpret_cast<const float*>(p)[idx];
}

}  // namespace nsb
