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
};

__device__ __forceinline__ float ld_any(const void* p, int dtype, size_t idx) {
    return dtype == kBF16 ? bf2f(reinterpret_cast<const __nv_bfloat16*>(p)[idx]) : reinterpret_cast<const float*>(p)[idx];
}

}  // namespace nsb
