// Shared definitions for the NeuralScript B200 kernels: error codes,
// activation functions (the reference formulas), bf16 helpers and the GEMM
// epilogue description shared by the tensor-core and SIMT GEMMs.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsb {

// Upper bound on device ordinals for per-device caches (kernel attributes).
constexpr int kMaxDevices = 64;

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
enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };  // kF16: fp16 outputs only (head + loss fusion)

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

// GELU for the bf16 tensor-core path: the tanh form of Hendrycks & Gimpel
// (Gaussian Error Linear Units, 2016),
//   GELU(x) ~= 0.5 x (1 + tanh(u)),  u = sqrt(2/pi) (x + 0.044715 x^3),
// evaluated with the hardware tanh approximation. It stays within ~3e-4 of
// the exact-erf GELU (x Phi(x)), below the resolution of the bf16 values this
// path produces, at a third of the instructions; the fp32 and TF32 modes keep
// the exact erff form of the reference. The derivative is that of the same
// tanh form, so forward and backward agree.
// 2^x for x <= 0 on the FMA/ALU pipes, without the special-function unit, so
// kernels whose exponentials saturate that unit (attention softmax, the
// cross-entropy pass) can move a share of them to the FP32 pipe.
// Cody-Waite range reduction: x = n + f with n = round(x) (adding 1.5 * 2^23
// leaves n in the low mantissa bits of t) and f in [-1/2, 1/2]; 2^f by a
// cubic fitted for this code (Lawson-weighted least squares on [-1/2, 1/2],
// maximum relative error 7.5e-5, below half a bf16 ulp); 2^n is added to the
// exponent field. x is clamped at -125 so the result stays a normal number
// (results there are about 2^-125, far under anything the callers keep).
__device__ __forceinline__ float exp2_poly3(float x) {
    x = fmaxf(x, -125.f);
    const float t = x + 12582912.f;
    const float f = x - (t - 12582912.f);
    const float p = fmaf(fmaf(fmaf(0.0551716648f, f, 0.2426111251f), f, 0.6932609677f), f, 0.9999280572f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Packed fp32 pairs (sm_100 fma/add .f32x2: two lanes of arithmetic per
// instruction), for the exponential-heavy loops of the softmax and the loss.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// exp2_poly3 of a pair (x <= 0), the polynomial on packed fp32 pairs
__device__ __forceinline__ void exp2_poly3_pair(float x0, float x1, float& y0, float& y1) {
    x0 = fmaxf(x0, -125.f);
    x1 = fmaxf(x1, -125.f);
    const uint64_t X = f2_pack(x0, x1);
    const uint64_t T = f2_add(X, f2_pack(12582912.f, 12582912.f));
    const uint64_t N = f2_add(T, f2_pack(-12582912.f, -12582912.f));
    const uint64_t F = f2_fma(N, f2_pack(-1.f, -1.f), X);
    uint64_t P = f2_fma(f2_pack(0.0551716648f, 0.0551716648f), F, f2_pack(0.2426111251f, 0.2426111251f));
    P = f2_fma(P, F, f2_pack(0.6932609677f, 0.6932609677f));
    P = f2_fma(P, F, f2_pack(0.9999280572f, 0.9999280572f));
    float p0, p1, t0, t1;
    f2_unpack(P, p0, p1);
    f2_unpack(T, t0, t1);
    y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
    y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_fast(float x) {
    const float x2 = x * x;
    const float u = x * fmaf(0.0356774081f, x2, 0.7978845608f);  // sqrt(2/pi) (x + 0.044715 x^3)
    const float hx = 0.5f * x;
    return fmaf(hx, tanh_approx(u), hx);
}
__device__ __forceinline__ float gelu_fast_deriv(float x) {
    const float x2 = x * x;
    const float u = x * fmaf(0.0356774081f, x2, 0.7978845608f);
    const float t = tanh_approx(u);
    const float du = fmaf(0.1070322243f, x2, 0.7978845608f);  // d u / dx
    // 0.5 (1 + t) + 0.5 x (1 - t^2) du
    return fmaf(0.5f * x * du, fmaf(-t, t, 1.f), fmaf(0.5f, t, 0.5f));
}
// gelu_fast / gelu_fast_deriv of a pair of values on packed fp32 pairs: the
// same operations in the same order (bit-identical results), half the FP32
// instructions.
__device__ __forceinline__ void gelu_fast2(float& x0, float& x1) {
    const uint64_t X = f2_pack(x0, x1);
    const uint64_t X2 = f2_mul(X, X);
    const uint64_t U = f2_mul(X, f2_fma(f2_pack(0.0356774081f, 0.0356774081f), X2, f2_pack(0.7978845608f, 0.7978845608f)));
    const uint64_t HX = f2_mul(f2_pack(0.5f, 0.5f), X);
    float u0, u1;
    f2_unpack(U, u0, u1);
    f2_unpack(f2_fma(HX, f2_pack(tanh_approx(u0), tanh_approx(u1)), HX), x0, x1);
}
__device__ __forceinline__ void gelu_fast_deriv2(float x0, float x1, float& d0, float& d1) {
    const uint64_t X = f2_pack(x0, x1);
    const uint64_t X2 = f2_mul(X, X);
    const uint64_t C0 = f2_pack(0.7978845608f, 0.7978845608f);
    const uint64_t U = f2_mul(X, f2_fma(f2_pack(0.0356774081f, 0.0356774081f), X2, C0));
    float u0, u1;
    f2_unpack(U, u0, u1);
    const float t0 = tanh_approx(u0), t1 = tanh_approx(u1);
    const uint64_t T = f2_pack(t0, t1);
    const uint64_t DU = f2_fma(f2_pack(0.1070322243f, 0.1070322243f), X2, C0);
    const uint64_t HALF = f2_pack(0.5f, 0.5f);
    const uint64_t A = f2_mul(f2_mul(HALF, X), DU);
    const uint64_t B = f2_fma(f2_pack(-t0, -t1), T, f2_pack(1.f, 1.f));
    f2_unpack(f2_fma(A, B, f2_fma(HALF, T, HALF)), d0, d1);
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
    // c16 holds IEEE fp16 instead of bf16 (TMA-store path only)
    bool c16_half = false;
    // LayerNorm of every output row (no affine, eps 1e-5) after alpha and
    // the residual add: c32 / c16 receive the normalised rows and
    // ln_rstd[row] the row's 1 / sqrt(var + eps). Tensor-core path with
    // N = 512 (one CTA owns whole rows).
    float* ln_rstd = nullptr;
    // Head GEMM + loss fusion (TMA-store path): the fp32 logit of column
    // ce_tgt[row] of every row goes to ce_tlogit[row] (the stored logits
    // are bf16; the loss takes the target's logit at full precision).
    const int* ce_tgt = nullptr;
    float* ce_tlogit = nullptr;
};

__device__ __forceinline__ float ld_any(const void* p, int dtype, size_t idx) {
    return dtype == kBF16 ? bf2f(reinterpret_cast<const __nv_bfloat16*>(p)[idx]) : reinterpret_cast<const float*>(p)[idx];
}

}  // namespace nsb
