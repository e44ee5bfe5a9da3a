// Elementwise and data-movement kernels: binary ops with their gradients,
// counter-based dropout, and the column/row copies of the reference's
// data-movement ops. All deterministic, all 16-byte vectorised where the
// pointers and widths allow it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsb {

enum BinopCode : int { kBinAdd = 0, kBinSub = 1, kBinMul = 2, kBinDiv = 3 };

// out = a (op) b elementwise over n values (the reference's ns_binop with a
// full-size right operand, src/codegen/codegen.cpp:1267-1278); fp32 and/or
// bf16 outputs.
int binop_fwd(const float* a, const float* b, size_t n, int code, float* out32, __nv_bfloat16* out16,
              cudaStream_t s);
// Gradients of out = a (op) b given dout: da and/or db (either may be null),
// each added to an existing running total when acc_a / acc_b is non-null
// (acc may alias the output).
int binop_bwd(const float* dout, const float* a, const float* b, size_t n, int code, const float* acc_a, float* da,
              const float* acc_b, float* db, cudaStream_t s);

// ---- counter-based dropout (Philox4x32-10) ---------------------------------
// Element i of a dropout site keeps its value with probability 1 - rate and
// is then scaled by 1 / (1 - rate). The keep decision is a pure function of
// (key, site, step, g) with g = base + i the element's index in the whole
// batch: uniform(g) = top 24 bits of word (g % 4) of
// Philox4x32-10(counter = {g / 4 low, g / 4 high, step, site}, key) / 2^24,
// kept when uniform >= rate. The backward regenerates the same mask, and a
// batch split over data-parallel ranks (base = the rank's first row times
// the width) draws exactly the masks of the unsplit batch.
struct DropoutSite {
    float rate = 0.f;
    uint32_t key0 = 0, key1 = 0;  // model seed
    uint32_t step = 0;            // training step (advances every train call)
    uint32_t site = 0;            // which dropout op of the network
    unsigned long long base = 0;  // index of element 0 in the whole batch
};

__host__ __device__ __forceinline__ void philox_round(uint32_t c[4], uint32_t k0, uint32_t k1) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
}

// Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011): counter c, key (k0, k1); the key
// advances by the Weyl constants (0x9E3779B9, 0xBB67AE85) between rounds.
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        philox_round(c, k0, k1);
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

// Keep multipliers (0 or 1 / (1 - rate)) of the four batch elements 4 q .. 4 q + 3.
__host__ __device__ __forceinline__ void dropout_mask4(const DropoutSite& d, unsigned long long q, float m[4]) {
    uint32_t c[4] = {(uint32_t)q, (uint32_t)(q >> 32), d.step, d.site};
    philox4x32_10(c, d.key0, d.key1);
    const float scale = 1.0f / (1.0f - d.rate);
#pragma unroll
    for (int j = 0; j < 4; j++) m[j] = (float)(c[j] >> 8) * (1.0f / 16777216.0f) >= d.rate ? scale : 0.f;
}

// out = x * mask (train) over n values; out32 / out16 optional.
int dropout_fwd(const float* x, size_t n, const DropoutSite& d, float* out32, __nv_bfloat16* out16, cudaStream_t s);
// dx = dy * mask (+ acc), the mask regenerated from the same site and step.
int dropout_bwd(const float* dy, size_t n, const DropoutSite& d, const float* acc, float* dx, cudaStream_t s);

// ---- data movement (reference cuda_backend.cpp:93-171) ---------------------
// Column forms on row-batched [M, C] values:
//   concat:  out[r, :] = [a[r, 0:ca] | b[r, 0:cb]]
//   slice:   out[r, c] = in[r, cs + c], c < ce - cs
//   index:   out[r, k] = in[r, idx[k]], k < L (0 where idx[k] is outside [0, C))
//   scatter: out[r, c] = upd[r, k] for the last k with idx[k] == c, else in[r, c]
// Each can also write a bf16 copy. idx is int64 as in the reference.
int concat_cols(const float* a, int ca, const float* b, int cb, int M, float* out32, __nv_bfloat16* out16,
                cudaStream_t s);
int slice_cols(const float* in, int M, int C, int cs, int ce, float* out32, __nv_bfloat16* out16, cudaStream_t s);
int index_cols(const float* in, int M, int C, const int64_t* idx, int L, float* out32, __nv_bfloat16* out16,
               cudaStream_t s);
int scatter_cols(const float* in, int M, int C, const int64_t* idx, int L, const float* upd, float* out32,
                 __nv_bfloat16* out16, cudaStream_t s);
// Row forms on whole tensors (static row counts):
//   concat_rows: [a (na rows) ; b (nb rows)], width D
//   slice_rows:  rows [rs, re) of a [*, C] tensor
//   index_rows:  out[k, :] = in[idx[k], :] (0 where idx[k] is outside [0, R))
//   scatter_rows: out[r, :] = upd[k, :] for the last k with idx[k] == r, else in[r, :]
//   transpose:   out[j, i] = in[i, j] for an [R, C] tensor
int concat_rows(const float* a, int na, const float* b, int nb, int D, float* out, cudaStream_t s);
int slice_rows(const float* in, int C, int rs, int re, float* out, cudaStream_t s);
int index_rows(const float* in, int R, int C, const int64_t* idx, int L, float* out, cudaStream_t s);
int scatter_rows(const float* in, int R, int C, const int64_t* idx, int L, const float* upd, float* out,
                 cudaStream_t s);
int transpose2d(const float* in, int R, int C, float* out, cudaStream_t s);

// Gradients of the column forms: the concat backward splits dout into da / db
// (each added to acc when given); slice and index scatter dout back into a
// zero [M, C] gradient (index adds duplicates in increasing k); scatter passes
// dout to in except at scattered columns and routes those to upd.
int concat_cols_bwd(const float* dout, int ca, int cb, int M, const float* acc_a, float* da, const float* acc_b,
                    float* db, cudaStream_t s);
int slice_cols_bwd(const float* dout, int M, int C, int cs, int ce, const float* acc, float* din, cudaStream_t s);
int index_cols_bwd(const float* dout, int M, int C, const int64_t* idx, int L, const float* acc, float* din,
                   cudaStream_t s);
int scatter_cols_bwd(const float* dout, int M, int C, const int64_t* idx, int L, const float* acc_in, float* din,
                     const float* acc_upd, float* dupd, cudaStream_t s);

}  // namespace nsb
