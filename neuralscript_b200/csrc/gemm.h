// Host interface of the dense GEMM used by every contraction on the hot
// path (layer GEMMs and their gradients, attention projections, MoE expert
// GEMMs, Newton-Schulz).
//
//   C[M,N] = epilogue( A[M,K] . B[N,K]^T )
//
// Operands are described by element type, leading dimension and major-ness:
//   K-major  : element (i, k) at ptr[i * ld + k]
//   MN-major : element (i, k) at ptr[k * ld + i]
// so a weight W[in,out] (row-major, as the reference blob stores it) is a
// MN-major B operand for the forward GEMM and a K-major B operand for the
// input-gradient GEMM, without any transposition.
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace nsb {

struct GemmOperand {
    const void* ptr = nullptr;
    int dtype = kF32;
    long long ld = 0;
    bool mn_major = false;
};

enum GemmEngine : int {
    kEngineAuto = 0,    // tcgen05 when the operands allow it, else SIMT
    kEngineSimt = 1,    // exact fp32 FMA (parity mode)
    kEngineTensor = 2,  // tcgen05 only (error if the operands do not allow it)
};

struct GemmDesc {
    int M = 0, N = 0, K = 0;
    GemmOperand a, b;
    Epilogue ep;
    int engine = kEngineAuto;
    // Grouped GEMM (MoE experts): group g covers output rows
    // [seg[g], seg[g+1]) (device array, each start a multiple of 128) and uses
    // the B matrix at b.ptr + g * b_group_stride elements.
    int groups = 1;
    const int* seg = nullptr;
    const int* seg_end = nullptr;  // optional: rows [seg[g], seg_end[g]) are real (the rest padding)
    long long b_group_stride = 0;
    // Grouped over K instead (per-expert weight gradients): group g reduces
    // k in [seg[g], seg_end[g]) and writes C at ep.c32 + g * c_group_stride.
    bool group_k = false;
    long long c_group_stride = 0;
    // Split-K workspace (fp32, >= splits * M * N floats); splits chosen by
    // the dispatcher when 0.
    float* workspace = nullptr;
    size_t workspace_floats = 0;
    int splits = 0;
};

// Returns 0 on success, a negative value on a launch/shape error.
// dev_err: device int that kernels set on a bounded-wait timeout.
int gemm(const GemmDesc& d, cudaStream_t stream, int* dev_err);

// Workspace (floats) the split-K path wants for this problem (0 = none).
size_t gemm_workspace_floats(const GemmDesc& d);

// True when gemm() would use the tcgen05 path for these operands.
bool gemm_uses_tensor_cores(const GemmDesc& d);

// Number of SMs of the current device (cached).
int num_sms();

}  // namespace nsb
