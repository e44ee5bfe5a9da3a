// Tensor-core attention forward (tcgen05 + TMEM + TMA) for bf16 q/k/v with
// head dim 64 and sequences of at most 256 positions (the configuration
// shape; longer sequences use the SIMT path in attention.cu).
//
// One CTA (4 warps) per (sequence b, head h, 128-query tile):
//   TMA      Q [128 x 64], K [256 x 64], V [256 x 64] straight out of the
//            fused qkv buffer (128-byte swizzle, no multicast)
//   MMA      S = Q K^T            (M=128, N=256, K=64)  -> TMEM cols [0,256)
//   softmax  thread r owns query row r: scale after the dot (as the
//            reference), max, exp, sum read from TMEM; P rounded to bf16 and
//            written to shared memory as a K-major swizzled operand
//   MMA      O = P V              (M=128, N=64, K=256; V is the MN-major B
//            operand in its natural row layout) -> TMEM cols [256,320)
//   epilogue ctx = O / rowsum (bf16), lse = max + log(rowsum) for the backward
// All waits are bounded and report through the error word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "attention.h"
#include "common.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace nsb {

namespace {
constexpr int kQ = 128;          // queries per CTA
constexpr int kKeys = 256;       // key tile (= max sequence length here)
constexpr int kDh = 64;          // head dim
constexpr int kQBytes = kQ * 128;        // 16 KB
constexpr int kKBytes = kKeys * 128;     // 32 KB
constexpr int kPChunk = kQ * 128;        // 64 keys x 128 rows, bf16 = 16 KB
constexpr int kPBytes = 4 * kPChunk;     // 64 KB
constexpr int kSmem = kQBytes + 2 * kKBytes + kPBytes + 1024 + 64;
constexpr uint32_t kIdescS = ptx::instr_desc(1, 0, 0, kQ, kKeys);
constexpr uint32_t kIdescO = ptx::instr_desc(1, 0, 1, kQ, kDh);
}  // namespace

__global__ void __launch_bounds__(128, 1)
    attn_tc_fwd_kernel(const __grid_constant__ CUtensorMap tqkv, int S, int H, int D, float scale,
                       __nv_bfloat16* __restrict__ ctx, long long ld_ctx, float* __restrict__ lse, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + kQBytes;
    uint8_t* sV = sK + kKBytes;
    uint8_t* sP = sV + kKBytes;
    uint64_t* ld_bar = reinterpret_cast<uint64_t*>(sP + kPBytes);
    uint64_t* mma_bar = ld_bar + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5;
    const int row0 = b * S;  // first row of this sequence in qkv
    const int q0 = qt * kQ;

    if (threadIdx.x == 0) {
        ptx::mbar_init(ld_bar, 1);
        ptx::mbar_init(mma_bar, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tqkv);
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (threadIdx.x == 0) {
        ptx::mbar_arrive_expect_tx(ld_bar, kQBytes + 2 * kKBytes);
        ptx::tma_load_2d(sQ, &tqkv, ld_bar, h * kDh, row0 + q0);
        ptx::tma_load_2d(sK, &tqkv, ld_bar, D + h * kDh, row0);
        ptx::tma_load_2d(sK + kKBytes / 2, &tqkv, ld_bar, D + h * kDh, row0 + 128);
        ptx::tma_load_2d(sV, &tqkv, ld_bar, 2 * D + h * kDh, row0);
        ptx::tma_load_2d(sV + kKBytes / 2, &tqkv, ld_bar, 2 * D + h * kDh, row0 + 128);
        ok = ptx::mbar_wait(ld_bar, 0, err, kErrTimeoutAttn);
        if (ok) {
            ptx::tc_fence_after();
            const uint32_t q = ptx::smem_u32(sQ), k = ptx::smem_u32(sK);
#pragma unroll
            for (int s = 0; s < kDh / 16; s++)
                ptx::mma_bf16(tmem, ptx::smem_desc(q + s * 32, 16, 1024, 2), ptx::smem_desc(k + s * 32, 16, 1024, 2),
                              kIdescS, s > 0);
        }
        ptx::mma_commit(mma_bar);
    }
    // ---- softmax: thread r owns query row r (TMEM lane r) ----
    ok = ptx::mbar_wait(mma_bar, 0, err, kErrTimeoutAttn) && ok;
    ptx::tc_fence_after();
    const int r = threadIdx.x;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < kKeys; c += 32) {
        uint32_t v[32];
        ptx::tmem_ld32(lane_base + c, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
            float s = __uint_as_float(v[j]) * scale;
            if (c + j < S) mx = fmaxf(mx, s);
        }
    }
    float sum = 0.f;
#pragma unroll 1
    for (int c = 0; c < kKeys; c += 32) {
        uint32_t v[32];
        ptx::tmem_ld32(lane_base + c, v);
        ptx::tmem_ld_wait();
        float p[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            float s = __uint_as_float(v[j]) * scale;
            p[j] = (c + j < S) ? expf(s - mx) : 0.f;
            sum += p[j];
        }
        // 32 keys = 4 granules of 16 bytes in 64-key chunk c/64, granule
        // index (c%64)/8 + g, XOR-swizzled by row % 8 (128-byte swizzle)
        uint8_t* chunk = sP + (c >> 6) * kPChunk + r * 128;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const int gi = ((c & 63) >> 3) + g;
            uint4 pk;
            __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int t = 0; t < 4; t++) h2[t] = __floats2bfloat162_rn(p[8 * g + 2 * t], p[8 * g + 2 * t + 1]);
            *reinterpret_cast<uint4*>(chunk + ((gi ^ (r & 7)) << 4)) = pk;
        }
    }
    ptx::fence_proxy_async();  // generic-proxy P writes -> tensor-core (async proxy) reads
    ptx::tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        ptx::tc_fence_after();
        if (ok) {
            const uint32_t pa = ptx::smem_u32(sP), vb = ptx::smem_u32(sV);
#pragma unroll
            for (int s = 0; s < kKeys / 16; s++) {
                const uint64_t ad = ptx::smem_desc(pa + (s >> 2) * kPChunk + (s & 3) * 32, 16, 1024, 2);
                const uint64_t bd = ptx::smem_desc(vb + s * 16 * 128, kKBytes, 1024, 2);
                ptx::mma_bf16(tmem + kKeys, ad, bd, kIdescO, s > 0);
            }
        }
        ptx::mma_commit(mma_bar);
    }
    ok = ptx::mbar_wait(mma_bar, 1, err, kErrTimeoutAttn) && ok;
    ptx::tc_fence_after();
    // ---- epilogue ----
    const int qi = q0 + r;
    const float inv = 1.f / sum;
#pragma unroll 1
    for (int c = 0; c < kDh; c += 32) {
        uint32_t v[32];
        ptx::tmem_ld32(lane_base + kKeys + c, v);
        ptx::tmem_ld_wait();
        if (ok && qi < S) {
            uint4* dst = reinterpret_cast<uint4*>(ctx + (size_t)(row0 + qi) * ld_ctx + h * kDh + c);
#pragma unroll
            for (int g = 0; g < 4; g++) {
                uint4 pk;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int t = 0; t < 4; t++)
                    h2[t] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * t]) * inv,
                                                  __uint_as_float(v[8 * g + 2 * t + 1]) * inv);
                dst[g] = pk;
            }
        }
    }
    if (ok && lse && qi < S) lse[((size_t)b * H + h) * S + qi] = mx + logf(sum);
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool attention_tc_supported(const AttnArgs& a) {
    if (a.dtype != kBF16 || a.dh != 64 || a.S > kKeys || a.S <= 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.qkv) & 15) || (a.ld_qkv * 2) % 16) return false;
    if ((reinterpret_cast<uintptr_t>(a.ctx) & 15) || (a.ld_ctx * 2) % 16) return false;
    return true;
}

int attention_tc_fwd(const AttnArgs& a, cudaStream_t s, int* err) {
    static EncodeTiledFn2 enc = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<EncodeTiledFn2>(f);
    });
    if (!enc) return -2;
    CUtensorMap m;
    const long long rows = (long long)a.B * a.S;
    cuuint64_t dims[2] = {(cuuint64_t)(3LL * a.D), (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(a.ld_qkv * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.qkv), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -2;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        attr = true;
    }
    dim3 grid((a.S + kQ - 1) / kQ, a.H, a.B);
    attn_tc_fwd_kernel<<<grid, 128, kSmem, s>>>(m, a.S, a.H, a.D, a.scale, reinterpret_cast<__nv_bfloat16*>(a.ctx),
                                                 a.ld_ctx, a.lse, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace nsb
