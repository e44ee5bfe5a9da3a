// Tensor-core attention forward (tcgen05 + TMEM + TMA) for bf16 q/k/v with
// head dim 64 and sequences of at most 256 positions (the configuration
// shape; longer sequences use the SIMT path in attention.cu).
//
// Persistent: one CTA (8 warps) per SM walks the work items (sequence b,
// head h, 128-query tile), Q/K/V double-buffered so the next item's TMA
// loads overlap this item's softmax:
//   TMA      Q [128 x 64], K [256 x 64], V [256 x 64] straight out of the
//            fused qkv buffer (128-byte swizzle, no multicast)
//   MMA      S = Q K^T            (M=128, N=256, K=64)  -> TMEM cols [0,256)
//   softmax  warp w owns query rows 32*(w%4).. and key half w/4; the two
//            halves of a row meet through shared memory for the max and the
//            sum. Scores are scaled after the dot product (as the
//            reference), exponentials use ex2 on log2e-prescaled values; P
//            is rounded to bf16 into shared memory as a K-major swizzled
//            operand
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
constexpr int kQ = 128;          // queries per item
constexpr int kKeys = 256;       // key tile (= max sequence length here)
constexpr int kDh = 64;          // head dim
constexpr int kQBytes = kQ * 128;        // 16 KB
constexpr int kKBytes = kKeys * 128;     // 32 KB
constexpr int kBufBytes = kQBytes + 2 * kKBytes;  // Q | K | V of one item: 80 KB
constexpr int kPChunk = kQ * 128;        // 64 keys x 128 rows, bf16 = 16 KB
constexpr int kPBytes = 4 * kPChunk;     // 64 KB
constexpr int kFwdThreads = 256;
constexpr int kSmem = 2 * kBufBytes + kPBytes + 2 * kQ * 4 + 64 + 1024;
constexpr uint32_t kIdescS = ptx::instr_desc(1, 0, 0, kQ, kKeys);
constexpr uint32_t kIdescO = ptx::instr_desc(1, 0, 1, kQ, kDh);
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
}  // namespace

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_tc_fwd_kernel(const __grid_constant__ CUtensorMap tqkv, int B, int S, int H, int D, float scale,
                       __nv_bfloat16* __restrict__ ctx, long long ld_ctx, float* __restrict__ lse, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sP = smem + 2 * kBufBytes;
    float* xch = reinterpret_cast<float*>(sP + kPBytes);  // [2][kQ] half-row max / sum exchange
    uint64_t* ld_bar = reinterpret_cast<uint64_t*>(xch + 2 * kQ);  // [2]
    uint64_t* s_bar = ld_bar + 2;  // S = QK^T of the current item done
    uint64_t* o_bar = s_bar + 1;   // O = PV of the current item done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_bar + 1);

    const int t = threadIdx.x, warp = t >> 5;
    const int lg = warp & 3, half = warp >> 2;
    const int r = lg * 32 + (t & 31);  // query row within the tile = TMEM lane
    const int qtiles = (S + kQ - 1) / kQ;
    const int items = B * H * qtiles;

    if (t == 0) {
        ptx::mbar_init(&ld_bar[0], 1);
        ptx::mbar_init(&ld_bar[1], 1);
        ptx::mbar_init(s_bar, 1);
        ptx::mbar_init(o_bar, 1);
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
    const uint32_t lane_base = tmem + ((uint32_t)(lg * 32) << 16);

    auto issue_load = [&](int it, int buf) {
        const int qt = it % qtiles, h = (it / qtiles) % H, b = it / (qtiles * H);
        const int row0 = b * S;
        uint8_t* sQ = smem + buf * kBufBytes;
        uint8_t* sK = sQ + kQBytes;
        uint8_t* sV = sK + kKBytes;
        ptx::mbar_arrive_expect_tx(&ld_bar[buf], kBufBytes);
        ptx::tma_load_2d(sQ, &tqkv, &ld_bar[buf], h * kDh, row0 + qt * kQ);
        ptx::tma_load_2d(sK, &tqkv, &ld_bar[buf], D + h * kDh, row0);
        ptx::tma_load_2d(sK + kKBytes / 2, &tqkv, &ld_bar[buf], D + h * kDh, row0 + 128);
        ptx::tma_load_2d(sV, &tqkv, &ld_bar[buf], 2 * D + h * kDh, row0);
        ptx::tma_load_2d(sV + kKBytes / 2, &tqkv, &ld_bar[buf], 2 * D + h * kDh, row0 + 128);
    };
    if (t == 0) {
        if ((int)blockIdx.x < items) issue_load(blockIdx.x, 0);
        if ((int)(blockIdx.x + gridDim.x) < items) issue_load(blockIdx.x + gridDim.x, 1);
    }

    bool ok = true;
    uint32_t sph = 0, oph = 0;
    const float sl2 = scale * kLog2e;  // score -> log2 units
    // S = Q K^T of the item in buffer `b` into TMEM columns [0, 256)
    auto issue_s = [&](int b) {
        const uint32_t q = ptx::smem_u32(smem + b * kBufBytes), k = q + kQBytes;
#pragma unroll
        for (int st = 0; st < kDh / 16; st++)
            ptx::mma_bf16(tmem, ptx::smem_desc(q + st * 32, 16, 1024, 2), ptx::smem_desc(k + st * 32, 16, 1024, 2),
                          kIdescS, st > 0);
    };
    // The S MMA of the next item is issued right behind this item's PV MMA,
    // so it runs while this item's epilogue reads O.
    if (t == 0 && (int)blockIdx.x < items) {
        ok = ptx::mbar_wait(&ld_bar[0], 0, err, kErrTimeoutAttn) && ok;
        ptx::tc_fence_after();
        if (ok) issue_s(0);
        ptx::mma_commit(s_bar);
    }
    int li = 0;
#pragma unroll 1
    for (int it = blockIdx.x; it < items; it += gridDim.x, li++) {
        const int buf = li & 1;
        const int qt = it % qtiles, h = (it / qtiles) % H, b = it / (qtiles * H);
        const int row0 = b * S, q0 = qt * kQ;
        const uint32_t aQ = ptx::smem_u32(smem + buf * kBufBytes);
        const uint32_t aK = aQ + kQBytes, aV = aK + kKBytes;
        (void)aK;
        ok = ptx::mbar_wait(s_bar, sph, err, kErrTimeoutAttn) && ok;
        sph ^= 1;
        ptx::tc_fence_after();
        // ---- softmax over this thread's 128 keys of row r ----
        // all four 32-column TMEM loads in flight, one wait; the row stays in
        // registers for both the max and the exponentials
        const int c_lo = half * 128;
        uint32_t sv[128];
        ptx::tmem_ld32(lane_base + c_lo, sv);
        ptx::tmem_ld32(lane_base + c_lo + 32, sv + 32);
        ptx::tmem_ld32(lane_base + c_lo + 64, sv + 64);
        ptx::tmem_ld32(lane_base + c_lo + 96, sv + 96);
        ptx::tmem_ld_wait();
        // eight independent partial maxima of the raw scores (short dependency
        // chains), scaled once; a key tile that lies wholly inside the
        // sequence needs no per-element mask
        const bool full_tile = c_lo + 128 <= S;
        float m8[8];
#pragma unroll
        for (int q = 0; q < 8; q++) m8[q] = -INFINITY;
        if (full_tile) {
#pragma unroll
            for (int j = 0; j < 128; j++) m8[j & 7] = fmaxf(m8[j & 7], __uint_as_float(sv[j]));
        } else {
#pragma unroll
            for (int j = 0; j < 128; j++)
                if (c_lo + j < S) m8[j & 7] = fmaxf(m8[j & 7], __uint_as_float(sv[j]));
        }
        float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        mx *= sl2;  // scale > 0: max of the scaled scores (-inf when no key is valid)
        xch[half * kQ + r] = mx;
        __syncthreads();
        mx = fmaxf(xch[r], xch[kQ + r]);
        float s8[8];
#pragma unroll
        for (int q = 0; q < 8; q++) s8[q] = 0.f;
#pragma unroll
        for (int c = 0; c < 128; c += 32) {
            float p[32];
            if (full_tile) {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    p[j] = ex2_approx(fmaf(__uint_as_float(sv[c + j]), sl2, -mx));
                    s8[j & 7] += p[j];
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    p[j] = (c_lo + c + j < S) ? ex2_approx(fmaf(__uint_as_float(sv[c + j]), sl2, -mx)) : 0.f;
                    s8[j & 7] += p[j];
                }
            }
            // 32 keys = 4 granules of 16 bytes in 64-key chunk (c_lo+c)/64,
            // granule index ((c_lo+c)%64)/8 + g, XOR-swizzled by row % 8
            uint8_t* chunk = sP + ((c_lo + c) >> 6) * kPChunk + r * 128;
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const int gi = (((c_lo + c) & 63) >> 3) + g;
                uint4 pk;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; e++) h2[e] = __floats2bfloat162_rn(p[8 * g + 2 * e], p[8 * g + 2 * e + 1]);
                *reinterpret_cast<uint4*>(chunk + ((gi ^ (r & 7)) << 4)) = pk;
            }
        }
        const float sum_part = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
        __syncthreads();  // everyone has read the max exchange
        xch[half * kQ + r] = sum_part;
        ptx::fence_proxy_async();  // generic-proxy P writes -> tensor-core (async proxy) reads
        ptx::tc_fence_before();
        __syncthreads();
        const float sum = xch[r] + xch[kQ + r];
        if (t == 0) {
            ptx::tc_fence_after();
            if (ok) {
                const uint32_t pa = ptx::smem_u32(sP);
#pragma unroll
                for (int s = 0; s < kKeys / 16; s++) {
                    const uint64_t ad = ptx::smem_desc(pa + (s >> 2) * kPChunk + (s & 3) * 32, 16, 1024, 2);
                    const uint64_t bd = ptx::smem_desc(aV + s * 16 * 128, kKBytes, 1024, 2);
                    ptx::mma_bf16(tmem + kKeys, ad, bd, kIdescO, s > 0);
                }
            }
            ptx::mma_commit(o_bar);
            // the next item's S (its Q/K were loaded two items ago)
            if (it + (int)gridDim.x < items) {
                ok = ptx::mbar_wait(&ld_bar[buf ^ 1], ((li + 1) >> 1) & 1, err, kErrTimeoutAttn) && ok;
                ptx::tc_fence_after();
                if (ok) issue_s(buf ^ 1);
                ptx::mma_commit(s_bar);
            }
        }
        ok = ptx::mbar_wait(o_bar, oph, err, kErrTimeoutAttn) && ok;
        oph ^= 1;
        ptx::tc_fence_after();
        // this item's Q/K/V buffer is free: load the item two steps ahead
        if (t == 0 && it + 2 * (int)gridDim.x < items) issue_load(it + 2 * gridDim.x, buf);
        // ---- epilogue: warp half h writes head columns [32*half, +32) ----
        const int qi = q0 + r;
        const float inv = 1.f / sum;
        uint32_t v[32];
        ptx::tmem_ld32(lane_base + kKeys + half * 32, v);
        ptx::tmem_ld_wait();
        if (ok && qi < S) {
            uint4* dst = reinterpret_cast<uint4*>(ctx + (size_t)(row0 + qi) * ld_ctx + h * kDh + half * 32);
#pragma unroll
            for (int g = 0; g < 4; g++) {
                uint4 pk;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; e++)
                    h2[e] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * e]) * inv,
                                                  __uint_as_float(v[8 * g + 2 * e + 1]) * inv);
                dst[g] = pk;
            }
            if (lse && half == 0) lse[((size_t)b * H + h) * S + qi] = mx * kLn2 + logf(sum);
        }
        ptx::tc_fence_before();
        __syncthreads();  // O and the exchange slots are read before the next item reuses them
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// Paired-tile forward for 128 < S <= 256 (the configuration's S = 256): one
// persistent CTA walks (sequence b, head h) items and computes BOTH 128-query
// tiles of an item, one per 4-warp group, so K and V are loaded once per item
// and every thread owns a whole query row (no exchange between warps):
//   warp 8 (one lane)  TMA loads (Q0 | Q1 | K | V, double-buffered by item)
//                      and every MMA:
//       S_g = Q_g K^T          (M=128, N=256, K=64) -> TMEM cols [256g, 256g+256)
//       O_g = P_g V            (M=128, N=64, K=256) -> TMEM cols [256g+128, +64),
//                              P_g read from TMEM (the .ts form: A in TMEM)
//   warps 4g..4g+3     softmax of tile g: row max over the 256 scores, then
//                      P = 2^(s*scale*log2e - max) rounded to bf16 and stored
//                      back into TMEM over the scores already read (two keys
//                      per 32-bit column, key 2j in the low half of column j),
//                      row sums in fp32 from the unrounded values; epilogue
//                      ctx = O / rowsum (bf16) and lse = max + log(rowsum).
// Ping-pong: a token passed between the groups lets only one group run its
// softmax at a time (it then has the exponential unit and the issue slots of
// the SM to itself) while the other waits for its PV product, writes its
// epilogue and receives its next S. The MMA lane issues each group's next S
// as soon as that group has read its O, ahead of the other group's PV.
// The softmax does its arithmetic on packed fp32 pairs (fma/add .f32x2) and
// takes the exponential of one pair in three on the FMA pipe (exp2_poly3),
// the rest on ex2.approx. All waits are bounded and report through the error
// word; after a timeout every role stops waiting.
namespace {
constexpr int kPairThreads = 288;                    // 8 softmax warps + 1 load/MMA warp
constexpr int kPairBuf = 2 * kQBytes + 2 * kKBytes;  // Q0 | Q1 | K | V = 96 KB
constexpr int kPairSmem = 2 * kPairBuf + 1024 + 128;
static_assert(kPairSmem <= 227 * 1024, "paired attention: shared memory above the per-block limit");

}  // namespace

__device__ __forceinline__ void store_row_bf16x64(__nv_bfloat16* dst, const uint32_t* v, float mul) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int g = 0; g < 8; g++) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; e++)
            h2[e] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * e]) * mul,
                                          __uint_as_float(v[8 * g + 2 * e + 1]) * mul);
        d[g] = pk;
    }
}

__global__ void __launch_bounds__(kPairThreads, 1)
    attn_tc_fwd_pair_kernel(const __grid_constant__ CUtensorMap tqkv, int B, int S, int H, int D, float scale,
                            __nv_bfloat16* __restrict__ ctx, long long ld_ctx, float* __restrict__ lse, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* ld_bar = reinterpret_cast<uint64_t*>(smem + 2 * kPairBuf);  // [2] by buffer
    uint64_t* s_bar = ld_bar + 2;     // [2] by group: S_g of the current item in TMEM
    uint64_t* p_bar = s_bar + 2;      // [2] P_g stored (128 arrivals)
    uint64_t* o_bar = p_bar + 2;      // [2] O_g of the current item in TMEM
    uint64_t* free_bar = o_bar + 2;   // [2] O_g read, the group's columns are free (128 arrivals)
    uint64_t* tok_bar = free_bar + 2; // [2] softmax token handed to group g (128 arrivals)
    uint64_t* drain_bar = tok_bar + 2;  // error path: all MMAs of this CTA complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

    const int t = threadIdx.x, warp = t >> 5;
    const int items = B * H;

    if (t == 0) {
        for (int i = 0; i < 2; i++) {
            ptx::mbar_init(&ld_bar[i], 1);
            ptx::mbar_init(&s_bar[i], 1);
            ptx::mbar_init(&p_bar[i], 128);
            ptx::mbar_init(&o_bar[i], 1);
            ptx::mbar_init(&free_bar[i], 128);
            ptx::mbar_init(&tok_bar[i], 128);
        }
        ptx::mbar_init(drain_bar, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 8) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 8) {
        if ((t & 31) == 0) {
            ptx::prefetch_tmap(&tqkv);
            auto issue_load = [&](int it, int buf) {
                const int h = it % H, b = it / H;
                const int row0 = b * S;
                uint8_t* sQ = smem + buf * kPairBuf;
                uint8_t* sK = sQ + 2 * kQBytes;
                uint8_t* sV = sK + kKBytes;
                ptx::mbar_arrive_expect_tx(&ld_bar[buf], kPairBuf);
                ptx::tma_load_2d(sQ, &tqkv, &ld_bar[buf], h * kDh, row0);
                ptx::tma_load_2d(sQ + kQBytes, &tqkv, &ld_bar[buf], h * kDh, row0 + kQ);
                ptx::tma_load_2d(sK, &tqkv, &ld_bar[buf], D + h * kDh, row0);
                ptx::tma_load_2d(sK + kKBytes / 2, &tqkv, &ld_bar[buf], D + h * kDh, row0 + 128);
                ptx::tma_load_2d(sV, &tqkv, &ld_bar[buf], 2 * D + h * kDh, row0);
                ptx::tma_load_2d(sV + kKBytes / 2, &tqkv, &ld_bar[buf], 2 * D + h * kDh, row0 + 128);
            };
            auto issue_s = [&](int g, int buf) {
                const uint32_t aQ = ptx::smem_u32(smem + buf * kPairBuf) + g * kQBytes;
                const uint32_t aK = ptx::smem_u32(smem + buf * kPairBuf) + 2 * kQBytes;
#pragma unroll
                for (int st = 0; st < kDh / 16; st++)
                    ptx::mma_bf16(tmem + 256 * g, ptx::smem_desc(aQ + st * 32, 16, 1024, 2),
                                  ptx::smem_desc(aK + st * 32, 16, 1024, 2), kIdescS, st > 0);
                ptx::mma_commit(&s_bar[g]);
            };
            auto issue_o = [&](int g, int buf) {
                const uint32_t aV = ptx::smem_u32(smem + buf * kPairBuf) + 2 * kQBytes + kKBytes;
#pragma unroll
                for (int s = 0; s < kKeys / 16; s++)
                    ptx::mma_bf16_ts(tmem + 256 * g + 128, tmem + 256 * g + 8 * s,
                                     ptx::smem_desc(aV + s * 16 * 128, kKBytes, 1024, 2), kIdescO, s > 0);
                ptx::mma_commit(&o_bar[g]);
            };
            // loads issued and not yet waited for, by buffer (drained on exit)
            int pending[2] = {0, 0};
            uint32_t ld_phase[2] = {0, 0};
            const int n = items > (int)blockIdx.x ? (items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
            auto item = [&](int li) { return (int)blockIdx.x + li * (int)gridDim.x; };
            auto wait_ld = [&](int buf) {
                ok = ptx::mbar_wait(&ld_bar[buf], ld_phase[buf], err, kErrTimeoutAttn);
                ld_phase[buf] ^= 1;
                pending[buf] = 0;
                ptx::tc_fence_after();
                return ok;
            };
            if (n > 0) {
                issue_load(item(0), 0);
                pending[0] = 1;
            }
            if (n > 1) {
                issue_load(item(1), 1);
                pending[1] = 1;
            }
            if (n > 0 && wait_ld(0)) {
                issue_s(0, 0);
                issue_s(1, 0);
            }
#pragma unroll 1
            for (int li = 0; li < n && ok; li++) {
                const int buf = li & 1;
                const bool more = li + 1 < n;
                ok = ptx::mbar_wait(&p_bar[0], li & 1, err, kErrTimeoutAttn);
                if (!ok) break;
                ptx::tc_fence_after();
                issue_o(0, buf);
                if (more) {
                    // group 0's next scores as soon as it has read O_0
                    ok = ptx::mbar_wait(&free_bar[0], li & 1, err, kErrTimeoutAttn);
                    if (!ok || !wait_ld(buf ^ 1)) break;
                    ptx::tc_fence_after();
                    issue_s(0, buf ^ 1);
                }
                ok = ptx::mbar_wait(&p_bar[1], li & 1, err, kErrTimeoutAttn);
                if (!ok) break;
                ptx::tc_fence_after();
                issue_o(1, buf);
                if (more) {
                    ok = ptx::mbar_wait(&free_bar[1], li & 1, err, kErrTimeoutAttn);
                    if (!ok) break;
                    ptx::tc_fence_after();
                    // both groups have read O of item li: every MMA reading
                    // its buffer is complete, so it takes item li + 2
                    if (li + 2 < n) {
                        issue_load(item(li + 2), buf);
                        pending[buf] = 1;
                    }
                    issue_s(1, buf ^ 1);
                }
            }
            // drain: no TMA write or MMA of this CTA may be in flight at exit
            // (no error word here, so these waits do not return early once
            // another role has recorded a timeout; each is still bounded)
            for (int i = 0; i < 2; i++)
                if (pending[i]) ptx::mbar_wait(&ld_bar[i], ld_phase[i], nullptr, 0);
            if (!ok) {
                ptx::mma_commit(drain_bar);
                ptx::mbar_wait(drain_bar, 0, nullptr, 0);
            }
        }
    } else {
        const int g = warp >> 2, lg = warp & 3;
        const int r = lg * 32 + (t & 31);  // query row within tile g = TMEM lane
        const uint32_t base = tmem + ((uint32_t)(lg * 32) << 16) + 256 * g;
        const float sl2 = scale * kLog2e;  // score -> log2 units
        const bool full = S >= kKeys;      // every key valid: no masking
        int li = 0;
#pragma unroll 1
        for (int it = blockIdx.x; it < items; it += gridDim.x, li++) {
            const int h = it % H, b = it / H;
            ok = ptx::mbar_wait(&s_bar[g], li & 1, err, kErrTimeoutAttn);
            if (!ok) break;
            // the token: group 0 takes it back from group 1's previous
            // softmax, group 1 from group 0's softmax of this item
            if (g == 1 || li > 0) {
                ok = ptx::mbar_wait(&tok_bar[g], (g == 1 ? li : li - 1) & 1, err, kErrTimeoutAttn);
                if (!ok) break;
            }
            ptx::tc_fence_after();
            // ---- row max: two round trips of 128 columns ----
            float m4[4];
#pragma unroll
            for (int q = 0; q < 4; q++) m4[q] = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < kKeys; c += 128) {
                uint32_t a[128];
#pragma unroll
                for (int k = 0; k < 4; k++) ptx::tmem_ld32(base + c + 32 * k, a + 32 * k);
#pragma unroll
                for (int k = 0; k < 4; k++) ptx::tmem_ld_wait_regs32(a + 32 * k);
                if (full) {
#pragma unroll
                    for (int j = 0; j < 128; j += 2)
                        m4[(j >> 1) & 3] = max3(m4[(j >> 1) & 3], __uint_as_float(a[j]), __uint_as_float(a[j + 1]));
                } else {
#pragma unroll
                    for (int j = 0; j < 128; j++)
                        if (c + j < S) m4[j & 3] = fmaxf(m4[j & 3], __uint_as_float(a[j]));
                }
            }
            float mx = fmaxf(max3(m4[0], m4[1], m4[2]), m4[3]);
            mx *= sl2;  // scale > 0: the max of the scaled scores (key 0 is always valid)
            // ---- P = 2^(s*sl2 - mx), bf16 pairs into TMEM column key/2 ----
            // 32-column chunks, the next chunk's TMEM load in flight while
            // this one is exponentiated. P of keys [c, c+32) lands in columns
            // [c/2, c/2+16), all already read (c/2 + 16 <= c + 32).
            const uint64_t SL2 = f2_pack(sl2, sl2), NMX = f2_pack(-mx, -mx);
            uint64_t s4[4];
#pragma unroll
            for (int q = 0; q < 4; q++) s4[q] = 0ull;
            auto emit = [&](const uint32_t* sv, int c) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const int j = 2 * e;
                    const uint64_t X = f2_fma(f2_pack(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])), SL2, NMX);
                    float x0, x1, p0, p1;
                    f2_unpack(X, x0, x1);
                    if (e % 3 == 2) {
                        exp2_poly3_pair(x0, x1, p0, p1);
                    } else {
                        p0 = ex2_approx(x0);
                        p1 = ex2_approx(x1);
                    }
                    if (!full) {
                        p0 = c + j < S ? p0 : 0.f;
                        p1 = c + j + 1 < S ? p1 : 0.f;
                    }
                    s4[e & 3] = f2_add(s4[e & 3], f2_pack(p0, p1));
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                    pk[e] = *reinterpret_cast<uint32_t*>(&h2);
                }
                ptx::tmem_st16(base + c / 2, pk);
            };
            {
                uint32_t ca[32], cb[32];
                ptx::tmem_ld32(base, ca);
                ptx::tmem_ld_wait_regs32(ca);
#pragma unroll 1
                for (int c = 0; c < kKeys; c += 64) {
                    ptx::tmem_ld32(base + c + 32, cb);
                    emit(ca, c);
                    ptx::tmem_ld_wait_regs32(cb);
                    if (c + 64 < kKeys) ptx::tmem_ld32(base + c + 64, ca);
                    emit(cb, c + 32);
                    if (c + 64 < kKeys) ptx::tmem_ld_wait_regs32(ca);
                }
            }
            const uint64_t s2 = f2_add(f2_add(s4[0], s4[1]), f2_add(s4[2], s4[3]));
            float sa, sb;
            f2_unpack(s2, sa, sb);
            const float sum = sa + sb;
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(&p_bar[g]);
            ptx::mbar_arrive(&tok_bar[g ^ 1]);  // the other group's softmax may start
            // ---- epilogue: O_g row r ----
            ok = ptx::mbar_wait(&o_bar[g], li & 1, err, kErrTimeoutAttn);
            if (!ok) break;
            ptx::tc_fence_after();
            uint32_t v[64];
            ptx::tmem_ld32(base + 128, v);
            ptx::tmem_ld32(base + 160, v + 32);
            ptx::tmem_ld_wait();
            ptx::tc_fence_before();
            ptx::mbar_arrive(&free_bar[g]);
            const int qi = g * kQ + r;
            if (qi < S) {
                const int row = b * S + qi;
                const float inv = 1.f / sum;
                store_row_bf16x64(ctx + (size_t)row * ld_ctx + h * kDh, v, inv);
                if (lse) lse[((size_t)b * H + h) * S + qi] = mx * kLn2 + logf(sum);
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// Tensor-core attention backward (bf16, head dim 64, S <= 256), the flash
// recomputation form of the reference's ns_attention_grad_kernel
// (src/codegen/cuda_backend.cpp:231-366, CPU ns_attention_bwd
// src/codegen/codegen.cpp:1785-1907): with P = exp(scale*QK^T - lse),
//   dV = P^T dO,  dP = dO V^T,  dS = P o (dP - rowdot(dO, O)),
//   dQ = scale * dS K,  dK = scale * dS^T Q.
// One CTA (8 warps) per (sequence b, head h) holds the whole sequence's
// Q, K, V, dO in shared memory (TMA, 128-byte swizzle) and walks the
// (key tile j, query tile i) pairs of 128 x 128:
//   MMA1  S^T = K_j Q_i^T, dP^T = V_j dO_i^T          -> TMEM cols [0,256)
//   elementwise: warp w owns key rows 32*(w%4).., query half w/4; P^T and
//         dS^T are rounded to bf16 into shared memory (K-major swizzled)
//   MMA2  dV_j += P^T dO_i, dK_j += dS^T Q_i          -> cols [256,384)
//         dQ_i += dS K_j (dS^T read as an MN-major A) -> cols [384,512)
// dK_j / dV_j are written when key tile j is done, dQ at the end, so every
// sum over keys or queries stays inside the CTA (no atomics). All waits are
// bounded and report through the error word.
namespace {
constexpr int kBT = 128;                 // key / query tile
constexpr int kTile = kBT * 128;         // 128 rows x 64 bf16 = 16 KB
constexpr int kBwdThreads = 256;
constexpr int kBwdSmem = 12 * kTile + 2 * 256 * 4 + 64 + 1024;
constexpr uint32_t kIdescT = ptx::instr_desc(1, 0, 0, kBT, kBT);   // S^T, dP^T
constexpr uint32_t kIdescKV = ptx::instr_desc(1, 0, 1, kBT, kDh);  // dV, dK
constexpr uint32_t kIdescQ = ptx::instr_desc(1, 1, 1, kBT, kDh);   // dQ
}  // namespace

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const uint32_t* v, float mul) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int g = 0; g < 4; g++) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; t++)
            h2[t] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * t]) * mul,
                                          __uint_as_float(v[8 * g + 2 * t + 1]) * mul);
        d[g] = pk;
    }
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_tc_bwd_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tctx, const __grid_constant__ CUtensorMap tdqkv, int S,
                       int H, int D, float scale, const __nv_bfloat16* __restrict__ ctx, long long ld_ctx,
                       const __nv_bfloat16* __restrict__ dctx, long long ld_dctx, const float* __restrict__ lse,
                       __nv_bfloat16* __restrict__ dqkv, long long ld_dqkv, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + 2 * kTile;
    uint8_t* sV = sK + 2 * kTile;
    uint8_t* sO = sV + 2 * kTile;  // dO
    uint8_t* sP = sO + 2 * kTile;  // P^T  [128 keys][128 queries] as two 64-query chunks
    uint8_t* sD = sP + 2 * kTile;  // dS^T, same layout
    float* lse_s = reinterpret_cast<float*>(sD + 2 * kTile);
    float* dv_s = lse_s + 256;
    uint64_t* ld_bar = reinterpret_cast<uint64_t*>(dv_s + 256);
    uint64_t* mma_bar = ld_bar + 1;  // MMA1 (S^T, dP^T) of the current step done
    uint64_t* o_bar = mma_bar + 1;   // MMA2 (dV, dK, dQ) of the previous step done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_bar + 1);

    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x, warp = t >> 5;
    const int lg = warp & 3, half = warp >> 2;
    const int r = lg * 32 + (t & 31);  // TMEM lane = tile row this thread reads
    const int row0 = b * S;
    const int nt = (S + kBT - 1) / kBT;

    if (t == 0) {
        ptx::mbar_init(ld_bar, 1);
        ptx::mbar_init(mma_bar, 1);
        ptx::mbar_init(o_bar, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tqkv);
        ptx::prefetch_tmap(&tdo);
        ptx::prefetch_tmap(&tctx);
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + ((uint32_t)(lg * 32) << 16);

    // Q, K, V, dO of the whole sequence, and O (ctx) into the P^T buffer,
    // which is free until the first step: rowdot(dO, O) is then computed
    // from shared memory instead of a second, latency-bound pass over global.
    if (t == 0) {
        ptx::mbar_arrive_expect_tx(ld_bar, nt * 5 * kTile);
        for (int x = 0; x < nt; x++) {
            const int y = row0 + x * kBT;
            ptx::tma_load_2d(sQ + x * kTile, &tqkv, ld_bar, h * kDh, y);
            ptx::tma_load_2d(sK + x * kTile, &tqkv, ld_bar, D + h * kDh, y);
            ptx::tma_load_2d(sV + x * kTile, &tqkv, ld_bar, 2 * D + h * kDh, y);
            ptx::tma_load_2d(sO + x * kTile, &tdo, ld_bar, h * kDh, y);
            ptx::tma_load_2d(sP + x * kTile, &tctx, ld_bar, h * kDh, y);
        }
    }
    bool ok = true;
    {
        const int q = t;
        const float L = q < S ? lse[((size_t)b * H + h) * S + q] : 0.f;
        ok = ptx::mbar_wait(ld_bar, 0, err, kErrTimeoutAttn);
        float dd = 0.f;
        if (ok && q < S) {
            // row q of the dO and O tiles; 16-byte granule g sits at g ^ (row % 8)
            const int rr = q & (kBT - 1);
            const uint8_t* go = sO + (q / kBT) * kTile + rr * 128;
            const uint8_t* oo = sP + (q / kBT) * kTile + rr * 128;
#pragma unroll
            for (int g = 0; g < kDh / 8; g++) {
                const uint4 a = *reinterpret_cast<const uint4*>(go + ((g ^ (rr & 7)) << 4));
                const uint4 c = *reinterpret_cast<const uint4*>(oo + ((g ^ (rr & 7)) << 4));
                const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
                const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 fa = __bfloat1622float2(a2[e]), fc = __bfloat1622float2(c2[e]);
                    dd = fmaf(fa.x, fc.x, dd);
                    dd = fmaf(fa.y, fc.y, dd);
                }
            }
        }
        if (q < 256) {
            lse_s[q] = L * kLog2e;  // log2 units: P = 2^(s * scale * log2e - lse2)
            dv_s[q] = dd;
        }
    }
    __syncthreads();  // O has been read: the P^T buffer is free again

    const uint32_t aQ = ptx::smem_u32(sQ), aK = ptx::smem_u32(sK), aV = ptx::smem_u32(sV), aO = ptx::smem_u32(sO);
    const uint32_t aP = ptx::smem_u32(sP), aD = ptx::smem_u32(sD);
    auto mma1 = [&](int j, int i) {
#pragma unroll
        for (int s = 0; s < kDh / 16; s++)
            ptx::mma_bf16(tmem, ptx::smem_desc(aK + j * kTile + s * 32, 16, 1024, 2),
                          ptx::smem_desc(aQ + i * kTile + s * 32, 16, 1024, 2), kIdescT, s > 0);
#pragma unroll
        for (int s = 0; s < kDh / 16; s++)
            ptx::mma_bf16(tmem + kBT, ptx::smem_desc(aV + j * kTile + s * 32, 16, 1024, 2),
                          ptx::smem_desc(aO + i * kTile + s * 32, 16, 1024, 2), kIdescT, s > 0);
    };
    auto mma2 = [&](int j, int i) {
#pragma unroll
        for (int s = 0; s < kBT / 16; s++) {
            const uint64_t pa = ptx::smem_desc(aP + (s >> 2) * kTile + (s & 3) * 32, 16, 1024, 2);
            const uint64_t ob = ptx::smem_desc(aO + i * kTile + s * 2048, kTile, 1024, 2);
            ptx::mma_bf16(tmem + 256, pa, ob, kIdescKV, (i > 0) || (s > 0));
        }
#pragma unroll
        for (int s = 0; s < kBT / 16; s++) {
            const uint64_t da = ptx::smem_desc(aD + (s >> 2) * kTile + (s & 3) * 32, 16, 1024, 2);
            const uint64_t qb = ptx::smem_desc(aQ + i * kTile + s * 2048, kTile, 1024, 2);
            ptx::mma_bf16(tmem + 320, da, qb, kIdescKV, (i > 0) || (s > 0));
        }
#pragma unroll
        for (int s = 0; s < kBT / 16; s++) {
            const uint64_t da = ptx::smem_desc(aD + s * 2048, kTile, 1024, 2);
            const uint64_t kb = ptx::smem_desc(aK + j * kTile + s * 2048, kTile, 1024, 2);
            ptx::mma_bf16(tmem + 384 + 64 * i, da, kb, kIdescQ, (j > 0) || (s > 0));
        }
    };
    // dK_j / dV_j: warps of the first half write dV, the second half dK
    auto write_kv = [&](int j) {
        uint32_t v[32];
        const int kg = j * kBT + r;
        const int col = (half == 0 ? 2 * D : D) + h * kDh;
        const float mul = half == 0 ? 1.f : scale;
#pragma unroll 1
        for (int c = 0; c < kDh; c += 32) {
            ptx::tmem_ld32(lane_base + 256 + half * 64 + c, v);
            ptx::tmem_ld_wait();
            if (ok && kg < S) store_bf16x32(dqkv + (size_t)(row0 + kg) * ld_dqkv + col + c, v, mul);
        }
    };

    if (t == 0) {
        ptx::tc_fence_after();
        if (ok) mma1(0, 0);
        ptx::mma_commit(mma_bar);
    }
    // Per step: wait for MMA1 of this step, compute P^T and dS^T in registers
    // (the previous step's MMA2 runs meanwhile), wait for that MMA2 (it reads
    // the P^T / dS^T buffers), store them, then issue the next step's MMA1
    // ahead of this step's MMA2.
    uint32_t mph = 0, oph = 0;
    const float sl2 = scale * kLog2e;
    const int steps = nt * nt;
#pragma unroll 1
    for (int st = 0; st < steps; st++) {
        const int j = st / nt, i = st % nt;
        ok = ptx::mbar_wait(mma_bar, mph, err, kErrTimeoutAttn) && ok;
        mph ^= 1;
        ptx::tc_fence_after();
        const int kg = j * kBT + r;
        const bool kval = kg < S;
        // both 32-column halves of S^T and dP^T in flight, one wait
        uint32_t sva[64], pva[64];
        ptx::tmem_ld32(lane_base + half * 64, sva);
        ptx::tmem_ld32(lane_base + half * 64 + 32, sva + 32);
        ptx::tmem_ld32(lane_base + kBT + half * 64, pva);
        ptx::tmem_ld32(lane_base + kBT + half * 64 + 32, pva + 32);
        ptx::tmem_ld_wait();
        // a (key tile, query tile) pair wholly inside the sequence needs no masks
        const bool full_pair = (j + 1) * kBT <= S && (i + 1) * kBT <= S;
        uint32_t pk[32], dk[32];  // 64 bf16 of P^T and of dS^T, packed in pairs
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 32) {
            const uint32_t* sv = sva + c0;
            const uint32_t* pv = pva + c0;
            const int q0 = i * kBT + half * 64 + c0;
            float p[32], ds[32];
            if (full_pair) {
                // per-query lse and rowdot(dO, O), four at a time (broadcast reads)
                const float4* l4 = reinterpret_cast<const float4*>(lse_s + q0);
                const float4* d4 = reinterpret_cast<const float4*>(dv_s + q0);
#pragma unroll
                for (int e4 = 0; e4 < 8; e4++) {
                    const float4 L = l4[e4], Dd = d4[e4];
                    const float Ls[4] = {L.x, L.y, L.z, L.w}, Ds[4] = {Dd.x, Dd.y, Dd.z, Dd.w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const int e = 4 * e4 + q;
                        const float pe = ex2_approx(fmaf(__uint_as_float(sv[e]), sl2, -Ls[q]));
                        p[e] = pe;
                        ds[e] = pe * (__uint_as_float(pv[e]) - Ds[q]);
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    const int qg = q0 + e;
                    const bool v = kval && qg < S;
                    const float pe = v ? ex2_approx(fmaf(__uint_as_float(sv[e]), sl2, -lse_s[qg])) : 0.f;
                    p[e] = pe;
                    ds[e] = v ? pe * (__uint_as_float(pv[e]) - dv_s[qg]) : 0.f;
                }
            }
#pragma unroll
            for (int e = 0; e < 16; e++) {
                __nv_bfloat162 a = __floats2bfloat162_rn(p[2 * e], p[2 * e + 1]);
                __nv_bfloat162 d = __floats2bfloat162_rn(ds[2 * e], ds[2 * e + 1]);
                pk[c0 / 2 + e] = *reinterpret_cast<uint32_t*>(&a);
                dk[c0 / 2 + e] = *reinterpret_cast<uint32_t*>(&d);
            }
        }
        if (st > 0) {
            ok = ptx::mbar_wait(o_bar, oph, err, kErrTimeoutAttn) && ok;  // MMA2 of step st-1
            oph ^= 1;
            ptx::tc_fence_after();
            if (i == 0) write_kv(j - 1);  // key tile j-1 is complete
        }
        // 64 queries = 8 granules of 16 bytes in this half's chunk, XOR-swizzled by row % 8
        uint8_t* prow = sP + half * kTile + r * 128;
        uint8_t* drow = sD + half * kTile + r * 128;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            *reinterpret_cast<uint4*>(prow + ((g ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
            *reinterpret_cast<uint4*>(drow + ((g ^ (r & 7)) << 4)) =
                make_uint4(dk[4 * g], dk[4 * g + 1], dk[4 * g + 2], dk[4 * g + 3]);
        }
        ptx::fence_proxy_async();  // generic-proxy P/dS writes -> tensor-core reads
        ptx::tc_fence_before();
        __syncthreads();
        if (t == 0) {
            ptx::tc_fence_after();
            if (st + 1 < steps) {
                if (ok) mma1((st + 1) / nt, (st + 1) % nt);  // S^T/dP^T columns were read before the barrier
                ptx::mma_commit(mma_bar);
            }
            if (ok) mma2(j, i);
            ptx::mma_commit(o_bar);
        }
    }
    ok = ptx::mbar_wait(o_bar, oph, err, kErrTimeoutAttn) && ok;
    ptx::tc_fence_after();
    // Final dK/dV tile and the dQ tiles. A tile that lies wholly inside the
    // sequence is staged (bf16, 128-byte swizzle) in the P^T / dS^T buffers,
    // free now, and written by TMA stores; a ragged tile is written row by
    // row (a 128-row box would run into the next sequence's rows).
    const int jl = nt - 1;
    if ((jl + 1) * kBT <= S) {
        uint32_t v[64];
        ptx::tmem_ld32(lane_base + 256 + half * 64, v);
        ptx::tmem_ld32(lane_base + 256 + half * 64 + 32, v + 32);
        ptx::tmem_ld_wait();
        const float mul = half == 0 ? 1.f : scale;  // dV | dK
        uint8_t* row = sP + half * kTile + r * 128;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            uint4 pk;
            __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; e++)
                h2[e] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * e]) * mul,
                                              __uint_as_float(v[8 * g + 2 * e + 1]) * mul);
            *reinterpret_cast<uint4*>(row + ((g ^ (r & 7)) << 4)) = pk;
        }
    } else {
        write_kv(jl);
    }
#pragma unroll 1
    for (int i = 0; i < nt; i++) {
        uint32_t v[32];
        ptx::tmem_ld32(lane_base + 384 + 64 * i + half * 32, v);
        ptx::tmem_ld_wait();
        const int qg = i * kBT + r;
        if ((i + 1) * kBT <= S) {
            // dQ_i: warps of the first half hold columns [0,32), the second [32,64)
            uint8_t* row = sD + i * kTile + r * 128;
#pragma unroll
            for (int g = 0; g < 4; g++) {
                uint4 pk;
                __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; e++)
                    h2[e] = __floats2bfloat162_rn(__uint_as_float(v[8 * g + 2 * e]) * scale,
                                                  __uint_as_float(v[8 * g + 2 * e + 1]) * scale);
                const int gi = half * 4 + g;
                *reinterpret_cast<uint4*>(row + ((gi ^ (r & 7)) << 4)) = pk;
            }
        } else if (ok && qg < S) {
            store_bf16x32(dqkv + (size_t)(row0 + qg) * ld_dqkv + h * kDh + half * 32, v, scale);
        }
    }
    ptx::fence_proxy_async();  // staged tiles -> TMA (async proxy) reads
    __syncthreads();
    if (t == 0 && ok) {
        if ((jl + 1) * kBT <= S) {
            ptx::tma_store_2d(&tdqkv, sP, 2 * D + h * kDh, row0 + jl * kBT);          // dV
            ptx::tma_store_2d(&tdqkv, sP + kTile, D + h * kDh, row0 + jl * kBT);      // dK
        }
        for (int i = 0; i < nt; i++)
            if ((i + 1) * kBT <= S) ptx::tma_store_2d(&tdqkv, sD + i * kTile, h * kDh, row0 + i * kBT);  // dQ
        ptx::bulk_commit();
        ptx::bulk_wait_all();  // the staging buffers must outlive the stores
    }
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

static EncodeTiledFn2 tmap_encoder() {
    static EncodeTiledFn2 enc = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<EncodeTiledFn2>(f);
    });
    return enc;
}

// 2D bf16 map over a row-major [rows, cols] matrix with row stride ld
// elements, 64 x 128 boxes, 128-byte swizzle.
static bool bf16_tmap(CUtensorMap* m, const void* base, long long cols, long long rows, long long ld) {
    EncodeTiledFn2 enc = tmap_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool aligned16(const void* p, long long ld) {
    return !(reinterpret_cast<uintptr_t>(p) & 15) && (ld * 2) % 16 == 0;
}

bool attention_tc_supported(const AttnArgs& a) {
    if (a.dtype != kBF16 || a.dh != 64 || a.S > kKeys || a.S <= 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.qkv) & 15) || (a.ld_qkv * 2) % 16) return false;
    if ((reinterpret_cast<uintptr_t>(a.ctx) & 15) || (a.ld_ctx * 2) % 16) return false;
    return true;
}

int attention_tc_fwd(const AttnArgs& a, cudaStream_t s, int* err) {
    CUtensorMap m;
    if (!bf16_tmap(&m, a.qkv, 3LL * a.D, (long long)a.B * a.S, a.ld_qkv)) return -2;
    static bool attr[kMaxDevices] = {};  // per device: the attribute belongs to the current one
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return -1;
    if (!attr[dev]) {
        cudaFuncSetAttribute(attn_tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        attr[dev] = true;
    }
    if (a.S > kQ) {  // two query tiles per sequence: the paired kernel
        static bool pattr[kMaxDevices] = {};
        if (!pattr[dev]) {
            cudaFuncSetAttribute(attn_tc_fwd_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem);
            pattr[dev] = true;
        }
        const int items = a.B * a.H;
        const int grid = items < num_sms() ? items : num_sms();
        attn_tc_fwd_pair_kernel<<<grid, kPairThreads, kPairSmem, s>>>(
            m, a.B, a.S, a.H, a.D, a.scale, reinterpret_cast<__nv_bfloat16*>(a.ctx), a.ld_ctx, a.lse, err);
        return cudaGetLastError() == cudaSuccess ? 0 : -5;
    }
    const int items = a.B * a.H * ((a.S + kQ - 1) / kQ);
    const int grid = items < num_sms() ? items : num_sms();
    attn_tc_fwd_kernel<<<grid, kFwdThreads, kSmem, s>>>(m, a.B, a.S, a.H, a.D, a.scale,
                                                        reinterpret_cast<__nv_bfloat16*>(a.ctx), a.ld_ctx, a.lse, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

bool attention_tc_bwd_supported(const AttnArgs& a) {
    if (a.dtype != kBF16 || a.dh != 64 || a.S > 2 * kBT || a.S <= 0 || !a.lse) return false;
    return aligned16(a.qkv, a.ld_qkv) && aligned16(a.ctx, a.ld_ctx) && aligned16(a.dctx, a.ld_dctx) &&
           aligned16(a.dqkv, a.ld_dqkv);
}

int attention_tc_bwd(const AttnArgs& a, cudaStream_t s, int* err) {
    CUtensorMap mq, mo, mc, md;
    const long long rows = (long long)a.B * a.S;
    if (!bf16_tmap(&mq, a.qkv, 3LL * a.D, rows, a.ld_qkv) || !bf16_tmap(&mo, a.dctx, a.D, rows, a.ld_dctx) ||
        !bf16_tmap(&mc, a.ctx, a.D, rows, a.ld_ctx) || !bf16_tmap(&md, a.dqkv, 3LL * a.D, rows, a.ld_dqkv))
        return -2;
    static bool attr[kMaxDevices] = {};  // per device: the attribute belongs to the current one
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return -1;
    if (!attr[dev]) {
        cudaFuncSetAttribute(attn_tc_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
        attr[dev] = true;
    }
    dim3 grid(a.H, a.B);
    attn_tc_bwd_kernel<<<grid, kBwdThreads, kBwdSmem, s>>>(
        mq, mo, mc, md, a.S, a.H, a.D, a.scale, reinterpret_cast<const __nv_bfloat16*>(a.ctx), a.ld_ctx,
        reinterpret_cast<const __nv_bfloat16*>(a.dctx), a.ld_dctx, a.lse, reinterpret_cast<__nv_bfloat16*>(a.dqkv),
        a.ld_dqkv, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace nsb
