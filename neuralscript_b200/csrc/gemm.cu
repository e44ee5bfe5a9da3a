// Dense GEMM for sm_100a.
//
// Tensor-core path: persistent, warp-specialised tcgen05 kernel.
//   warp 0      TMA producer (one elected thread): A and B tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle, no multicast)
//   warp 1      MMA issuer (one thread) + TMEM owner: tcgen05.mma into a
//               double-buffered fp32 accumulator in TMEM (2 x BN columns)
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, fused epilogue
//               (residual / act' / activation / bf16 cast), global stores
// The accumulator double buffer lets the epilogue of tile i overlap the MMAs
// of tile i+1. K-major and MN-major operands are both read straight from
// their storage layout (the shared-memory descriptor encodes the major-ness),
// so no transposed copies are needed for forward, input-gradient or
// weight-gradient GEMMs. Split-K (for weight gradients, whose K is the row
// count) writes fp32 partials that a second kernel sums in a fixed order, so
// results are deterministic.
//
// SIMT path: fp32 FMA, each output accumulated sequentially in k, for the
// pure-fp32 parity mode and for shapes TMA cannot describe.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "gemm.h"
#include "ptx.cuh"

namespace nsb {

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// ---------------------------------------------------------------------------
// Epilogue helpers (shared by all paths)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void epi_apply(const Epilogue& ep, int row, int col, float v) {
    v *= ep.alpha;
    if (ep.add) v += ep.add_scale * ep.add[(size_t)row * ep.ld_add + col];
    if (ep.row_scale) v *= ep.row_scale[row];
    if (ep.dz) v *= act_deriv(ld_any(ep.dz, ep.dz_dtype, (size_t)row * ep.ld_dz + col), ep.dz_act);
    if (ep.z) {
        size_t zi = (size_t)row * ep.ld_z + col;
        if (ep.z_dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(ep.z)[zi] = f2bf(v);
        else reinterpret_cast<float*>(ep.z)[zi] = v;
    }
    if (ep.act) v = act_fwd(v, ep.act);
    int orow = ep.out_rows ? ep.out_rows[row] : row;
    if (ep.c32) {
        if (ep.col_block) {
            const int b = col / ep.col_block;
            ep.c32[b * ep.col_block_stride + (size_t)orow * ep.ld_c32 + (col - b * ep.col_block)] = v;
        } else {
            ep.c32[(size_t)orow * ep.ld_c32 + col] = v;
        }
    }
    if (ep.c16) ep.c16[(size_t)orow * ep.ld_c16 + col] = f2bf(v);
}

// Epilogue of 32 consecutive columns of one row held in registers, split in
// the order the outputs need it: pre() = alpha, residual, row scale and
// activation derivative (the value stored as z), act() = the activation.
// ncols < 32 marks a ragged last chunk (scalar, guarded loads); full chunks
// use 16-byte loads (leading dimensions multiples of 8 elements, col0 a
// multiple of 32).
template <bool FAST>
__device__ __forceinline__ void epi_pre32(const Epilogue& ep, int row, int col0, float* v, int ncols,
                                          const float* pre_add = nullptr, const uint4* pre_dz = nullptr) {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] *= ep.alpha;
    if (ep.add && pre_add) {
        // residual already loaded (full chunk)
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] += ep.add_scale * pre_add[j];
    } else if (ep.add) {
        const float* a = ep.add + (size_t)row * ep.ld_add + col0;
        if (ncols == 32) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 t = reinterpret_cast<const float4*>(a)[j];
                v[4 * j] += ep.add_scale * t.x;
                v[4 * j + 1] += ep.add_scale * t.y;
                v[4 * j + 2] += ep.add_scale * t.z;
                v[4 * j + 3] += ep.add_scale * t.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (j < ncols) v[j] += ep.add_scale * a[j];
        }
    }
    if (ep.row_scale) {
        float sc = ep.row_scale[row];
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] *= sc;
    }
    if (ep.dz) {
        float z[32];
        if (ncols == 32 && ep.dz_dtype == kBF16) {
            const uint4* a = pre_dz ? pre_dz
                                    : reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(ep.dz) +
                                                                     (size_t)row * ep.ld_dz + col0);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint4 t = a[j];
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&t);
#pragma unroll
                for (int q = 0; q < 8; q++) z[8 * j + q] = bf2f(h[q]);
            }
        } else if (ncols == 32) {
            const float4* a = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ep.dz) +
                                                              (size_t)row * ep.ld_dz + col0);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 t = a[j];
                z[4 * j] = t.x;
                z[4 * j + 1] = t.y;
                z[4 * j + 2] = t.z;
                z[4 * j + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                z[j] = j < ncols ? ld_any(ep.dz, ep.dz_dtype, (size_t)row * ep.ld_dz + col0 + j) : 0.f;
        }
        switch (ep.dz_act) {
            case kRelu:
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] *= act_deriv(z[j], kRelu);
                break;
            case kGelu:
                if constexpr (FAST) {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float d0, d1;
                        gelu_fast_deriv2(z[j], z[j + 1], d0, d1);
                        v[j] *= d0;
                        v[j + 1] *= d1;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] *= act_deriv(z[j], kGelu);
                }
                break;
            default:
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] *= act_deriv(z[j], ep.dz_act);
        }
    }
}

template <bool FAST>
__device__ __forceinline__ void epi_act32(int act, float* v) {
    switch (act) {
        case kIdentity:
            break;
        case kRelu:
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = act_fwd(v[j], kRelu);
            break;
        case kGelu:
            if constexpr (FAST) {
#pragma unroll
                for (int j = 0; j < 32; j += 2) gelu_fast2(v[j], v[j + 1]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = act_fwd(v[j], kGelu);
            }
            break;
        case kGeluMoe:
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = act_fwd(v[j], kGeluMoe);
            break;
        default:
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = act_fwd(v[j], act);
    }
}

__device__ __forceinline__ void store32_f32(float* dst, const float* v) {
#pragma unroll
    for (int j = 0; j < 8; j++)
        reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
__device__ __forceinline__ void store32_bf16(__nv_bfloat16* dst, const float* v) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint4 t;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&t);
#pragma unroll
        for (int q = 0; q < 4; q++) h[q] = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
        reinterpret_cast<uint4*>(dst)[j] = t;
    }
}

// Full 32-column chunk with direct (per-row) stores.
template <bool FAST>
__device__ __forceinline__ void epi_apply32_vec(const Epilogue& ep, int row, int col0, float* v) {
    epi_pre32<FAST>(ep, row, col0, v, 32);
    if (ep.z) {
        if (ep.z_dtype == kBF16)
            store32_bf16(reinterpret_cast<__nv_bfloat16*>(ep.z) + (size_t)row * ep.ld_z + col0, v);
        else
            store32_f32(reinterpret_cast<float*>(ep.z) + (size_t)row * ep.ld_z + col0, v);
    }
    epi_act32<FAST>(ep.act, v);
    int orow = ep.out_rows ? ep.out_rows[row] : row;
    if (ep.c32) store32_f32(ep.c32 + (size_t)orow * ep.ld_c32 + col0, v);
    if (ep.c16) store32_bf16(ep.c16 + (size_t)orow * ep.ld_c16 + col0, v);
}

// ---------------------------------------------------------------------------
// tcgen05 kernel
// ---------------------------------------------------------------------------
struct TcParams {
    int M, N, K;
    int m_tiles, n_tiles, k_blocks, splits, kb_per_split;
    int total_units;
    int vec_ok;
    Epilogue ep;
    float* workspace;  // splits > 1: raw fp32 partials [splits][M][N]
    int* err;
    // grouped: group g owns rows [seg[g], seg[g+1]); B rows offset g * N
    int groups;
    const int* seg;
    const int* seg_end;
    int max_m_tiles_per_group;
    int tma_out;  // outputs leave through the TMA-store epilogue (tz / tc32 / tc16)
    int bk;       // K elements per k-block
    // grouped, MN-major B: group g's [K, N] matrix starts at row g * K of
    // the B tensor map (groups stacked along K)
    int b_kgroup;
    // grouped over K: unit -> (group, m tile, n tile), k-blocks over the
    // group's rows [seg[g], seg_end[g]) rounded up to a k-block; C of group g
    // at ep.c32 + g * c_group_stride
    int group_k;
    long long c_group_stride;
    // static round-robin units (grid = min(units, SMs)) instead of cluster
    // launch control; for grouped GEMMs, whose many empty units are then
    // skipped without a scheduling round trip
    int static_sched;
};

template <int BN, bool TF32>
struct TcCfg {
    static constexpr int BM = 128;
    static constexpr int ELEM = TF32 ? 4 : 2;
    // K extent of a stage in bytes. The whole-row tile (BN = 512) takes
    // 64-byte K rows (64-byte swizzle for K-major operands), so that four
    // 40 KB stages fit beside the epilogue staging instead of two of 80 KB.
    static constexpr int ROW_BYTES = BN == 512 ? 64 : 128;
    static constexpr int BK = ROW_BYTES / ELEM;  // K elements per stage
    static constexpr int CHUNK = 128 / ELEM;  // MN elements per 128-byte chunk
    static constexpr int KSTEP = TF32 ? 8 : 16;  // K per MMA instruction (32 bytes)
    static constexpr int KSTEPS = BK / KSTEP;    // MMA instructions per stage and N slice
    static constexpr int A_BYTES = BM * ROW_BYTES;
    static constexpr int B_BYTES = BN * ROW_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // K-major operands: 8-row swizzle atoms of ROW_BYTES-byte rows
    static constexpr uint32_t K_SBO = 8 * ROW_BYTES;
    static constexpr uint32_t K_LAYOUT = ROW_BYTES == 128 ? 2 : 4;  // 128- or 64-byte swizzle
    // BN = 512 (whole-row LayerNorm mode): one accumulator spanning all of
    // TMEM, filled by two N = 256 MMAs per k step
    static constexpr int NACC = BN == 512 ? 1 : 2;
    static constexpr int NMMA = BN == 512 ? 256 : BN;  // N of one MMA instruction
    static constexpr int STAGES = BN == 512 ? 5 : (BN == 256 ? 4 : 6);
    static constexpr int TMEM_COLS = NACC * BN;
    // MN-major operands: 128-byte chunks along M/N, BK k-rows each. bf16 uses
    // the 16-byte-granule 128B swizzle (8-row atoms, SBO 1024); tf32 needs the
    // 32-byte-granule variant (4-row atoms, SBO 512).
    static constexpr uint32_t MN_LAYOUT = TF32 ? 1 : 2;
    static constexpr uint32_t MN_SBO = TF32 ? 512 : 1024;
    // epilogue staging: per epilogue warp two 2 KB buffers (32 rows x 64 B);
    // one for the whole-row tile, whose fifth stage takes the difference
    static constexpr int NSTG = BN == 512 ? 1 : 2;
    static constexpr int STAGING = 8 * NSTG * 2048;
    static constexpr int SMEM = STAGES * STAGE_BYTES + STAGING + 1024 /*align*/ + 512 /*barriers, queue*/ +
                                (BN == 512 ? 2048 : 0) /*LayerNorm row statistics*/;
    static_assert(SMEM <= 227 * 1024, "dynamic shared memory above the 227 KB per-block limit");
};

// Decode a work unit into (m0, n0, kb0, kb1, split, group); returns false
// for an empty grouped tile.
__device__ __forceinline__ bool tc_decode(const TcParams& p, int u, int BN, int& m0, int& n0, int& kb0, int& kb1,
                                          int& split, int& g, int& row_end) {
    split = u % p.splits;
    int tile = u / p.splits;
    int m_blk, n_blk;
    if (p.group_k) {
        const int per_group = p.m_tiles * p.n_tiles;
        g = tile / per_group;
        const int t = tile % per_group;
        m0 = (t / p.n_tiles) * 128;
        n0 = (t % p.n_tiles) * BN;
        row_end = p.M;
        kb0 = p.seg[g] / p.bk;
        kb1 = (p.seg_end[g] + p.bk - 1) / p.bk;
        return true;
    }
    if (p.groups > 1) {
        // tile -> (group, m within group, n)
        int per_group = p.max_m_tiles_per_group * p.n_tiles;
        g = tile / per_group;
        int t = tile % per_group;
        m_blk = t / p.n_tiles;
        n_blk = t % p.n_tiles;
        int s0 = p.seg[g], s1 = p.seg_end ? p.seg_end[g] : p.seg[g + 1];
        m0 = s0 + m_blk * 128;
        if (m0 >= s1) return false;
        row_end = s1;
    } else {
        g = 0;
        m_blk = tile / p.n_tiles;
        n_blk = tile % p.n_tiles;
        m0 = m_blk * 128;
        row_end = p.M;
    }
    n0 = n_blk * BN;
    kb0 = split * p.kb_per_split;
    kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
    return true;
}

// One unit of work for a CTA: a tile (or split-K slice) and its k-block range.
struct Work {
    int m0, n0, kb0, kb1, split, g, row_end;
};

constexpr int kQueue = 4;  // depth of the work-unit queue from the scheduler to the MMA / epilogue warps

constexpr int kEpiWarps = 8;                    // two per TMEM lane quarter
constexpr int kTcThreads = 64 + 32 * kEpiWarps;  // producer warp + MMA warp + epilogue

template <int BN, bool TF32, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ CUtensorMap tz, const __grid_constant__ CUtensorMap tc32,
                   const __grid_constant__ CUtensorMap tc16, const TcParams p) {
    using C = TcCfg<BN, TF32>;
    static_assert(kEpiWarps == 8, "staging is sized for 8 epilogue warps");
    constexpr uint32_t IDESC = ptx::instr_desc(TF32 ? 2 : 1, A_MN ? 1 : 0, B_MN ? 1 : 0, C::BM, C::NMMA);
    static_assert(BN != 512 || (!A_MN && B_MN), "the 512-wide mode takes a K-major A and an MN-major B");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;
    uint4* clc_resp = reinterpret_cast<uint4*>(staging + C::STAGING);  // 16-byte aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(clc_resp + 1);
    uint64_t* empty = full + C::STAGES;
    uint64_t* acc_full = empty + C::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* clc_bar = acc_empty + 2;
    uint64_t* q_full = clc_bar + 1;
    uint64_t* q_empty = q_full + kQueue;
    uint64_t* ln_bar = q_empty + kQueue;  // LayerNorm mode: epilogue row-statistics exchange
    int* unit_q = reinterpret_cast<int*>(ln_bar + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(unit_q + kQueue);
    float* ln_xch = reinterpret_cast<float*>(staging + C::STAGING + 512);  // [2 passes][2 halves][128 rows]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&acc_full[a], 1);
            ptx::mbar_init(&acc_empty[a], 32 * kEpiWarps);
        }
        ptx::mbar_init(clc_bar, 1);
        for (int q = 0; q < kQueue; q++) {
            ptx::mbar_init(&q_full[q], 1);
            ptx::mbar_init(&q_empty[q], 1 + kEpiWarps);  // the MMA thread + one lane per epilogue warp
        }
        ptx::mbar_init(ln_bar, 32 * kEpiWarps);
        ptx::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tmap(&ta);
        ptx::prefetch_tmap(&tb);
        if (p.tma_out) {
            if (p.ep.z) ptx::prefetch_tmap(&tz);
            if (p.ep.c32) ptx::prefetch_tmap(&tc32);
            if (p.ep.c16) ptx::prefetch_tmap(&tc16);
        }
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- scheduler + TMA producer ----------------
            // Work units are handed out dynamically: this CTA starts with unit
            // blockIdx.x and then takes over units of CTAs that have not been
            // launched yet (cluster launch control: try_cancel). SMs busy with
            // other work (e.g. a collective running beside this GEMM) simply
            // launch fewer CTAs. Units reach the MMA and epilogue warps in
            // order through the shared-memory queue.
            int stage = 0;
            uint32_t phase = 0;
            int qslot = 0;
            uint32_t qphase = 0, clc_phase = 0;
            bool alive = true;     // false after a timed-out wait (error recorded)
            bool pending = false;  // a try_cancel response is in flight
            auto push = [&](int unit) -> bool {
                if (!ptx::mbar_wait(&q_empty[qslot], qphase ^ 1, p.err, kErrTimeoutProducer)) return false;
                unit_q[qslot] = unit;
                ptx::mbar_arrive(&q_full[qslot]);
                if (++qslot == kQueue) {
                    qslot = 0;
                    qphase ^= 1;
                }
                return true;
            };
            int unit = blockIdx.x;
            while (alive) {
                // ask for the next unit while this one's tiles load
                if (!p.static_sched) {
                    ptx::mbar_arrive_expect_tx(clc_bar, 16);
                    ptx::clc_try_cancel(clc_resp, clc_bar);
                    pending = true;
                }
                Work w;
                if (tc_decode(p, unit, BN, w.m0, w.n0, w.kb0, w.kb1, w.split, w.g, w.row_end)) {
                    alive = push(unit);
                    const int m0 = w.m0;
                    // B row (row-grouped, K-major B: groups stacked along N)
                    const int nb = (p.groups > 1 && !p.group_k && !p.b_kgroup) ? w.g * p.N + w.n0 : w.n0;
                    const int kb_row = p.b_kgroup ? w.g * p.K : 0;  // MN-major grouped B: stacked along K
                    for (int kb = w.kb0; alive && kb < w.kb1; kb++) {
                        if (!ptx::mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer)) {
                            alive = false;
                            break;
                        }
                        uint8_t* sa = smem + stage * C::STAGE_BYTES;
                        uint8_t* sb = sa + C::A_BYTES;
                        ptx::mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                        if (!A_MN) {
                            ptx::tma_load_2d(sa, &ta, &full[stage], kb * C::BK, m0);
                        } else {
#pragma unroll
                            for (int c = 0; c < C::BM / C::CHUNK; c++)
                                ptx::tma_load_2d(sa + c * (C::BK * 128), &ta, &full[stage], m0 + c * C::CHUNK,
                                                 kb * C::BK);
                        }
                        if (!B_MN) {
                            ptx::tma_load_2d(sb, &tb, &full[stage], kb * C::BK, nb);
                        } else {
#pragma unroll
                            for (int c = 0; c < BN / C::CHUNK; c++)
                                ptx::tma_load_2d(sb + c * (C::BK * 128), &tb, &full[stage], nb + c * C::CHUNK,
                                                 kb_row + kb * C::BK);
                        }
                        if (++stage == C::STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                if (p.static_sched) {
                    unit += gridDim.x;
                    if (unit >= p.total_units) break;
                    continue;
                }
                // the response is awaited on every path, so none is in flight at exit
                const bool got = ptx::mbar_wait(clc_bar, clc_phase, p.err, kErrTimeoutProducer);
                pending = false;
                clc_phase ^= 1;
                if (!got) {
                    alive = false;
                    break;
                }
                int next;
                if (!ptx::clc_query(clc_resp, next)) break;  // no unlaunched CTA left
                unit = next;
            }
            (void)pending;
            if (alive) push(-1);  // end of work
            // Drain: wait until every issued load has landed before the CTA
            // can exit (bounded).
            for (int s = 0; s < C::STAGES; s++) {
                // the last use of stage s completed if its empty barrier
                // passed; wait for the consumer side to release it
                ptx::mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer);
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            int qslot = 0;
            uint32_t qphase = 0;
            Work w;
            for (;;) {
                if (!ptx::mbar_wait(&q_full[qslot], qphase, p.err, kErrTimeoutMma)) goto mma_done;
                const int unit = unit_q[qslot];
                ptx::mbar_arrive(&q_empty[qslot]);
                if (++qslot == kQueue) {
                    qslot = 0;
                    qphase ^= 1;
                }
                if (unit < 0) break;
                tc_decode(p, unit, BN, w.m0, w.n0, w.kb0, w.kb1, w.split, w.g, w.row_end);
                const int kb0 = w.kb0;
                if (!ptx::mbar_wait(&acc_empty[acc], acc_phase ^ 1, p.err, kErrTimeoutMma)) goto mma_done;
                ptx::tc_fence_after();
                const uint32_t d = tmem_base + acc * BN;
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!ptx::mbar_wait(&full[stage], phase, p.err, kErrTimeoutMma)) goto mma_done;
                    ptx::tc_fence_after();
                    const uint32_t sa = ptx::smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                    for (int h = 0; h < BN / C::NMMA; h++) {
                        // N-slice h of the tile: MN-major B in 128-byte column chunks,
                        // K-major B in ROW_BYTES-byte rows
                        const uint32_t sbh =
                            sb + h * (B_MN ? (C::NMMA / C::CHUNK) * C::BK * 128 : C::NMMA * C::ROW_BYTES);
#pragma unroll
                        for (int k = 0; k < C::KSTEPS; k++) {
                            uint64_t ad =
                                A_MN ? ptx::smem_desc(sa + k * C::KSTEP * 128, C::BK * 128, C::MN_SBO, C::MN_LAYOUT)
                                     : ptx::smem_desc(sa + k * 32, 16, C::K_SBO, C::K_LAYOUT);
                            uint64_t bd =
                                B_MN ? ptx::smem_desc(sbh + k * C::KSTEP * 128, C::BK * 128, C::MN_SBO, C::MN_LAYOUT)
                                     : ptx::smem_desc(sbh + k * 32, 16, C::K_SBO, C::K_LAYOUT);
                            uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
                            if (TF32) ptx::mma_tf32(d + h * C::NMMA, ad, bd, IDESC, accum);
                            else ptx::mma_bf16(d + h * C::NMMA, ad, bd, IDESC, accum);
                        }
                    }
                    ptx::mma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                ptx::mma_commit(&acc_full[acc]);
                if (C::NACC == 2) acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        mma_done:;
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // warp w reads TMEM lanes [32*(w%4), +32) (its hardware lane quarter)
        // and half (w-2)/4 of the tile's columns
        const int lane_grp = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r_in_tile = lane_grp * 32 + lane;
        constexpr int HALF_COLS = BN / 2;
        constexpr bool FAST = !TF32;
        // TMA-store staging: two 2 KB buffers of 32 rows x 64 bytes, 64-byte
        // swizzle (16-byte granule j of row r at j ^ ((r >> 1) & 3)), which is
        // also conflict-free for the row-per-thread writes. Every box (32
        // bf16 or 16 fp32 columns) fills one buffer; the buffers alternate,
        // so writing one overlaps the store of the other (the whole-row tile
        // keeps one buffer per warp and waits for its previous store).
        uint8_t* stg = staging + (warp - 2) * (C::NSTG * 2048);
        int sbuf = 0;
        auto stage_store = [&](const CUtensorMap* map, const uint4* g4, int x, int y) {
            uint8_t* buf = stg + sbuf * 2048;
            if (lane == 0) {
                if (C::NSTG == 2) ptx::bulk_wait_read1();
                else ptx::bulk_wait_read0();
            }
            __syncwarp();
            uint8_t* rowp = buf + lane * 64;
#pragma unroll
            for (int j = 0; j < 4; j++) *reinterpret_cast<uint4*>(rowp + ((j ^ ((lane >> 1) & 3)) << 4)) = g4[j];
            ptx::fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                ptx::tma_store_2d(map, buf, x, y);
                ptx::bulk_commit();
            }
            if (C::NSTG == 2) sbuf ^= 1;
        };
        auto out_f32 = [&](const CUtensorMap* map, const float* v, int col0, int y) {
            const uint4* g8 = reinterpret_cast<const uint4*>(v);
            stage_store(map, g8, col0, y);
            if (col0 + 16 < p.N) stage_store(map, g8 + 4, col0 + 16, y);  // uniform
        };
        auto out_bf16 = [&](const CUtensorMap* map, const float* v, int col0, int y) {
            uint4 g4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&g4[j]);
#pragma unroll
                for (int q = 0; q < 4; q++) h[q] = __floats2bfloat162_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
            }
            stage_store(map, g4, col0, y);
        };
        auto out_f16 = [&](const CUtensorMap* map, const float* v, int col0, int y) {
            uint4 g4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                __half2* h = reinterpret_cast<__half2*>(&g4[j]);
#pragma unroll
                for (int q = 0; q < 4; q++) h[q] = __floats2half2_rn(v[8 * j + 2 * q], v[8 * j + 2 * q + 1]);
            }
            stage_store(map, g4, col0, y);
        };
        // TMA-store path, after epi_pre32: the pre-activation, the
        // activation and the outputs of 32 columns (col0 < N); rows >= M and
        // columns >= N of a box are clipped by the store
        auto store_tma = [&](int col0, int y, float* v) {
            if (p.ep.z) {
                if (p.ep.z_dtype == kBF16) out_bf16(&tz, v, col0, y);
                else out_f32(&tz, v, col0, y);
            }
            epi_act32<FAST>(p.ep.act, v);
            if (p.ep.c32) out_f32(&tc32, v, col0, y);
            if (p.ep.c16) {
                if (p.ep.c16_half) out_f16(&tc16, v, col0, y);
                else out_bf16(&tc16, v, col0, y);
            }
        };
        // Direct-store path: finish 32 accumulator columns (col0 < N) of
        // this thread's row.
        auto finish = [&](const Work& w, int col0, float* v) {
            const int row = w.m0 + r_in_tile;
            if (row >= w.row_end) return;
            const bool full = p.vec_ok && col0 + 32 <= p.N;
            if (p.group_k) {
                // per-group weight gradient: plain fp32 store
                float* dst = p.ep.c32 + (size_t)w.g * p.c_group_stride + (size_t)row * p.ep.ld_c32 + col0;
                if (full) {
                    store32_f32(dst, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (col0 + j < p.N) dst[j] = v[j];
                }
                return;
            }
            if (p.splits > 1) {
                float* ws = p.workspace + ((size_t)w.split * p.M + row) * p.N + col0;
                if (full) {
                    store32_f32(ws, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (col0 + j < p.N) ws[j] = v[j];
                }
            } else if (full && !p.ep.col_block) {
                epi_apply32_vec<FAST>(p.ep, row, col0, v);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (col0 + j < p.N) epi_apply(p.ep, row, col0 + j, v[j]);
            }
        };
        // Epilogue operands of a full 32-column chunk of this thread's row
        // (the fp32 residual, the bf16 activation input of act'), loaded one
        // chunk ahead of their use (TMA-store path, vectorisable operands).
        const bool ahead_add = p.tma_out && p.vec_ok && p.ep.add != nullptr;
        const bool ahead_dz = p.tma_out && p.vec_ok && p.ep.dz != nullptr && p.ep.dz_dtype == kBF16;
        float addv[32];
        uint4 dzv[4];
        auto load_ahead = [&](const Work& w, int col0) -> bool {
            const int row = w.m0 + r_in_tile;
            if (!(ahead_add || ahead_dz) || row >= w.row_end || col0 + 32 > p.N) return false;
            if (ahead_add) {
                const float4* a = reinterpret_cast<const float4*>(p.ep.add + (size_t)row * p.ep.ld_add + col0);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 t = a[j];
                    addv[4 * j] = t.x;
                    addv[4 * j + 1] = t.y;
                    addv[4 * j + 2] = t.z;
                    addv[4 * j + 3] = t.w;
                }
            }
            if (ahead_dz) {
                const uint4* a = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.ep.dz) +
                                                                (size_t)row * p.ep.ld_dz + col0);
#pragma unroll
                for (int j = 0; j < 4; j++) dzv[j] = a[j];
            }
            return true;
        };
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t ln_phase = 0;
        int qslot = 0;
        uint32_t qphase = 0;
        Work w;
        for (;;) {
            int unit = -1;
            if (lane == 0) {
                if (ptx::mbar_wait(&q_full[qslot], qphase, p.err, kErrTimeoutEpilogue)) unit = unit_q[qslot];
                ptx::mbar_arrive(&q_empty[qslot]);
            }
            unit = __shfl_sync(0xffffffffu, unit, 0);
            if (++qslot == kQueue) {
                qslot = 0;
                qphase ^= 1;
            }
            if (unit < 0) break;
            tc_decode(p, unit, BN, w.m0, w.n0, w.kb0, w.kb1, w.split, w.g, w.row_end);
            if constexpr (BN == 512) {
                // ---- whole-row LayerNorm (N = 512) ----
                // This warp owns 256 columns (half `half`) of its 32 rows; the
                // two halves of a row meet through shared memory twice (the
                // sum, then the centred sum of squares), each time on an
                // mbarrier with a bounded wait. Pass 1 forms x = alpha*acc +
                // add_scale*residual (the residual read once, the next 32
                // columns' loads in flight while this chunk is summed) and
                // writes x back over the accumulator in TMEM; passes 2 and 3
                // read x from TMEM only.
                const int row = w.m0 + r_in_tile;
                const bool rvalid = row < w.row_end;
                const int cb = half * 256;
                const uint32_t tb = tmem_base + ((uint32_t)(lane_grp * 32) << 16) + cb;
                const bool okw = ptx::mbar_wait(&acc_full[0], acc_phase, p.err, kErrTimeoutEpilogue);
                ptx::tc_fence_after();
                const bool has_add = okw && p.ep.add != nullptr && rvalid;
                const float4* addp =
                    has_add ? reinterpret_cast<const float4*>(p.ep.add + (size_t)row * p.ep.ld_add + cb) : nullptr;
                float s1 = 0.f;
                if (okw) {
                    float4 nxt[8];
                    if (has_add) {
#pragma unroll
                        for (int j = 0; j < 8; j++) nxt[j] = addp[j];
                    }
#pragma unroll 1
                    for (int c = 0; c < 256; c += 32) {
                        float4 cur[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) cur[j] = nxt[j];
                        if (has_add && c + 32 < 256) {
#pragma unroll
                            for (int j = 0; j < 8; j++) nxt[j] = addp[(c + 32) / 4 + j];
                        }
                        uint32_t r[32];
                        ptx::tmem_ld32(tb + c, r);
                        ptx::tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            float v = __uint_as_float(r[j]) * p.ep.alpha;
                            if (has_add) {
                                const float4 t = cur[j / 4];
                                const float a = (j & 3) == 0 ? t.x : (j & 3) == 1 ? t.y : (j & 3) == 2 ? t.z : t.w;
                                v = fmaf(p.ep.add_scale, a, v);
                            }
                            s1 += v;
                            r[j] = __float_as_uint(v);
                        }
                        ptx::tmem_st16(tb + c, r);
                        ptx::tmem_st16(tb + c + 16, r + 16);
                    }
                    ptx::tmem_st_wait();
                }
                // x of 64 columns from TMEM (passes 2 and 3)
                auto ld_x64 = [&](int c, uint32_t* r) {
                    ptx::tmem_ld32(tb + c, r);
                    ptx::tmem_ld32(tb + c + 32, r + 32);
                    ptx::tmem_ld_wait();
                };
                ln_xch[half * 128 + r_in_tile] = s1;
                ptx::mbar_arrive(ln_bar);
                const bool ok1 = ptx::mbar_wait(ln_bar, ln_phase, p.err, kErrTimeoutEpilogue);
                ln_phase ^= 1;
                const float mean = (ln_xch[r_in_tile] + ln_xch[128 + r_in_tile]) * (1.f / 512.f);
                float s2 = 0.f;
                if (okw) {
#pragma unroll 1
                    for (int c = 0; c < 256; c += 64) {
                        uint32_t r[64];
                        ld_x64(c, r);
#pragma unroll
                        for (int j = 0; j < 64; j++) {
                            const float dv = __uint_as_float(r[j]) - mean;
                            s2 = fmaf(dv, dv, s2);
                        }
                    }
                }
                ln_xch[256 + half * 128 + r_in_tile] = s2;
                ptx::mbar_arrive(ln_bar);
                const bool ok2 = ptx::mbar_wait(ln_bar, ln_phase, p.err, kErrTimeoutEpilogue);
                ln_phase ^= 1;
                const float var = (ln_xch[256 + r_in_tile] + ln_xch[384 + r_in_tile]) * (1.f / 512.f);
                const float rstd = 1.f / sqrtf(var + 1e-5f);
                const int y0 = w.m0 + lane_grp * 32;
                if (okw && y0 < p.M) {  // rows >= M of the box are clipped by the store
#pragma unroll 1
                    for (int c = 0; c < 256; c += 32) {
                        uint32_t r[32];
                        ptx::tmem_ld32(tb + c, r);
                        ptx::tmem_ld_wait();
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) v[j] = (__uint_as_float(r[j]) - mean) * rstd;
                        if (p.ep.c32) out_f32(&tc32, v, cb + c, y0);
                        if (p.ep.c16) out_bf16(&tc16, v, cb + c, y0);
                    }
                }
                if (half == 0 && rvalid && okw) p.ep.ln_rstd[row] = rstd;
                ptx::tc_fence_before();
                ptx::mbar_arrive(&acc_empty[0]);
                acc_phase ^= 1;
                if (!okw || !ok1 || !ok2) break;
                continue;
            }
            const int c_begin = half * HALF_COLS, c_end = (half + 1) * HALF_COLS;
            // target column of this thread's row (head + loss fusion)
            const int ce_t = (p.ep.ce_tgt && w.m0 + r_in_tile < w.row_end) ? p.ep.ce_tgt[w.m0 + r_in_tile] : -1;
            // the first chunk's operands load while this tile's MMAs run
            bool have = load_ahead(w, w.n0 + c_begin);
            if (!ptx::mbar_wait(&acc_full[acc], acc_phase, p.err, kErrTimeoutEpilogue)) break;
            ptx::tc_fence_after();
#pragma unroll 1
            for (int c = c_begin; c < c_end; c += 32) {
                uint32_t r[32];
                ptx::tmem_ld32(tmem_base + ((uint32_t)(lane_grp * 32) << 16) + acc * BN + c, r);
                ptx::tmem_ld_wait();
                const int col0 = w.n0 + c;
                if (col0 >= p.N) continue;  // uniform across the warp
                float v[32];
                const bool no_k = w.kb1 <= w.kb0;  // empty k range (a group with no rows): C = 0
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = no_k ? 0.f : __uint_as_float(r[j]);
                if (p.tma_out) {
                    const int y = w.m0 + lane_grp * 32;
                    if (y >= p.M) continue;  // slab entirely past M: nothing to store (uniform)
                    const int row = w.m0 + r_in_tile;
                    const int nc = col0 + 32 <= p.N ? 32 : p.N - col0;
                    if (row < w.row_end)
                        epi_pre32<FAST>(p.ep, row, col0, v, nc, have && ahead_add ? addv : nullptr,
                                        have && ahead_dz ? dzv : nullptr);
                    if (ce_t >= col0 && ce_t < col0 + nc) {  // this chunk holds the target logit
                        float tv = 0.f;
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j == ce_t) tv = v[j];
                        p.ep.ce_tlogit[row] = tv;
                    }
                    // the next chunk's operands load while this chunk is stored
                    have = c + 32 < c_end && load_ahead(w, col0 + 32);
                    store_tma(col0, y, v);
                } else {
                    finish(w, col0, v);
                }
            }
            ptx::tc_fence_before();
            ptx::mbar_arrive(&acc_empty[acc]);
            if (C::NACC == 2) acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
        if (p.tma_out && lane == 0) ptx::bulk_wait_all();
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Sum split-K partials in split order, then the full epilogue; four
// consecutive columns per thread when N % 4 == 0 and the workspace is aligned.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int M, int N, Epilogue ep, int vec4) {
    const size_t total = (size_t)M * N;
    if (vec4 == 2) {
        // Plain fp32 output (weight gradients): alpha, an optional fp32
        // residual, column blocks of a multiple of 4; the splits' partials are
        // loaded four at a time and summed in split order, one 16-byte store.
        const size_t i4 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (4 * i4 >= total) return;
        const float4* w4 = reinterpret_cast<const float4*>(ws) + i4;
        const size_t stride4 = total / 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        int s = 0;
        for (; s + 4 <= splits; s += 4) {
            float4 w[4];
#pragma unroll
            for (int k = 0; k < 4; k++) w[k] = __ldcs(w4 + (size_t)(s + k) * stride4);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                v.x += w[k].x;
                v.y += w[k].y;
                v.z += w[k].z;
                v.w += w[k].w;
            }
        }
        for (; s < splits; s++) {
            const float4 w = __ldcs(w4 + (size_t)s * stride4);
            v.x += w.x;
            v.y += w.y;
            v.z += w.z;
            v.w += w.w;
        }
        const int row = (int)(4 * i4 / N), col = (int)(4 * i4 % N);
        v.x *= ep.alpha;
        v.y *= ep.alpha;
        v.z *= ep.alpha;
        v.w *= ep.alpha;
        if (ep.add) {
            const float4 a = *reinterpret_cast<const float4*>(ep.add + (size_t)row * ep.ld_add + col);
            v.x += ep.add_scale * a.x;
            v.y += ep.add_scale * a.y;
            v.z += ep.add_scale * a.z;
            v.w += ep.add_scale * a.w;
        }
        float* dst;
        if (ep.col_block) {
            const int b = col / ep.col_block;
            dst = ep.c32 + b * ep.col_block_stride + (size_t)row * ep.ld_c32 + (col - b * ep.col_block);
        } else {
            dst = ep.c32 + (size_t)row * ep.ld_c32 + col;
        }
        *reinterpret_cast<float4*>(dst) = v;
        return;
    }
    if (vec4) {
        const size_t i4 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (4 * i4 >= total) return;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < splits; s++) {
            const float4 w = __ldcs(reinterpret_cast<const float4*>(ws + (size_t)s * total) + i4);
            v.x += w.x;
            v.y += w.y;
            v.z += w.z;
            v.w += w.w;
        }
        const int row = (int)(4 * i4 / N), col = (int)(4 * i4 % N);
        epi_apply(ep, row, col, v.x);
        epi_apply(ep, row, col + 1, v.y);
        epi_apply(ep, row, col + 2, v.z);
        epi_apply(ep, row, col + 3, v.w);
        return;
    }
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    int row = (int)(idx / N), col = (int)(idx % N);
    float v = 0.f;
    for (int s = 0; s < splits; s++) v += ws[(size_t)s * total + idx];
    epi_apply(ep, row, col, v);
}

// ---------------------------------------------------------------------------
// SIMT fp32 kernel: 64x64 tile, 256 threads, 4x4 outputs per thread, each
// output accumulated with fmaf in increasing k.
// ---------------------------------------------------------------------------
struct SimtParams {
    int M, N, K;
    GemmOperand a, b;
    Epilogue ep;
    int groups;
    const int* seg;
    const int* seg_end;
    long long b_group_stride;
    bool group_k;
    long long c_group_stride;
};

__device__ __forceinline__ float ld_op(const GemmOperand& o, long long i, long long k) {
    size_t idx = o.mn_major ? (size_t)(k * o.ld + i) : (size_t)(i * o.ld + k);
    return ld_any(o.ptr, o.dtype, idx);
}

// Narrow outputs (N <= 32, e.g. a 10-class head) with a K-major A: each
// warp owns kNarrowRows rows of C; lane l takes the 8 consecutive k of
// every 256-wide k step starting at 8 l (one 16-byte load of bf16 A per
// row, two for fp32); B is staged in shared memory per 256-k step as fp32
// with an odd row stride; one butterfly reduction per output at the end.
// For the tensor-core precision modes only: its summation order differs
// from the k-sequential fp32 parity kernel.
constexpr int kNarrowK = 256;
constexpr int kNarrowWarps = 8;
constexpr int kNarrowRows = 4;
template <int NMAX, typename TA>
__global__ void __launch_bounds__(32 * kNarrowWarps) gemm_narrow_kernel(const SimtParams p) {
    __shared__ float Bs[kNarrowK * (NMAX + 1)];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kNarrowWarps + warp) * kNarrowRows;
    const TA* A = reinterpret_cast<const TA*>(p.a.ptr);
    float acc[kNarrowRows][NMAX];
#pragma unroll
    for (int r = 0; r < kNarrowRows; r++)
#pragma unroll
        for (int n = 0; n < NMAX; n++) acc[r][n] = 0.f;
    for (int k0 = 0; k0 < p.K; k0 += kNarrowK) {
        const int kn = min(kNarrowK, p.K - k0);
        __syncthreads();
        for (int i = threadIdx.x; i < kNarrowK * NMAX; i += blockDim.x) {
            const int kk = i / NMAX, n = i % NMAX;
            Bs[kk * (NMAX + 1) + n] = (n < p.N && kk < kn) ? ld_op(p.b, n, k0 + kk) : 0.f;
        }
        __syncthreads();
        const int kl = 8 * lane;  // this lane's 8 k within the step
        if (kl >= kn) continue;
#pragma unroll
        for (int r = 0; r < kNarrowRows; r++) {
            const int row = row0 + r;
            if (row >= p.M) break;
            float a[8];
            const TA* src = A + (size_t)row * p.a.ld + k0 + kl;
            if (kl + 8 <= kn) {
                if constexpr (sizeof(TA) == 2) {
                    const uint4 t = *reinterpret_cast<const uint4*>(src);
                    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&t);
#pragma unroll
                    for (int j = 0; j < 8; j++) a[j] = bf2f(h[j]);
                } else {
                    const float4 t0 = reinterpret_cast<const float4*>(src)[0];
                    const float4 t1 = reinterpret_cast<const float4*>(src)[1];
                    a[0] = t0.x; a[1] = t0.y; a[2] = t0.z; a[3] = t0.w;
                    a[4] = t1.x; a[5] = t1.y; a[6] = t1.z; a[7] = t1.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) a[j] = kl + j < kn ? ld_any(src, p.a.dtype, j) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float* b = Bs + (kl + j) * (NMAX + 1);
#pragma unroll
                for (int n = 0; n < NMAX; n++) acc[r][n] = fmaf(a[j], b[n], acc[r][n]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kNarrowRows; r++) {
        const int row = row0 + r;
        float mine = 0.f;
#pragma unroll
        for (int n = 0; n < NMAX; n++) {
            float s = acc[r][n];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == n) mine = s;
        }
        if (row < p.M && lane < p.N) epi_apply(p.ep, row, lane, mine);
    }
}

__global__ void __launch_bounds__(256) gemm_simt_kernel(const SimtParams p) {
    __shared__ float As[16][64 + 1];
    __shared__ float Bs[16][64 + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    int g = 0, row_end = p.M;
    GemmOperand b = p.b;
    Epilogue ep = p.ep;
    int kbeg = 0, kend = p.K;
    int mbase = m0;
    if (p.groups > 1 && !p.group_k) {
        // blockIdx.z = group; rows [seg[g], seg_end[g])
        g = blockIdx.z;
        int s0 = p.seg[g], s1 = p.seg_end ? p.seg_end[g] : p.seg[g + 1];
        if (s0 + m0 >= s1) return;
        row_end = s1;
        mbase = s0 + m0;
        b.ptr = (const char*)b.ptr + (size_t)g * p.b_group_stride * (b.dtype == kBF16 ? 2 : 4);
    } else if (p.group_k) {
        // blockIdx.z = group; reduce k in [seg[g], seg_end[g]); C block g
        g = blockIdx.z;
        kbeg = p.seg[g];
        kend = p.seg_end ? p.seg_end[g] : p.seg[g + 1];
        if (ep.c32) ep.c32 += (size_t)g * p.c_group_stride;
        if (ep.c16) ep.c16 += (size_t)g * p.c_group_stride;
    }
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
    for (int k0 = kbeg; k0 < kend; k0 += 16) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            int kk = e / 64, ii = e % 64;
            int gm = mbase + ii, gk = k0 + kk, gn = n0 + ii;
            As[kk][ii] = (gm < row_end && gk < kend) ? ld_op(p.a, gm, gk) : 0.f;
            Bs[kk][ii] = (gn < p.N && gk < kend) ? ld_op(b, gn, gk) : 0.f;
        }
        __syncthreads();
        const int kmax = min(16, kend - k0);
        for (int kk = 0; kk < kmax; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int row = mbase + ty + 16 * i;
        if (row >= row_end) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int col = n0 + tx + 16 * j;
            if (col < p.N) epi_apply(ep, row, col, acc[i][j]);
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// 2D map over a row-major [outer, inner] array with leading dimension ld
// (elements); box {box_inner, box_outer}; 128-byte swizzle (32-byte granules
// when atom32: MN-major tf32 operands; 64-byte swizzle when sw64: K-major
// operands of 64-byte K rows).
static bool make_map(CUtensorMap* m, const void* ptr, int dtype, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer, bool atom32 = false, bool sw64 = false) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return false;
    const int es = dtype == kBF16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                            : (sw64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B),
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Output map for the TMA-store epilogue: row-major [rows, cols] with leading
// dimension ld; boxes of 32 rows x 64 bytes with 64-byte swizzle (bf16: 32
// columns, fp32: 16 columns), so every box fills one 2 KB staging buffer.
static bool make_out_map(CUtensorMap* m, const void* ptr, int dtype, long long cols, long long rows, long long ld) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return false;
    const int es = dtype == kF32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)(64 / es), 32};
    cuuint32_t estr[2] = {1, 1};
    return enc(m,
               dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                              : (dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32),
               2,
               const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool operand_tc_ok(const GemmOperand& o) {
    const int es = o.dtype == kBF16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(o.ptr) & 15) != 0) return false;
    if ((o.ld * es) % 16 != 0) return false;
    return true;
}

bool gemm_uses_tensor_cores(const GemmDesc& d) {
    if (d.engine == kEngineSimt) return false;
    if (d.a.dtype != d.b.dtype) return false;
    if (!operand_tc_ok(d.a) || !operand_tc_ok(d.b)) return false;
    if (d.M <= 0 || d.N <= 0 || d.K <= 0) return false;
    // very narrow outputs waste a 128-wide tile; the SIMT kernel is cheaper
    if (d.N < 32) return false;
    if (d.groups > 1) {
        const int bk = d.a.dtype == kBF16 ? 64 : 32;
        if (d.group_k) {
            // both operands stored token-major ([K rows][M or N]); segment
            // starts are multiples of 128 rows and rows past a segment's end
            // up to the next k-block are zero (MoE dispatch padding)
            if (!d.a.mn_major || !d.b.mn_major || !d.seg || !d.seg_end || !d.ep.c32) return false;
            if (d.ep.add || d.ep.c16 || d.ep.z || d.ep.act || d.ep.dz || d.ep.row_scale || d.ep.out_rows) return false;
            return true;
        }
        // row groups: one 2D tensor map over all groups' B matrices, stacked
        // along N (K-major) or along K (MN-major, K a whole number of k-blocks)
        if (!d.b.mn_major) return d.b_group_stride == (long long)d.N * d.b.ld;
        return d.b_group_stride == (long long)d.K * d.b.ld && d.K % bk == 0;
    }
    return true;
}

// 256-wide tiles whenever N allows; grouped GEMMs only when N is a whole
// number of tiles (a K-major B stacked along N must not straddle groups).
// (128-wide tiles for the N = 512 layers measured slower: ff2 49 -> 62 us.)
static int pick_bn(const GemmDesc& d) {
    if (d.ep.ln_rstd) return 512;  // whole-row LayerNorm mode
    return d.N >= 256 && (d.groups == 1 || d.N % 256 == 0) ? 256 : 128;
}

static void pick_splits(const GemmDesc& d, int bn, int& splits, int& kb_per_split, int k_blocks) {
    splits = 1;
    if (d.groups == 1 && !d.ep.ln_rstd) {  // (a row's LayerNorm needs its whole K sum)
        const int tiles = ((d.M + 127) / 128) * ((d.N + bn - 1) / bn);
        const int sms = num_sms();
        if (d.splits > 0) splits = d.splits;
        else if (tiles < sms / 2 && k_blocks >= 16) {
            // as many splits as keep every unit in one wave
            splits = sms / tiles;
            splits = min(splits, k_blocks / 8);
            splits = max(splits, 1);
        }
    }
    kb_per_split = (k_blocks + splits - 1) / splits;
    splits = (k_blocks + kb_per_split - 1) / kb_per_split;
}

size_t gemm_workspace_floats(const GemmDesc& d) {
    if (!gemm_uses_tensor_cores(d)) return 0;
    const int bn = pick_bn(d);
    const int bk = d.a.dtype == kBF16 ? 64 : 32;
    const int kblocks = (d.K + bk - 1) / bk;
    int splits, kbps;
    pick_splits(d, bn, splits, kbps, kblocks);
    return splits > 1 ? (size_t)splits * d.M * d.N : 0;
}

struct OutMaps {
    CUtensorMap z, c32, c16;
};

template <int BN, bool TF32, bool A_MN, bool B_MN>
static cudaError_t launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om, const TcParams& p,
                             cudaStream_t s) {
    using C = TcCfg<BN, TF32>;
    auto k = gemm_tc_kernel<BN, TF32, A_MN, B_MN>;
    // the attribute belongs to the current device: set it once per device
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (!attr[dev]) {
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        attr[dev] = true;
    }
    // one CTA per unit; running CTAs take over the units of CTAs not yet
    // launched (static scheduling: one CTA per SM, units round-robin)
    int grid = p.static_sched ? min(p.total_units, num_sms()) : p.total_units;
    if (grid <= 0) return cudaSuccess;
    k<<<grid, kTcThreads, C::SMEM, s>>>(ta, tb, om.z, om.c32, om.c16, p);
    return cudaGetLastError();
}

template <int BN, bool TF32>
static cudaError_t launch_tc_majors(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps& om,
                                    const TcParams& p, bool amn, bool bmn, cudaStream_t s) {
    if (!amn && !bmn) return launch_tc<BN, TF32, false, false>(ta, tb, om, p, s);
    if (!amn && bmn) return launch_tc<BN, TF32, false, true>(ta, tb, om, p, s);
    if (amn && !bmn) return launch_tc<BN, TF32, true, false>(ta, tb, om, p, s);
    return launch_tc<BN, TF32, true, true>(ta, tb, om, p, s);
}

static bool ep_vec_ok(const GemmDesc& d) {
    const Epilogue& e = d.ep;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (e.add && (e.ld_add % 4 || !al(e.add))) return false;
    if (e.dz && (e.ld_dz % 8 || !al(e.dz))) return false;
    if (e.z && (e.ld_z % 8 || !al(e.z))) return false;
    if (e.c32 && (e.ld_c32 % 4 || !al(e.c32))) return false;
    if (e.c16 && (e.ld_c16 % 8 || !al(e.c16))) return false;
    if (d.workspace && !al(d.workspace)) return false;
    if (d.N % 4) return false;
    return true;
}

static int gemm_tc(const GemmDesc& d, cudaStream_t s, int* dev_err) {
    const bool tf32 = d.a.dtype == kF32;
    const int bn = pick_bn(d);
    // K elements per stage: 128-byte K rows, 64-byte rows for the whole-row
    // tile (TcCfg::ROW_BYTES)
    const bool row64 = bn == 512;
    const int bk = (tf32 ? 32 : 64) / (row64 ? 2 : 1);
    const int chunk = tf32 ? 32 : 64;
    CUtensorMap ta, tb;
    // A: M x K. K-major -> array [M][ld] (inner K); MN-major -> [K][ld] (inner M)
    bool ok;
    if (!d.a.mn_major) ok = make_map(&ta, d.a.ptr, d.a.dtype, d.K, d.M, d.a.ld, bk, 128, false, row64);
    else ok = make_map(&ta, d.a.ptr, d.a.dtype, d.M, d.K, d.a.ld, chunk, bk, tf32);
    if (!ok) return -2;
    const bool b_kgroup = d.groups > 1 && !d.group_k && d.b.mn_major;
    const long long brows = (d.groups > 1 && !d.group_k && !b_kgroup) ? (long long)d.N * d.groups : d.N;
    const long long bk_rows = b_kgroup ? (long long)d.K * d.groups : d.K;
    if (!d.b.mn_major) ok = make_map(&tb, d.b.ptr, d.b.dtype, d.K, brows, d.b.ld, bk, bn, false, row64);
    else ok = make_map(&tb, d.b.ptr, d.b.dtype, brows, bk_rows, d.b.ld, chunk, bk, tf32);
    if (!ok) return -2;

    TcParams p;
    p.M = d.M;
    p.N = d.N;
    p.K = d.K;
    p.m_tiles = (d.M + 127) / 128;
    p.n_tiles = (d.N + bn - 1) / bn;
    p.k_blocks = (d.K + bk - 1) / bk;
    pick_splits(d, bn, p.splits, p.kb_per_split, p.k_blocks);
    p.ep = d.ep;
    p.err = dev_err;
    p.groups = d.groups;
    p.seg = d.seg;
    p.seg_end = d.seg_end;
    p.max_m_tiles_per_group = p.m_tiles;
    p.bk = bk;
    p.b_kgroup = b_kgroup ? 1 : 0;
    p.group_k = d.group_k ? 1 : 0;
    p.c_group_stride = d.c_group_stride;
    p.static_sched = d.groups > 1 ? 1 : 0;
    p.workspace = nullptr;
    if (p.splits > 1) {
        if (!d.workspace || d.workspace_floats < (size_t)p.splits * d.M * d.N) return -3;
        p.workspace = d.workspace;
    }
    p.vec_ok = ep_vec_ok(d) ? 1 : 0;
    if (d.group_k) {
        p.total_units = d.groups * p.m_tiles * p.n_tiles;
    } else if (d.groups > 1) {
        p.total_units = d.groups * p.max_m_tiles_per_group * p.n_tiles * p.splits;
    } else {
        p.total_units = p.m_tiles * p.n_tiles * p.splits;
    }
    // TMA-store epilogue: plain row-major outputs of a single (non-split,
    // non-grouped, non-scattered) GEMM; the store clips rows >= M, cols >= N
    OutMaps om;
    memset(&om, 0, sizeof(om));
    p.tma_out = 0;
    // (row-grouped GEMMs too: a tile never crosses an expert's 128-row
    // padded segment, and padding rows, whose operand rows are zero, store
    // zeros)
    if (p.vec_ok && !d.group_k && p.splits == 1 && !d.ep.out_rows && !d.ep.col_block &&
        (d.ep.z || d.ep.c32 || d.ep.c16)) {
        bool okm = true;
        if (d.ep.z) okm = okm && make_out_map(&om.z, d.ep.z, d.ep.z_dtype, d.N, d.M, d.ep.ld_z);
        if (d.ep.c32) okm = okm && make_out_map(&om.c32, d.ep.c32, kF32, d.N, d.M, d.ep.ld_c32);
        if (d.ep.c16) okm = okm && make_out_map(&om.c16, d.ep.c16, d.ep.c16_half ? kF16 : kBF16, d.N, d.M, d.ep.ld_c16);
        p.tma_out = okm ? 1 : 0;
    }
    if (d.ep.ce_tgt && (!p.tma_out || !d.ep.ce_tlogit)) return -6;  // captured on the TMA-store path
    if (d.ep.c16_half && !p.tma_out) return -6;
    if (d.ep.ln_rstd) {
        // whole-row LayerNorm: N = 512, K-major A, MN-major B, no split, TMA stores
        if (d.N != 512 || d.groups != 1 || d.a.mn_major || !d.b.mn_major || p.splits != 1 || !p.tma_out ||
            d.ep.z || d.ep.act || d.ep.dz || d.ep.row_scale || d.ep.ce_tgt || d.ep.c16_half)
            return -7;
    }
    cudaError_t e;
    if (bn == 512) {
        e = tf32 ? launch_tc<512, true, false, true>(ta, tb, om, p, s) : launch_tc<512, false, false, true>(ta, tb, om, p, s);
    } else if (bn == 256) {
        e = tf32 ? launch_tc_majors<256, true>(ta, tb, om, p, d.a.mn_major, d.b.mn_major, s)
                 : launch_tc_majors<256, false>(ta, tb, om, p, d.a.mn_major, d.b.mn_major, s);
    } else {
        e = tf32 ? launch_tc_majors<128, true>(ta, tb, om, p, d.a.mn_major, d.b.mn_major, s)
                 : launch_tc_majors<128, false>(ta, tb, om, p, d.a.mn_major, d.b.mn_major, s);
    }
    if (e != cudaSuccess) return -5;
    if (p.splits > 1) {
        size_t total = (size_t)d.M * d.N;
        int vec4 = d.N % 4 == 0 && !(reinterpret_cast<uintptr_t>(p.workspace) & 15);
        // the plain fp32-output form (every 16-byte group of a row in one
        // column block, 16-byte aligned rows) takes the vector path
        const Epilogue& e2 = d.ep;
        if (vec4 && e2.c32 && !e2.c16 && !e2.z && !e2.dz && !e2.act && !e2.row_scale && !e2.out_rows &&
            (e2.col_block % 4) == 0 && (e2.col_block_stride % 4) == 0 && (e2.ld_c32 % 4) == 0 &&
            !(reinterpret_cast<uintptr_t>(e2.c32) & 15) &&
            (!e2.add || ((e2.ld_add % 4) == 0 && !(reinterpret_cast<uintptr_t>(e2.add) & 15))))
            vec4 = 2;
        const size_t threads = vec4 ? total / 4 : total;
        splitk_reduce_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(p.workspace, p.splits, d.M, d.N, d.ep,
                                                                             vec4);
        if (cudaGetLastError() != cudaSuccess) return -5;
    }
    return 0;
}

static int gemm_simt(const GemmDesc& d, cudaStream_t s) {
    SimtParams p;
    // narrow kernel: K-major A whose rows are 16-byte aligned
    const int aes = d.a.dtype == kBF16 ? 2 : 4;
    const bool narrow = d.engine != kEngineSimt && d.groups == 1 && d.N <= 32 && !d.ep.out_rows &&
                        !d.ep.col_block && !d.a.mn_major && (reinterpret_cast<uintptr_t>(d.a.ptr) & 15) == 0 &&
                        (d.a.ld * aes) % 16 == 0;
    p.M = d.M;
    p.N = d.N;
    p.K = d.K;
    p.a = d.a;
    p.b = d.b;
    p.ep = d.ep;
    p.groups = d.groups;
    p.seg = d.seg;
    p.seg_end = d.seg_end;
    p.b_group_stride = d.b_group_stride;
    p.group_k = d.group_k;
    p.c_group_stride = d.c_group_stride;
    if (narrow) {
        const int rows = kNarrowWarps * kNarrowRows;
        const unsigned blocks = (unsigned)((d.M + rows - 1) / rows);
        const bool h = d.a.dtype == kBF16;
        if (d.N <= 16) {
            if (h) gemm_narrow_kernel<16, __nv_bfloat16><<<blocks, 32 * kNarrowWarps, 0, s>>>(p);
            else gemm_narrow_kernel<16, float><<<blocks, 32 * kNarrowWarps, 0, s>>>(p);
        } else {
            if (h) gemm_narrow_kernel<32, __nv_bfloat16><<<blocks, 32 * kNarrowWarps, 0, s>>>(p);
            else gemm_narrow_kernel<32, float><<<blocks, 32 * kNarrowWarps, 0, s>>>(p);
        }
        return cudaGetLastError() == cudaSuccess ? 0 : -5;
    }
    dim3 grid((d.N + 63) / 64, (d.M + 63) / 64, d.groups);
    if (grid.x == 0 || grid.y == 0) return 0;
    gemm_simt_kernel<<<grid, 256, 0, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int gemm(const GemmDesc& d, cudaStream_t s, int* dev_err) {
    if (d.M < 0 || d.N < 0 || d.K < 0) return -1;
    if (d.M == 0 || d.N == 0) return 0;
    if (!d.a.ptr || !d.b.ptr || d.a.ld <= 0 || d.b.ld <= 0) return -1;
    if (!d.ep.c32 && !d.ep.c16 && !d.ep.z) return -1;
    if (d.engine == kEngineTensor && !gemm_uses_tensor_cores(d)) return -1;
    if (gemm_uses_tensor_cores(d)) return gemm_tc(d, s, dev_err);
    return gemm_simt(d, s);
}

}  // namespace nsb
