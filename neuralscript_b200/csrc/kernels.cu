// Memory-bound kernels of the hot path. One warp per row for row-wise ops
// (coalesced 128-bit accesses, warp-shuffle reductions), grid-stride
// elementwise kernels sized to the SM count, and fixed-order reductions
// everywhere (no float atomics), so every result is run-to-run bitwise
// reproducible.
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace nsb {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// Block-wide sum in a fixed order (warp trees, then warp 0 over the partials).
__device__ float block_sum(float v, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = 0.f;
    if (w == 0) {
        r = lane < nw ? sh[lane] : 0.f;
        r = warp_sum(r);
        if (lane == 0) sh[32] = r;
    }
    __syncthreads();
    return sh[32];
}
__device__ float block_max(float v, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        float r = lane < nw ? sh[lane] : -INFINITY;
        r = warp_max(r);
        if (lane == 0) sh[32] = r;
    }
    __syncthreads();
    return sh[32];
}

inline unsigned grid_for(size_t n, int per_block) {
    size_t g = (n + per_block - 1) / per_block;
    size_t cap = (size_t)num_sms() * 16;
    if (g > cap) g = cap;
    if (g == 0) g = 1;
    return (unsigned)g;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int launch_ok() { return cudaGetLastError() == cudaSuccess ? 0 : -5; }

}  // namespace

// ---------------------------------------------------------------------------
// Embedding
// ---------------------------------------------------------------------------
__global__ void embedding_fwd_kernel(const float* __restrict__ W, const float* __restrict__ ids, int M, int V, int D,
                                     float* __restrict__ out32, __nv_bfloat16* __restrict__ out16, int vec) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        long long k = (long long)ids[r];  // truncation toward zero, as the reference's (int64_t) cast
        if (k < 0 || k >= V) k = 0;
        const float* src = W + (size_t)k * D;
        if (vec) {
            for (int c = lane * 4; c < D; c += 128) {
                float4 t = *reinterpret_cast<const float4*>(src + c);
                if (out32) *reinterpret_cast<float4*>(out32 + (size_t)r * D + c) = t;
                if (out16) {
                    __nv_bfloat162 a = __floats2bfloat162_rn(t.x, t.y), b = __floats2bfloat162_rn(t.z, t.w);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t*>(&a);
                    u.y = *reinterpret_cast<uint32_t*>(&b);
                    *reinterpret_cast<uint2*>(out16 + (size_t)r * D + c) = u;
                }
            }
        } else {
            for (int c = lane; c < D; c += 32) {
                float t = src[c];
                if (out32) out32[(size_t)r * D + c] = t;
                if (out16) out16[(size_t)r * D + c] = f2bf(t);
            }
        }
    }
}

int embedding_fwd(const float* W, const float* ids, int M, int V, int D, float* out32, __nv_bfloat16* out16,
                  cudaStream_t s) {
    if (M <= 0) return 0;
    int vec = (D % 4 == 0) && aligned16(W) && (!out32 || aligned16(out32)) && (!out16 || (reinterpret_cast<uintptr_t>(out16) & 7) == 0);
    embedding_fwd_kernel<<<grid_for((size_t)M, 8), 256, 0, s>>>(W, ids, M, V, D, out32, out16, vec);
    return launch_ok();
}

size_t embedding_bwd_scratch_bytes(int M, int V) {
    // count[V], offset[V], cursor[V], rows[M], then the large-bucket flag
    return sizeof(int) * ((size_t)3 * V + M) + 64;
}

// Zeroes p[0, n) and, when given, the flag word.
__global__ void zero_ints_kernel(int* p, size_t n, int* flag = nullptr) {
    if (flag && blockIdx.x == 0 && threadIdx.x == 0) *flag = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = 0;
}

// Bucket sizes; *big becomes 1 when some bucket grows past kEmbWarpRows rows
// (the bitmap kernel then has work).
constexpr int kEmbWarpRows = 32;
__global__ void emb_count_kernel(const float* __restrict__ ids, int M, int V, int* count, int* big) {
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M; r += gridDim.x * blockDim.x) {
        long long v = (long long)ids[r];
        if (v >= 0 && v < V) {
            if (atomicAdd(&count[v], 1) == kEmbWarpRows) *big = 1;  // integer counts: order-independent
        }
    }
}

// Exclusive prefix sum of n ints, one block of 1024 threads: each thread
// owns a contiguous run, runs are combined by warp-shuffle scans. Runs of up
// to kScanRun elements (n <= 16384) are read into registers in one batch of
// independent loads and written from there; longer runs loop over global.
constexpr int kScanRun = 16;
__global__ void __launch_bounds__(1024) scan_kernel(const int* __restrict__ in, int* __restrict__ out, int n) {
    __shared__ int warp_tot[32];
    const int per = (n + 1023) / 1024;
    const int b0 = threadIdx.x * per;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const bool small = per <= kScanRun;
    int vals[kScanRun];
    int local = 0;
    if (small) {
#pragma unroll
        for (int i = 0; i < kScanRun; i++) vals[i] = (i < per && b0 + i < n) ? in[b0 + i] : 0;
#pragma unroll
        for (int i = 0; i < kScanRun; i++) local += vals[i];
    } else {
        for (int i = 0; i < per; i++)
            if (b0 + i < n) local += in[b0 + i];
    }
    int x = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    if (w == 0) {
        int t = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, t, o);
            if (lane >= o) t += y;
        }
        warp_tot[lane] = t;
    }
    __syncthreads();
    int excl = x - local + (w > 0 ? warp_tot[w - 1] : 0);
    if (small) {
#pragma unroll
        for (int i = 0; i < kScanRun; i++)
            if (i < per && b0 + i < n) {
                out[b0 + i] = excl;
                excl += vals[i];
            }
    } else {
        for (int i = 0; i < per; i++) {
            const int k = b0 + i;
            if (k < n) {
                out[k] = excl;
                excl += in[k];
            }
        }
    }
}

__global__ void emb_fill_kernel(const float* __restrict__ ids, int M, int V, const int* __restrict__ offset,
                                int* cursor, int* rows) {
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M; r += gridDim.x * blockDim.x) {
        long long v = (long long)ids[r];
        if (v >= 0 && v < V) {
            int slot = atomicAdd(&cursor[v], 1);  // slot order is arbitrary; the reduce sorts by row
            rows[offset[v] + slot] = r;
        }
    }
}

// Sum of the listed dOut rows (ascending row order) into dst for D = 128*CH:
// each lane owns CH float4 columns; rows are loaded G at a time (the loads of
// a partial last group predicated off) before any is added, so a warp keeps
// up to G*CH independent 16-byte loads in flight while the sums stay in row
// order (bit-identical to a one-row-at-a-time loop).
template <int CH, int G>
__device__ __forceinline__ void emb_sum_rows(const float* __restrict__ dout, int D, const int* rows_sorted, int n,
                                             float* __restrict__ dst, int lane) {
    float4 acc[CH];
#pragma unroll
    for (int c = 0; c < CH; c++) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < n; q += G) {
        float4 t[G][CH];
#pragma unroll
        for (int u = 0; u < G; u++) {
            if (q + u < n) {
                const float4* r = reinterpret_cast<const float4*>(dout + (size_t)rows_sorted[q + u] * D) + lane;
#pragma unroll
                for (int c = 0; c < CH; c++) t[u][c] = __ldcs(r + 32 * c);
            }
        }
#pragma unroll
        for (int u = 0; u < G; u++)
            if (q + u < n) {
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    acc[c].x += t[u][c].x; acc[c].y += t[u][c].y; acc[c].z += t[u][c].z; acc[c].w += t[u][c].w;
                }
            }
    }
    float4* d4 = reinterpret_cast<float4*>(dst) + lane;
#pragma unroll
    for (int c = 0; c < CH; c++) d4[32 * c] = acc[c];
}

// Buckets of at most kEmbWarpRows rows: one warp per vocabulary row gathers
// the rows that hit it, orders them by row index (bitonic sort across the
// warp) and sums their gradients in that order. The sorted row ids are
// staged in shared memory so the column loops (where only some lanes may be
// active for narrow rows) never shuffle across inactive lanes. Larger
// buckets are left to emb_big_kernel.
// CH > 0: D = 128*CH with 16-byte aligned rows (one instantiation per width,
// so each gets its own register budget); CH = 0: any D.
template <int CH>
__global__ void __launch_bounds__(256) emb_reduce_kernel(const float* __restrict__ dout, int D, int V,
                                                         const int* __restrict__ count,
                                                         const int* __restrict__ offset,
                                                         const int* __restrict__ rows, float* __restrict__ dW,
                                                         int vec) {
    __shared__ int sorted[8][32];  // blockDim.x == 256
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    for (int v = blockIdx.x * warps + wi; v < V; v += gridDim.x * warps) {
        const int n = count[v];
        if (n > kEmbWarpRows) continue;
        const int* rv = rows + offset[v];
        float* dst = dW + (size_t)v * D;
        if (n == 0) {
            for (int c = lane; c < D; c += 32) dst[c] = 0.f;
            continue;
        }
        int key = lane < n ? rv[lane] : 0x7fffffff;
        // warp bitonic sort, ascending (all 32 lanes participate)
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
                int other = __shfl_xor_sync(kFull, key, j);
                bool up = (lane & k) == 0;
                bool lower = (lane & j) == 0;
                int mn = min(key, other), mx = max(key, other);
                key = (lower == up) ? mn : mx;
            }
        }
        sorted[wi][lane] = key;
        __syncwarp();
        if constexpr (CH > 0) {
            emb_sum_rows<CH, (CH <= 2 ? 4 : (CH == 4 ? 2 : 1))>(dout, D, sorted[wi], n, dst, lane);
        } else if (vec) {
            for (int c = lane * 4; c < D; c += 128) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int q = 0; q < n; q++) {
                    float4 t = *reinterpret_cast<const float4*>(dout + (size_t)sorted[wi][q] * D + c);
                    acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
                }
                *reinterpret_cast<float4*>(dst + c) = acc;
            }
        } else {
            for (int c = lane; c < D; c += 32) {
                float acc = 0.f;
                for (int q = 0; q < n; q++) acc += dout[(size_t)sorted[wi][q] * D + c];
                dst[c] = acc;
            }
        }
        __syncwarp();
    }
}

// Buckets of more than kEmbWarpRows rows (frequent ids), one CTA per bucket
// at a time. The bucket's row list (filled in arbitrary order) is ordered in
// linear time through a bitmap of row indices in shared memory, one window
// of kEmbBitmapRows rows at a time: every row of the bucket that falls in the
// window sets its bit (atomicOr: order-independent), then every thread walks
// the set bits in ascending order and adds those rows into its own column
// slice. Each column is thus a sequential sum over ascending rows, as in the
// reference's loop, for any bucket size (work O(n + M/32) per bucket).
constexpr int kEmbBitmapRows = 262144;  // 32 KB bitmap
constexpr int kEmbBigThreads = 256;
__global__ void __launch_bounds__(kEmbBigThreads) emb_big_kernel(const float* __restrict__ dout, int M, int D, int V,
                                                               const int* __restrict__ count,
                                                               const int* __restrict__ offset,
                                                               const int* __restrict__ rows, float* __restrict__ dW,
                                                               int vec, const int* __restrict__ big) {
    __shared__ unsigned bits[kEmbBitmapRows / 32];
    if (*big == 0) return;  // no bucket above kEmbWarpRows rows (uniform)
    const int tid = threadIdx.x;
    const int slots = vec ? D / 4 : D;  // float4 or scalar columns
    for (int v = blockIdx.x; v < V; v += gridDim.x) {
        const int n = count[v];
        if (n <= kEmbWarpRows) continue;  // uniform across the CTA
        const int* rv = rows + offset[v];
        float* dst = dW + (size_t)v * D;
        for (int s0 = 0; s0 < slots; s0 += kEmbBigThreads) {  // column chunks of one slot per thread
            const int slot = s0 + tid;
            const bool mine = slot < slots;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int w0 = 0; w0 < M; w0 += kEmbBitmapRows) {
                const int wrows = min(kEmbBitmapRows, M - w0), words = (wrows + 31) / 32;
                for (int i = tid; i < words; i += kEmbBigThreads) bits[i] = 0u;
                __syncthreads();
                for (int i = tid; i < n; i += kEmbBigThreads) {
                    const int r = rv[i] - w0;
                    if (r >= 0 && r < wrows) atomicOr(&bits[r >> 5], 1u << (r & 31));
                }
                __syncthreads();
                if (mine) {
                    int pend[4];
                    int np = 0;
                    for (int q = 0; q < words; q++) {
                        unsigned b = bits[q];
                        while (b) {
                            pend[np++] = w0 + q * 32 + __ffs(b) - 1;
                            b &= b - 1;
                            if (np == 4) {
                                if (vec) {
                                    float4 t[4];
#pragma unroll
                                    for (int u = 0; u < 4; u++)
                                        t[u] = __ldcs(reinterpret_cast<const float4*>(dout + (size_t)pend[u] * D) + slot);
#pragma unroll
                                    for (int u = 0; u < 4; u++) {
                                        acc.x += t[u].x; acc.y += t[u].y; acc.z += t[u].z; acc.w += t[u].w;
                                    }
                                } else {
                                    float t[4];
#pragma unroll
                                    for (int u = 0; u < 4; u++) t[u] = dout[(size_t)pend[u] * D + slot];
#pragma unroll
                                    for (int u = 0; u < 4; u++) acc.x += t[u];
                                }
                                np = 0;
                            }
                        }
                    }
                    for (int u = 0; u < np; u++) {
                        if (vec) {
                            const float4 t = __ldcs(reinterpret_cast<const float4*>(dout + (size_t)pend[u] * D) + slot);
                            acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
                        } else {
                            acc.x += dout[(size_t)pend[u] * D + slot];
                        }
                    }
                }
                __syncthreads();  // before the next window clears the bitmap
            }
            if (mine) {
                if (vec) reinterpret_cast<float4*>(dst)[slot] = acc;
                else dst[slot] = acc.x;
            }
        }
    }
}

// The order of the gradient's sums depends on the ids alone: the counting
// sort (zero, count, scan, fill) can run before the gradient exists.
int embedding_bwd_sort(const float* ids, int M, int V, void* scratch, cudaStream_t s) {
    int* count = reinterpret_cast<int*>(scratch);
    int* offset = count + V;
    int* cursor = offset + V;
    int* rows = cursor + V;
    int* big = rows + M;  // in the 64 bytes past the row list
    zero_ints_kernel<<<grid_for((size_t)V * 3, 256), 256, 0, s>>>(count, (size_t)V * 3, big);
    if (M > 0) emb_count_kernel<<<grid_for((size_t)M, 256), 256, 0, s>>>(ids, M, V, count, big);
    scan_kernel<<<1, 1024, 0, s>>>(count, offset, V);
    if (M > 0) emb_fill_kernel<<<grid_for((size_t)M, 256), 256, 0, s>>>(ids, M, V, offset, cursor, rows);
    return launch_ok();
}

// The ordered sums into dW from the sort embedding_bwd_sort left in scratch.
int embedding_bwd_sum(const float* dout, int M, int V, int D, float* dW, const void* scratch, cudaStream_t s) {
    const int* count = reinterpret_cast<const int*>(scratch);
    const int* offset = count + V;
    const int* cursor = offset + V;
    const int* rows = cursor + V;
    const int* big = rows + M;
    int vec = (D % 4 == 0) && aligned16(dout) && aligned16(dW);
    const unsigned rg = grid_for((size_t)V, 8);
    if (vec && D == 512) emb_reduce_kernel<4><<<rg, 256, 0, s>>>(dout, D, V, count, offset, rows, dW, vec);
    else if (vec && D == 256) emb_reduce_kernel<2><<<rg, 256, 0, s>>>(dout, D, V, count, offset, rows, dW, vec);
    else if (vec && D == 128) emb_reduce_kernel<1><<<rg, 256, 0, s>>>(dout, D, V, count, offset, rows, dW, vec);
    else if (vec && D == 1024) emb_reduce_kernel<8><<<rg, 256, 0, s>>>(dout, D, V, count, offset, rows, dW, vec);
    else emb_reduce_kernel<0><<<rg, 256, 0, s>>>(dout, D, V, count, offset, rows, dW, vec);
    if (M > kEmbWarpRows) {
        // a few CTAs per SM walk the vocabulary (all return at once when the
        // count kernel saw no bucket above 32 rows); buckets of <= 32 rows
        // are skipped after one read of their count
        const unsigned nbig = (unsigned)(V < 148 * 4 ? V : 148 * 4);
        emb_big_kernel<<<nbig, kEmbBigThreads, 0, s>>>(dout, M, D, V, count, offset, rows, dW, vec, big);
    }
    return launch_ok();
}

int embedding_bwd(const float* dout, const float* ids, int M, int V, int D, float* dW, void* scratch,
                  cudaStream_t s) {
    const int rc = embedding_bwd_sort(ids, M, V, scratch, s);
    if (rc) return rc;
    return embedding_bwd_sum(dout, M, V, D, dW, scratch, s);
}

// ---------------------------------------------------------------------------
// Allocation-free embedding gradient
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at the point they need the
// embedding gradient: code running inside a custom allocator or memory-pool
// callback, a host that has handed all device memory to its own pool, or a
// runtime that forbids cudaMalloc after start-up. For them the sort scratch
// (counts, offsets, cursors and the row list) lives in this fixed device
// array instead of a caller buffer. Every GPU that loads the library holds
// it (kNoAllocScratchBytes) until the process exits.
constexpr int kNoAllocMaxRows = 262144;
constexpr int kNoAllocMaxVocab = 65536;
constexpr size_t kNoAllocScratchBytes = sizeof(int) * ((size_t)3 * kNoAllocMaxVocab + kNoAllocMaxRows) + 64;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device. In host code the symbol
// itself is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
static void* noalloc_scratch_ptr() {
    static std::mutex mu;
    static void* ptrs[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
        ptrs[dev] = p;
    }
    return ptrs[dev];
}

}  // namespace nsb

// The extern "C" entry point is declared in include/ns_b200_ops.h.
extern "C" int nsb_op_embedding_bwd_noalloc(const float* dout, const float* ids, int M, int V, int D, float* dW,
                                            void* stream) {
    if (M < 0 || V <= 0 || D <= 0 || !dout || !ids || !dW) return -1;
    if (M > nsb::kNoAllocMaxRows || V > nsb::kNoAllocMaxVocab) return -2;  // beyond the fixed scratch
    if (stream) {
        // the scratch address is the current device's: the stream must be on it
        int sdev = -1, cur = -1;
        if (cudaStreamGetDevice((cudaStream_t)stream, &sdev) != cudaSuccess || cudaGetDevice(&cur) != cudaSuccess ||
            sdev != cur)
            return -4;
    }
    void* scratch = nsb::noalloc_scratch_ptr();
    if (!scratch) return -3;
    // embedding_bwd zeroes the counters it needs at the start of every call
    return nsb::embedding_bwd(dout, ids, M, V, D, dW, scratch, (cudaStream_t)stream);
}

namespace nsb {

// ---------------------------------------------------------------------------
// LayerNorm (no affine, eps 1e-5) — reference ns_layernorm / ns_layernorm_grad
// ---------------------------------------------------------------------------
__global__ void layernorm_fwd_kernel(const float* __restrict__ x, int M, int D, float* __restrict__ out32,
                                     __nv_bfloat16* __restrict__ out16) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float* xr = x + (size_t)r * D;
        float s = 0.f;
        for (int c = lane; c < D; c += 32) s += xr[c];
        const float mean = warp_sum(s) / (float)D;
        float q = 0.f;
        for (int c = lane; c < D; c += 32) {
            float d = xr[c] - mean;
            q += d * d;
        }
        const float var = warp_sum(q) / (float)D;
        const float inv = 1.f / sqrtf(var + 1e-5f);
        for (int c = lane; c < D; c += 32) {
            float y = (xr[c] - mean) * inv;
            if (out32) out32[(size_t)r * D + c] = y;
            if (out16) out16[(size_t)r * D + c] = f2bf(y);
        }
    }
}

// D a multiple of 128, D <= 1024: the row stays in registers (float4 per
// lane per 128 columns), one HBM read and one write per element.
template <int NV>
__global__ void layernorm_fwd_vec_kernel(const float* __restrict__ x, int M, float* __restrict__ out32,
                                         __nv_bfloat16* __restrict__ out16) {
    constexpr int D = NV * 128;
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * D);
        float4 v[NV];
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            v[i] = xr[lane + 32 * i];
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
        const float mean = warp_sum(s) / (float)D;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + b * b) + (c * c + d * d);
        }
        const float var = warp_sum(q) / (float)D;
        const float inv = 1.f / sqrtf(var + 1e-5f);
#pragma unroll
        for (int i = 0; i < NV; i++) {
            float4 y = make_float4((v[i].x - mean) * inv, (v[i].y - mean) * inv, (v[i].z - mean) * inv,
                                   (v[i].w - mean) * inv);
            const int c = 4 * (lane + 32 * i);
            if (out32) *reinterpret_cast<float4*>(out32 + (size_t)r * D + c) = y;
            if (out16) {
                __nv_bfloat162 a = __floats2bfloat162_rn(y.x, y.y), b = __floats2bfloat162_rn(y.z, y.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&a);
                u.y = *reinterpret_cast<uint32_t*>(&b);
                *reinterpret_cast<uint2*>(out16 + (size_t)r * D + c) = u;
            }
        }
    }
}

int layernorm_fwd(const float* x, int M, int D, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (M <= 0) return 0;
    const bool vec = D % 128 == 0 && D <= 1024 && aligned16(x) && (!out32 || aligned16(out32)) &&
                     (!out16 || (reinterpret_cast<uintptr_t>(out16) & 7) == 0);
    unsigned g = grid_for((size_t)M, 8);
    if (vec) {
        switch (D / 128) {
            case 1: layernorm_fwd_vec_kernel<1><<<g, 256, 0, s>>>(x, M, out32, out16); break;
            case 2: layernorm_fwd_vec_kernel<2><<<g, 256, 0, s>>>(x, M, out32, out16); break;
            case 4: layernorm_fwd_vec_kernel<4><<<g, 256, 0, s>>>(x, M, out32, out16); break;
            case 8: layernorm_fwd_vec_kernel<8><<<g, 256, 0, s>>>(x, M, out32, out16); break;
            default: layernorm_fwd_kernel<<<g, 256, 0, s>>>(x, M, D, out32, out16);
        }
    } else {
        layernorm_fwd_kernel<<<g, 256, 0, s>>>(x, M, D, out32, out16);
    }
    return launch_ok();
}

__global__ void layernorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                     const float* __restrict__ add, int M, int D, float* __restrict__ dx32,
                                     __nv_bfloat16* __restrict__ dx16) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float* xr = x + (size_t)r * D;
        const float* dr = dy + (size_t)r * D;
        float sx = 0.f, sd = 0.f;
        for (int c = lane; c < D; c += 32) {
            sx += xr[c];
            sd += dr[c];
        }
        const float mean_x = warp_sum(sx) / (float)D;
        const float mean_d = warp_sum(sd) / (float)D;
        float vq = 0.f, gq = 0.f;
        for (int c = lane; c < D; c += 32) {
            float xc = xr[c] - mean_x;
            vq += xc * xc;
            gq += xc * dr[c];
        }
        const float var = warp_sum(vq) / (float)D;
        const float gamma = warp_sum(gq) / (float)D;
        const float inv = 1.f / sqrtf(var + 1e-5f);
        for (int c = lane; c < D; c += 32) {
            float xc = xr[c] - mean_x;
            float o = (dr[c] - mean_d - xc * gamma) * inv;
            if (add) o += add[(size_t)r * D + c];
            if (dx32) dx32[(size_t)r * D + c] = o;
            if (dx16) dx16[(size_t)r * D + c] = f2bf(o);
        }
    }
}

// FROM_Y: x holds the LayerNorm OUTPUT y and rstd[r] the row's
// 1 / sqrt(var + eps) (a LayerNorm fused into its producer's GEMM); the
// centred input is then y / rstd, so the pre-LayerNorm sum is never needed.
template <int NV, bool FROM_Y>
__global__ void layernorm_bwd_vec_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                         const float* __restrict__ rstd, const float* __restrict__ add, int M,
                                         float* __restrict__ dx32, __nv_bfloat16* __restrict__ dx16) {
    constexpr int D = NV * 128;
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * D);
        const float4* dr = reinterpret_cast<const float4*>(dy + (size_t)r * D);
        float4 xv[NV], dv[NV];
        float sx = 0.f, sd = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            xv[i] = xr[lane + 32 * i];
            dv[i] = dr[lane + 32 * i];
            sx += (xv[i].x + xv[i].y) + (xv[i].z + xv[i].w);
            sd += (dv[i].x + dv[i].y) + (dv[i].z + dv[i].w);
        }
        float mean_x = 0.f, inv;
        if (FROM_Y) {
            // x - mean(x) = y * sigma
            inv = rstd[r];
            const float sig = 1.f / inv;
#pragma unroll
            for (int i = 0; i < NV; i++) {
                xv[i].x *= sig;
                xv[i].y *= sig;
                xv[i].z *= sig;
                xv[i].w *= sig;
            }
        } else {
            mean_x = warp_sum(sx) / (float)D;
        }
        const float mean_d = warp_sum(sd) / (float)D;
        float vq = 0.f, gq = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            float a = xv[i].x - mean_x, b = xv[i].y - mean_x, c = xv[i].z - mean_x, d = xv[i].w - mean_x;
            vq += (a * a + b * b) + (c * c + d * d);
            gq += (a * dv[i].x + b * dv[i].y) + (c * dv[i].z + d * dv[i].w);
        }
        const float gamma = warp_sum(gq) / (float)D;
        if (!FROM_Y) {
            const float var = warp_sum(vq) / (float)D;
            inv = 1.f / sqrtf(var + 1e-5f);
        }
#pragma unroll
        for (int i = 0; i < NV; i++) {
            const int c = 4 * (lane + 32 * i);
            float4 o;
            o.x = (dv[i].x - mean_d - (xv[i].x - mean_x) * gamma) * inv;
            o.y = (dv[i].y - mean_d - (xv[i].y - mean_x) * gamma) * inv;
            o.z = (dv[i].z - mean_d - (xv[i].z - mean_x) * gamma) * inv;
            o.w = (dv[i].w - mean_d - (xv[i].w - mean_x) * gamma) * inv;
            if (add) {
                float4 a = *reinterpret_cast<const float4*>(add + (size_t)r * D + c);
                o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
            }
            if (dx32) *reinterpret_cast<float4*>(dx32 + (size_t)r * D + c) = o;
            if (dx16) {
                __nv_bfloat162 a = __floats2bfloat162_rn(o.x, o.y), b = __floats2bfloat162_rn(o.z, o.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&a);
                u.y = *reinterpret_cast<uint32_t*>(&b);
                *reinterpret_cast<uint2*>(dx16 + (size_t)r * D + c) = u;
            }
        }
    }
}

int layernorm_bwd(const float* dy, const float* x, const float* add, int M, int D, float* dx32, __nv_bfloat16* dx16,
                  cudaStream_t s) {
    if (M <= 0) return 0;
    const bool vec = D % 128 == 0 && D <= 1024 && aligned16(x) && aligned16(dy) && (!add || aligned16(add)) &&
                     (!dx32 || aligned16(dx32)) && (!dx16 || (reinterpret_cast<uintptr_t>(dx16) & 7) == 0);
    unsigned g = grid_for((size_t)M, 8);
    if (vec) {
        switch (D / 128) {
            case 1: layernorm_bwd_vec_kernel<1, false><<<g, 256, 0, s>>>(dy, x, nullptr, add, M, dx32, dx16); break;
            case 2: layernorm_bwd_vec_kernel<2, false><<<g, 256, 0, s>>>(dy, x, nullptr, add, M, dx32, dx16); break;
            case 4: layernorm_bwd_vec_kernel<4, false><<<g, 256, 0, s>>>(dy, x, nullptr, add, M, dx32, dx16); break;
            case 8: layernorm_bwd_vec_kernel<8, false><<<g, 256, 0, s>>>(dy, x, nullptr, add, M, dx32, dx16); break;
            default: layernorm_bwd_kernel<<<g, 256, 0, s>>>(dy, x, add, M, D, dx32, dx16);
        }
    } else {
        layernorm_bwd_kernel<<<g, 256, 0, s>>>(dy, x, add, M, D, dx32, dx16);
    }
    return launch_ok();
}

int layernorm_bwd_from_output(const float* dy, const float* y, const float* rstd, const float* add, int M, int D,
                              float* dx32, __nv_bfloat16* dx16, cudaStream_t s) {
    if (M <= 0) return 0;
    const bool vec = D % 128 == 0 && D <= 1024 && aligned16(y) && aligned16(dy) && (!add || aligned16(add)) &&
                     (!dx32 || aligned16(dx32)) && (!dx16 || (reinterpret_cast<uintptr_t>(dx16) & 7) == 0);
    if (!vec || !rstd) return -1;
    unsigned g = grid_for((size_t)M, 8);
    switch (D / 128) {
        case 1: layernorm_bwd_vec_kernel<1, true><<<g, 256, 0, s>>>(dy, y, rstd, add, M, dx32, dx16); break;
        case 2: layernorm_bwd_vec_kernel<2, true><<<g, 256, 0, s>>>(dy, y, rstd, add, M, dx32, dx16); break;
        case 4: layernorm_bwd_vec_kernel<4, true><<<g, 256, 0, s>>>(dy, y, rstd, add, M, dx32, dx16); break;
        case 8: layernorm_bwd_vec_kernel<8, true><<<g, 256, 0, s>>>(dy, y, rstd, add, M, dx32, dx16); break;
        default: return -1;
    }
    return launch_ok();
}

// ---------------------------------------------------------------------------
// Cross-entropy forward + seed gradient (reference ns_cross_entropy /
// ns_loss_grad, src/codegen/codegen.cpp:1582-1613), one CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ce_kernel(const float* __restrict__ logits, const float* __restrict__ labels,
                                                 const int* __restrict__ targets, int M, int C, float denom,
                                                 float* __restrict__ row_loss, float* __restrict__ d32,
                                                 __nv_bfloat16* __restrict__ d16) {
    __shared__ float sh[33];
    for (int r = blockIdx.x; r < M; r += gridDim.x) {
        const float* x = logits + (size_t)r * C;
        float mx = -INFINITY;
        for (int j = threadIdx.x; j < C; j += blockDim.x) mx = fmaxf(mx, x[j]);
        mx = block_max(mx, sh);
        float se = 0.f;
        for (int j = threadIdx.x; j < C; j += blockDim.x) se += expf(x[j] - mx);
        se = block_sum(se, sh);
        const int t = targets ? targets[r] : -1;
        float loss = 0.f;
        for (int j = threadIdx.x; j < C; j += blockDim.x) {
            const float p = expf(x[j] - mx) / se;
            const float y = labels ? labels[(size_t)r * C + j] : (j == t ? 1.f : 0.f);
            if (y > 0.f) loss -= logf(p);
            const float d = (p - y) / denom;
            if (d32) d32[(size_t)r * C + j] = d;
            if (d16) d16[(size_t)r * C + j] = f2bf(d);
        }
        loss = block_sum(loss, sh);
        if (threadIdx.x == 0) row_loss[r] = loss;
    }
}

// Single-pass form for rows of C = 1024*NV classes: 256 threads hold the
// row in registers (NV float4 each), so the logits are read once and the
// gradient written once.
template <int NV>
__global__ void __launch_bounds__(256) ce_rows_vec_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ labels,
                                                          const int* __restrict__ targets, int M, float denom,
                                                          float* __restrict__ row_loss, float* __restrict__ d32,
                                                          __nv_bfloat16* __restrict__ d16) {
    constexpr int C = 1024 * NV;
    __shared__ float sh[33];
    for (int r = blockIdx.x; r < M; r += gridDim.x) {
        const float4* x4 = reinterpret_cast<const float4*>(logits + (size_t)r * C);
        float4 e[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) e[v] = __ldcs(x4 + v * 256 + threadIdx.x);
        float mx = -INFINITY;
#pragma unroll
        for (int v = 0; v < NV; v++) mx = fmaxf(fmaxf(mx, fmaxf(e[v].x, e[v].y)), fmaxf(e[v].z, e[v].w));
        mx = block_max(mx, sh);
        // exp of arguments in [-inf, 0] through the hardware exp2 path
        // (__expf: a few ulp here, far inside the tolerances) and one
        // reciprocal per row: this kernel moves 3/4 of a GB per step, and
        // with the accurate expf and two divisions per element it is bound
        // by instruction issue rather than by HBM.
        float se = 0.f;
#pragma unroll
        for (int v = 0; v < NV; v++) {
            e[v].x = __expf(e[v].x - mx);
            e[v].y = __expf(e[v].y - mx);
            e[v].z = __expf(e[v].z - mx);
            e[v].w = __expf(e[v].w - mx);
            se += (e[v].x + e[v].y) + (e[v].z + e[v].w);
        }
        se = block_sum(se, sh);
        const float inv_se = 1.f / se, inv_denom = 1.f / denom;
        const int t = targets ? targets[r] : -1;
        float loss = 0.f;
#pragma unroll
        for (int v = 0; v < NV; v++) {
            const int j0 = 4 * (v * 256 + threadIdx.x);
            float4 y;
            if (labels) {
                y = __ldcs(reinterpret_cast<const float4*>(labels + (size_t)r * C) + v * 256 + threadIdx.x);
            } else {
                y.x = j0 == t ? 1.f : 0.f;
                y.y = j0 + 1 == t ? 1.f : 0.f;
                y.z = j0 + 2 == t ? 1.f : 0.f;
                y.w = j0 + 3 == t ? 1.f : 0.f;
            }
            float4 p;
            p.x = e[v].x * inv_se;
            p.y = e[v].y * inv_se;
            p.z = e[v].z * inv_se;
            p.w = e[v].w * inv_se;
            if (y.x > 0.f) loss -= logf(p.x);
            if (y.y > 0.f) loss -= logf(p.y);
            if (y.z > 0.f) loss -= logf(p.z);
            if (y.w > 0.f) loss -= logf(p.w);
            float4 d;
            d.x = (p.x - y.x) * inv_denom;
            d.y = (p.y - y.y) * inv_denom;
            d.z = (p.z - y.z) * inv_denom;
            d.w = (p.w - y.w) * inv_denom;
            if (d32) __stcs(reinterpret_cast<float4*>(d32 + (size_t)r * C) + v * 256 + threadIdx.x, d);
            if (d16) {
                __nv_bfloat162 a = __floats2bfloat162_rn(d.x, d.y), b = __floats2bfloat162_rn(d.z, d.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&a);
                u.y = *reinterpret_cast<uint32_t*>(&b);
                __stcs(reinterpret_cast<uint2*>(d16 + (size_t)r * C) + v * 256 + threadIdx.x, u);
            }
        }
        loss = block_sum(loss, sh);
        if (threadIdx.x == 0) row_loss[r] = loss;
    }
}

// Second half of the head GEMM + cross-entropy fusion: the GEMM left the
// logits in g16 as fp16 (a 2^-11 relative step: the softmax inputs need more
// than bf16's 2^-8) and the fp32 target logit in tlogit. One warp per row:
// pass 1 streams the row for its maximum and sum of exponentials (online,
// log2 units), pass 2 re-reads it (now in L1/L2) and overwrites it with the
// bf16 seed gradient (softmax - onehot) / denom; the row loss is
// log-sum-exp - logit[target]. Exponentials on ex2.approx (a few ulp, far
// inside the bf16 resolution of the seed).
__device__ __forceinline__ float ex2_approx_f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(256) ce_finish_kernel(void* __restrict__ g16, int M, int C,
                                                        const int* __restrict__ targets,
                                                        const float* __restrict__ tlogit, float denom,
                                                        float* __restrict__ row_loss) {
    constexpr float kL2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int n8 = C / 8;  // 8 bf16 per 16-byte load
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        uint4* row = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(g16) + (size_t)r * C);
        float m = -INFINITY, s = 0.f;
        int q = lane;
        for (; q + 96 < n8; q += 128) {  // four loads in flight
            uint4 u[4];
#pragma unroll
            for (int k = 0; k < 4; k++) u[k] = row[q + 32 * k];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const __half2* h = reinterpret_cast<const __half2*>(&u[k]);
                float x[8];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = __half22float2(h[e]);
                    x[2 * e] = f.x * kL2e;
                    x[2 * e + 1] = f.y * kL2e;
                }
                float cm = fmaxf(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])), fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7])));
                const float nm = fmaxf(m, cm);
                s *= ex2_approx_f(m - nm);
#pragma unroll
                for (int e = 0; e < 8; e++) s += ex2_approx_f(x[e] - nm);
                m = nm;
            }
        }
        for (; q < n8; q += 32) {
            const uint4 u = row[q];
            const __half2* h = reinterpret_cast<const __half2*>(&u);
            float x[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(h[e]);
                x[2 * e] = f.x * kL2e;
                x[2 * e + 1] = f.y * kL2e;
            }
            float cm = x[0];
#pragma unroll
            for (int e = 1; e < 8; e++) cm = fmaxf(cm, x[e]);
            const float nm = fmaxf(m, cm);
            s *= ex2_approx_f(m - nm);
#pragma unroll
            for (int e = 0; e < 8; e++) s += ex2_approx_f(x[e] - nm);
            m = nm;
        }
        // combine the lanes' (max, sum)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
            const float nm = fmaxf(m, om);
            s = s * ex2_approx_f(m - nm) + os * ex2_approx_f(om - nm);
            m = nm;
        }
        const float lse2 = m + __log2f(s);
        const int t = targets[r];
        if (lane == 0) row_loss[r] = (t >= 0 && t < C) ? (lse2 - tlogit[r] * kL2e) * kLn2 : 0.f;
        const float inv = 1.f / denom;
        auto seed_word = [&](uint4 u, int q2) {
            const __half2* hi = reinterpret_cast<const __half2*>(&u);
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 x = __half22float2(hi[e]);
                const int j = 8 * q2 + 2 * e;
                float a = ex2_approx_f(fmaf(x.x, kL2e, -lse2)), b = ex2_approx_f(fmaf(x.y, kL2e, -lse2));
                a -= j == t ? 1.f : 0.f;
                b -= j + 1 == t ? 1.f : 0.f;
                h[e] = __floats2bfloat162_rn(a * inv, b * inv);
            }
            __stcs(row + q2, u);
        };
        // the second pass also keeps four 16-byte loads in flight per lane
        int q2 = lane;
        for (; q2 + 96 < n8; q2 += 128) {
            uint4 u[4];
#pragma unroll
            for (int k = 0; k < 4; k++) u[k] = row[q2 + 32 * k];
#pragma unroll
            for (int k = 0; k < 4; k++) seed_word(u[k], q2 + 32 * k);
        }
        for (; q2 < n8; q2 += 32) seed_word(row[q2], q2);
    }
}

// The same pass for rows of at most 16384 classes with the row held in
// registers: a block of TPB threads reads its row once (NV 16-byte words of
// 8 fp16 per thread) and writes the seed once. The warp-per-row form above
// re-reads each row, and with an SM full of warps each holding a row the
// re-read no longer finds it in L2. Row maximum on packed halves (exact);
// the row sum on ex2.approx (the loss needs it to fp32 accuracy); the seed
// 2^(x log2e - lse2) on exp2_poly3 (relative error 7.5e-5, inside the bf16
// rounding of the seed) so that each element costs one MUFU exponential.
template <int NV, int TPB>
__global__ void __launch_bounds__(TPB) ce_finish_reg_kernel(void* __restrict__ g16, int M, int C,
                                                            const int* __restrict__ targets,
                                                            const float* __restrict__ tlogit, float denom,
                                                            float* __restrict__ row_loss) {
    constexpr float kL2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
    constexpr int W = TPB / 32;
    constexpr uint32_t kNegInf2 = 0xfc00fc00u;  // two fp16 -inf: padding past the row end
    __shared__ float red[2][W];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int n8 = C / 8;
    const float inv = 1.f / denom;
    // the next row's loads are issued before this row's reductions, so each
    // block keeps a row in flight while it works on the other
    uint4 nx[NV];
    auto load_row = [&](int rr) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(g16) + (size_t)rr * C);
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int q = tid + TPB * k;
            nx[k] = q < n8 ? __ldcs(src + q) : make_uint4(kNegInf2, kNegInf2, kNegInf2, kNegInf2);
        }
    };
    if ((int)blockIdx.x < M) load_row(blockIdx.x);
    for (int r = blockIdx.x; r < M; r += gridDim.x) {
        uint4* row = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(g16) + (size_t)r * C);
        uint4 u[NV];
#pragma unroll
        for (int k = 0; k < NV; k++) u[k] = nx[k];
        if (r + (int)gridDim.x < M) load_row(r + gridDim.x);
        const int t = targets[r];
        const float tl = tlogit[r];
        __half2 hm = *reinterpret_cast<const __half2*>(&u[0].x);
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const __half2* h = reinterpret_cast<const __half2*>(&u[k]);
#pragma unroll
            for (int e = 0; e < 4; e++) hm = __hmax2(hm, h[e]);
        }
        float mx = fmaxf(__low2float(hm), __high2float(hm));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[0][w] = mx;
        __syncthreads();
        mx = red[0][0];
#pragma unroll
        for (int i = 1; i < W; i++) mx = fmaxf(mx, red[0][i]);
        const float m2 = mx * kL2e;
        float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const __half2* h = reinterpret_cast<const __half2*>(&u[k]);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(h[e]);
                sp[e] += ex2_approx_f(fmaf(f.x, kL2e, -m2)) + ex2_approx_f(fmaf(f.y, kL2e, -m2));
            }
        }
        float s = (sp[0] + sp[1]) + (sp[2] + sp[3]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[1][w] = s;
        __syncthreads();
        s = red[1][0];
#pragma unroll
        for (int i = 1; i < W; i++) s += red[1][i];
        const float lse2 = m2 + __log2f(s);
        if (tid == 0) row_loss[r] = (t >= 0 && t < C) ? (lse2 - tl * kL2e) * kLn2 : 0.f;
        const uint64_t L2E = f2_pack(kL2e, kL2e), NL = f2_pack(-lse2, -lse2), INV = f2_pack(inv, inv);
#pragma unroll
        for (int k = 0; k < NV; k++) {
            const int q = tid + TPB * k;
            if (q >= n8) continue;
            const __half2* h = reinterpret_cast<const __half2*>(&u[k]);
            float y[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(h[e]);
                float a, b;
                f2_unpack(f2_fma(f2_pack(f.x, f.y), L2E, NL), a, b);
                exp2_poly3_pair(a, b, y[2 * e], y[2 * e + 1]);
            }
            if ((unsigned)(t - 8 * q) < 8u) {  // the target class lies in this word
#pragma unroll
                for (int e = 0; e < 8; e++) y[e] -= 8 * q + e == t ? 1.f : 0.f;
            }
            uint4 o;
            __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float a, b;
                f2_unpack(f2_mul(f2_pack(y[2 * e], y[2 * e + 1]), INV), a, b);
                ob[e] = __floats2bfloat162_rn(a, b);
            }
            __stcs(row + q, o);
        }
    }
}

// One resident wave of the register-resident loss pass: each block pipelines
// its rows, so a block that waited for a free SM would start unpipelined.
template <int NV, int TPB>
static void ce_finish_reg_launch(void* g16, int M, int C, const int* targets, const float* tlogit, float denom,
                                 float* row_loss, cudaStream_t s) {
    static int per_sm = 0;
    if (per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ce_finish_reg_kernel<NV, TPB>, TPB, 0) != cudaSuccess)
            n = 1;
        per_sm = n > 0 ? n : 1;
    }
    const unsigned blocks = (unsigned)min(M, num_sms() * per_sm);
    ce_finish_reg_kernel<NV, TPB><<<blocks, TPB, 0, s>>>(g16, M, C, targets, tlogit, denom, row_loss);
}

int cross_entropy_finish(void* g16, int M, int C, const int* targets, const float* tlogit, float denom,
                         float* row_loss, cudaStream_t s) {
    if (M <= 0) return 0;
    if (C % 8 || (reinterpret_cast<uintptr_t>(g16) & 15)) return -1;
    const int n8 = C / 8;
    if (n8 <= 1024) {
        const int nv = (n8 + 127) / 128;
        if (nv == 1)
            ce_finish_reg_launch<1, 128>(g16, M, C, targets, tlogit, denom, row_loss, s);
        else if (nv == 2)
            ce_finish_reg_launch<2, 128>(g16, M, C, targets, tlogit, denom, row_loss, s);
        else if (nv <= 4)
            ce_finish_reg_launch<4, 128>(g16, M, C, targets, tlogit, denom, row_loss, s);
        else
            ce_finish_reg_launch<8, 128>(g16, M, C, targets, tlogit, denom, row_loss, s);
    } else if (n8 <= 2048) {
        ce_finish_reg_launch<8, 256>(g16, M, C, targets, tlogit, denom, row_loss, s);
    } else {
        const unsigned blocks = (unsigned)min((M + 7) / 8, num_sms() * 8);
        ce_finish_kernel<<<blocks, 256, 0, s>>>(g16, M, C, targets, tlogit, denom, row_loss);
    }
    return launch_ok();
}

int cross_entropy_fwd_bwd(const float* logits, const float* labels, const int* targets, int M, int C, float denom,
                          float* row_loss, float* d32, __nv_bfloat16* d16, cudaStream_t s) {
    if (M <= 0) return 0;
    const bool vec = C % 1024 == 0 && C <= 16384 && aligned16(logits) && (!labels || aligned16(labels)) &&
                     (!d32 || aligned16(d32)) && (!d16 || (reinterpret_cast<uintptr_t>(d16) & 7) == 0);
    unsigned g = (unsigned)min(M, num_sms() * 8);
    if (vec) {
        switch (C / 1024) {
#define NSB_CE(NV) \
    case NV: ce_rows_vec_kernel<NV><<<g, 256, 0, s>>>(logits, labels, targets, M, denom, row_loss, d32, d16); break;
            NSB_CE(1) NSB_CE(2) NSB_CE(3) NSB_CE(4) NSB_CE(5) NSB_CE(6) NSB_CE(7) NSB_CE(8)
            NSB_CE(9) NSB_CE(10) NSB_CE(11) NSB_CE(12) NSB_CE(13) NSB_CE(14) NSB_CE(15) NSB_CE(16)
#undef NSB_CE
        }
    } else {
        ce_kernel<<<g, 256, 0, s>>>(logits, labels, targets, M, C, denom, row_loss, d32, d16);
    }
    return launch_ok();
}

__global__ void mse_kernel(const float* __restrict__ p, const float* __restrict__ y, int M, int C, float denom,
                           float* __restrict__ row_loss, float* __restrict__ d32, __nv_bfloat16* __restrict__ d16) {
    __shared__ float sh[33];
    for (int r = blockIdx.x; r < M; r += gridDim.x) {
        float acc = 0.f;
        for (int j = threadIdx.x; j < C; j += blockDim.x) {
            size_t i = (size_t)r * C + j;
            float e = p[i] - y[i];
            acc += e * e;
            float d = 2.0f * e / denom;
            if (d32) d32[i] = d;
            if (d16) d16[i] = f2bf(d);
        }
        acc = block_sum(acc, sh);
        if (threadIdx.x == 0) row_loss[r] = acc;
    }
}

// Warp per row, 4 columns per lane per step (C a multiple of 4, rows
// 16-byte aligned): no block-wide reduction per row.
__global__ void mse_vec_kernel(const float* __restrict__ p, const float* __restrict__ y, int M, int C, float denom,
                               float* __restrict__ row_loss, float* __restrict__ d32,
                               __nv_bfloat16* __restrict__ d16) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float4* pr = reinterpret_cast<const float4*>(p + (size_t)r * C);
        const float4* yr = reinterpret_cast<const float4*>(y + (size_t)r * C);
        float acc = 0.f;
        for (int j = lane; j < C / 4; j += 32) {
            const float4 a = pr[j], b = yr[j];
            const float e0 = a.x - b.x, e1 = a.y - b.y, e2 = a.z - b.z, e3 = a.w - b.w;
            acc += e0 * e0;
            acc += e1 * e1;
            acc += e2 * e2;
            acc += e3 * e3;
            const float4 d = make_float4(2.0f * e0 / denom, 2.0f * e1 / denom, 2.0f * e2 / denom, 2.0f * e3 / denom);
            if (d32) reinterpret_cast<float4*>(d32 + (size_t)r * C)[j] = d;
            if (d16) {
                uint2 h;
                reinterpret_cast<__nv_bfloat162*>(&h)[0] = __floats2bfloat162_rn(d.x, d.y);
                reinterpret_cast<__nv_bfloat162*>(&h)[1] = __floats2bfloat162_rn(d.z, d.w);
                reinterpret_cast<uint2*>(d16 + (size_t)r * C)[j] = h;
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) row_loss[r] = acc;
    }
}

int mse_fwd_bwd(const float* p, const float* y, int M, int C, float denom, float* row_loss, float* d32,
                __nv_bfloat16* d16, cudaStream_t s) {
    if (M <= 0) return 0;
    auto al = [](const void* q) { return !(reinterpret_cast<uintptr_t>(q) & 15); };
    if (C % 4 == 0 && al(p) && al(y) && (!d32 || al(d32)) && (!d16 || al(d16))) {
        const int blocks = min((M + 7) / 8, num_sms() * 16);
        mse_vec_kernel<<<blocks, 256, 0, s>>>(p, y, M, C, denom, row_loss, d32, d16);
        return launch_ok();
    }
    mse_kernel<<<(unsigned)min(M, num_sms() * 8), 256, 0, s>>>(p, y, M, C, denom, row_loss, d32, d16);
    return launch_ok();
}

// Sum of n floats in a fixed order (one block; float4 loads when aligned).
__global__ void __launch_bounds__(1024) reduce_sum_kernel(const float* __restrict__ x, int n, float scale, float* out) {
    __shared__ float sh[33];
    float acc = 0.f;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = x4[i];
            acc += (v.x + v.y) + (v.z + v.w);
        }
        for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) acc += x[i];
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) acc += x[i];
    }
    acc = block_sum(acc, sh);
    if (threadIdx.x == 0) *out = acc * scale;
}

int reduce_sum(const float* x, int n, float scale, float* out, cudaStream_t s) {
    reduce_sum_kernel<<<1, 1024, 0, s>>>(x, n, scale, out);
    return launch_ok();
}

// ---------------------------------------------------------------------------
// Elementwise
// ---------------------------------------------------------------------------
__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, size_t n, float* __restrict__ o32,
                           __nv_bfloat16* __restrict__ o16) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = a[i] + b[i];
        if (o32) o32[i] = v;
        if (o16) o16[i] = f2bf(v);
    }
}
int add_f32(const float* a, const float* b, size_t n, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (n == 0) return 0;
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, n, out32, out16);
    return launch_ok();
}

__global__ void act_fwd_kernel(const float* __restrict__ x, size_t n, int act, float* __restrict__ o32,
                               __nv_bfloat16* __restrict__ o16) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = act_fwd(x[i], act);
        if (o32) o32[i] = v;
        if (o16) o16[i] = f2bf(v);
    }
}
int act_fwd_f32(const float* x, size_t n, int act, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (n == 0) return 0;
    act_fwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, act, out32, out16);
    return launch_ok();
}

__global__ void act_bwd_kernel(const float* __restrict__ dy, const void* __restrict__ z, int z_dtype, int act,
                               const float* __restrict__ add, size_t n, float* __restrict__ o32,
                               __nv_bfloat16* __restrict__ o16) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = dy[i] * act_deriv(ld_any(z, z_dtype, i), act);
        if (add) v += add[i];
        if (o32) o32[i] = v;
        if (o16) o16[i] = f2bf(v);
    }
}
int act_bwd(const float* dy, const void* z, int z_dtype, int act, const float* add, size_t n, float* out32,
            __nv_bfloat16* out16, cudaStream_t s) {
    if (n == 0) return 0;
    act_bwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(dy, z, z_dtype, act, add, n, out32, out16);
    return launch_ok();
}

__global__ void f2bf_kernel(const float* __restrict__ x, size_t n, __nv_bfloat16* __restrict__ o) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        o[i] = f2bf(x[i]);
}
// 8 elements per thread per step: two 16-byte loads, one 16-byte store
__global__ void f2bf_x8_kernel(const float4* __restrict__ x, size_t n8, uint4* __restrict__ o) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
        const float4 a = x[2 * i], b = x[2 * i + 1];
        uint4 r;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
        h[0] = __floats2bfloat162_rn(a.x, a.y);
        h[1] = __floats2bfloat162_rn(a.z, a.w);
        h[2] = __floats2bfloat162_rn(b.x, b.y);
        h[3] = __floats2bfloat162_rn(b.z, b.w);
        o[i] = r;
    }
}
int f32_to_bf16(const float* x, size_t n, __nv_bfloat16* out, cudaStream_t s) {
    if (n == 0) return 0;
    if (n % 8 == 0 && !(reinterpret_cast<uintptr_t>(x) & 15) && !(reinterpret_cast<uintptr_t>(out) & 15)) {
        const size_t n8 = n / 8;
        const size_t cap = (size_t)num_sms() * 16;
        const size_t blocks = (n8 + 255) / 256;
        f2bf_x8_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, s>>>(reinterpret_cast<const float4*>(x), n8,
                                                                               reinterpret_cast<uint4*>(out));
        return launch_ok();
    }
    f2bf_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, out);
    return launch_ok();
}

// reference ns_softmax (codegen.cpp:1293-1302), one warp per row
__global__ void softmax_kernel(const float* __restrict__ x, int M, int C, float* __restrict__ o32,
                               __nv_bfloat16* __restrict__ o16) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < M; r += gridDim.x * warps) {
        const float* xr = x + (size_t)r * C;
        float mx = -INFINITY;
        for (int j = lane; j < C; j += 32) mx = fmaxf(mx, xr[j]);
        mx = warp_max(mx);
        float s = 0.f;
        for (int j = lane; j < C; j += 32) s += expf(xr[j] - mx);
        s = warp_sum(s);
        for (int j = lane; j < C; j += 32) {
            float v = expf(xr[j] - mx) / s;
            if (o32) o32[(size_t)r * C + j] = v;
            if (o16) o16[(size_t)r * C + j] = f2bf(v);
        }
    }
}
int softmax_rows(const float* x, int M, int C, float* out32, __nv_bfloat16* out16, cudaStream_t s) {
    if (M <= 0) return 0;
    softmax_kernel<<<grid_for((size_t)M, 8), 256, 0, s>>>(x, M, C, out32, out16);
    return launch_ok();
}

__global__ void pack_weight_kernel(const float* __restrict__ src, int rows, int cols, void* dst, int dtype,
                                   long long ld, int off) {
    size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / cols, c = i % cols;
        size_t o = r * ld + off + c;
        if (dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(dst)[o] = f2bf(src[i]);
        else reinterpret_cast<float*>(dst)[o] = src[i];
    }
}
int pack_weight(const float* src, int rows, int cols, void* dst, int dst_dtype, long long ld_dst, int col_off,
                cudaStream_t s) {
    size_t n = (size_t)rows * cols;
    if (n == 0) return 0;
    pack_weight_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, rows, cols, dst, dst_dtype, ld_dst, col_off);
    return launch_ok();
}

// ---------------------------------------------------------------------------
// Optimizers
// ---------------------------------------------------------------------------
// codegen.cpp:3108-3120 per element.
__device__ __forceinline__ float adamw_elem(float w, float gg, float& m, float& v, float b1t, float b2t,
                                            const AdamHyper& h) {
    m = h.beta1 * m + h.one_minus_beta1 * gg;
    v = h.beta2 * v + h.one_minus_beta2 * gg * gg;
    const float mh = m / b1t, vh = v / b2t;
    return w - ((h.lr * mh / (sqrtf(vh) + h.eps)) + (h.decay * h.lr) * w);
}

__device__ __forceinline__ long long wk_index(const AdamTensor& t, long long i) {
    const long long r = i / t.wk_cols, c = i - r * t.wk_cols;
    return r * t.wk_ld + t.wk_off + c;
}

__device__ __forceinline__ void adamw_body(const AdamTensor& t, const AdamHyper& h) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long first = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (t.vec4) {
        const long long n4 = t.n >> 2;
        for (long long i = first; i < n4; i += stride) {
            const float4 g = __ldcs(reinterpret_cast<const float4*>(t.g) + i);
            float4 m = __ldcs(reinterpret_cast<const float4*>(t.m) + i);
            float4 v = __ldcs(reinterpret_cast<const float4*>(t.v) + i);
            float4 w = __ldcs(reinterpret_cast<const float4*>(t.w) + i);
            w.x = adamw_elem(w.x, g.x, m.x, v.x, t.b1t, t.b2t, h);
            w.y = adamw_elem(w.y, g.y, m.y, v.y, t.b1t, t.b2t, h);
            w.z = adamw_elem(w.z, g.z, m.z, v.z, t.b1t, t.b2t, h);
            w.w = adamw_elem(w.w, g.w, m.w, v.w, t.b1t, t.b2t, h);
            __stcs(reinterpret_cast<float4*>(t.m) + i, m);
            __stcs(reinterpret_cast<float4*>(t.v) + i, v);
            reinterpret_cast<float4*>(t.w)[i] = w;
            if (t.wk) {
                const long long o = wk_index(t, 4 * i);
                if (t.wk_bf16) {
                    __nv_bfloat162 a = __floats2bfloat162_rn(w.x, w.y), b = __floats2bfloat162_rn(w.z, w.w);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t*>(&a);
                    u.y = *reinterpret_cast<uint32_t*>(&b);
                    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(t.wk) + o) = u;
                } else {
                    *reinterpret_cast<float4*>(reinterpret_cast<float*>(t.wk) + o) = w;
                }
            }
        }
        return;
    }
    for (long long i = first; i < t.n; i += stride) {
        float m = t.m[i], v = t.v[i];
        const float w = adamw_elem(t.w[i], t.g[i], m, v, t.b1t, t.b2t, h);
        t.m[i] = m;
        t.v[i] = v;
        t.w[i] = w;
        if (t.wk) {
            const long long o = wk_index(t, i);
            if (t.wk_bf16) reinterpret_cast<__nv_bfloat16*>(t.wk)[o] = f2bf(w);
            else reinterpret_cast<float*>(t.wk)[o] = w;
        }
    }
}

struct AdamBatch {
    AdamTensor t[kAdamBatch];
};

// blockIdx.y selects the tensor
__global__ void __launch_bounds__(256) adamw_batch_kernel(const __grid_constant__ AdamBatch b, AdamHyper h) {
    adamw_body(b.t[blockIdx.y], h);
}
__global__ void adamw_single_kernel(AdamTensor t, AdamHyper h) { adamw_body(t, h); }

void adamw_prepare(AdamTensor& t) {
    const bool a16 = aligned16(t.w) && aligned16(t.g) && aligned16(t.m) && aligned16(t.v);
    bool ok = a16 && t.n % 4 == 0;
    if (ok && t.wk) {
        const uintptr_t al = t.wk_bf16 ? 8 : 16;
        ok = t.wk_cols % 4 == 0 && t.wk_ld % 4 == 0 && t.wk_off % 4 == 0 &&
             (reinterpret_cast<uintptr_t>(t.wk) & (al - 1)) == 0;
    }
    t.vec4 = ok ? 1 : 0;
}

int adamw_single(AdamTensor t, AdamHyper h, cudaStream_t s) {
    if (t.n <= 0) return 0;
    adamw_prepare(t);
    adamw_single_kernel<<<grid_for((size_t)(t.vec4 ? t.n / 4 : t.n), 256), 256, 0, s>>>(t, h);
    return launch_ok();
}

int adamw_multi(const AdamTensor* ts, int count, AdamHyper h, cudaStream_t s) {
    for (int b0 = 0; b0 < count; b0 += kAdamBatch) {
        const int nb = count - b0 < kAdamBatch ? count - b0 : kAdamBatch;
        AdamBatch batch;
        long long maxw = 0;
        for (int i = 0; i < nb; i++) {
            batch.t[i] = ts[b0 + i];
            adamw_prepare(batch.t[i]);
            const long long wn = batch.t[i].vec4 ? batch.t[i].n / 4 : batch.t[i].n;
            if (wn > maxw) maxw = wn;
        }
        if (maxw <= 0) continue;
        long long blocks = (maxw + 255) / 256, cap = (long long)num_sms() * 4;
        dim3 grid((unsigned)(blocks < cap ? blocks : cap), nb);
        adamw_batch_kernel<<<grid, 256, 0, s>>>(batch, h);
        if (launch_ok()) return -5;
    }
    return 0;
}

__global__ void muon_momentum_kernel(float* m, const float* g, long long n, float mu) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        m[i] = mu * m[i] + g[i];
}
int muon_momentum(float* m, const float* g, long long n, float momentum, cudaStream_t s) {
    if (n <= 0) return 0;
    muon_momentum_kernel<<<grid_for((size_t)n, 256), 256, 0, s>>>(m, g, n, momentum);
    return launch_ok();
}

// Modified Gram-Schmidt (reference ns_orthonom, codegen.cpp:1617-1633).
__global__ void __launch_bounds__(1024) mgs_kernel(float* G, int M, int N) {
    __shared__ float sh[33];
    const bool tr = M < N;
    const int R = tr ? N : M, Cn = tr ? M : N;
    auto at = [&](int k, int j) -> float& { return tr ? G[(size_t)j * R + k] : G[(size_t)k * N + j]; };
    for (int j = 0; j < Cn; j++) {
        for (int i = 0; i < j; i++) {
            float d = 0.f;
            for (int k = threadIdx.x; k < R; k += blockDim.x) d += at(k, i) * at(k, j);
            d = block_sum(d, sh);
            for (int k = threadIdx.x; k < R; k += blockDim.x) at(k, j) -= d * at(k, i);
            __syncthreads();
        }
        float nr = 0.f;
        for (int k = threadIdx.x; k < R; k += blockDim.x) nr += at(k, j) * at(k, j);
        nr = sqrtf(block_sum(nr, sh)) + 1e-30f;
        for (int k = threadIdx.x; k < R; k += blockDim.x) at(k, j) /= nr;
        __syncthreads();
    }
}
int mgs_orthonormalize(float* G, int r, int c, cudaStream_t s) {
    mgs_kernel<<<1, 1024, 0, s>>>(G, r, c);
    return launch_ok();
}

__global__ void muon_apply_kernel(float* w, const float* o, float* m, long long n, float le, float decay_lr, int zero_m,
                                  __nv_bfloat16* __restrict__ w16) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float wi = w[i];
        const float wn = wi - (le * o[i] + decay_lr * wi);
        w[i] = wn;
        if (w16) w16[i] = f2bf(wn);
        if (zero_m) m[i] = 0.f;
    }
}
int muon_apply(float* w, const float* o, float* m, long long n, float le, float decay_lr, int zero_m, cudaStream_t s,
               __nv_bfloat16* w16) {
    if (n <= 0) return 0;
    muon_apply_kernel<<<grid_for((size_t)n, 256), 256, 0, s>>>(w, o, m, n, le, decay_lr, zero_m, w16);
    return launch_ok();
}

// Frobenius normalisation out = x / (||x|| + eps): per-block partial sums
// of squares, then a scaling pass that also writes the bf16 copy the
// Newton-Schulz GEMMs read (when out16 is given). 16-byte accesses when n is
// a multiple of 4 and the buffers are aligned.
__global__ void sumsq_partial_kernel(const float* __restrict__ x, long long n, int vec, float* part) {
    __shared__ float sh[33];
    float acc = 0.f;
    const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x, st = (long long)gridDim.x * blockDim.x;
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (long long i = t0; i < n / 4; i += st) {
            const float4 v = x4[i];
            acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (long long i = t0; i < n; i += st) acc += x[i] * x[i];
    }
    acc = block_sum(acc, sh);
    if (threadIdx.x == 0) part[blockIdx.x] = acc;
}
__global__ void scale_by_norm_kernel(const float* __restrict__ x, long long n, int vec, const float* part, int nparts,
                                     float eps, float* __restrict__ out, __nv_bfloat16* __restrict__ out16) {
    __shared__ float inv;
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int i = 0; i < nparts; i++) s += part[i];
        inv = 1.f / (sqrtf(s) + eps);
    }
    __syncthreads();
    const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x, st = (long long)gridDim.x * blockDim.x;
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (long long i = t0; i < n / 4; i += st) {
            float4 v = x4[i];
            v.x *= inv;
            v.y *= inv;
            v.z *= inv;
            v.w *= inv;
            reinterpret_cast<float4*>(out)[i] = v;
            if (out16) {
                uint2 h;
                reinterpret_cast<__nv_bfloat162*>(&h)[0] = __floats2bfloat162_rn(v.x, v.y);
                reinterpret_cast<__nv_bfloat162*>(&h)[1] = __floats2bfloat162_rn(v.z, v.w);
                reinterpret_cast<uint2*>(out16)[i] = h;
            }
        }
    } else {
        for (long long i = t0; i < n; i += st) {
            out[i] = x[i] * inv;
            if (out16) out16[i] = f2bf(out[i]);
        }
    }
}
int frob_normalize(const float* x, long long n, float eps, float* out, float* scratch, cudaStream_t s,
                   __nv_bfloat16* out16) {
    const int parts = 512;
    auto al = [](const void* q, int b) { return !(reinterpret_cast<uintptr_t>(q) & (b - 1)); };
    const int vec = n % 4 == 0 && al(x, 16) && al(out, 16) && (!out16 || al(out16, 8));
    sumsq_partial_kernel<<<parts, 256, 0, s>>>(x, n, vec, scratch);
    const size_t work = vec ? (size_t)n / 4 : (size_t)n;
    scale_by_norm_kernel<<<grid_for(work, 256), 256, 0, s>>>(x, n, vec, scratch, parts, eps, out, out16);
    return launch_ok();
}

}  // namespace nsb
