// engram_backward.cu -- K3: row gradients of the overlay.
//
// The result reproduces the reference's accumulation order exactly.  The
// reference sums duplicate rows with index_put_(accumulate=True) over idx lists
// built in ascending (t, h) order (engraft/replica/seq.py:401-441): serially on
// one CPU thread, and after a stable sort of the indices on CUDA.  Here:
//   1. a stable LSD radix sort (8-bit digits) of the hit entries keyed by overlay
//      slot; entry values are flat indices t*n_heads+h, so each slot's entries
//      come out in ascending (t, h) order.  Ranks inside a tile come from warp
//      __match_any_sync groups plus per-warp digit counts (no comparison sort);
//      block offsets come from a per-digit row scan (256 blocks);
//   2. segment starts per slot from the sorted keys;
//   3. one streaming segmented reduction: blocks take segment-aligned chunks
//      of the sorted entries (dynamically), stage their row offsets in shared
//      memory, stream the rows through a kStages-deep cp.async ring, and every
//      thread adds its own columns in order, writing a slot's row when its
//      segment ends.
// Every term is added from +0 in ascending (t, h) order in fp32, so the result
// is bit-identical to the reference and independent of scheduling.
#include <algorithm>
#include <mutex>

#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsItems = 16;
constexpr int kRsTile = kRsThreads * kRsItems;
constexpr int kScanThreads = 1024;
constexpr int kRedThreads = 256;
#ifndef ENGRAM_RED_CHUNK
#define ENGRAM_RED_CHUNK 256
#endif
#ifndef ENGRAM_RED_STAGES
#define ENGRAM_RED_STAGES 4
#endif
constexpr int kChunk = ENGRAM_RED_CHUNK;  // nominal sorted entries per work chunk (snapped to segment starts)
constexpr int kMetaCap = 4096;            // entries whose row offsets and keys a block stages at a time
constexpr int kStageBytes = 16384;        // rows per pipeline stage (>= 4 rows of <= 4 KB)
constexpr int kStages = ENGRAM_RED_STAGES;
constexpr int kRedSmem = kStages * kStageBytes + kMetaCap * 4 + (kMetaCap + 1) * 4;

constexpr int kBigChunk = 4 * kChunk;  // chunks longer than this (long segments) are scheduled first

// counters[] in the workspace
constexpr int kCntHits = 0, kCntChunkNext = 1, kCntBig = 2, kCntBigNext = 3;

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct Workspace {
    int32_t* keys[2];
    int32_t* vals[2];
    uint32_t* block_hist;
    uint32_t* digit_tot;
    int32_t* seg_begin;
    int32_t* chunk_lo;  // [max_chunks + 1] segment-aligned chunk bounds
    int32_t* big;       // [max_chunks] ids of long chunks
    int32_t* counters;
    int64_t bytes;
    int nblk;
};

Workspace layout(void* base, int64_t N, int64_t R) {
    Workspace w{};
    const int64_t nblk = (N + kRsTile - 1) / kRsTile;
    w.nblk = (int)(nblk > 0 ? nblk : 1);
    char* p = static_cast<char*>(base);
    int64_t off = 0;
    auto take = [&](int64_t bytes) {
        char* r = p ? p + off : nullptr;
        off += align256(bytes);
        return r;
    };
    for (int k = 0; k < 2; k++) {
        w.keys[k] = reinterpret_cast<int32_t*>(take(4 * N));
        w.vals[k] = reinterpret_cast<int32_t*>(take(4 * N));
    }
    w.block_hist = reinterpret_cast<uint32_t*>(take(4 * 256 * (int64_t)w.nblk));
    w.digit_tot = reinterpret_cast<uint32_t*>(take(4 * 256));
    w.seg_begin = reinterpret_cast<int32_t*>(take(4 * (R + 1)));
    const int64_t max_chunks = N / kChunk + 1;
    w.chunk_lo = reinterpret_cast<int32_t*>(take(4 * (max_chunks + 1)));
    w.big = reinterpret_cast<int32_t*>(take(4 * max_chunks));
    w.counters = reinterpret_cast<int32_t*>(take(64));
    w.bytes = off;
    return w;
}

// Exclusive scan of one value per thread over a block of `nthreads` (multiple of
// 32, <= 1024); returns the exclusive prefix, *total gets the block sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < nwarps ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(kFull, s, o);
            if (lane >= o) s += y;
        }
        if (lane < nwarps) warp_sums[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    if (total) *total = warp_sums[nwarps - 1];
    const uint32_t res = before + x - v;
    __syncthreads();  // warp_sums may be reused by the caller
    return res;
}

// Pass histogram: digit counts of this block's tile, stored digit-major.
__global__ void __launch_bounds__(kRsThreads) k_rs_hist(const int32_t* __restrict__ keys, const int32_t* n_dev,
                                                        int64_t n_static, int shift, uint32_t* block_hist, int nblk,
                                                        int32_t* counters) {
    __shared__ uint32_t h[256];
    for (int d = threadIdx.x; d < 256; d += kRsThreads) h[d] = 0;
    if (counters && blockIdx.x == 0 && threadIdx.x == 0) {
        counters[kCntChunkNext] = 0;
        counters[kCntBig] = 0;
        counters[kCntBigNext] = 0;
    }
    __syncthreads();
    const int64_t n = n_dev ? (int64_t)*n_dev : n_static;
    const int64_t begin = (int64_t)blockIdx.x * kRsTile;
    int32_t kr[kRsItems];
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int64_t i = begin + (int64_t)sub * kRsThreads + threadIdx.x;
        kr[sub] = i < n ? __ldg(keys + i) : -1;
    }
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++)
        if (kr[sub] >= 0) atomicAdd(&h[(kr[sub] >> shift) & 255], 1u);
    __syncthreads();
    for (int d = threadIdx.x; d < 256; d += kRsThreads) block_hist[(int64_t)d * nblk + blockIdx.x] = h[d];
}

// Block d: exclusive scan, in place, of digit d's counts over the blocks; digit_tot[d] = total.
__global__ void __launch_bounds__(kScanThreads) k_rs_rowscan(uint32_t* block_hist, int nblk, uint32_t* digit_tot) {
    __shared__ uint32_t wsum[32];
    uint32_t* row = block_hist + (int64_t)blockIdx.x * nblk;
    uint32_t carry = 0;
    for (int base = 0; base < nblk; base += kScanThreads) {
        const int i = base + threadIdx.x;
        const uint32_t v = i < nblk ? row[i] : 0u;
        uint32_t tot;
        const uint32_t ex = block_exclusive_scan(v, wsum, &tot);
        if (i < nblk) row[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) digit_tot[blockIdx.x] = carry;
}

// Stable scatter of one pass.  vals_in == nullptr: the value is the index.
// total_out (nullable): receives the number of entries sorted (the hit count).
// The tile's keys (and values) are loaded into registers up front, so the 16
// sub-tiles cost one memory latency; per-warp digit counts alternate between
// two shared buffers so each sub-tile needs two block barriers.
__global__ void __launch_bounds__(kRsThreads) k_rs_scatter(const int32_t* __restrict__ keys_in,
                                                           const int32_t* __restrict__ vals_in, const int32_t* n_dev,
                                                           int64_t n_static, int shift,
                                                           const uint32_t* __restrict__ block_off,
                                                           const uint32_t* __restrict__ digit_tot, int nblk,
                                                           int32_t* __restrict__ keys_out,
                                                           int32_t* __restrict__ vals_out, int32_t* total_out) {
    __shared__ uint32_t wcnt[2][kRsWarps][256];
    __shared__ uint32_t run[256];
    __shared__ uint32_t wsum[32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n = n_dev ? (int64_t)*n_dev : n_static;
    const int64_t begin = (int64_t)blockIdx.x * kRsTile;
    int32_t kr[kRsItems], vr[kRsItems];
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int64_t i = begin + (int64_t)sub * kRsThreads + tid;
        kr[sub] = i < n ? __ldg(keys_in + i) : -1;
        vr[sub] = vals_in ? (i < n ? __ldg(vals_in + i) : 0) : (int32_t)i;
    }
    for (int k = tid; k < 2 * kRsWarps * 256; k += kRsThreads) (&wcnt[0][0][0])[k] = 0;
    {
        const uint32_t dt = digit_tot[tid];  // kRsThreads == 256 digits
        uint32_t tot;
        const uint32_t base = block_exclusive_scan(dt, wsum, &tot);  // contains a barrier
        run[tid] = base + block_off[(int64_t)tid * nblk + blockIdx.x];
        if (total_out && blockIdx.x == 0 && tid == 0) *total_out = (int32_t)tot;
    }
    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int B = sub & 1;
        const int32_t key = kr[sub];
        const bool valid = key >= 0;
        const int digit = valid ? ((key >> shift) & 255) : (256 + lane);
        const unsigned peers = __match_any_sync(kFull, digit);
        const int rank = __popc(peers & lt);
        if (valid && rank == 0) wcnt[B][warp][digit] = (uint32_t)__popc(peers);
        __syncthreads();
        {
            const int d = tid;
            uint32_t acc = run[d];
#pragma unroll
            for (int w = 0; w < kRsWarps; w++) {
                const uint32_t c = wcnt[B][w][d];
                wcnt[B][w][d] = acc;
                wcnt[B ^ 1][w][d] = 0;  // ready for the next sub-tile
                acc += c;
            }
            run[d] = acc;
        }
        __syncthreads();
        if (valid) {
            const uint32_t pos = wcnt[B][warp][digit] + (uint32_t)rank;
            keys_out[pos] = key;
            vals_out[pos] = vr[sub];
        }
    }
}

// seg_begin[s] = number of sorted entries with key < s, for s in [0, R].
__global__ void k_seg_begin(const int32_t* __restrict__ keys, const int32_t* counters, int64_t R,
                            int32_t* __restrict__ seg_begin) {
    const int64_t n = counters[kCntHits];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (n == 0) {
        for (int64_t s = tid; s <= R; s += stride) seg_begin[s] = 0;
        return;
    }
    for (int64_t i = tid; i < n; i += stride) {
        const int32_t k = keys[i];
        const int32_t prev = i == 0 ? -1 : keys[i - 1];
        for (int64_t s = (int64_t)prev + 1; s <= k; s++) seg_begin[s] = (int32_t)i;
        if (i == n - 1)
            for (int64_t s = (int64_t)k + 1; s <= R; s++) seg_begin[s] = (int32_t)n;
    }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Offset, in 16-byte units, of the upstream-gradient row of flat entry i = t*n_heads + h.
template <int MODE>
__device__ __forceinline__ uint32_t grad_row16(int64_t i, int dim, int n_heads, int hpn) {
    if (MODE == ENGRAM_MODE_CONCAT_F32) return (uint32_t)((i * (int64_t)dim) >> 2);
    const int64_t t = i / n_heads;
    const int h = (int)(i - t * n_heads);
    return (uint32_t)((t * hpn * dim + (int64_t)(h % hpn) * dim) >> 3);
}

// First segment start at or after sorted entry e (e in [0, n]).
__device__ __forceinline__ int64_t snap_to_segment(const int32_t* __restrict__ keys,
                                                   const int32_t* __restrict__ seg_begin, int64_t e, int64_t n) {
    if (e <= 0) return 0;
    if (e >= n) return n;
    const int32_t k = __ldg(keys + e);
    if (__ldg(keys + e - 1) != k) return e;
    return __ldg(seg_begin + k + 1);
}

// chunk_lo[j] = first segment start at or after j*kChunk, j in [0, n_chunks];
// chunks longer than kBigChunk are listed in big[] so they start first.
__global__ void k_chunks(const int32_t* __restrict__ keys, const int32_t* __restrict__ seg_begin, int32_t* counters,
                         int32_t* __restrict__ chunk_lo, int32_t* __restrict__ big) {
    const int64_t n = counters[kCntHits];
    const int64_t nchunks = (n + kChunk - 1) / kChunk;
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j <= nchunks; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lo = snap_to_segment(keys, seg_begin, j * kChunk, n);
        chunk_lo[j] = (int32_t)lo;
        if (j < nchunks) {
            const int64_t hi = snap_to_segment(keys, seg_begin, (j + 1) * kChunk, n);
            if (hi - lo > kBigChunk) big[atomicAdd(counters + kCntBig, 1)] = (int32_t)j;
        }
    }
}

// Streaming segmented reduction over the slot-sorted entries.  Blocks take
// chunks of ~kChunk entries whose bounds are snapped to segment starts (so a
// segment never spans two blocks; a long segment makes one long chunk).  A
// chunk's row offsets and keys are staged in shared memory, then its rows
// stream through a kStages-deep cp.async ring while thread c adds column c of
// every row in order and writes the slot's row when its segment ends.  Slots
// without entries get zero rows.  NJ = columns per thread (dim <= 256*NJ).
template <int MODE, int NJ>
__global__ void __launch_bounds__(kRedThreads) k_reduce(const int32_t* __restrict__ keys,
                                                        const int32_t* __restrict__ vals,
                                                        const int32_t* __restrict__ seg_begin,
                                                        const int32_t* __restrict__ chunk_lo,
                                                        const int32_t* __restrict__ big, int32_t* counters,
                                                        int64_t R, int dim, int n_heads, int hpn,
                                                        const uint8_t* __restrict__ grad,
                                                        float* __restrict__ grad_rows) {
    constexpr int ES = MODE == ENGRAM_MODE_CONCAT_F32 ? 4 : 2;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* m_off = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes);
    int32_t* m_key = reinterpret_cast<int32_t*>(m_off + kMetaCap);
    __shared__ int s_job;
    const int tid = threadIdx.x;
    const int64_t n = counters[kCntHits];
    const int64_t nchunks = (n + kChunk - 1) / kChunk;
    const int row_bytes = dim * ES;
    const int chunks16 = row_bytes >> 4;
    const int rps = kStageBytes / row_bytes;  // rows per stage
    const uint4* g16 = reinterpret_cast<const uint4*>(grad);
    // when the 16-byte pieces of a row divide the block, every thread copies one
    // fixed piece of every r_step-th row (no division in the copy loop)
    const bool fixed_piece = chunks16 <= kRedThreads && (kRedThreads % chunks16) == 0;
    const int my_p = fixed_piece ? tid % chunks16 : 0;
    const int my_r = fixed_piece ? tid / chunks16 : 0;
    const int r_step = fixed_piece ? kRedThreads / chunks16 : 1;

    const int n_big = counters[kCntBig];
    while (true) {
        // long chunks first (their sequential chains are the critical path), then the rest in order
        if (tid == 0) {
            int j = -1;
            const int b = atomicAdd(counters + kCntBigNext, 1);
            if (b < n_big) {
                j = big[b];
            } else {
                while (true) {
                    const int c = atomicAdd(counters + kCntChunkNext, 1);
                    if (c >= nchunks) break;
                    if (chunk_lo[c + 1] - chunk_lo[c] <= kBigChunk) { j = c; break; }
                }
            }
            s_job = j;
        }
        __syncthreads();
        const int64_t j = s_job;
        __syncthreads();
        if (j < 0) break;
        const int64_t lo = chunk_lo[j];
        const int64_t hi = chunk_lo[j + 1];
        float acc[NJ];
#pragma unroll
        for (int q = 0; q < NJ; q++) acc[q] = 0.f;
        for (int64_t m0 = lo; m0 < hi; m0 += kMetaCap) {
            const int mn = (int)(hi - m0 < kMetaCap ? hi - m0 : kMetaCap);
            for (int e = tid; e <= mn; e += kRedThreads) {
                if (e < mn) {
                    m_off[e] = grad_row16<MODE>(__ldg(vals + m0 + e), dim, n_heads, hpn);
                    m_key[e] = __ldg(keys + m0 + e);
                } else {
                    m_key[e] = (m0 + e < hi) ? __ldg(keys + m0 + e) : -1;  // key after the last staged entry
                }
            }
            __syncthreads();
            const int nst = (mn + rps - 1) / rps;
            auto issue = [&](int st) {
                if (st < nst) {
                    uint8_t* buf = smem + (st % kStages) * kStageBytes;
                    const int r0 = st * rps;
                    const int nr = min(rps, mn - r0);
                    if (fixed_piece) {  // thread copies piece my_p of rows my_r, my_r + r_step, ...
                        for (int r = my_r; r < nr; r += r_step)
                            cp_async16(buf + r * row_bytes + my_p * 16, g16 + m_off[r0 + r] + my_p);
                    } else {
                        for (int c = tid; c < nr * chunks16; c += kRedThreads) {
                            const int r = c / chunks16, p = c - r * chunks16;
                            cp_async16(buf + r * row_bytes + p * 16, g16 + m_off[r0 + r] + p);
                        }
                    }
                }
                cp_async_commit();
            };
#pragma unroll 1
            for (int st = 0; st < kStages - 1; st++) issue(st);
#pragma unroll 1
            for (int st = 0; st < nst; st++) {
                cp_async_wait<kStages - 2>();
                __syncthreads();
                issue(st + kStages - 1);
                const uint8_t* buf = smem + (st % kStages) * kStageBytes;
                const int r0 = st * rps;
                const int nr = min(rps, mn - r0);
                // 4 rows per step: their shared-memory loads issue together, the adds stay in row order
                constexpr int U = 4;
#pragma unroll 1
                for (int r = 0; r < nr; r += U) {
                    float x[U][NJ];
                    int32_t kk[U + 1];
#pragma unroll
                    for (int u = 0; u <= U; u++) kk[u] = (r + u <= nr) ? m_key[r0 + r + u] : -2;
#pragma unroll
                    for (int u = 0; u < U; u++) {
#pragma unroll
                        for (int q = 0; q < NJ; q++) {
                            const int c = tid + kRedThreads * q;
                            x[u][q] = 0.f;
                            if (r + u < nr && c < dim) {
                                const uint8_t* row = buf + (r + u) * row_bytes;
                                if (MODE == ENGRAM_MODE_CONCAT_F32)
                                    x[u][q] = reinterpret_cast<const float*>(row)[c];
                                else
                                    x[u][q] = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(row)[c] << 16);
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        if (r + u < nr) {
#pragma unroll
                            for (int q = 0; q < NJ; q++) acc[q] = __fadd_rn(acc[q], x[u][q]);
                            if (kk[u + 1] != kk[u]) {  // last entry of its segment
                                float* dst = grad_rows + (int64_t)kk[u] * dim;
#pragma unroll
                                for (int q = 0; q < NJ; q++) {
                                    const int c = tid + kRedThreads * q;
                                    if (c < dim) dst[c] = acc[q];
                                    acc[q] = 0.f;
                                }
                            }
                        }
                    }
                }
            }
            cp_async_wait<0>();
            __syncthreads();  // stage buffers and metadata are reused next
        }
    }
    // slots without entries
    const int lane = tid & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + tid) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t s = warp0; s < R; s += nwarps) {
        if (__ldg(seg_begin + s) == __ldg(seg_begin + s + 1)) {
            float4* dst = reinterpret_cast<float4*>(grad_rows + s * dim);
            for (int c = lane; c < (dim >> 2); c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

int grid_for_chunks(const Workspace& w);

template <int MODE, int NJ>
void launch_reduce(const Workspace& w, const int32_t* keys, const int32_t* vals, int64_t R, int dim, int n_heads,
                   int hpn, const void* grad, float* grad_rows, cudaStream_t s) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaFuncSetAttribute(k_reduce<MODE, NJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRedSmem);
        configured[dev] = true;
    }
    const int grid = sm_count() * 2;
    k_chunks<<<grid_for_chunks(w), 256, 0, s>>>(keys, w.seg_begin, w.counters, w.chunk_lo, w.big);
    k_reduce<MODE, NJ><<<grid, kRedThreads, kRedSmem, s>>>(keys, vals, w.seg_begin, w.chunk_lo, w.big, w.counters, R,
                                                          dim, n_heads, hpn,
                                                          static_cast<const uint8_t*>(grad), grad_rows);
}

int grid_for(int64_t work, int threads, int per_sm) {
    const int64_t want = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int64_t g = want < cap ? want : cap;
    return (int)(g > 0 ? g : 1);
}

int grid_for_chunks(const Workspace& w) { return grid_for((int64_t)w.nblk * kRsTile / kChunk + 2, 256, 4); }

}  // namespace

extern "C" int64_t engram_backward_workspace_bytes(int64_t n, int32_t n_heads, int64_t R) {
    if (n < 0 || n_heads < 1 || R < 0) return ENGRAM_ERR_ARG;
    return layout(nullptr, n * n_heads, R).bytes;
}

extern "C" int engram_backward(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                               int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                               void* workspace, int64_t workspace_bytes, void* stream) {
    if (n < 0 || R < 0 || n_heads < 1 || n_heads > ENGRAM_MAX_HEADS || heads_per_ngram < 1) return ENGRAM_ERR_ARG;
    if (mode != ENGRAM_MODE_CONCAT_F32 && mode != ENGRAM_MODE_PAIRSUM_ADD_BF16) return ENGRAM_ERR_ARG;
    if (dim <= 0 || dim > 1024 || (mode == ENGRAM_MODE_CONCAT_F32 ? dim % 4 : dim % 8)) return ENGRAM_ERR_FORMAT;
    if (mode == ENGRAM_MODE_PAIRSUM_ADD_BF16 && n_heads != 2 * heads_per_ngram) return ENGRAM_ERR_FORMAT;
    if (R >= (1LL << 24) || n * n_heads >= (1LL << 31)) return ENGRAM_ERR_RANGE;
    const int64_t grad_bytes = mode == ENGRAM_MODE_CONCAT_F32 ? n * n_heads * (int64_t)dim * 4
                                                              : n * (int64_t)heads_per_ngram * dim * 2;
    if ((grad_bytes >> 4) >= (1LL << 32)) return ENGRAM_ERR_RANGE;
    if (R == 0) return ENGRAM_OK;
    if (!grad_rows || !aligned16(grad_rows)) return ENGRAM_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        return cudaMemsetAsync(grad_rows, 0, sizeof(float) * (size_t)R * dim, s) == cudaSuccess ? ENGRAM_OK
                                                                                                 : ENGRAM_ERR_CUDA;
    }
    if (!slots || !grad || !aligned16(grad)) return ENGRAM_ERR_ARG;
    const int64_t N = n * n_heads;
    Workspace w = layout(workspace, N, R);
    if (!workspace || workspace_bytes < w.bytes) return ENGRAM_ERR_WORKSPACE;

    int bits = 0;
    while ((1LL << bits) < R) bits++;
    const int passes = bits <= 8 ? 1 : (bits + 7) / 8;
    int cur = 0;
    for (int pass = 0; pass < passes; pass++) {
        const int shift = 8 * pass;
        const int32_t* kin = pass == 0 ? slots : w.keys[cur];
        const int32_t* vin = pass == 0 ? nullptr : w.vals[cur];
        const int32_t* n_dev = pass == 0 ? nullptr : w.counters + kCntHits;
        const int out = pass == 0 ? 0 : 1 - cur;
        k_rs_hist<<<w.nblk, kRsThreads, 0, s>>>(kin, n_dev, N, shift, w.block_hist, w.nblk,
                                                pass == 0 ? w.counters : nullptr);
        k_rs_rowscan<<<256, kScanThreads, 0, s>>>(w.block_hist, w.nblk, w.digit_tot);
        k_rs_scatter<<<w.nblk, kRsThreads, 0, s>>>(kin, vin, n_dev, N, shift, w.block_hist, w.digit_tot, w.nblk,
                                                     w.keys[out], w.vals[out],
                                                     pass == 0 ? w.counters + kCntHits : nullptr);
        cur = out;
    }
    k_seg_begin<<<grid_for(N, 256, 8), 256, 0, s>>>(w.keys[cur], w.counters, R, w.seg_begin);
    const int nj = (dim + kRedThreads - 1) / kRedThreads;
    if (mode == ENGRAM_MODE_CONCAT_F32) {
        if (nj <= 1) launch_reduce<ENGRAM_MODE_CONCAT_F32, 1>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
        else if (nj <= 2) launch_reduce<ENGRAM_MODE_CONCAT_F32, 2>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
        else launch_reduce<ENGRAM_MODE_CONCAT_F32, 4>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
    } else {
        if (nj <= 1) launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 1>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
        else if (nj <= 2) launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 2>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
        else launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 4>(w, w.keys[cur], w.vals[cur], R, dim, n_heads, heads_per_ngram, grad, grad_rows, s);
    }
    count_launches(3 * passes + 3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

// ---- engram_backward_noalloc ---------------------------------------------------
// The same row-gradient computation for callers that cannot allocate device
// memory on their hot path: the scratch comes from this file-scope array
// instead of a caller workspace.  Host code must not pass the array's name to
// a kernel (on the host it is only a stand-in symbol); its device address is
// looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ENGRAM_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (set-up on first use).
int noalloc_scratch(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ENGRAM_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return ENGRAM_ERR_CUDA;
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return ENGRAM_OK;
}
}  // namespace

extern "C" int engram_backward_noalloc(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                                       int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                                       void* stream) {
    if (n < 0 || R < 0 || n_heads < 1 || n_heads > ENGRAM_MAX_HEADS) return ENGRAM_ERR_ARG;
    if (R >= (1LL << 24) || n * n_heads >= (1LL << 31)) return ENGRAM_ERR_RANGE;
    if (layout(nullptr, n * n_heads, R).bytes > ENGRAM_NOALLOC_SCRATCH_BYTES) return ENGRAM_ERR_WORKSPACE;
    void* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != ENGRAM_OK) return st;
    return engram_backward(slots, n, n_heads, heads_per_ngram, mode, grad, dim, R, grad_rows, scratch,
                           ENGRAM_NOALLOC_SCRATCH_BYTES, stream);
}
