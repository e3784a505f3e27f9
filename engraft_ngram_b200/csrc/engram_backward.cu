// engram_backward.cu -- K3: row gradients of the overlay.
//
// The result reproduces the reference's accumulation order exactly.  The
// reference sums duplicate rows with index_put_(accumulate=True) over idx lists
// built in ascending (t, h) order (engraft/replica/seq.py:401-441): serially on
// one CPU thread, and after a stable sort of the indices on CUDA.  Here:
//   1. a stable LSD radix sort (8-bit digits) of the hit entries keyed by overlay
//      slot; entry values are flat indices t*n_heads+h, so each slot's entries
//      come out in ascending (t, h) order.  Ranks inside a tile come from
//      per-warp running digit counts and, inside a warp, from one ballot per
//      digit bit (no comparison sort); block offsets come from a per-digit
//      row scan (256 blocks);
//   2. segment starts per slot from the sorted keys;
//   3. one segmented reduction in which every warp runs its own jobs.  First
//      the segments longer than kLongRows entries, split by columns: one job
//      per 64-byte slice, so the long sequential chains of the hot slots start
//      at once, on many SMs.  Then every warp streams the remaining entries
//      (whole segments, taken in jobs from an atomic counter) through a private
//      cp.async ring: lane l copies and adds its own 16-byte column vectors of
//      every row and the warp writes a slot's row when its segment ends.
// Every term is added from +0 in ascending (t, h) order in fp32, so the result
// is bit-identical to the reference and independent of scheduling.
#include <algorithm>
#include <climits>
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
// segmented reduction
#ifndef ENGRAM_RED_ROWS
#define ENGRAM_RED_ROWS 16
#endif
#ifndef ENGRAM_RED_LONG_GI
#define ENGRAM_RED_LONG_GI 5
#endif
#ifndef ENGRAM_RED_CPW
#define ENGRAM_RED_CPW 8
#endif
constexpr int kRedWarps = 4;                            // warps per block; each warp runs its own jobs
constexpr int kShortRows = ENGRAM_RED_ROWS;             // 512-byte rows in flight per warp in short jobs
constexpr int kShortWarpSmem = (kShortRows + 8) * 512;  // its ring, with one spare batch
constexpr int kChunksPerWarp = ENGRAM_RED_CPW;          // short chunks per warp, for balance
constexpr int kMinChunk = 32, kMaxChunk = 2048;         // short-chunk size bounds (entries)
#ifndef ENGRAM_RED_LONGROWS
#define ENGRAM_RED_LONGROWS 256
#endif
constexpr int kLongRows = ENGRAM_RED_LONGROWS;          // segments longer than this are split by columns
constexpr int kSliceBytes = 64;                         // column slice of a long-segment job
constexpr int kLongGI = ENGRAM_RED_LONG_GI;             // 32-row groups in flight in a long job
constexpr int kLongRingGroups = kLongGI + 1;
constexpr int kLongValSlots = 2 * kLongGI + 1;
constexpr int kLongWarpSmem = kLongRingGroups * 32 * kSliceBytes + kLongValSlots * 32 * 4;
constexpr int kWarpSmem = kLongWarpSmem > kShortWarpSmem ? kLongWarpSmem : kShortWarpSmem;  // per warp
constexpr int kRedSmem = kRedWarps * kWarpSmem;

// Short-chunk ring: lane-owned 16-byte column vectors, NV per lane.
template <int NV>
struct ShortRing {
    static constexpr int D = kShortRows / NV;                   // rows in flight
    static constexpr int U = D >= 16 ? 4 : (D >= 8 ? 2 : 1);    // rows per commit group
    static constexpr int GI = D / U;                            // commit groups in flight
    static constexpr int ROWS = D + U;                          // ring rows: one spare batch
    static_assert(D <= 32 && D % U == 0 && 32 % U == 0 && GI >= 2, "short-chunk ring");
    static_assert(ROWS * NV * 512 <= kShortWarpSmem, "short-chunk ring");
};

// counters[] in the workspace
constexpr int kCntHits = 0, kCntLongNext = 1, kCntLong = 2, kCntChunks = 3, kCntShortNext = 4, kCntMedium = 5;

// Entries per short chunk: about kChunksPerWarp chunks per warp of the reduce grid.
__host__ __device__ inline int64_t chunk_size(int64_t n, int warps) {
    const int64_t parts = (int64_t)kChunksPerWarp * warps;
    const int64_t per = (n + parts - 1) / parts;
    const int64_t k = (per + 7) / 8 * 8;
    return k < kMinChunk ? kMinChunk : (k > kMaxChunk ? kMaxChunk : k);
}

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct Workspace {
    int32_t* keys[2];
    int32_t* vals[2];
    uint32_t* block_hist;
    uint32_t* digit_tot;
    int32_t* seg_begin;
    int32_t* chunk_lo;  // [max_chunks] short entries of each chunk: [chunk_lo, chunk_hi)
    int32_t* chunk_hi;
    int32_t* long_seg;    // [max_chunks] slots whose segments are split by columns
    int32_t* medium_seg;  // [max_chunks] slots whose segments are short jobs of their own
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
    const int64_t max_chunks = N / kMinChunk + 2;
    w.chunk_lo = reinterpret_cast<int32_t*>(take(4 * max_chunks));
    w.chunk_hi = reinterpret_cast<int32_t*>(take(4 * max_chunks));
    w.long_seg = reinterpret_cast<int32_t*>(take(4 * max_chunks));
    w.medium_seg = reinterpret_cast<int32_t*>(take(4 * max_chunks));
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
        counters[kCntLongNext] = 0;
        counters[kCntLong] = 0;
        counters[kCntChunks] = 0;
        counters[kCntShortNext] = 0;
        counters[kCntMedium] = 0;
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
// Warp w of the block owns the tile's entries [w*512, (w+1)*512) (sub-tile s,
// lane l -> entry w*512 + 32*s + l), so an entry's rank is: the block's offset
// for its digit, plus the counts of that digit in the earlier warps, plus the
// warp's running count before this sub-tile, plus its rank among the lanes of
// this sub-tile with the same digit (found with one ballot per digit bit).  The running counts are kept per warp in
// shared memory without block barriers; one scan over the warps per digit
// follows the whole tile.
__global__ void __launch_bounds__(kRsThreads) k_rs_scatter(const int32_t* __restrict__ keys_in,
                                                           const int32_t* __restrict__ vals_in, const int32_t* n_dev,
                                                           int64_t n_static, int shift,
                                                           const uint32_t* __restrict__ block_off,
                                                           const uint32_t* __restrict__ digit_tot, int nblk,
                                                           int32_t* __restrict__ keys_out,
                                                           int32_t* __restrict__ vals_out, int32_t* total_out) {
    __shared__ uint32_t wcnt[kRsWarps][256];
    __shared__ uint32_t run[256];
    __shared__ uint32_t wsum[32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n = n_dev ? (int64_t)*n_dev : n_static;
    const int64_t wbase = (int64_t)blockIdx.x * kRsTile + (int64_t)warp * (kRsItems * 32);
    int32_t kr[kRsItems], vr[kRsItems];
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int64_t i = wbase + 32 * sub + lane;
        kr[sub] = i < n ? __ldg(keys_in + i) : -1;
        vr[sub] = vals_in ? (i < n ? __ldg(vals_in + i) : 0) : (int32_t)i;
    }
#pragma unroll
    for (int w = 0; w < kRsWarps; w++) wcnt[w][tid] = 0;  // kRsThreads == 256 digits
    {
        const uint32_t dt = digit_tot[tid];
        uint32_t tot;
        const uint32_t base = block_exclusive_scan(dt, wsum, &tot);  // contains a barrier
        run[tid] = base + block_off[(int64_t)tid * nblk + blockIdx.x];
        if (total_out && blockIdx.x == 0 && tid == 0) *total_out = (int32_t)tot;
    }
    const unsigned lt = (1u << lane) - 1u;
    uint32_t* cnt = wcnt[warp];
    uint32_t lrank[kRsItems];
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int32_t key = kr[sub];
        const bool valid = key >= 0;
        const int digit = (key >> shift) & 255;
        // lanes holding the same digit: one ballot per digit bit (invalid lanes match no one)
        unsigned peers = __ballot_sync(kFull, valid);
#pragma unroll
        for (int b = 0; b < 8; b++) {
            const unsigned m = __ballot_sync(kFull, (digit >> b) & 1);
            peers &= ((digit >> b) & 1) ? m : ~m;
        }
        const uint32_t rank = (uint32_t)__popc(peers & lt);
        const uint32_t before = valid ? cnt[digit] : 0u;
        __syncwarp();
        if (valid && rank == 0) cnt[digit] = before + (uint32_t)__popc(peers);
        __syncwarp();
        lrank[sub] = before + rank;
    }
    __syncthreads();
    {
        uint32_t acc = run[tid];
#pragma unroll
        for (int w = 0; w < kRsWarps; w++) {
            const uint32_t c = wcnt[w][tid];
            wcnt[w][tid] = acc;
            acc += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int sub = 0; sub < kRsItems; sub++) {
        const int32_t key = kr[sub];
        if (key >= 0) {
            const uint32_t pos = cnt[(key >> shift) & 255] + lrank[sub];
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

// Division of flat indices (< 2^31) by n_heads (<= 32) as a multiply and shift:
// with s = 32 + ceil(log2 d) and m = ceil(2^s / d) < 2^33, (x*m) >> s == x / d
// for every x < 2^s / d, which covers x < 2^32, and x*m stays below 2^64.
struct HeadDiv {
    uint64_t m;
    int s;
};

inline HeadDiv head_div(int d) {
    int lg = 0;
    while ((1 << lg) < d) lg++;
    const int s = 32 + lg;
    return {((1ULL << s) + (uint64_t)d - 1) / (uint64_t)d, s};
}

// Offset, in 16-byte units, of the upstream-gradient row of flat entry
// i = t*n_heads + h: CONCAT row i; PAIRSUM row t, group h % hpn (n_heads == 2*hpn).
struct GradRows {
    int dim, n_heads, hpn;
    HeadDiv hd;
    template <int MODE>
    __device__ __forceinline__ uint32_t off16(uint32_t i) const {
        if (MODE == ENGRAM_MODE_CONCAT_F32) return (uint32_t)(((uint64_t)i * (uint32_t)dim) >> 2);
        const uint32_t t = (uint32_t)(((uint64_t)i * hd.m) >> hd.s);
        const uint32_t h = i - t * (uint32_t)n_heads;
        const uint32_t r = h >= (uint32_t)hpn ? h - (uint32_t)hpn : h;
        return (uint32_t)(((uint64_t)(t * (uint32_t)hpn + r) * (uint32_t)dim) >> 3);
    }
};

// First segment start at or after sorted entry e (e in [0, n]).
__device__ __forceinline__ int64_t snap_to_segment(const int32_t* __restrict__ keys,
                                                   const int32_t* __restrict__ seg_begin, int64_t e, int64_t n) {
    if (e <= 0) return 0;
    if (e >= n) return n;
    const int32_t k = __ldg(keys + e);
    if (__ldg(keys + e - 1) != k) return e;
    return __ldg(seg_begin + k + 1);
}

// Where the row gradient of slot s is written: the dense [R, dim] array, or
// (data-parallel ranks over peer memory) the receive buffer of the rank that
// owns s.  Owners hold contiguous near-equal shards (the first R % world ranks
// one row more); owner o's buffer is [world, size_o, dim] and this rank writes
// block `rank` of it, so the owner finds every rank's partial row gradients in
// its own memory.
struct RowDst {
    float* dense;
    float* const* owners;  // device array [world] of receive buffers, or null
    int64_t R;
    int world, rank;
    __device__ __forceinline__ float* row(int64_t s, int dim) const {
        if (!owners) return dense + s * dim;
        const int64_t base = R / world, extra = R % world, big = extra * (base + 1);
        int64_t o, lo, size;
        if (s < big) {
            o = s / (base + 1);
            lo = o * (base + 1);
            size = base + 1;
        } else {
            o = extra + (s - big) / base;
            lo = big + (o - extra) * base;
            size = base;
        }
        return owners[o] + ((int64_t)rank * size + (s - lo)) * dim;
    }
};

// Work split of the segmented reduction.  With K = the chunk size chosen from
// the hit count, chunk j spans [first segment start >= j*K, first segment
// start >= (j+1)*K).  A segment longer than K can only sit at a chunk's head or
// tail (one strictly inside would be shorter than K), so trimming those gives
// the chunk's short entries [chunk_lo[j], chunk_hi[j]); each trimmed segment
// is listed once, by the chunk that holds it: in long_seg[] when it is longer
// than max(K, kLongRows) (split by columns), else in medium_seg[] (a short job
// of its own).
__global__ void k_chunks(const int32_t* __restrict__ keys, const int32_t* __restrict__ seg_begin, int32_t* counters,
                         int warps, int32_t* __restrict__ chunk_lo, int32_t* __restrict__ chunk_hi,
                         int32_t* __restrict__ long_seg, int32_t* __restrict__ medium_seg) {
    const int64_t n = counters[kCntHits];
    const int64_t K = chunk_size(n, warps);
    const int64_t TL = K > kLongRows ? K : kLongRows;
    const int64_t nchunks = (n + K - 1) / K;
    if (blockIdx.x == 0 && threadIdx.x == 0) counters[kCntChunks] = (int32_t)nchunks;
    auto list = [&](int32_t k, int64_t len) {
        if (len > TL) long_seg[atomicAdd(counters + kCntLong, 1)] = k;
        else medium_seg[atomicAdd(counters + kCntMedium, 1)] = k;
    };
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < nchunks; j += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = snap_to_segment(keys, seg_begin, j * K, n);
        int64_t hi = snap_to_segment(keys, seg_begin, (j + 1) * K, n);
        if (lo < hi) {  // head segment (it starts at lo)
            const int32_t k = __ldg(keys + lo);
            const int64_t end = __ldg(seg_begin + k + 1);
            if (end - lo > K) {
                list(k, end - lo);
                lo = end;
            }
        }
        if (lo < hi) {  // tail segment (it ends at hi)
            const int32_t k = __ldg(keys + hi - 1);
            const int64_t begin = __ldg(seg_begin + k);
            if (hi - begin > K) {
                list(k, hi - begin);
                hi = begin;
            }
        }
        chunk_lo[j] = (int32_t)lo;
        chunk_hi[j] = (int32_t)(hi > lo ? hi : lo);
    }
}

template <bool F32>
__device__ __forceinline__ void add_vec16(float2* acc, const uint4 w) {
    if (F32) {
        acc[0] = __fadd2_rn(acc[0], make_float2(__uint_as_float(w.x), __uint_as_float(w.y)));
        acc[1] = __fadd2_rn(acc[1], make_float2(__uint_as_float(w.z), __uint_as_float(w.w)));
    } else {
        acc[0] = __fadd2_rn(acc[0], make_float2(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u)));
        acc[1] = __fadd2_rn(acc[1], make_float2(__uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u)));
        acc[2] = __fadd2_rn(acc[2], make_float2(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u)));
        acc[3] = __fadd2_rn(acc[3], make_float2(__uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u)));
    }
}

// The short jobs (medium segments first, then the short chunks) as one
// continuous row stream per warp.  Jobs are taken from an atomic counter while
// the stream's 32-row metadata windows are fetched, two windows ahead of the
// adds, so the ring never drains between jobs.  Lane l owns the 16-byte column
// vectors l, l+32, ... (NV of them) of every row: it copies exactly those
// bytes into its part of the ring and adds exactly those, so the ring needs no
// cross-lane synchronisation.  D rows are in flight, committed in batches of U.
// Every job is a run of whole segments, so a segment ends where its key
// changes or its job ends, and the warp then writes the slot's row.
template <int MODE, int NV>
__device__ __forceinline__ void reduce_stream(uint8_t* __restrict__ ring, const int lane,
                                              const int32_t* __restrict__ keys, const int32_t* __restrict__ vals,
                                              const int32_t* __restrict__ seg_begin,
                                              const int32_t* __restrict__ chunk_lo,
                                              const int32_t* __restrict__ chunk_hi,
                                              const int32_t* __restrict__ medium_seg, int32_t* counters,
                                              const int64_t n_medium, const int64_t n_jobs, const GradRows& G,
                                              const uint4* __restrict__ g16, const RowDst& out) {
    using RG = ShortRing<NV>;
    constexpr int D = RG::D, U = RG::U, GI = RG::GI, ROWS = RG::ROWS;
    constexpr bool F32 = MODE == ENGRAM_MODE_CONCAT_F32;
    constexpr int CPV = F32 ? 4 : 8;  // columns per 16-byte vector
    const int dim = G.dim;
    const int nvec = dim / CPV;
    auto slot = [&](int s, int q) { return ring + (s * NV + q) * 512 + lane * 16; };
    // job cursor (warp-uniform): entries [jlo, jhi) of the current job not yet in a window
    int64_t jlo = 0, jhi = 0;
    bool exhausted = false;
    auto next_job = [&]() {
        while (true) {
            int j = 0;
            if (lane == 0) j = atomicAdd(counters + kCntShortNext, 1);
            j = __shfl_sync(kFull, j, 0);
            if (j >= n_jobs) return false;
            int64_t lo, hi;
            if (j < n_medium) {
                const int32_t key = __ldg(medium_seg + j);
                lo = __ldg(seg_begin + key);
                hi = __ldg(seg_begin + key + 1);
            } else {
                lo = __ldg(chunk_lo + (j - n_medium));
                hi = __ldg(chunk_hi + (j - n_medium));
            }
            if (lo < hi) {
                jlo = lo;
                jhi = hi;
                return true;
            }
        }
    };
    // maps the next 32 stream rows to entries (taking jobs as needed); returns how many it mapped
    auto fetch = [&](int32_t& k, int32_t& kn, int32_t& v) {
        k = -1;
        kn = -1;
        v = 0;
        int filled = 0;
        while (filled < 32) {
            if (jlo >= jhi) {
                if (exhausted || !next_job()) {
                    exhausted = true;
                    break;
                }
            }
            const int64_t avail = jhi - jlo;
            const int take = avail < 32 - filled ? (int)avail : 32 - filled;
            if (lane >= filled && lane < filled + take) {
                const int64_t e = jlo + (lane - filled);
                k = __ldg(keys + e);
                v = __ldg(vals + e);
                if (e + 1 < jhi) kn = __ldg(keys + e + 1);
            }
            filled += take;
            jlo += take;
        }
        return filled;
    };
    auto finish = [&](int32_t k, int32_t kn, int32_t v, uint32_t& off, int32_t& key, unsigned& last) {
        off = k >= 0 ? G.off16<MODE>((uint32_t)v) : 0u;
        key = k;
        last = __ballot_sync(kFull, k >= 0 && k != kn);
    };
    // A = window being added, B = the next one, C = raw loads of the one after;
    // `end` = stream length, known once a window comes back short
    uint32_t offA, offB;
    int32_t keyA, keyB, ck, ckn, cv;
    unsigned lastA, lastB;
    int end = INT_MAX;
    {
        int32_t k0, kn0, v0, k1, kn1, v1;
        int f = fetch(k0, kn0, v0);
        if (f < 32) end = f;
        f = fetch(k1, kn1, v1);
        if (f < 32 && end == INT_MAX) end = 32 + f;
        f = fetch(ck, ckn, cv);
        if (f < 32 && end == INT_MAX) end = 64 + f;
        finish(k0, kn0, v0, offA, keyA, lastA);
        finish(k1, kn1, v1, offB, keyB, lastB);
    }
    if (end == 0) return;
    auto issue = [&](int y, uint32_t off_src, int s) {  // stream row y into ring row s
        const uint32_t o = __shfl_sync(kFull, off_src, y & 31);
        if (y < end) {
#pragma unroll
            for (int q = 0; q < NV; q++)
                if (lane + 32 * q < nvec) cp_async16(slot(s, q), g16 + o + lane + 32 * q);
        }
    };
#pragma unroll 1
    for (int b = 0; b < GI; b++) {  // rows 0 .. D-1, all in window A
#pragma unroll
        for (int u = 0; u < U; u++) issue(b * U + u, offA, b * U + u);
        cp_async_commit();
    }
    float2 acc[NV][CPV / 2];
#pragma unroll
    for (int q = 0; q < NV; q++)
#pragma unroll
        for (int i = 0; i < CPV / 2; i++) acc[q][i] = make_float2(0.f, 0.f);
    int cs = 0, is = D;  // ring rows of the batch added / issued
#pragma unroll 1
    for (int x0 = 0; x0 < end; x0 += U) {
        if (x0 > 0 && (x0 & 31) == 0) {
            offA = offB;
            keyA = keyB;
            lastA = lastB;
            finish(ck, ckn, cv, offB, keyB, lastB);
            const int f = fetch(ck, ckn, cv);
            if (f < 32 && end == INT_MAX) end = x0 + 64 + f;
        }
        cp_async_wait<GI - 1>();
        uint4 v[U][NV];
#pragma unroll
        for (int u = 0; u < U; u++)
#pragma unroll
            for (int q = 0; q < NV; q++)
                v[u][q] = (x0 + u < end && lane + 32 * q < nvec) ? *reinterpret_cast<const uint4*>(slot(cs + u, q))
                                                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (x0 + u < end) {
#pragma unroll
                for (int q = 0; q < NV; q++) add_vec16<F32>(acc[q], v[u][q]);
                const int rr = (x0 + u) & 31;
                if ((lastA >> rr) & 1u) {  // the row ends its segment: write the slot's gradient row
                    const int32_t key = __shfl_sync(kFull, keyA, rr);
                    float* dst = out.row(key, dim);
#pragma unroll
                    for (int q = 0; q < NV; q++) {
                        if (lane + 32 * q < nvec) {
                            float4* d4 = reinterpret_cast<float4*>(dst + (lane + 32 * q) * CPV);
#pragma unroll
                            for (int i = 0; i < CPV / 4; i++)
                                d4[i] = make_float4(acc[q][2 * i].x, acc[q][2 * i].y, acc[q][2 * i + 1].x,
                                                    acc[q][2 * i + 1].y);
                        }
#pragma unroll
                        for (int i = 0; i < CPV / 2; i++) acc[q][i] = make_float2(0.f, 0.f);
                    }
                }
            }
        }
        __syncwarp();  // the ring rows refilled below were read in the previous batch
        const int y0 = x0 + D;
        const uint32_t osrc = ((y0 >> 5) != (x0 >> 5)) ? offB : offA;
#pragma unroll
        for (int u = 0; u < U; u++) issue(y0 + u, osrc, is + u);
        cp_async_commit();
        cs += U;
        if (cs == ROWS) cs = 0;
        is += U;
        if (is == ROWS) is = 0;
    }
    cp_async_wait<0>();
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}

// One kSliceBytes column slice of one long segment [a, b) (slot `key`), by one
// warp.  Lane l copies the slice of rows 32g+l (group g); lane w < words adds
// 4-byte word w of every row in order.  kLongGI groups are in flight; the flat
// indices of the rows travel through a per-lane shared-memory queue filled by
// cp.async 2*kLongGI groups ahead, so no load latency sits on the issue path.
template <int MODE>
__device__ __forceinline__ void reduce_long(uint8_t* __restrict__ ws, const int lane, const int64_t a, const int64_t b,
                                            const int32_t key, const int slice, const int32_t* __restrict__ vals,
                                            const GradRows& G, const uint4* __restrict__ g16, const RowDst& out) {
    const int dim = G.dim;
    constexpr bool F32 = MODE == ENGRAM_MODE_CONCAT_F32;
    constexpr int GI = kLongGI, RG = kLongRingGroups, VS = kLongValSlots, SB = kSliceBytes;
    uint8_t* ring = ws;
    int32_t* vq = reinterpret_cast<int32_t*>(ws + RG * 32 * SB);
    const int row_bytes = F32 ? dim * 4 : dim * 2;
    const int p0 = slice * (SB / 16);
    const int np = min(SB / 16, row_bytes / 16 - p0);  // 16-byte pieces in this slice
    const int words = np * 4;
    const int n = (int)(b - a);
    const int ngroups = (n + 31) >> 5;
    auto load_val = [&](int g) {
        if (32 * g + lane < n) cp_async4(vq + (g % VS) * 32 + lane, vals + a + 32LL * g + lane);
    };
    auto issue_rows = [&](int g) {
        if (32 * g + lane < n) {
            const uint32_t o = G.off16<MODE>((uint32_t)vq[(g % VS) * 32 + lane]);
            uint8_t* dst = ring + ((g % RG) * 32 + lane) * SB;
            for (int p = 0; p < np; p++) cp_async16(dst + p * 16, g16 + o + p0 + p);
        }
    };
#pragma unroll 1
    for (int g = 0; g < 2 * GI; g++) load_val(g);
    cp_async_commit();
    cp_async_wait<0>();
#pragma unroll 1
    for (int g = 0; g < GI; g++) {
        issue_rows(g);
        cp_async_commit();
    }
    float2 acc = make_float2(0.f, 0.f);
    float accf = 0.f;
#pragma unroll 1
    for (int it = 0; it < ngroups; it++) {
        cp_async_wait<GI - 1>();
        __syncwarp();  // other lanes' copies of group it are visible; group it-1's ring rows are free
        // refill group it-1's ring rows first, so the copies' address arithmetic overlaps the adds
        issue_rows(it + GI);
        load_val(it + 2 * GI);
        cp_async_commit();
        const uint8_t* gp = ring + (it % RG) * 32 * SB + lane * 4;
        const int nr = min(32, n - 32 * it);
        if (lane < words) {
            if (nr == 32) {
                uint32_t w[32];
#pragma unroll
                for (int u = 0; u < 32; u++) w[u] = *reinterpret_cast<const uint32_t*>(gp + u * SB);
#pragma unroll
                for (int u = 0; u < 32; u++) {
                    if (F32) accf = __fadd_rn(accf, __uint_as_float(w[u]));
                    else acc = __fadd2_rn(acc, make_float2(__uint_as_float(w[u] << 16), __uint_as_float(w[u] & 0xffff0000u)));
                }
            } else {
#pragma unroll 1
                for (int r = 0; r < nr; r++) {
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(gp + r * SB);
                    if (F32) accf = __fadd_rn(accf, __uint_as_float(w));
                    else acc = __fadd2_rn(acc, make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)));
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncwarp();
    if (lane < words) {
        const int word = p0 * 4 + lane;
        if (F32) out.row(key, dim)[word] = accf;
        else reinterpret_cast<float2*>(out.row(key, dim))[word] = acc;
    }
}

// Segmented reduction over the slot-sorted entries.  Every warp first takes
// column slices of the long segments (an atomic counter), so the longest
// sequential chains start at once; then it joins the short jobs (medium
// segments first, then the short chunks) as one row stream.  Slots without
// entries get zero rows.  NV = 16-byte column vectors per lane in short jobs
// (row bytes <= 512*NV).
template <int MODE, int NV>
__global__ void __launch_bounds__(kRedWarps * 32) k_reduce(const int32_t* __restrict__ keys,
                                                           const int32_t* __restrict__ vals,
                                                           const int32_t* __restrict__ seg_begin,
                                                           const int32_t* __restrict__ chunk_lo,
                                                           const int32_t* __restrict__ chunk_hi,
                                                           const int32_t* __restrict__ long_seg,
                                                           const int32_t* __restrict__ medium_seg,
                                                           int32_t* counters, int64_t R, const GradRows G,
                                                           const uint8_t* __restrict__ grad, const RowDst out) {
    constexpr int ES = MODE == ENGRAM_MODE_CONCAT_F32 ? 4 : 2;
    const int dim = G.dim;
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t* ws = smem + warp * kWarpSmem;
    const uint4* g16 = reinterpret_cast<const uint4*>(grad);
    const int n_slices = (dim * ES + kSliceBytes - 1) / kSliceBytes;
    const int64_t n_long_jobs = (int64_t)counters[kCntLong] * n_slices;
    while (true) {
        int j = 0;
        if (lane == 0) j = atomicAdd(counters + kCntLongNext, 1);
        j = __shfl_sync(kFull, j, 0);
        if (j >= n_long_jobs) break;
        const int32_t key = __ldg(long_seg + j / n_slices);
        reduce_long<MODE>(ws, lane, __ldg(seg_begin + key), __ldg(seg_begin + key + 1), key, j % n_slices, vals, G,
                          g16, out);
        __syncwarp();  // the short stream lays the ring out differently
    }
    const int64_t n_medium = counters[kCntMedium];
    const int64_t n_jobs = n_medium + counters[kCntChunks];
    reduce_stream<MODE, NV>(ws, lane, keys, vals, seg_begin, chunk_lo, chunk_hi, medium_seg, counters, n_medium,
                            n_jobs, G, g16, out);
    // slots without entries
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t s = warp0; s < R; s += nwarps) {
        if (__ldg(seg_begin + s) == __ldg(seg_begin + s + 1)) {
            float4* dst = reinterpret_cast<float4*>(out.row(s, dim));
            for (int c = lane; c < (dim >> 2); c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// Blocks of `kernel` that fit at once on one SM (set-up on first use per device).
template <typename F>
int blocks_per_sm(F kernel, int threads, int smem, int* cache) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 1;
    if (cache[dev] == 0) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, smem) != cudaSuccess || b < 1) b = 1;
        cache[dev] = b;
    }
    return cache[dev];
}

int grid_for(int64_t work, int threads, int per_sm);

template <int MODE, int NV>
void launch_reduce(const Workspace& w, const int32_t* keys, const int32_t* vals, int64_t N, int64_t R, int dim,
                   int n_heads, int hpn, const void* grad, const RowDst& out, cudaStream_t s) {
    static int per_sm[64] = {0};
    const int grid = sm_count() * blocks_per_sm(k_reduce<MODE, NV>, kRedWarps * 32, kRedSmem, per_sm);
    k_chunks<<<grid_for(N / kMinChunk + 2, 256, 4), 256, 0, s>>>(keys, w.seg_begin, w.counters, grid * kRedWarps,
                                                                   w.chunk_lo, w.chunk_hi, w.long_seg, w.medium_seg);
    k_reduce<MODE, NV><<<grid, kRedWarps * 32, kRedSmem, s>>>(keys, vals, w.seg_begin, w.chunk_lo, w.chunk_hi,
                                                               w.long_seg, w.medium_seg, w.counters, R,
                                                               GradRows{dim, n_heads, hpn, head_div(n_heads)},
                                                               static_cast<const uint8_t*>(grad), out);
}

int grid_for(int64_t work, int threads, int per_sm) {
    const int64_t want = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int64_t g = want < cap ? want : cap;
    return (int)(g > 0 ? g : 1);
}

}  // namespace

extern "C" int64_t engram_backward_workspace_bytes(int64_t n, int32_t n_heads, int64_t R) {
    if (n < 0 || n_heads < 1 || R < 0) return ENGRAM_ERR_ARG;
    return layout(nullptr, n * n_heads, R).bytes;
}

namespace {

__global__ void k_zero_rows(RowDst out, int64_t R, int dim) {
    const int64_t q = dim >> 2, total = R * q;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x)
        reinterpret_cast<float4*>(out.row(k / q, dim))[k % q] = make_float4(0.f, 0.f, 0.f, 0.f);
}

int backward_impl(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram, int32_t mode,
                  const void* grad, int32_t dim, int64_t R, const RowDst& out, void* workspace,
                  int64_t workspace_bytes, void* stream) {
    if (n < 0 || R < 0 || n_heads < 1 || n_heads > ENGRAM_MAX_HEADS || heads_per_ngram < 1) return ENGRAM_ERR_ARG;
    if (mode != ENGRAM_MODE_CONCAT_F32 && mode != ENGRAM_MODE_PAIRSUM_ADD_BF16) return ENGRAM_ERR_ARG;
    if (dim <= 0 || dim > 1024 || (mode == ENGRAM_MODE_CONCAT_F32 ? dim % 4 : dim % 8)) return ENGRAM_ERR_FORMAT;
    if (mode == ENGRAM_MODE_PAIRSUM_ADD_BF16 && n_heads != 2 * heads_per_ngram) return ENGRAM_ERR_FORMAT;
    if (R >= (1LL << 24) || n * n_heads >= (1LL << 31)) return ENGRAM_ERR_RANGE;
    const int64_t grad_bytes = mode == ENGRAM_MODE_CONCAT_F32 ? n * n_heads * (int64_t)dim * 4
                                                              : n * (int64_t)heads_per_ngram * dim * 2;
    if ((grad_bytes >> 4) >= (1LL << 32)) return ENGRAM_ERR_RANGE;
    if (R == 0) return ENGRAM_OK;
    if (out.owners ? (out.world < 1 || out.rank < 0 || out.rank >= out.world)
                   : (!out.dense || !aligned16(out.dense)))
        return ENGRAM_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) {
        k_zero_rows<<<grid_for(R * (dim >> 2), 256, 8), 256, 0, s>>>(out, R, dim);
        count_launches(1);
        return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
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
    const int nvec = mode == ENGRAM_MODE_CONCAT_F32 ? dim / 4 : dim / 8;  // 16-byte column vectors per row
    const int32_t* K = w.keys[cur];
    const int32_t* V = w.vals[cur];
    const int hpn = heads_per_ngram;
    if (mode == ENGRAM_MODE_CONCAT_F32) {
        if (nvec <= 32) launch_reduce<ENGRAM_MODE_CONCAT_F32, 1>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
        else if (nvec <= 64) launch_reduce<ENGRAM_MODE_CONCAT_F32, 2>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
        else if (nvec <= 128) launch_reduce<ENGRAM_MODE_CONCAT_F32, 4>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
        else launch_reduce<ENGRAM_MODE_CONCAT_F32, 8>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
    } else {
        if (nvec <= 32) launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 1>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
        else if (nvec <= 64) launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 2>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
        else launch_reduce<ENGRAM_MODE_PAIRSUM_ADD_BF16, 4>(w, K, V, N, R, dim, n_heads, hpn, grad, out, s);
    }
    count_launches(3 * passes + 3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

}  // namespace

extern "C" int engram_backward(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                               int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                               void* workspace, int64_t workspace_bytes, void* stream) {
    return backward_impl(slots, n, n_heads, heads_per_ngram, mode, grad, dim, R, RowDst{grad_rows, nullptr, R, 1, 0},
                         workspace, workspace_bytes, stream);
}

extern "C" int engram_backward_to_owners(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                                         int32_t mode, const void* grad, int32_t dim, int64_t R,
                                         const void* owner_bufs, int32_t world, int32_t rank, void* workspace,
                                         int64_t workspace_bytes, void* stream) {
    if (!owner_bufs) return ENGRAM_ERR_ARG;
    return backward_impl(slots, n, n_heads, heads_per_ngram, mode, grad, dim, R,
                         RowDst{nullptr, static_cast<float* const*>(owner_bufs), R, world, rank}, workspace,
                         workspace_bytes, stream);
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
