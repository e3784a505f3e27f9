// engram_rowset.cu -- sets of global table rows on the device (bitmaps).
//
// The row-set builders around the descent are set algebra over global row ids:
// build_all_read_row_set (engraft/descend_corpus.py:1409-1430) is the union of
// the rows every prefix position of every training fragment reads;
// build_rows_var (engraft/replica/distill.py:401-457) takes unions and
// differences of census row lists, minus the rows read at excluded positions,
// and returns them sorted; sum_overlays (engraft/replica/overlay_sum.py:36-112)
// needs the sorted union of the rows of several .pleo files and each file row's
// index in it.  The reference builds Python sets position by position.
//
// Here a set is a bitmap of n_rows bits (40 MB for a 320 M-row table):
//   - marking the rows read at positions hashes each (position, head) with the
//     table's constants (the same hash_row as the forward) and sets its bit;
//     a plain read first skips the atomic for bits already set (Zipf-hot rows);
//   - unions, differences and intersections are one word-wise pass;
//   - the sorted id list comes from one scan of per-word popcounts: block sums,
//     an exclusive scan of the block sums, then each block writes its ids in
//     order; the per-word exclusive prefix stays in the workspace, so the index
//     of any member in the sorted list is one popcount away (engram_rowset_index).
#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kTileWords = 2048;  // words per block in the scan (8 per thread)
constexpr int kScanThreads = 256;
constexpr int kScanItems = kTileWords / kScanThreads;
constexpr int kTopThreads = 1024;

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct RsWorkspace {
    uint32_t* word_prefix;  // [words] exclusive popcount prefix of each word
    uint32_t* tile_sum;     // [tiles + 1] popcounts per tile, then their exclusive scan
    int64_t bytes;
    int64_t tiles;
};

RsWorkspace rs_layout(void* base, int64_t words) {
    RsWorkspace w{};
    w.tiles = (words + kTileWords - 1) / kTileWords;
    char* p = static_cast<char*>(base);
    int64_t off = 0;
    auto take = [&](int64_t b) {
        char* r = p ? p + off : nullptr;
        off += align256(b);
        return r;
    };
    w.word_prefix = reinterpret_cast<uint32_t*>(take(4 * (words > 0 ? words : 1)));
    w.tile_sum = reinterpret_cast<uint32_t*>(take(4 * (w.tiles + 1)));
    w.bytes = off;
    return w;
}

__device__ __forceinline__ void set_bit(uint32_t* bitmap, int64_t g) {
    uint32_t* w = bitmap + (g >> 5);
    const uint32_t m = 1u << (g & 31);
    if ((*reinterpret_cast<volatile uint32_t*>(w) & m) == 0u) atomicOr(w, m);
}

// Rows read at positions: one thread per (position, head).
__global__ void k_mark_positions(engram_table T, const int32_t* __restrict__ tokens, int64_t n_tokens,
                                 const int32_t* __restrict__ seg_start, const int64_t* __restrict__ positions,
                                 int64_t n, uint32_t* bitmap) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total;
         k += (int64_t)gridDim.x * blockDim.x) {
        int64_t i;
        int h;
        split_pair(k, nh, i, h);
        int64_t t = positions ? __ldg(positions + i) : i;
        t = t < 0 ? 0 : (t >= n_tokens ? n_tokens - 1 : t);
        const int32_t g = hash_row(T, htab, tokens, seg_start, t, h);
        if (g >= 0 && g < T.n_rows) set_bit(bitmap, g);
    }
}

__global__ void k_mark_ids(const int32_t* __restrict__ ids, int64_t n, int64_t n_rows, uint32_t* bitmap) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const int32_t g = __ldg(ids + k);
        if (g >= 0 && g < n_rows) set_bit(bitmap, g);
    }
}

__global__ void k_combine(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, int64_t words, int op,
                          uint32_t* __restrict__ out) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < words;
         k += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t x = __ldg(a + k), y = __ldg(b + k);
        out[k] = op == 0 ? (x | y) : (op == 1 ? (x & ~y) : (x & y));
    }
}

// Exclusive scan of one value per thread over the block; *total = block sum.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
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
        if (lane < nwarps) warp_sums[lane] = s;
    }
    __syncthreads();
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    if (total) *total = warp_sums[nwarps - 1];
    const uint32_t r = before + x - v;
    __syncthreads();
    return r;
}

// Per tile: popcount sum.  Thread j covers words [tile + j*8, +8).
__global__ void __launch_bounds__(kScanThreads) k_tile_sums(const uint32_t* __restrict__ bitmap, int64_t words,
                                                            uint32_t* __restrict__ tile_sum) {
    __shared__ uint32_t ws[32];
    const int64_t w0 = (int64_t)blockIdx.x * kTileWords + (int64_t)threadIdx.x * kScanItems;
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; i++)
        if (w0 + i < words) c += (uint32_t)__popc(__ldg(bitmap + w0 + i));
    uint32_t tot;
    block_scan(c, ws, &tot);
    if (threadIdx.x == 0) tile_sum[blockIdx.x] = tot;
}

// Exclusive scan of tile_sum[0..tiles) in place (one block); tile_sum[tiles] = total.
__global__ void __launch_bounds__(kTopThreads) k_tile_scan(uint32_t* tile_sum, int64_t tiles, int64_t* count) {
    __shared__ uint32_t ws[32];
    const int64_t per = (tiles + kTopThreads - 1) / kTopThreads;
    const int64_t lo = threadIdx.x * per, hi = lo + per < tiles ? lo + per : tiles;
    uint32_t s = 0;
    for (int64_t k = lo; k < hi; k++) s += tile_sum[k];
    uint32_t tot;
    uint32_t run = block_scan(s, ws, &tot);
    for (int64_t k = lo; k < hi; k++) {
        const uint32_t x = tile_sum[k];
        tile_sum[k] = run;
        run += x;
    }
    if (threadIdx.x == 0) {
        tile_sum[tiles] = tot;
        if (count) *count = (int64_t)tot;
    }
}

// Per tile: word prefixes, and (ids_out != null) the members in ascending order,
// at most `capacity` of them.
__global__ void __launch_bounds__(kScanThreads) k_tile_write(const uint32_t* __restrict__ bitmap, int64_t words,
                                                             const uint32_t* __restrict__ tile_sum,
                                                             uint32_t* __restrict__ word_prefix,
                                                             int32_t* __restrict__ ids_out, int64_t capacity) {
    __shared__ uint32_t ws[32];
    const int64_t w0 = (int64_t)blockIdx.x * kTileWords + (int64_t)threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    uint32_t c = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        v[i] = w0 + i < words ? __ldg(bitmap + w0 + i) : 0u;
        c += (uint32_t)__popc(v[i]);
    }
    uint32_t run = tile_sum[blockIdx.x] + block_scan(c, ws, nullptr);
#pragma unroll
    for (int i = 0; i < kScanItems; i++) {
        if (w0 + i < words) {
            word_prefix[w0 + i] = run;
            if (ids_out) {
                uint32_t x = v[i];
                uint32_t pos = run;
                while (x) {
                    const int b = __ffs(x) - 1;
                    if (pos < capacity) ids_out[pos] = (int32_t)((w0 + i) * 32 + b);
                    pos++;
                    x &= x - 1;
                }
            }
            run += (uint32_t)__popc(v[i]);
        }
    }
}

// index_out[k] = position of ids[k] in the sorted member list, or -1 if it is not a member.
__global__ void k_index(const uint32_t* __restrict__ bitmap, int64_t words, const uint32_t* __restrict__ word_prefix,
                        const int32_t* __restrict__ ids, int64_t n, int32_t* __restrict__ index_out) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const int32_t g = __ldg(ids + k);
        int32_t r = -1;
        if (g >= 0 && (g >> 5) < words) {
            const uint32_t w = __ldg(bitmap + (g >> 5));
            const uint32_t m = 1u << (g & 31);
            if (w & m) r = (int32_t)(__ldg(word_prefix + (g >> 5)) + (uint32_t)__popc(w & (m - 1u)));
        }
        index_out[k] = r;
    }
}

// acc[index[k]] += data[k] - base[k], one thread per (row, column); the rows of
// one launch have distinct targets (the caller splits repeated rows into rounds).
__global__ void k_overlay_accumulate(float* __restrict__ acc, const int32_t* __restrict__ index,
                                     const float* __restrict__ data, const float* __restrict__ base, int64_t n,
                                     int dim) {
    const int64_t total = n * dim;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = e / dim;
        const int c = (int)(e - k * dim);
        const int32_t r = __ldg(index + k);
        if (r >= 0) {
            float* a = acc + (int64_t)r * dim + c;
            *a = __fadd_rn(*a, __fsub_rn(__ldg(data + e), __ldg(base + e)));
        }
    }
}

// The same with repeated targets, in one launch: order lists the rows k sorted
// by index[k], stable (ascending k among equal targets).  The thread of
// (j, c) with j the first of a run of equal targets adds the run's rows to
// column c one after another, in file order, as np.add.at applies them.
__global__ void k_overlay_accumulate_runs(float* __restrict__ acc, const int32_t* __restrict__ index,
                                          const int64_t* __restrict__ order, const float* __restrict__ data,
                                          const float* __restrict__ base, int64_t n, int dim) {
    const int64_t total = n * dim;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e / dim;
        const int c = (int)(e - j * dim);
        const int32_t r = __ldg(index + __ldg(order + j));
        if (r < 0 || (j > 0 && __ldg(index + __ldg(order + j - 1)) == r)) continue;
        float* a = acc + (int64_t)r * dim + c;
        float v = *a;
        for (int64_t q = j; q < n; q++) {
            const int64_t k = __ldg(order + q);
            if (q > j && __ldg(index + k) != r) break;
            v = __fadd_rn(v, __fsub_rn(__ldg(data + k * dim + c), __ldg(base + k * dim + c)));
        }
        *a = v;
    }
}

int grid_for(int64_t work) {
    const int64_t want = (work + 255) / 256, cap = (int64_t)sm_count() * 8;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

extern "C" int64_t engram_rowset_words(int64_t n_rows) {
    if (n_rows < 0 || n_rows > (1LL << 31)) return ENGRAM_ERR_RANGE;
    return (n_rows + 31) / 32;
}

extern "C" int engram_rowset_mark(const engram_table* t, const int32_t* tokens, int64_t n_tokens,
                                  const int32_t* seg_start, const int64_t* positions, int64_t n, uint32_t* bitmap,
                                  void* stream) {
    if (!t || n < 0 || n_tokens < 0) return ENGRAM_ERR_ARG;
    if (!positions && n > n_tokens) return ENGRAM_ERR_RANGE;
    if (n == 0) return ENGRAM_OK;
    if (!tokens || !bitmap || n_tokens == 0) return ENGRAM_ERR_ARG;
    if (n * (int64_t)t->n_heads >= (1LL << 40)) return ENGRAM_ERR_RANGE;
    k_mark_positions<<<grid_for(n * t->n_heads), 256, 0, (cudaStream_t)stream>>>(*t, tokens, n_tokens, seg_start,
                                                                                 positions, n, bitmap);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_rowset_mark_ids(const int32_t* ids, int64_t n, int64_t n_rows, uint32_t* bitmap, void* stream) {
    if (n < 0 || n_rows < 0 || n_rows > (1LL << 31)) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!ids || !bitmap) return ENGRAM_ERR_ARG;
    k_mark_ids<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(ids, n, n_rows, bitmap);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_rowset_combine(const uint32_t* a, const uint32_t* b, int64_t words, int32_t op, uint32_t* out,
                                     void* stream) {
    if (words < 0 || op < 0 || op > 2) return ENGRAM_ERR_ARG;
    if (words == 0) return ENGRAM_OK;
    if (!a || !b || !out) return ENGRAM_ERR_ARG;
    k_combine<<<grid_for(words), 256, 0, (cudaStream_t)stream>>>(a, b, words, op, out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int64_t engram_rowset_workspace_bytes(int64_t words) {
    if (words < 0) return ENGRAM_ERR_ARG;
    return rs_layout(nullptr, words).bytes;
}

extern "C" int engram_rowset_extract(const uint32_t* bitmap, int64_t words, int32_t* ids_out, int64_t capacity,
                                     int64_t* count, void* workspace, int64_t workspace_bytes, void* stream) {
    if (words < 0 || capacity < 0 || !count) return ENGRAM_ERR_ARG;
    if (words > (1LL << 26)) return ENGRAM_ERR_RANGE;  // 2^31 rows
    cudaStream_t s = (cudaStream_t)stream;
    if (words == 0) return cudaMemsetAsync(count, 0, sizeof(int64_t), s) == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
    if (!bitmap || (capacity > 0 && !ids_out)) return ENGRAM_ERR_ARG;
    RsWorkspace w = rs_layout(workspace, words);
    if (!workspace || workspace_bytes < w.bytes) return ENGRAM_ERR_WORKSPACE;
    k_tile_sums<<<(int)w.tiles, kScanThreads, 0, s>>>(bitmap, words, w.tile_sum);
    k_tile_scan<<<1, kTopThreads, 0, s>>>(w.tile_sum, w.tiles, count);
    k_tile_write<<<(int)w.tiles, kScanThreads, 0, s>>>(bitmap, words, w.tile_sum, w.word_prefix,
                                                       capacity > 0 ? ids_out : nullptr, capacity);
    count_launches(3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_rowset_index(const uint32_t* bitmap, int64_t words, const void* workspace,
                                   int64_t workspace_bytes, const int32_t* ids, int64_t n, int32_t* index_out,
                                   void* stream) {
    if (words < 0 || n < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!bitmap || !ids || !index_out || !workspace) return ENGRAM_ERR_ARG;
    RsWorkspace w = rs_layout(const_cast<void*>(workspace), words);
    if (workspace_bytes < w.bytes) return ENGRAM_ERR_WORKSPACE;
    k_index<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(bitmap, words, w.word_prefix, ids, n, index_out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_overlay_accumulate(float* acc, const int32_t* index, const int64_t* order, const float* data,
                                         const float* base, int64_t n, int32_t dim, void* stream) {
    if (n < 0 || dim <= 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!acc || !index || !data || !base) return ENGRAM_ERR_ARG;
    if (order)
        k_overlay_accumulate_runs<<<grid_for(n * dim), 256, 0, (cudaStream_t)stream>>>(acc, index, order, data, base,
                                                                                       n, dim);
    else
        k_overlay_accumulate<<<grid_for(n * dim), 256, 0, (cudaStream_t)stream>>>(acc, index, data, base, n, dim);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
