// engram_stage.cu -- push staging of a row-sharded table (owner(g) = g mod W,
// local row g / W) across the GPUs of one box, the rows moving as NVLink stores.
//
// Each rank's stage buffer holds every row its next forward reads, grouped by
// owner: block o is the rows rank o owns, in (output row, head) order.  So an
// owner writes each requester's block as one contiguous run -- full-width
// stores over NVLink -- and the forward reads the stage through a row index
// (engram_forward_indirect).  Per batch:
//   requester (engram_stage_plan, local): hash its output rows; count, per
//     owner and per 32-row tile, the heads the owner serves; exclusive scan
//     over (owner, tile) -> plan[o * (tiles + 1) + t] = index in the stage of
//     the first row of tile t served by o (plan[o * (tiles + 1) + tiles] = end
//     of block o); row_index[i * nh + h] = the stage index of head h of row i;
//   owner (engram_stage_push, after a barrier): for every requester r (itself
//     included) and every tile of r's batch, hash the tile from r's tokens,
//     list the rows it owns in the same order, and copy them from its shard to
//     stage_r + plan_r[o][t] rows.
// Both sides enumerate a tile's rows in the same order (row i ascending, then
// head h ascending), so they agree on every index without exchanging it.
#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kStageMaxWorld = 16;  // owners packed as 4-bit fields
constexpr int kPlanWarps = 8;
constexpr int kPushWarps = 8;
constexpr int kPushLoads = 8;

struct Owners {
    uint32_t world;
    int wshift;  // log2(world) for a power of two, else -1
    __device__ __forceinline__ void of(int32_t g, uint32_t& o, uint32_t& l) const {
        if (wshift >= 0) {
            o = (uint32_t)g & (world - 1u);
            l = (uint32_t)g >> wshift;
        } else {
            l = (uint32_t)g / world;
            o = (uint32_t)g - l * world;
        }
    }
};

Owners owners_for(int world) {
    return Owners{(uint32_t)world, (world & (world - 1)) == 0 ? __builtin_ctz((unsigned)world) : -1};
}

// Tokens and segment starts possibly in another GPU's memory: plain loads
// through L2, not the read-only path.
__device__ __forceinline__ TokCtx load_ctx_cg(const engram_table& T, const int32_t* tokens, const int32_t* seg_start,
                                              int64_t t) {
    TokCtx c;
    c.lo = seg_start ? __ldcg(seg_start + t) : 0;
#pragma unroll
    for (int s = 0; s < ENGRAM_MAX_CTX; s++) c.x[s] = (s < T.ngram_size && t - s >= 0) ? __ldcg(tokens + t - s) : 0;
    return c;
}

// Owner of each head of output row i, 4 bits per head (heads 0..15 in lo, 16..31 in hi).
__device__ __forceinline__ void head_owners(const engram_table& T, const HeadTab& H, const TokCtx& c, int64_t t,
                                            const Owners& ow,
                                            unsigned long long& lo, unsigned long long& hi) {
    lo = hi = 0ull;
    for (int h = 0; h < T.n_heads; h++) {
        uint32_t o, l;
        ow.of(hash_ctx(T, H, c, t, h), o, l);
        if (h < 16) lo |= (unsigned long long)o << (4 * h);
        else hi |= (unsigned long long)o << (4 * (h - 16));
    }
}

__device__ __forceinline__ unsigned owned_mask(unsigned long long lo, unsigned long long hi, int nh, uint32_t o) {
    unsigned m = 0;
    for (int h = 0; h < nh; h++) {
        const uint32_t x = (uint32_t)((h < 16 ? lo >> (4 * h) : hi >> (4 * (h - 16))) & 15ull);
        if (x == o) m |= 1u << h;
    }
    return m;
}

__device__ __forceinline__ int warp_exclusive(int v, int lane, int& total) {
    int x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(kFull, x, d);
        if (lane >= d) x += y;
    }
    total = __shfl_sync(kFull, x, 31);
    return x - v;
}

// Per (owner, tile): heads of the tile served by the owner.  One warp per tile.
__global__ void __launch_bounds__(kPlanWarps * 32) k_plan_count(engram_table T, const int32_t* __restrict__ tokens,
                                                                const int32_t* __restrict__ seg_start, int64_t t0,
                                                                int64_t n, Owners ow, int64_t tiles,
                                                                int32_t* __restrict__ plan) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t tile = (int64_t)blockIdx.x * kPlanWarps + warp; tile < tiles;
         tile += (int64_t)gridDim.x * kPlanWarps) {
        const int64_t i = tile * 32 + lane;
        unsigned long long lo = 0, hi = 0;
        if (i < n) head_owners(T, htab, load_ctx(T, tokens, seg_start, t0 + i), t0 + i, ow, lo, hi);
        for (uint32_t o = 0; o < ow.world; o++) {
            const unsigned m = i < n ? owned_mask(lo, hi, T.n_heads, o) : 0u;
            int c = __popc(m);
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) c += __shfl_xor_sync(kFull, c, d);
            if (lane == 0) plan[o * (tiles + 1) + tile] = c;
        }
    }
}

// Exclusive scan of plan[0, m) in place, entries at tile index `tiles` of each
// owner counting as 0 (they receive the end of the owner's block).  One block.
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) k_plan_scan(int32_t* __restrict__ plan, int64_t m, int64_t tiles) {
    __shared__ int64_t part[kScanThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t per = (m + kScanThreads - 1) / kScanThreads;
    const int64_t lo = tid * per, hi = lo + per < m ? lo + per : m;
    auto val = [&](int64_t k) -> int64_t { return (k % (tiles + 1)) == tiles ? 0 : (int64_t)plan[k]; };
    int64_t s = 0;
    for (int64_t k = lo; k < hi; k++) s += val(k);
    int64_t x = s;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int64_t y = __shfl_up_sync(kFull, x, d);
        if (lane >= d) x += y;
    }
    if (lane == 31) part[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int64_t p = part[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int64_t y = __shfl_up_sync(kFull, p, d);
            if (lane >= d) p += y;
        }
        part[lane] = p;
    }
    __syncthreads();
    int64_t run = x - s + (warp > 0 ? part[warp - 1] : 0);
    for (int64_t k = lo; k < hi; k++) {
        const int64_t v = val(k);
        plan[k] = (int32_t)run;
        run += v;
    }
}

// row_index[i * nh + h] = stage index of head h of output row i.  One warp per tile.
__global__ void __launch_bounds__(kPlanWarps * 32) k_plan_index(engram_table T, const int32_t* __restrict__ tokens,
                                                                const int32_t* __restrict__ seg_start, int64_t t0,
                                                                int64_t n, Owners ow, int64_t tiles,
                                                                const int32_t* __restrict__ plan,
                                                                int32_t* __restrict__ row_index) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nh = T.n_heads;
    for (int64_t tile = (int64_t)blockIdx.x * kPlanWarps + warp; tile < tiles;
         tile += (int64_t)gridDim.x * kPlanWarps) {
        const int64_t i = tile * 32 + lane;
        unsigned long long lo = 0, hi = 0;
        if (i < n) head_owners(T, htab, load_ctx(T, tokens, seg_start, t0 + i), t0 + i, ow, lo, hi);
        for (uint32_t o = 0; o < ow.world; o++) {
            const unsigned m = i < n ? owned_mask(lo, hi, nh, o) : 0u;
            int total;
            const int ex = warp_exclusive(__popc(m), lane, total);
            if (total == 0) continue;
            int k = __ldg(plan + o * (tiles + 1) + tile) + ex;
            for (unsigned b = m; b; b &= b - 1) row_index[i * nh + (__ffs(b) - 1)] = k++;
        }
    }
}

// Owner side: for every requester r (this rank included) and every tile of r's
// batch, this rank's rows of the tile go to stage_r from row plan_r[rank][t]
// on, contiguously.  One warp per (requester, tile); the owned rows' local
// indices are listed in shared memory, then the warp copies 16-byte pieces,
// kPushLoads per lane in flight, consecutive lanes writing consecutive pieces.
// The next unit's tokens and plan entry load while this unit copies.
template <int PIECES>  // row_stride / 16, or 0: read from T
__global__ void __launch_bounds__(kPushWarps * 32) k_stage_push(engram_table T, const int32_t* const* toks,
                                                               const int32_t* const* segs,
                                                               const int32_t* const* plans, int64_t t0, int64_t n,
                                                               uint8_t* const* stages, Owners ow, int rank,
                                                               int first_r) {
    extern __shared__ int32_t plist[];
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nh = T.n_heads;
    int32_t* list = plist + warp * 32 * nh;
    const int pieces = PIECES > 0 ? PIECES : (int)(T.row_stride >> 4);
    const int64_t stride = T.row_stride;
    const uint8_t* shard = static_cast<const uint8_t*>(T.rows);
    const int W = (int)ow.world;
    const int64_t tiles = (n + 31) >> 5;
    const int64_t jobs = tiles * W;
    const int64_t step = (int64_t)gridDim.x * kPushWarps;
    auto ptr_of = [&](const void* arr, int r) {
        return reinterpret_cast<const void*>(__ldg(reinterpret_cast<const unsigned long long*>(arr) + r));
    };
    // requesters in the order first_r, first_r + 1, ...: ranks start on different peers
    auto decode = [&](int64_t jb, int& r, int64_t& tile) {
        const int64_t q = jb / tiles;
        r = (int)((q + first_r) % W);
        tile = jb - q * tiles;
    };
    auto load = [&](int64_t jb, TokCtx& c, int32_t& base) {
        int r;
        int64_t tile;
        decode(jb, r, tile);
        const int64_t i = tile * 32 + lane;
        if (i < n)
            c = load_ctx_cg(T, static_cast<const int32_t*>(ptr_of(toks, r)),
                            segs ? static_cast<const int32_t*>(ptr_of(segs, r)) : nullptr, t0 + i);
        base = lane == 0 ? __ldcg(static_cast<const int32_t*>(ptr_of(plans, r)) + rank * (tiles + 1) + tile) : 0;
    };
    int64_t job = (int64_t)blockIdx.x * kPushWarps + warp;
    TokCtx c{};
    int32_t base = 0;
    if (job < jobs) load(job, c, base);
    for (; job < jobs; job += step) {
        int r;
        int64_t tile;
        decode(job, r, tile);
        const int64_t i = tile * 32 + lane;
        const TokCtx cur = c;
        const int32_t cur_base = __shfl_sync(kFull, base, 0);
        if (job + step < jobs) load(job + step, c, base);
        unsigned m = 0;  // the heads of row i whose rows live here
        if (i < n)
            for (int h = 0; h < nh; h++) {
                uint32_t o, l;
                ow.of(hash_ctx(T, htab, cur, t0 + i, h), o, l);
                if ((int)o == rank) m |= 1u << h;
            }
        int total;
        int k = warp_exclusive(__popc(m), lane, total);
        for (unsigned b = m; b; b &= b - 1) {  // their local rows, in head order (the hash again: no local array)
            uint32_t o, l;
            ow.of(hash_ctx(T, htab, cur, t0 + i, __ffs(b) - 1), o, l);
            list[k++] = (int32_t)l;
        }
        __syncwarp();
        uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(ptr_of(stages, r))) + (int64_t)cur_base * stride;
        const int npieces = total * pieces;
        for (int j0 = 0; j0 < npieces; j0 += 32 * kPushLoads) {
            uint4 v[kPushLoads];
#pragma unroll
            for (int u = 0; u < kPushLoads; u++) {
                const int j = j0 + u * 32 + lane;
                if (j < npieces) {
                    const int q = j / pieces;
                    const int p = j - q * pieces;
                    v[u] = __ldg(reinterpret_cast<const uint4*>(shard + (int64_t)list[q] * stride + p * 16));
                }
            }
#pragma unroll
            for (int u = 0; u < kPushLoads; u++) {
                const int j = j0 + u * 32 + lane;
                if (j < npieces) *reinterpret_cast<uint4*>(dst + (int64_t)j * 16) = v[u];
            }
        }
        __syncwarp();  // the list is rewritten by the next unit
    }
}

int check_stage_table(const engram_table* t, int64_t t0, int64_t n, int32_t world) {
    if (!t || t0 < 0 || n < 0 || world < 1) return ENGRAM_ERR_ARG;
    if (world > kStageMaxWorld) return ENGRAM_ERR_RANGE;
    if (t->row_stride % 16 || t->n_heads < 1 || t->n_heads > 32) return ENGRAM_ERR_FORMAT;
    if (n * (int64_t)t->n_heads >= ((int64_t)1 << 31)) return ENGRAM_ERR_RANGE;
    return ENGRAM_OK;
}

}  // namespace

extern "C" int64_t engram_stage_plan_words(int64_t n, int32_t world) {
    if (n < 0 || world < 1) return ENGRAM_ERR_ARG;
    return (int64_t)world * ((n + 31) / 32 + 1);
}

extern "C" int engram_stage_plan(const engram_table* t, const int32_t* tokens, const int32_t* seg_start, int64_t t0,
                                 int64_t n, int32_t world, int32_t* plan, int32_t* row_index, void* stream) {
    const int st = check_stage_table(t, t0, n, world);
    if (st != ENGRAM_OK) return st;
    if (n == 0) return ENGRAM_OK;
    if (!tokens || !plan || !row_index) return ENGRAM_ERR_ARG;
    const Owners ow = owners_for(world);
    const int64_t tiles = (n + 31) / 32;
    const int64_t m = (int64_t)world * (tiles + 1);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t want = (tiles + kPlanWarps - 1) / kPlanWarps, cap = (int64_t)sm_count() * 8;
    const int blocks = (int)(want < cap ? want : cap);
    k_plan_count<<<blocks, kPlanWarps * 32, 0, s>>>(*t, tokens, seg_start, t0, n, ow, tiles, plan);
    k_plan_scan<<<1, kScanThreads, 0, s>>>(plan, m, tiles);
    k_plan_index<<<blocks, kPlanWarps * 32, 0, s>>>(*t, tokens, seg_start, t0, n, ow, tiles, plan, row_index);
    count_launches(3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_stage_push(const engram_table* t, const void* token_ptrs, const void* seg_ptrs,
                                 const void* plan_ptrs, int64_t t0, int64_t n, const void* stage_ptrs, int32_t world,
                                 int32_t rank, int32_t max_blocks, void* stream) {
    const int st = check_stage_table(t, t0, n, world);
    if (st != ENGRAM_OK) return st;
    if (rank < 0 || rank >= world || max_blocks < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!t->rows || !token_ptrs || !plan_ptrs || !stage_ptrs) return ENGRAM_ERR_ARG;
    const int smem = kPushWarps * 32 * t->n_heads * (int)sizeof(int32_t);
    const int64_t jobs = ((n + 31) / 32) * world;
    const int64_t want = (jobs + kPushWarps - 1) / kPushWarps;
    const int64_t cap = max_blocks > 0 ? max_blocks : (int64_t)sm_count() * 2;
    const int blocks = (int)(want < cap ? want : cap);
    cudaStream_t s = (cudaStream_t)stream;
    const Owners ow = owners_for(world);
    const auto* tk = static_cast<const int32_t* const*>(token_ptrs);
    const auto* sg = static_cast<const int32_t* const*>(seg_ptrs);
    const auto* pl = static_cast<const int32_t* const*>(plan_ptrs);
    auto* sp = static_cast<uint8_t* const*>(stage_ptrs);
    const int first = (rank + 1) % world;
    if (t->row_stride == 144) k_stage_push<9><<<blocks, kPushWarps * 32, smem, s>>>(*t, tk, sg, pl, t0, n, sp, ow, rank, first);
    else k_stage_push<0><<<blocks, kPushWarps * 32, smem, s>>>(*t, tk, sg, pl, t0, n, sp, ow, rank, first);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
