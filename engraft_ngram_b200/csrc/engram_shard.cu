// engram_shard.cu -- the row-sharded table across W GPUs (owner(id) = id mod W).
//
// Each rank keeps only the rows it owns (global id g lives on rank g % W at local
// index g / W).  Per step a rank:
//   1. hashes its positions (engram_hash) and probes the overlay;
//   2. engram_shard_requests: inserts every table row it needs (overlay hits
//      excluded) into a hash set -- one request per distinct row --, groups the
//      distinct ids by owner (send_ids, per-owner counts) and records, for every
//      (position, head), where that row will sit in the reply buffer (row_index);
//   3. exchanges ids with NCCL all-to-all-v (host code); each owner copies the
//      requested rows out of its shard with engram_shard_gather; the quantised
//      rows travel back with a second all-to-all-v;
//   4. runs the forward with row_index pointing into the received rows
//      (engram_forward_indirect).
// No kernel here reads another GPU's memory: remote rows arrive in local HBM
// through NCCL before any kernel touches them.
#include <climits>

#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr int kMaxWorld = 64;

__device__ __forceinline__ uint32_t set_home(int32_t key, int64_t capacity) { return map_home(key, capacity); }

// Exclusive scan of one value per thread over the block (blockDim a multiple of
// 32, <= 1024); *total = the block's sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < nwarps ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < nwarps) warp_sums[lane] = s;
    }
    __syncthreads();
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    *total = warp_sums[nwarps - 1];
    const uint32_t res = before + x - v;
    __syncthreads();
    return res;
}

__global__ void k_set_clear(int32_t* keys, int64_t capacity, int64_t* counts, int world) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < capacity; i += stride) keys[i] = -1;
    if (blockIdx.x == 0 && threadIdx.x < 2 * world) counts[threadIdx.x] = 0;  // counts[world] + cursors[world]
}

// Inserts the ids that the table must serve (slot < 0) into the set.
__global__ void k_set_insert(const int32_t* __restrict__ ids, const int32_t* __restrict__ slots, int64_t n,
                             int32_t* keys, int64_t capacity) {
    const uint32_t mask = (uint32_t)capacity - 1u;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += stride) {
        if (slots && slots[k] >= 0) continue;
        const int32_t g = ids[k];
        if (g < 0) continue;  // an entry the plan does not request
        uint32_t pos = set_home(g, capacity);
        for (int64_t probe = 0; probe < capacity; probe++) {
            // a plain read first: repeated ids (Zipf-hot rows) then need no atomic
            const int32_t seen = *reinterpret_cast<volatile int32_t*>(keys + pos);
            if (seen == g) break;
            if (seen == -1) {
                const int32_t prev = atomicCAS(keys + pos, -1, g);
                if (prev == -1 || prev == g) break;
            }
            pos = (pos + 1u) & mask;
        }
    }
}

// Per-owner counts of the distinct ids, aggregated per block in shared memory
// (one global atomic per owner per block; the ids of a hot table would
// otherwise serialise on W counters).
__global__ void k_owner_count(const int32_t* __restrict__ keys, int64_t capacity, int world,
                              unsigned long long* counts) {
    __shared__ unsigned int c[kMaxWorld];
    for (int o = threadIdx.x; o < world; o += blockDim.x) c[o] = 0;
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < capacity; e += stride) {
        const int32_t g = keys[e];
        if (g >= 0) atomicAdd(c + (g % world), 1u);
    }
    __syncthreads();
    for (int o = threadIdx.x; o < world; o += blockDim.x)
        if (c[o]) atomicAdd(counts + o, (unsigned long long)c[o]);
}

// send_ids grouped by owner; vals[e] = the entry's position in send_ids (= in the
// reply).  Each block reserves one range per owner, then places its entries
// inside the ranges with shared-memory counters.
__global__ void k_owner_scatter(const int32_t* __restrict__ keys, int32_t* __restrict__ vals, int64_t capacity,
                                int world, const unsigned long long* counts, unsigned long long* cursors,
                                int32_t* __restrict__ send_ids) {
    __shared__ unsigned long long off[kMaxWorld];
    __shared__ unsigned int c[kMaxWorld];
    __shared__ unsigned long long base[kMaxWorld];
    if (threadIdx.x == 0) {
        unsigned long long acc = 0;
        for (int o = 0; o < world; o++) {
            off[o] = acc;
            acc += counts[o];
        }
    }
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t e0 = (int64_t)blockIdx.x * blockDim.x; e0 < capacity; e0 += stride) {
        for (int o = threadIdx.x; o < world; o += blockDim.x) c[o] = 0;
        __syncthreads();
        const int64_t e = e0 + threadIdx.x;
        const int32_t g = e < capacity ? keys[e] : -1;
        unsigned int local = 0;
        if (g >= 0) local = atomicAdd(c + (g % world), 1u);
        __syncthreads();
        for (int o = threadIdx.x; o < world; o += blockDim.x)
            base[o] = c[o] ? off[o] + atomicAdd(cursors + o, (unsigned long long)c[o]) : 0ull;
        __syncthreads();
        if (g >= 0) {
            const unsigned long long pos = base[g % world] + local;
            send_ids[pos] = g;
            vals[e] = (int32_t)pos;
        }
        __syncthreads();
    }
}

__global__ void k_row_index(const int32_t* __restrict__ ids, const int32_t* __restrict__ slots, int64_t n,
                            const int32_t* __restrict__ keys, const int32_t* __restrict__ vals, int64_t capacity,
                            int32_t* __restrict__ row_index) {
    const uint32_t mask = (uint32_t)capacity - 1u;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += stride) {
        int32_t r = -1;
        if (!(slots && slots[k] >= 0)) {
            const int32_t g = ids[k];
            uint32_t pos = set_home(g, capacity);
            for (int64_t probe = 0; probe < capacity; probe++) {
                const int32_t key = keys[pos];
                if (key == g) {
                    r = vals[pos];
                    break;
                }
                if (key == -1) break;
                pos = (pos + 1u) & mask;
            }
        }
        row_index[k] = r;
    }
}

// The rows a rank reads from other ranks (engram_shard_plan): for each
// (position, head) of positions t0..t0+n-1, the global id when another rank
// owns it and the overlay does not serve it, else -1.  One thread per pair.
__global__ void k_plan_ids(engram_table T, engram_overlay OV, const int32_t* __restrict__ tokens,
                           const int32_t* __restrict__ seg_start, int64_t t0, int64_t n, int world, int rank,
                           int32_t* __restrict__ out) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        int64_t i;
        int h;
        split_pair(k, nh, i, h);
        const int32_t g = hash_row(T, htab, tokens, seg_start, t0 + i, h);
        const bool remote = (int)((uint32_t)g % (uint32_t)world) != rank;
        out[k] = (remote && overlay_slot(OV, g) < 0) ? g : -1;
    }
}

// row_index[k] = the position of ids[k] in send_ids (its row in the reply), or
// -1 for an entry not requested (ids[k] < 0); ids and row_index may be the same
// array (each thread reads its entry before writing it).
__global__ void k_row_index_inplace(const int32_t* ids, int64_t n, const int32_t* __restrict__ keys,
                                    const int32_t* __restrict__ vals, int64_t capacity, int32_t* row_index) {
    const uint32_t mask = (uint32_t)capacity - 1u;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += stride) {
        const int32_t g = ids[k];
        int32_t r = -1;
        if (g >= 0) {
            uint32_t pos = set_home(g, capacity);
            for (int64_t probe = 0; probe < capacity; probe++) {
                const int32_t key = keys[pos];
                if (key == g) {
                    r = vals[pos];
                    break;
                }
                if (key == -1) break;
                pos = (pos + 1u) & mask;
            }
        }
        row_index[k] = r;
    }
}

// out[k] = shard row (ids[k] / world); one thread per 16-byte word.
__global__ void k_shard_gather(const uint8_t* __restrict__ shard, int64_t stride, int64_t n_local,
                               const int32_t* __restrict__ ids, int64_t n, int world, uint8_t* __restrict__ out) {
    const int64_t words = stride >> 4;
    const int64_t total = n * words;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = w / words, p = w - k * words;
        const int64_t local = (int64_t)ids[k] / world;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (ids[k] >= 0 && local < n_local) v = __ldg(reinterpret_cast<const uint4*>(shard + local * stride) + p);
        reinterpret_cast<uint4*>(out + k * stride)[p] = v;
    }
}

// engram_shard_route: the requests of a batch grouped by owner, one per
// (position, head) served by another rank and not by the overlay, without
// deduplication.  Tiles of kRouteTile entries: k_route_count hashes a tile,
// writes each entry's id (or -1) and the tile's per-owner counts; k_route_scan
// turns the counts into each tile's first slot per owner (owner-major); then
// k_route_scatter places every requested id in its owner's group (the order
// inside a group is free) and records its slot as the entry's row index.
constexpr int kRouteThreads = 256, kRouteItems = 8, kRouteTile = kRouteThreads * kRouteItems;

__global__ void __launch_bounds__(kRouteThreads) k_route_count(engram_table T, engram_overlay OV,
                                                               const int32_t* __restrict__ tokens,
                                                               const int32_t* __restrict__ seg_start, int64_t t0,
                                                               int64_t n, int world, int rank,
                                                               int32_t* __restrict__ ids, uint32_t* __restrict__ tile_cnt) {
    __shared__ uint32_t cnt[kMaxWorld];
    __shared__ HeadTab htab;
    for (int o = threadIdx.x; o < world; o += blockDim.x) cnt[o] = 0;
    head_tab_fill(htab, T);
    __syncthreads();
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    const int64_t base = (int64_t)blockIdx.x * kRouteTile;
#pragma unroll
    for (int it = 0; it < kRouteItems; it++) {
        const int64_t k = base + it * kRouteThreads + threadIdx.x;
        if (k >= total) break;
        int64_t i;
        int h;
        split_pair(k, nh, i, h);
        const int32_t g = hash_row(T, htab, tokens, seg_start, t0 + i, h);
        const int o = (int)((uint32_t)g % (uint32_t)world);
        const bool req = o != rank && overlay_slot(OV, g) < 0;
        ids[k] = req ? g : -1;
        if (req) atomicAdd(cnt + o, 1u);
    }
    __syncthreads();
    for (int o = threadIdx.x; o < world; o += blockDim.x) tile_cnt[(int64_t)blockIdx.x * world + o] = cnt[o];
}

// One block: tile_cnt[b][o] -> the first slot of tile b's ids for owner o
// (owners in ascending order, tiles in ascending order inside an owner);
// counts[o] = requests for owner o.
__global__ void __launch_bounds__(1024) k_route_scan(uint32_t* tile_cnt, int nblk, int world,
                                                     unsigned long long* counts) {
    __shared__ uint32_t warp_sums[32];
    __shared__ unsigned long long carry;
    if (threadIdx.x == 0) carry = 0ull;
    __syncthreads();
    for (int o = 0; o < world; o++) {
        const unsigned long long owner_base = carry;
        for (int b0 = 0; b0 < nblk; b0 += blockDim.x) {
            const int b = b0 + threadIdx.x;
            const uint32_t v = b < nblk ? tile_cnt[(int64_t)b * world + o] : 0u;
            uint32_t tot;
            const uint32_t ex = block_exclusive_scan(v, warp_sums, &tot);
            if (b < nblk) tile_cnt[(int64_t)b * world + o] = (uint32_t)(carry + ex);
            __syncthreads();
            if (threadIdx.x == 0) carry += tot;
            __syncthreads();
        }
        if (threadIdx.x == 0) counts[o] = carry - owner_base;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kRouteThreads) k_route_scatter(const int32_t* ids, int64_t total, int world,
                                                                 const uint32_t* __restrict__ tile_first,
                                                                 int32_t* __restrict__ send_ids, int32_t* row_index) {
    __shared__ uint32_t cur[kMaxWorld];
    for (int o = threadIdx.x; o < world; o += blockDim.x) cur[o] = tile_first[(int64_t)blockIdx.x * world + o];
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kRouteTile;
#pragma unroll
    for (int it = 0; it < kRouteItems; it++) {
        const int64_t k = base + it * kRouteThreads + threadIdx.x;
        if (k >= total) break;
        const int32_t g = ids[k];
        int32_t r = -1;
        if (g >= 0) {
            r = (int32_t)atomicAdd(cur + (int)((uint32_t)g % (uint32_t)world), 1u);
            send_ids[r] = g;
        }
        row_index[k] = r;
    }
}

// engram_shard_route_push: the requests of a batch written straight into their
// owners' memory.  Requester `rank` owns region `rank` of every owner's request
// buffer (region entries of int32 ids) and of its send buffer (region rows).
// k_route_push hashes a tile of (position, head) pairs and counts each owner's
// requests in shared memory; the tile's ids are staged there grouped by owner,
// one atomic per owner on the global counters reserves the tile's slots, and
// the block then writes each owner's ids as one contiguous run (consecutive
// threads, consecutive addresses: coalesced stores over NVLink).  Each pair is
// tagged with owner * region + slot.  k_route_finish turns the tags into rows
// of the receive buffer (owners' blocks in ascending owner order, so row = the
// counts of lower owners + slot) and block 0 stores each count into its
// owner's count array (entry `rank`).  The order inside an owner's block
// depends on which tile reserved first; the forward reads every pair's own
// row, so its output does not.
constexpr int kPushThreads = 256, kPushItems = 8, kPushTile = kPushThreads * kPushItems;

__global__ void __launch_bounds__(kPushThreads) k_route_push(engram_table T, engram_overlay OV,
                                                             const int32_t* __restrict__ tokens,
                                                             const int32_t* __restrict__ seg_start, int64_t t0,
                                                             int64_t n, int world, int rank,
                                                             const unsigned long long* __restrict__ id_ptrs,
                                                             int64_t region, unsigned long long* __restrict__ cnt,
                                                             int32_t* __restrict__ row_index) {
    __shared__ uint32_t tile_cnt[kMaxWorld];
    __shared__ uint32_t tile_off[kMaxWorld + 1];        // first staged entry of each owner
    __shared__ unsigned long long first[kMaxWorld];     // first slot of each owner's run in its region
    __shared__ int32_t staged[kPushTile];
    __shared__ uint8_t staged_owner[kPushTile];
    __shared__ HeadTab htab;
    for (int o = threadIdx.x; o < world; o += blockDim.x) tile_cnt[o] = 0;
    head_tab_fill(htab, T);
    __syncthreads();
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    const int64_t base = (int64_t)blockIdx.x * kPushTile;
    int32_t g[kPushItems];
    uint32_t loc[kPushItems];
#pragma unroll
    for (int it = 0; it < kPushItems; it++) {
        const int64_t k = base + it * kPushThreads + threadIdx.x;
        g[it] = -1;
        if (k < total) {
            int64_t i;
            int h;
            split_pair(k, nh, i, h);
            const int32_t id = hash_row(T, htab, tokens, seg_start, t0 + i, h);
            const int o = (int)((uint32_t)id % (uint32_t)world);
            if (o != rank && overlay_slot(OV, id) < 0) {
                g[it] = id;
                loc[it] = atomicAdd(tile_cnt + o, 1u);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t acc = 0;
        for (int o = 0; o < world; o++) {
            tile_off[o] = acc;
            acc += tile_cnt[o];
        }
        tile_off[world] = acc;
    }
    for (int o = threadIdx.x; o < world; o += blockDim.x)
        first[o] = tile_cnt[o] ? atomicAdd(cnt + o, (unsigned long long)tile_cnt[o]) : 0ull;
    __syncthreads();
#pragma unroll
    for (int it = 0; it < kPushItems; it++) {
        const int64_t k = base + it * kPushThreads + threadIdx.x;
        if (k >= total) break;
        int32_t tag = -1;
        if (g[it] >= 0) {
            const int o = (int)((uint32_t)g[it] % (uint32_t)world);
            const uint32_t e = tile_off[o] + loc[it];
            staged[e] = g[it];
            staged_owner[e] = (uint8_t)o;
            tag = (int32_t)(o * region + (int64_t)first[o] + loc[it]);  // slot < region: at most region pairs
        }
        row_index[k] = tag;
    }
    __syncthreads();
    const uint32_t staged_n = tile_off[world];
    for (uint32_t e = threadIdx.x; e < staged_n; e += blockDim.x) {
        const int o = staged_owner[e];
        const int64_t slot = (int64_t)first[o] + (e - tile_off[o]);
        reinterpret_cast<int32_t*>(id_ptrs[o])[(int64_t)rank * region + slot] = staged[e];
    }
}

__global__ void __launch_bounds__(256) k_route_finish(int64_t total, int world, int rank, int64_t region,
                                                      const unsigned long long* __restrict__ cnt,
                                                      const unsigned long long* __restrict__ count_ptrs,
                                                      int32_t* __restrict__ row_index) {
    __shared__ long long before[kMaxWorld];
    if (threadIdx.x == 0) {
        long long acc = 0;
        for (int o = 0; o < world; o++) {
            before[o] = acc;
            acc += (long long)cnt[o];
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < world && threadIdx.x != rank)
        reinterpret_cast<long long*>(count_ptrs[threadIdx.x])[rank] = (long long)cnt[threadIdx.x];
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += stride) {
        const int32_t tag = row_index[k];
        if (tag >= 0) {
            const int o = (int)(tag / region);
            row_index[k] = (int32_t)(before[o] + (tag - o * region));
        }
    }
}

// Owner side of the pushed exchange (engram_shard_serve_pushed): requester r's
// ids for this owner are entries [0, counts[r]) of region r of req_ids (this
// GPU's memory, written by r's route); the rows land in region r of send_rows,
// in the same order.  A warp serves 32 send rows at a time: lane l looks up
// row g0 + l once, then the warp copies the 32 rows word by word with
// kServeLoads 16-byte loads per lane in flight.  Ids that are not this
// owner's, or past its shard, give zero rows.
__global__ void __launch_bounds__(256) k_serve_pushed(const uint8_t* __restrict__ shard, int64_t stride,
                                                      int64_t n_local, int world, int rank,
                                                      const int32_t* __restrict__ req_ids,
                                                      const long long* __restrict__ req_counts, int64_t region,
                                                      uint8_t* __restrict__ send_rows) {
    __shared__ long long base[kMaxWorld + 1];  // first flattened row of each requester
    if (threadIdx.x == 0) {
        long long acc = 0;
        for (int r = 0; r < world; r++) {
            base[r] = acc;
            long long c = r == rank ? 0 : req_counts[r];
            acc += c < 0 ? 0 : (c > region ? region : c);
        }
        base[world] = acc;
    }
    __syncthreads();
    const int64_t total = base[world];
    const int words = (int)(stride >> 4);
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    constexpr int kServeLoads = 8;
    for (int64_t g0 = warp0 * 32; g0 < total; g0 += nwarps * 32) {
        const int64_t f = g0 + lane;
        int64_t src = -1, dst_row = -1;  // byte offset of the row in the shard (-1: zero row); its row in send_rows
        if (f < total) {
            int r = 0;
            while (r + 1 < world && base[r + 1] <= f) r++;
            dst_row = (int64_t)r * region + (f - base[r]);
            const int32_t g = req_ids[dst_row];
            const int64_t local = (int64_t)g / world;
            if (g >= 0 && (int)(g % world) == rank && local < n_local) src = local * stride;
        }
        const int pairs = 32 * words;
        for (int p0 = 0; p0 < pairs; p0 += 32 * kServeLoads) {
            uint4 v[kServeLoads];
            int64_t dst[kServeLoads];
#pragma unroll
            for (int u = 0; u < kServeLoads; u++) {
                const int p = p0 + u * 32 + lane;
                const int rr = p / words, w = p - rr * words;
                const int src_lane = rr < 32 ? rr : 0;
                const int64_t s_off = __shfl_sync(0xffffffffu, src, src_lane);
                const int64_t d_row = __shfl_sync(0xffffffffu, dst_row, src_lane);
                dst[u] = -1;
                if (p < pairs && d_row >= 0) {
                    v[u] = s_off >= 0 ? __ldg(reinterpret_cast<const uint4*>(shard + s_off) + w)
                                      : make_uint4(0u, 0u, 0u, 0u);
                    dst[u] = d_row * stride + 16 * w;
                }
            }
#pragma unroll
            for (int u = 0; u < kServeLoads; u++)
                if (dst[u] >= 0) __stcg(reinterpret_cast<uint4*>(send_rows + dst[u]), v[u]);
        }
    }
}

int grid(int64_t work) {
    const int64_t want = (work + 255) / 256, cap = (int64_t)sm_count() * 8;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

extern "C" int engram_shard_requests(const int32_t* ids, const int32_t* slots, int64_t n, int32_t world,
                                     int32_t* set_keys, int32_t* set_vals, int64_t capacity, int32_t* send_ids,
                                     int64_t* counts, int32_t* row_index, void* stream) {
    if (n < 0 || world < 1 || world > kMaxWorld) return ENGRAM_ERR_ARG;
    if (!set_keys || !set_vals || !send_ids || !counts || !row_index) return ENGRAM_ERR_ARG;
    if (n > 0 && !ids) return ENGRAM_ERR_ARG;
    if ((capacity & (capacity - 1)) != 0 || capacity < 2 * n || capacity < 2 || capacity > (1LL << 31))
        return ENGRAM_ERR_RANGE;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(counts);
    k_set_clear<<<grid(capacity), 256, 0, s>>>(set_keys, capacity, counts, world);
    k_set_insert<<<grid(n), 256, 0, s>>>(ids, slots, n, set_keys, capacity);
    k_owner_count<<<grid(capacity), 256, 0, s>>>(set_keys, capacity, world, cnt);
    k_owner_scatter<<<grid(capacity), 256, 0, s>>>(set_keys, set_vals, capacity, world, cnt, cnt + world, send_ids);
    k_row_index<<<grid(n), 256, 0, s>>>(ids, slots, n, set_keys, set_vals, capacity, row_index);
    count_launches(5);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_shard_gather(const void* shard_rows, int64_t stride, int64_t n_local, const int32_t* ids,
                                   int64_t n, int32_t world, void* out, void* stream) {
    if (n < 0 || world < 1 || stride <= 0 || (stride & 15) || n_local < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!shard_rows || !ids || !out || !aligned16(shard_rows) || !aligned16(out)) return ENGRAM_ERR_ARG;
    k_shard_gather<<<grid(n * (stride >> 4)), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(shard_rows), stride, n_local, ids, n, world, static_cast<uint8_t*>(out));
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_shard_plan(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                 const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                 int32_t* set_keys, int32_t* set_vals, int64_t capacity, int32_t* send_ids,
                                 int64_t* counts, int32_t* row_index, void* stream) {
    if (!t || t0 < 0 || n < 0 || world < 1 || world > kMaxWorld || rank < 0 || rank >= world) return ENGRAM_ERR_ARG;
    if (!set_keys || !set_vals || !send_ids || !counts || !row_index) return ENGRAM_ERR_ARG;
    if (n > 0 && !tokens) return ENGRAM_ERR_ARG;
    const int64_t entries = n * t->n_heads;
    if ((capacity & (capacity - 1)) != 0 || capacity < 2 * entries || capacity < 2 || capacity > (1LL << 31))
        return ENGRAM_ERR_RANGE;
    engram_overlay OV{nullptr, 0, nullptr, nullptr, 0};
    if (ov && ov->n_rows > 0) {
        OV = *ov;
        if (!OV.map_keys || !OV.map_slots || (OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows)
            return ENGRAM_ERR_ARG;
    }
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(counts);
    k_set_clear<<<grid(capacity), 256, 0, s>>>(set_keys, capacity, counts, world);
    int launched = 1;
    if (entries > 0) {
        k_plan_ids<<<grid(entries), 256, 0, s>>>(*t, OV, tokens, seg_start, t0, n, world, rank, row_index);
        k_set_insert<<<grid(entries), 256, 0, s>>>(row_index, nullptr, entries, set_keys, capacity);
        k_owner_count<<<grid(capacity), 256, 0, s>>>(set_keys, capacity, world, cnt);
        k_owner_scatter<<<grid(capacity), 256, 0, s>>>(set_keys, set_vals, capacity, world, cnt, cnt + world, send_ids);
        k_row_index_inplace<<<grid(entries), 256, 0, s>>>(row_index, entries, set_keys, set_vals, capacity, row_index);
        launched += 5;
    }
    count_launches(launched);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int64_t engram_shard_route_scratch_words(int64_t n, int32_t n_heads, int32_t world) {
    if (n < 0 || n_heads < 1 || world < 1 || world > kMaxWorld) return ENGRAM_ERR_ARG;
    const int64_t tiles = (n * n_heads + kRouteTile - 1) / kRouteTile;
    return (tiles > 0 ? tiles : 1) * world;
}

extern "C" int engram_shard_route(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                  const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                  uint32_t* scratch, int64_t scratch_words, int32_t* send_ids, int64_t* counts,
                                  int32_t* row_index, void* stream) {
    if (!t || t0 < 0 || n < 0 || world < 1 || world > kMaxWorld || rank < 0 || rank >= world) return ENGRAM_ERR_ARG;
    if (!scratch || !send_ids || !counts || !row_index || (n > 0 && !tokens)) return ENGRAM_ERR_ARG;
    const int64_t entries = n * t->n_heads;
    const int64_t tiles = (entries + kRouteTile - 1) / kRouteTile;
    if (scratch_words < (tiles > 0 ? tiles : 1) * world) return ENGRAM_ERR_WORKSPACE;
    if (tiles > INT_MAX) return ENGRAM_ERR_RANGE;
    engram_overlay OV{nullptr, 0, nullptr, nullptr, 0};
    if (ov && ov->n_rows > 0) {
        OV = *ov;
        if (!OV.map_keys || !OV.map_slots || (OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows)
            return ENGRAM_ERR_ARG;
    }
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(counts);
    if (tiles == 0) {
        cudaMemsetAsync(counts, 0, sizeof(int64_t) * world, s);
        return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
    }
    k_route_count<<<(int)tiles, kRouteThreads, 0, s>>>(*t, OV, tokens, seg_start, t0, n, world, rank, row_index, scratch);
    k_route_scan<<<1, 1024, 0, s>>>(scratch, (int)tiles, world, cnt);
    k_route_scatter<<<(int)tiles, kRouteThreads, 0, s>>>(row_index, entries, world, scratch, send_ids, row_index);
    count_launches(3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_shard_route_push(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                       const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                       const void* id_ptrs, const void* count_ptrs, int64_t region, int64_t* counts,
                                       int32_t* row_index, void* stream) {
    if (!t || t0 < 0 || n < 0 || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || region < 1)
        return ENGRAM_ERR_ARG;
    if (!id_ptrs || !count_ptrs || !counts || !row_index || (n > 0 && !tokens)) return ENGRAM_ERR_ARG;
    const int64_t entries = n * t->n_heads;
    if (entries > region) return ENGRAM_ERR_RANGE;
    if ((int64_t)world * region > INT32_MAX) return ENGRAM_ERR_RANGE;
    engram_overlay OV{nullptr, 0, nullptr, nullptr, 0};
    if (ov && ov->n_rows > 0) {
        OV = *ov;
        if (!OV.map_keys || !OV.map_slots || (OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows)
            return ENGRAM_ERR_ARG;
    }
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(counts);
    cudaMemsetAsync(counts, 0, sizeof(int64_t) * world, s);
    const int64_t tiles = (entries + kPushTile - 1) / kPushTile;
    if (tiles > INT_MAX) return ENGRAM_ERR_RANGE;
    int launched = 0;
    if (tiles > 0) {
        k_route_push<<<(int)tiles, kPushThreads, 0, s>>>(*t, OV, tokens, seg_start, t0, n, world, rank,
                                                         static_cast<const unsigned long long*>(id_ptrs), region, cnt,
                                                         row_index);
        launched++;
    }
    // publishes the counts (zero for an empty batch) even when there is nothing to route
    k_route_finish<<<grid(entries > 0 ? entries : 1), 256, 0, s>>>(entries, world, rank, region, cnt,
                                                                   static_cast<const unsigned long long*>(count_ptrs),
                                                                   row_index);
    count_launches(launched + 1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_shard_serve_pushed(const void* shard_rows, int64_t stride, int64_t n_local, int32_t world,
                                         int32_t rank, const int32_t* req_ids, const int64_t* req_counts,
                                         int64_t region, void* send_rows, void* stream) {
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || stride <= 0 || (stride & 15) || n_local < 0 ||
        region < 1)
        return ENGRAM_ERR_ARG;
    if (world == 1) return ENGRAM_OK;
    if (!shard_rows || !req_ids || !req_counts || !send_rows || !aligned16(shard_rows) || !aligned16(send_rows))
        return ENGRAM_ERR_ARG;
    const int64_t cap = (int64_t)sm_count() * 8;
    k_serve_pushed<<<(int)cap, 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(shard_rows), stride, n_local, world, rank, req_ids,
        reinterpret_cast<const long long*>(req_counts), region, static_cast<uint8_t*>(send_rows));
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
