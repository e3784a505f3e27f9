// engram_scan.cu -- bulk hash + overlay hit scan over a token corpus
// (engraft/damage.py:168-224 scan_hits, with ngram_rows :68-104).
//
// For every position: the 16 global rows (the hash of engram_hash, no
// segments), their overlay slots, and per hit position the number of overlay
// rows read, the max and the sum of their dnorm values.  Per overlay row, the
// number of reads.  Three launches:
//   A. each block scores a tile of kTile positions (a 16-lane group per
//      position: lane h hashes head h and probes the overlay map; the group's
//      first lane forms max and sum in the reference's order) and counts the
//      tile's hit positions;
//   B. exclusive scan of the tile counts;
//   C. each block writes its hit positions, in position order, at its offset.
// The sum follows numpy's float32 pairwise reduction of a 16-wide row
// (((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), r_j = v_j + v_{j+8}), so the result
// is bit-identical to the reference.
#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr int kTile = 256;
constexpr int kScanBlockThreads = 1024;
constexpr unsigned kFull = 0xffffffffu;

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct ScanWs {
    int32_t* nhit;
    float* dmax;
    float* dsum;
    uint32_t* tile_cnt;
    int64_t bytes;
    int64_t ntiles;
};

ScanWs scan_layout(void* base, int64_t n) {
    ScanWs w{};
    w.ntiles = (n + kTile - 1) / kTile;
    char* p = static_cast<char*>(base);
    int64_t off = 0;
    auto take = [&](int64_t b) {
        char* r = p ? p + off : nullptr;
        off += align256(b);
        return r;
    };
    w.nhit = reinterpret_cast<int32_t*>(take(4 * n));
    w.dmax = reinterpret_cast<float*>(take(4 * n));
    w.dsum = reinterpret_cast<float*>(take(4 * n));
    w.tile_cnt = reinterpret_cast<uint32_t*>(take(4 * (w.ntiles + 1)));
    w.bytes = off;
    return w;
}

// numpy's pairwise float32 sum of a row of m values held by lanes 0..m-1 of a
// 16-lane group; evaluated by the group's lane 0 (see the file comment).
__device__ __forceinline__ float np_pairwise_sum(const float* v, int m) {
    if (m < 8) {
        float res = 0.0f;
        for (int i = 0; i < m; i++) res = __fadd_rn(res, v[i]);
        return res;
    }
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; k++) r[k] = v[k];
    int i = 8;
    for (; i + 8 <= m; i += 8)
#pragma unroll
        for (int k = 0; k < 8; k++) r[k] = __fadd_rn(r[k], v[i + k]);
    float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                          __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
    for (; i < m; i++) res = __fadd_rn(res, v[i]);
    return res;
}

__global__ void __launch_bounds__(256) k_scan_score(engram_table T, engram_overlay OV, const int32_t* __restrict__ tokens,
                                                    int64_t t0, int64_t n, int64_t last_t,
                                                    const float* __restrict__ dnorm,
                                                    unsigned long long* __restrict__ read_count, ScanWs w) {
    __shared__ uint32_t s_cnt;
    __shared__ HeadTab htab;
    if (threadIdx.x == 0) s_cnt = 0;
    head_tab_fill(htab, T);
    __syncthreads();
    const int lane = threadIdx.x & 31, sub = lane & 15, grp = threadIdx.x >> 4;  // 16 groups of 16 lanes
    const int nh = T.n_heads;
    const unsigned gmask = (lane < 16) ? 0x0000ffffu : 0xffff0000u;
    const int64_t base = (int64_t)blockIdx.x * kTile;
    for (int r = grp; r < kTile; r += 16) {
        const int64_t i = base + r;
        const bool live = i < n;
        const int64_t t = t0 + i;
        float v = 0.0f;
        bool match = false;
        if (live && sub < nh) {
            const int32_t gid = hash_row(T, htab, tokens, nullptr, t, sub);
            const int32_t slot = overlay_slot(OV, gid);
            match = slot >= 0;
            if (match) {
                v = __ldg(dnorm + slot);
                atomicAdd(read_count + slot, 1ull);
            }
        }
        const unsigned b = __ballot_sync(kFull, match) & gmask;
        const int n_hit = __popc(b);
        float vals[16];
#pragma unroll
        for (int h = 0; h < 16; h++) vals[h] = __shfl_sync(kFull, v, h, 16);
        if (sub == 0 && live) {
            const int m = nh < 16 ? nh : 16;
            float dmax = vals[0];
            for (int h = 1; h < m; h++) dmax = fmaxf(dmax, vals[h]);
            const bool listed = n_hit > 0 && t != last_t;
            w.nhit[i] = listed ? n_hit : 0;
            w.dmax[i] = dmax;
            w.dsum[i] = np_pairwise_sum(vals, m);
            if (listed) atomicAdd(&s_cnt, 1u);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) w.tile_cnt[blockIdx.x] = s_cnt;
}

// Exclusive scan of tile_cnt[0..ntiles) in place (one block); total -> *n_hits.
__global__ void __launch_bounds__(kScanBlockThreads) k_scan_tiles(uint32_t* a, int64_t len, int64_t* n_hits) {
    __shared__ uint32_t part[kScanBlockThreads];
    const int tid = threadIdx.x;
    const int64_t per = (len + kScanBlockThreads - 1) / kScanBlockThreads;
    const int64_t lo = tid * per, hi = (lo + per < len) ? lo + per : len;
    uint32_t s = 0;
    for (int64_t k = lo; k < hi; k++) s += a[k];
    part[tid] = s;
    __syncthreads();
    for (int off = 1; off < kScanBlockThreads; off <<= 1) {
        const uint32_t x = tid >= off ? part[tid - off] : 0u;
        __syncthreads();
        part[tid] += x;
        __syncthreads();
    }
    uint32_t run = part[tid] - s;
    for (int64_t k = lo; k < hi; k++) {
        const uint32_t x = a[k];
        a[k] = run;
        run += x;
    }
    if (tid == kScanBlockThreads - 1) *n_hits = (int64_t)part[tid];
}

// Ordered write of the tile's listed positions.
__global__ void __launch_bounds__(kTile) k_scan_emit(int64_t t0, int64_t n, int64_t pos_base, ScanWs w,
                                                     int64_t* __restrict__ pos_out, int32_t* __restrict__ nhit_out,
                                                     float* __restrict__ dmax_out, float* __restrict__ dsum_out) {
    __shared__ uint32_t wsum[kTile / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t i = (int64_t)blockIdx.x * kTile + tid;
    const int32_t nh = i < n ? w.nhit[i] : 0;
    const bool listed = nh > 0;
    const unsigned b = __ballot_sync(kFull, listed);
    if (lane == 0) wsum[warp] = __popc(b);
    __syncthreads();
    uint32_t before = 0;
    for (int k = 0; k < warp; k++) before += wsum[k];
    if (listed) {
        const uint64_t o = (uint64_t)w.tile_cnt[blockIdx.x] + before + __popc(b & ((1u << lane) - 1u));
        pos_out[o] = pos_base + t0 + i;
        nhit_out[o] = nh;
        dmax_out[o] = w.dmax[i];
        dsum_out[o] = w.dsum[i];
    }
}

}  // namespace

extern "C" int64_t engram_scan_hits_workspace_bytes(int64_t n) {
    if (n < 0) return ENGRAM_ERR_ARG;
    return scan_layout(nullptr, n).bytes;
}

extern "C" int engram_scan_hits(const engram_table* t, const int32_t* tokens, int64_t t0, int64_t n, int64_t pos_base,
                                int32_t exclude_last, const engram_overlay* ov, const float* dnorm, int64_t* pos_out,
                                int32_t* nhit_out, float* dmax_out, float* dsum_out, int64_t* n_hits,
                                int64_t* read_count, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!t || !ov || t0 < 0 || n < 0 || !n_hits) return ENGRAM_ERR_ARG;
    if (t->n_heads > 16) return ENGRAM_ERR_FORMAT;
    if (n >= (1LL << 31)) return ENGRAM_ERR_RANGE;
    engram_overlay OV = *ov;
    if (OV.n_rows < 0) return ENGRAM_ERR_ARG;
    if (OV.n_rows > 0) {
        if (!OV.map_keys || !OV.map_slots || !dnorm || !read_count) return ENGRAM_ERR_ARG;
        if ((OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows) return ENGRAM_ERR_RANGE;
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (n == 0) return cudaMemsetAsync(n_hits, 0, sizeof(int64_t), s) == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
    if (!tokens || !pos_out || !nhit_out || !dmax_out || !dsum_out) return ENGRAM_ERR_ARG;
    ScanWs w = scan_layout(workspace, n);
    if (!workspace || workspace_bytes < w.bytes) return ENGRAM_ERR_WORKSPACE;
    const int64_t last_t = exclude_last ? t0 + n - 1 : -1;
    k_scan_score<<<(int)w.ntiles, 256, 0, s>>>(*t, OV, tokens, t0, n, last_t, dnorm,
                                               reinterpret_cast<unsigned long long*>(read_count), w);
    k_scan_tiles<<<1, kScanBlockThreads, 0, s>>>(w.tile_cnt, w.ntiles, n_hits);
    k_scan_emit<<<(int)w.ntiles, kTile, 0, s>>>(t0, n, pos_base, w, pos_out, nhit_out, dmax_out, dsum_out);
    count_launches(3);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
