// engram_forward.cu -- K1 (hash) and the fused K1+K2 forward: hash -> overlay
// probe -> gather + dequantise -> emit (CONCAT fp32, or pair-sum added into a
// bf16 residual stream).
//
// One warp per position (grid-stride over positions).  Lane h < n_heads hashes
// head h and probes the overlay map; the warp then streams the position's
// output in 16-byte chunks, lane-contiguous so every store is a full 512-byte
// warp transaction, and every chunk's source row (table or overlay) is picked
// by a shuffle from the lane that owns its head.  Loads of U chunks are issued
// before any is consumed, so each warp keeps U row reads in flight.
#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr unsigned kFull = 0xffffffffu;

struct PosHeads {
    int32_t gid;   // this lane's head: global row id
    int32_t slot;  // overlay slot or -1
    int32_t row;   // row in T.rows serving it (the global id, or an index into gathered rows)
};

// Output row i -> token position: pm.at(i), or pos[i] for an explicit position
// list (decode-style calls), clamped into [0, n_tokens).
struct PosMap {
    int64_t t0;
    const int64_t* pos;
    int64_t n_tokens;
    const int32_t* rix;  // nullable: row of (output row i, head h) in T.rows is rix[i*n_heads + h]
    // nullable: the table is row-sharded over `world` ranks (row g at local row
    // g / world of rank g % world's shard, shard[rank] = its address in this
    // process, e.g. peer memory mapped over NVLink); wshift = log2(world) when
    // world is a power of two, else -1
    const uint8_t* const* shard = nullptr;
    uint32_t world = 1;
    int wshift = 0;
    // nullable (sharded reads only): rows of other ranks already copied into
    // this GPU's memory, head h of output row i at stage + (i * nh + h) * stride
    // (engram_stage_sharded); rows owned by `rank` are still read in place
    const uint8_t* stage = nullptr;
    uint32_t rank = 0;
    // nullable (exchanged reads): this rank's own shard, read in place; the
    // rows of other ranks sit in `stage`, the row of head h of output row i at
    // stage + srix[i * nh + h] * stride (engram_shard_plan's row_index)
    const uint8_t* local = nullptr;
    const int32_t* srix = nullptr;
    __device__ __host__ __forceinline__ bool sharded() const { return shard != nullptr || local != nullptr; }
    // Owner rank o of global row r and its row l in that rank's shard.
    __device__ __forceinline__ void owner_of(int32_t r, uint32_t& o, uint32_t& l) const {
        if (wshift >= 0) {
            o = (uint32_t)r & (world - 1u);
            l = (uint32_t)r >> wshift;
        } else {
            l = (uint32_t)r / world;
            o = (uint32_t)r - l * world;
        }
    }
    // Address of row r serving head h of output row i: T.rows + r * stride, its
    // staged copy, or the row in its owner's shard.
    __device__ __forceinline__ const uint8_t* row_ptr(const uint8_t* rows, int64_t stride, int32_t r, int64_t i,
                                                      int h, int nh) const {
        if (!sharded()) return rows + (int64_t)r * stride;
        uint32_t o, l;
        owner_of(r, o, l);
        if (o != rank) {
            if (srix != nullptr) {  // an entry the plan did not request reads row 0 (never used)
                const int32_t k = __ldg(srix + i * nh + h);
                return stage + (int64_t)(k < 0 ? 0 : k) * stride;
            }
            if (stage != nullptr) return stage + (i * nh + h) * stride;
        } else if (local != nullptr) {
            return local + (int64_t)l * stride;
        }
        const uint8_t* base =
            reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(shard) + o));
        return base + (int64_t)l * stride;
    }
    // row_ptr with the exchanged-read row index srix[i * nh + h] already loaded
    // (k_pre; ignored for every other layout).
    __device__ __forceinline__ const uint8_t* row_ptr_pre(const uint8_t* rows, int64_t stride, int32_t r, int32_t k_pre,
                                                          int64_t i, int h, int nh) const {
        if (srix == nullptr || !sharded()) return row_ptr(rows, stride, r, i, h, nh);
        uint32_t o, l;
        owner_of(r, o, l);
        if (o != rank) return stage + (int64_t)(k_pre < 0 ? 0 : k_pre) * stride;
        if (local != nullptr) return local + (int64_t)l * stride;
        const uint8_t* base =
            reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(shard) + o));
        return base + (int64_t)l * stride;
    }
    // Row number in T.rows that serves head h of output row i (the global id
    // unless the rows were gathered into a local buffer, see engram_forward_indirect).
    __device__ __forceinline__ int32_t row(int64_t i, int h, int nh, int32_t gid) const {
        if (rix == nullptr) return gid;
        const int32_t r = __ldg(rix + i * nh + h);
        return r < 0 ? 0 : r;
    }
    __device__ __forceinline__ int64_t at(int64_t i) const {
        if (pos == nullptr) return t0 + i;
        const int64_t p = __ldg(pos + i);
        return p < 0 ? 0 : (p >= n_tokens ? n_tokens - 1 : p);
    }
};

__device__ __forceinline__ PosHeads heads_of(const engram_table& T, const HeadTab& H, const engram_overlay& OV,
                                             const TokCtx& c, const PosMap& pm, int64_t i, int lane) {
    PosHeads r{0, -1, 0};
    if (lane < T.n_heads) {
        r.gid = hash_ctx(T, H, c, pm.at(i), lane);
        r.slot = overlay_slot(OV, r.gid);
        r.row = pm.row(i, lane, T.n_heads, r.gid);
    }
    return r;
}

__device__ __forceinline__ void write_heads(const PosHeads& ph, int64_t i, int nh, int lane, int32_t* ids_out,
                                            int32_t* slots_out, unsigned long long& hits) {
    if (lane < nh) {
        if (ids_out) ids_out[i * nh + lane] = ph.gid;
        if (slots_out) slots_out[i * nh + lane] = ph.slot;
    }
    const unsigned hb = __ballot_sync(kFull, lane < nh && ph.slot >= 0);
    hits += (unsigned long long)__popc(hb);
}

__device__ __forceinline__ void flush_hits(unsigned long long hits, unsigned long long* hit_count, int lane) {
    if (hit_count && lane == 0 && hits) atomicAdd(hit_count, hits);
}

__global__ void __launch_bounds__(256) k_hash(engram_table T, const int32_t* __restrict__ tokens,
                                              const int32_t* __restrict__ seg_start, PosMap pm, int64_t n,
                                              int32_t* __restrict__ ids_out) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        int64_t i;
        int h;
        split_pair(k, nh, i, h);
        ids_out[k] = hash_row(T, htab, tokens, seg_start, pm.at(i), h);
    }
}

// Copies every row of another rank that the sharded forward over the same
// output rows reads into this GPU's memory: head h of output row i to
// stage + (i * nh + h) * stride.  One warp per output row; each lane keeps up
// to kStageLoads 16-byte pieces in flight.  Rows of this rank are skipped (the
// forward reads them in place), so are the heads the overlay serves (the
// forward reads their fp32 rows; OV.n_rows == 0: no overlay).
constexpr int kStageLoads = 8;
__global__ void __launch_bounds__(256) k_stage_sharded(engram_table T, engram_overlay OV,
                                                       const int32_t* __restrict__ tokens,
                                                       const int32_t* __restrict__ seg_start, PosMap pm, int64_t n,
                                                       uint8_t* __restrict__ stage) {
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nh = T.n_heads;
    const int pieces = (int)(T.row_stride >> 4);
    const int total = nh * pieces;
    const unsigned long long* shard = reinterpret_cast<const unsigned long long*>(pm.shard);
    for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; i < n; i += nw) {
        int32_t gid = 0;
        bool copy = false;  // another rank's row that the overlay does not replace
        if (lane < nh) {
            const int64_t t = pm.at(i);
            gid = hash_ctx(T, htab, load_ctx(T, tokens, seg_start, t), t, lane);
            uint32_t o, l;
            pm.owner_of(gid, o, l);
            copy = o != pm.rank && overlay_slot(OV, gid) < 0;
        }
        const unsigned want = __ballot_sync(kFull, copy);
        uint8_t* srow = stage + i * nh * T.row_stride;
        for (int j0 = 0; j0 < total; j0 += 32 * kStageLoads) {
            uint4 v[kStageLoads];
            int dst[kStageLoads];  // byte offset in srow, -1: nothing to copy
#pragma unroll
            for (int u = 0; u < kStageLoads; u++) {
                const int j = j0 + u * 32 + lane;
                const int h = j / pieces;
                const int p = j - h * pieces;
                const int32_t g = __shfl_sync(kFull, gid, h < nh ? h : 0);
                dst[u] = -1;
                if (j < total && ((want >> h) & 1u)) {
                    uint32_t o, l;
                    pm.owner_of(g, o, l);
                    const uint8_t* src = reinterpret_cast<const uint8_t*>(__ldg(shard + o)) +
                                         (int64_t)l * T.row_stride + p * 16;
                    v[u] = *reinterpret_cast<const uint4*>(src);
                    dst[u] = h * (int)T.row_stride + p * 16;
                }
            }
#pragma unroll
            for (int u = 0; u < kStageLoads; u++)
                if (dst[u] >= 0) __stcg(reinterpret_cast<uint4*>(srow + dst[u]), v[u]);
        }
    }
}

// Raw bytes of 4 (Raw4) or 8 (Raw8) consecutive values of a resident IQ4 row,
// loaded ahead and dequantised when consumed; F32 rows are loaded as values.
struct Raw4 {
    uint32_t q;    // 4 code bytes
    uint32_t h0;   // IQ4_NL: fp16 d; IQ4_XS: d | scales_h << 16
    uint32_t h1;   // IQ4_XS: scales_l
};
struct Raw8 {
    uint2 q;       // 8 code bytes
    uint32_t h0, h1;
};

template <int FMT>
__device__ __forceinline__ Raw4 raw4(const uint8_t* __restrict__ row, int c, int dim) {
    Raw4 r{0u, 0u, 0u};
    if (FMT == ENGRAM_FMT_IQ4_NL) {
        const int nb = dim >> 5, b = c >> 3, j0 = (c & 7) << 2;
        r.q = __ldg(reinterpret_cast<const uint32_t*>(row + b * 16 + (j0 & 15)));
        r.h0 = __ldg(reinterpret_cast<const unsigned short*>(row + 16 * nb + 2 * b));
    } else if (FMT == ENGRAM_FMT_IQ4_XS) {
        const uint8_t* base = row + (c >> 6) * 144;
        const int w = c & 63, ib = w >> 3, j0 = (w & 7) << 2;
        r.q = __ldg(reinterpret_cast<const uint32_t*>(base + ib * 16 + (j0 & 15)));
        const uint2 hdr = __ldg(reinterpret_cast<const uint2*>(base + 128));
        r.h0 = hdr.x;
        r.h1 = hdr.y;
    }
    return r;
}

template <int FMT>
__device__ __forceinline__ Raw8 raw8(const uint8_t* __restrict__ row, int c, int dim) {
    Raw8 r{make_uint2(0u, 0u), 0u, 0u};
    if (FMT == ENGRAM_FMT_IQ4_NL) {
        const int nb = dim >> 5, b = c >> 2, k = c & 3;
        r.q = __ldg(reinterpret_cast<const uint2*>(row + b * 16 + (k & 1) * 8));
        r.h0 = __ldg(reinterpret_cast<const unsigned short*>(row + 16 * nb + 2 * b));
    } else if (FMT == ENGRAM_FMT_IQ4_XS) {
        const uint8_t* base = row + (c >> 5) * 144;
        const int w = c & 31, ib = w >> 2, k = w & 3;
        r.q = __ldg(reinterpret_cast<const uint2*>(base + ib * 16 + (k & 1) * 8));
        const uint2 hdr = __ldg(reinterpret_cast<const uint2*>(base + 128));
        r.h0 = hdr.x;
        r.h1 = hdr.y;
    }
    return r;
}

// Dequantisation, bit-exact with the reference: IQ4_NL y = kv*d
// (engraft/table.py:164-168); IQ4_XS dl = d*(ls-32), y = dl*kv
// (engraft/replica/dequant.py:175-186).
template <int FMT>
__device__ __forceinline__ float block_scale(uint32_t h0, uint32_t h1, int ib) {
    if (FMT == ENGRAM_FMT_IQ4_NL) return half_bits_to_float(h0 & 0xffffu);
    const int ls = (int)(((h1 >> (4 * ib)) & 15u) | (((h0 >> (16 + 2 * ib)) & 3u) << 4));
    return __fmul_rn(half_bits_to_float(h0 & 0xffffu), (float)(ls - 32));
}

template <int FMT>
__device__ __forceinline__ float4 dq4(const Raw4& r, int c, const float* kv) {
    const int j0 = FMT == ENGRAM_FMT_IQ4_NL ? ((c & 7) << 2) : (((c & 63) & 7) << 2);
    const int ib = FMT == ENGRAM_FMT_IQ4_NL ? 0 : ((c & 63) >> 3);
    const float d = block_scale<FMT>(r.h0, r.h1, ib);
    const int sh = j0 >= 16 ? 4 : 0;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float q = kv[(r.q >> (8 * k + sh)) & 15u];
        v[k] = FMT == ENGRAM_FMT_IQ4_NL ? __fmul_rn(q, d) : __fmul_rn(d, q);
    }
    return make_float4(v[0], v[1], v[2], v[3]);
}

template <int FMT>
__device__ __forceinline__ void dq8(const Raw8& r, int c, const float* kv, float* v) {
    const int k = FMT == ENGRAM_FMT_IQ4_NL ? (c & 3) : ((c & 31) & 3);
    const int ib = FMT == ENGRAM_FMT_IQ4_NL ? 0 : ((c & 31) >> 2);
    const float d = block_scale<FMT>(r.h0, r.h1, ib);
    const int sh = (k >> 1) * 4;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float q0 = kv[(r.q.x >> (8 * j + sh)) & 15u];
        const float q1 = kv[(r.q.y >> (8 * j + sh)) & 15u];
        v[j] = FMT == ENGRAM_FMT_IQ4_NL ? __fmul_rn(q0, d) : __fmul_rn(d, q0);
        v[4 + j] = FMT == ENGRAM_FMT_IQ4_NL ? __fmul_rn(q1, d) : __fmul_rn(d, q1);
    }
}

__device__ __forceinline__ void ld_f8(const float* __restrict__ src, float* v) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// CONCAT: out[i, h, :] = row(h) for positions i; U float4 chunks per lane per round.
// Per position: the next position's tokens are prefetched, every table-row
// load of the round is issued before any value is used, overlay rows (L2
// resident) are read when consumed.
template <int FMT, int U>
__global__ void __launch_bounds__(256, 2) k_forward_concat(engram_table T, engram_overlay OV,
                                                           const int32_t* __restrict__ tokens,
                                                           const int32_t* __restrict__ seg_start, PosMap pm,
                                                           int64_t n, float* __restrict__ out, int32_t* ids_out,
                                                           int32_t* slots_out, unsigned long long* hit_count) {
    __shared__ float s_kv[16];
    __shared__ HeadTab htab;
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
    head_tab_fill(htab, T);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nh = T.n_heads, dim = T.dim;
    const int cpr = dim >> 2;  // float4 chunks per row
    const int cpp = nh * cpr;  // chunks per position
    const uint8_t* rows = static_cast<const uint8_t*>(T.rows);
    const float* ovr = OV.rows;
    unsigned long long hits = 0;
    TokCtx nxt{};
    if (warp0 < n) nxt = load_ctx(T, tokens, seg_start, pm.at(warp0));
    for (int64_t i = warp0; i < n; i += nwarps) {
        const TokCtx cur = nxt;
        const PosHeads ph = heads_of(T, htab, OV, cur, pm, i, lane);
        write_heads(ph, i, nh, lane, ids_out, slots_out, hits);
        if (i + nwarps < n) nxt = load_ctx(T, tokens, seg_start, pm.at(i + nwarps));
        float4* dst = reinterpret_cast<float4*>(out + i * (int64_t)nh * dim);
        for (int base = 0; base < cpp; base += 32 * U) {
            float4 v[U];
            Raw4 raw[U];
            int32_t sl[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = base + u * 32 + lane;
                const int h = c / cpr;
                const int cc = c - h * cpr;
                const int hs = h < nh ? h : 0;
                const int32_t g = __shfl_sync(kFull, ph.row, hs);
                const int32_t s = __shfl_sync(kFull, ph.slot, hs);
                sl[u] = s;
                if (c < cpp) {
                    if (FMT == ENGRAM_FMT_F32) {
                        const float* src = s >= 0 ? ovr + (int64_t)s * dim : reinterpret_cast<const float*>(pm.row_ptr(rows, T.row_stride, g, i, h, nh));
                        v[u] = __ldg(reinterpret_cast<const float4*>(src) + cc);
                    } else if (s < 0) {
                        raw[u] = raw4<FMT>(pm.row_ptr(rows, T.row_stride, g, i, h, nh), cc, dim);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = base + u * 32 + lane;
                if (c < cpp) {
                    if (FMT != ENGRAM_FMT_F32) {
                        const int h = c / cpr;
                        const int cc = c - h * cpr;
                        v[u] = sl[u] >= 0 ? __ldg(reinterpret_cast<const float4*>(ovr + (int64_t)sl[u] * dim) + cc)
                                          : dq4<FMT>(raw[u], cc, s_kv);
                    }
                    __stcs(dst + c, v[u]);
                }
            }
        }
    }
    flush_hits(hits, hit_count, lane);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// bf16 residual chunk + (a + b), rounded to nearest even.
__device__ __forceinline__ uint4 pair_add(const uint4& r, const float* a, const float* b) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float s0 = __fadd_rn(a[2 * k], b[2 * k]);
        const float s1 = __fadd_rn(a[2 * k + 1], b[2 * k + 1]);
        o[k] = pack_bf16x2(__fadd_rn(bf16_lo(w[k]), s0), __fadd_rn(bf16_hi(w[k]), s1));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// PAIRSUM_ADD: residual[i, g*dim + c] += row(g)[c] + row(hpn+g)[c] in bf16.
// Per position: the residual chunks are loaded before the hash (they do not
// depend on it), the next position's tokens are prefetched, and every table
// row load of the round is issued before any value is used.
template <int FMT, int U>
__global__ void __launch_bounds__(256, 2) k_forward_pairsum(engram_table T, engram_overlay OV,
                                                            const int32_t* __restrict__ tokens,
                                                            const int32_t* __restrict__ seg_start, PosMap pm,
                                                            int64_t n, __nv_bfloat16* __restrict__ out,
                                                            int32_t* ids_out, int32_t* slots_out,
                                                            unsigned long long* hit_count) {
    __shared__ float s_kv[16];
    __shared__ HeadTab htab;
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
    head_tab_fill(htab, T);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int nh = T.n_heads, hpn = T.heads_per_ngram, dim = T.dim;
    const int cpr = dim >> 3;   // 8-value chunks per row
    const int cpp = hpn * cpr;  // chunks per position (one residual row of hpn*dim)
    const uint8_t* rows = static_cast<const uint8_t*>(T.rows);
    const float* ovr = OV.rows;
    unsigned long long hits = 0;
    TokCtx nxt{};
    if (warp0 < n) nxt = load_ctx(T, tokens, seg_start, pm.at(warp0));
    for (int64_t i = warp0; i < n; i += nwarps) {
        const TokCtx cur = nxt;
        uint4* res = reinterpret_cast<uint4*>(out + i * (int64_t)hpn * dim);
        PosHeads ph{0, -1};
        for (int base = 0; base < cpp; base += 32 * U) {
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int c = base + u * 32 + lane;
                if (c < cpp) r[u] = __ldcs(res + c);
            }
            if (base == 0) {
                ph = heads_of(T, htab, OV, cur, pm, i, lane);
                write_heads(ph, i, nh, lane, ids_out, slots_out, hits);
                if (i + nwarps < n) nxt = load_ctx(T, tokens, seg_start, pm.at(i + nwarps));
            }
            if constexpr (FMT == ENGRAM_FMT_F32) {
                float fa[U][8], fb[U][8];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = base + u * 32 + lane;
                    const int g = c / cpr;
                    const int cc = c - g * cpr;
                    const int gs = g < hpn ? g : 0;
                    const int32_t ga = __shfl_sync(kFull, ph.row, gs);
                    const int32_t s0 = __shfl_sync(kFull, ph.slot, gs);
                    const int32_t gb = __shfl_sync(kFull, ph.row, hpn + gs);
                    const int32_t s1 = __shfl_sync(kFull, ph.slot, hpn + gs);
                    if (c < cpp) {
                        ld_f8(s0 >= 0 ? ovr + (int64_t)s0 * dim + 8 * cc
                                      : reinterpret_cast<const float*>(pm.row_ptr(rows, T.row_stride, ga, i, gs, nh)) + 8 * cc, fa[u]);
                        ld_f8(s1 >= 0 ? ovr + (int64_t)s1 * dim + 8 * cc
                                      : reinterpret_cast<const float*>(pm.row_ptr(rows, T.row_stride, gb, i, hpn + gs, nh)) + 8 * cc, fb[u]);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = base + u * 32 + lane;
                    if (c < cpp) __stcs(res + c, pair_add(r[u], fa[u], fb[u]));
                }
            } else {
                Raw8 ra[U], rb[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = base + u * 32 + lane;
                    const int g = c / cpr;
                    const int cc = c - g * cpr;
                    const int gs = g < hpn ? g : 0;
                    const int32_t ga = __shfl_sync(kFull, ph.row, gs);
                    const int32_t s0 = __shfl_sync(kFull, ph.slot, gs);
                    const int32_t gb = __shfl_sync(kFull, ph.row, hpn + gs);
                    const int32_t s1 = __shfl_sync(kFull, ph.slot, hpn + gs);
                    if (c < cpp) {
                        if (s0 < 0) ra[u] = raw8<FMT>(pm.row_ptr(rows, T.row_stride, ga, i, gs, nh), cc, dim);
                        if (s1 < 0) rb[u] = raw8<FMT>(pm.row_ptr(rows, T.row_stride, gb, i, hpn + gs, nh), cc, dim);
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = base + u * 32 + lane;
                    const int g = c / cpr;
                    const int gs = g < hpn ? g : 0;
                    const int32_t s0 = __shfl_sync(kFull, ph.slot, gs);  // slots re-read: fewer live registers
                    const int32_t s1 = __shfl_sync(kFull, ph.slot, hpn + gs);
                    if (c < cpp) {
                        const int cc = c - g * cpr;
                        float a[8], b[8];
                        if (s0 >= 0) ld_f8(ovr + (int64_t)s0 * dim + 8 * cc, a);
                        else dq8<FMT>(ra[u], cc, s_kv, a);
                        if (s1 >= 0) ld_f8(ovr + (int64_t)s1 * dim + 8 * cc, b);
                        else dq8<FMT>(rb[u], cc, s_kv, b);
                        __stcs(res + c, pair_add(r[u], a, b));
                    }
                }
            }
        }
    }
    flush_hits(hits, hit_count, lane);
}

// ---- PAIRSUM_ADD for IQ4 tables: shared-memory staged, double-buffered warps ----
//
// Each warp owns two shared-memory buffers of one position each (the bf16
// residual row + the 16 resident table rows).  While position i is computed
// from one buffer, position i+nw's rows are already being copied into the
// other by cp.async, so no register holds data in flight and the hash, probe
// and DRAM latencies of one position hide behind the work of another.  The
// table rows are fetched even for heads the overlay serves (so the copies do
// not wait for the map probe); overlay rows are read from global memory (they
// stay L2-resident) when consumed.  Lane q of a group row handles values
// {32u+4m..+3} and {32u+16+4m..+3} (u = q/4, m = q%4): the low and high
// nibbles of the same four code bytes, decoded together through a 256-entry
// (kv[b&15], kv[b>>4]) table, with paired fp32 multiplies and adds.
constexpr int kStagedWarps = 4;
constexpr int kPairTableBytes = 256 * 8;

__device__ __forceinline__ void cp_async16_f(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit_f() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_f() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

// 8 values (two runs of 4) of one row at lane chunk q: v[k] = (value at 32u+4m+k, value at 32u+16+4m+k).
template <int FMT>
__device__ __forceinline__ void row_pairs(const uint8_t* row_smem, const float* ov_row, int q, int dim,
                                          const float2* pair_tab, float2* v) {
    const int u = q >> 2, m = q & 3;
    if (ov_row != nullptr) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(ov_row + 32 * u + 4 * m));
        const float4 b = __ldg(reinterpret_cast<const float4*>(ov_row + 32 * u + 16 + 4 * m));
        v[0] = make_float2(a.x, b.x);
        v[1] = make_float2(a.y, b.y);
        v[2] = make_float2(a.z, b.z);
        v[3] = make_float2(a.w, b.w);
        return;
    }
    uint32_t qs;
    float d;
    if (FMT == ENGRAM_FMT_IQ4_XS) {
        const uint8_t* sb = row_smem + (u >> 3) * 144;
        const int ib = u & 7;
        qs = *reinterpret_cast<const uint32_t*>(sb + ib * 16 + 4 * m);
        const uint2 hdr = *reinterpret_cast<const uint2*>(sb + 128);
        d = block_scale<ENGRAM_FMT_IQ4_XS>(hdr.x, hdr.y, ib);
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = __fmul2_rn(f2(d), pair_tab[(qs >> (8 * k)) & 0xffu]);
    } else {
        const int nb = dim >> 5;
        qs = *reinterpret_cast<const uint32_t*>(row_smem + u * 16 + 4 * m);
        d = half_bits_to_float(*reinterpret_cast<const unsigned short*>(row_smem + 16 * nb + 2 * u));
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = __fmul2_rn(pair_tab[(qs >> (8 * k)) & 0xffu], f2(d));
    }
}

template <int FMT>
__global__ void __launch_bounds__(kStagedWarps * 32) k_forward_pairsum_staged(
    engram_table T, engram_overlay OV, const int32_t* __restrict__ tokens, const int32_t* __restrict__ seg_start,
    PosMap pm, int64_t n, __nv_bfloat16* __restrict__ out, int32_t* ids_out, int32_t* slots_out,
    unsigned long long* hit_count, int buf_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    float2* pair_tab = reinterpret_cast<float2*>(smem);
    for (int b = threadIdx.x; b < 256; b += blockDim.x) pair_tab[b] = make_float2(kKvIq4[b & 15], kKvIq4[b >> 4]);
    __shared__ HeadTab htab;
    head_tab_fill(htab, T);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* wbuf = smem + kPairTableBytes + warp * 2 * buf_bytes;
    const int64_t nw = (int64_t)gridDim.x * kStagedWarps;
    int64_t i = (int64_t)blockIdx.x * kStagedWarps + warp;
    if (i >= n) return;  // no block-wide barrier follows
    const int nh = T.n_heads, hpn = T.heads_per_ngram, dim = T.dim;
    const int res_bytes = hpn * dim * 2;
    const int pieces = (int)(T.row_stride >> 4);
    const int row_pieces = nh * pieces;
    const uint8_t* rows = static_cast<const uint8_t*>(T.rows);

    auto issue = [&](int64_t pos, int32_t gid, int b) {
        uint8_t* bb = wbuf + b * buf_bytes;
        const uint4* src = reinterpret_cast<const uint4*>(out + pos * (int64_t)hpn * dim);
        for (int c = lane; c < (res_bytes >> 4); c += 32) cp_async16_f(bb + c * 16, src + c);
        for (int j0 = 0; j0 < row_pieces; j0 += 32) {
            const int j = j0 + lane;
            const int h = j / pieces;
            const int p = j - h * pieces;
            const int32_t g = __shfl_sync(kFull, gid, h < nh ? h : 0);
            if (j < row_pieces)
                cp_async16_f(bb + res_bytes + h * T.row_stride + p * 16, pm.row_ptr(rows, T.row_stride, g, pos, h, nh) + p * 16);
        }
        cp_async_commit_f();
    };

    TokCtx ctx = load_ctx(T, tokens, seg_start, pm.at(i));
    int32_t gid = lane < nh ? hash_ctx(T, htab, ctx, pm.at(i), lane) : 0;
    issue(i, lane < nh ? pm.row(i, lane, nh, gid) : 0, 0);
    int32_t slot = lane < nh ? overlay_slot(OV, gid) : -1;
    int64_t inext = i + nw;
    if (inext < n) ctx = load_ctx(T, tokens, seg_start, pm.at(inext));
    unsigned long long hits = 0;
    int b = 0;
    for (; i < n; i += nw, inext += nw) {
        const bool has_next = inext < n;
        int32_t gid_n = 0;
        if (has_next) {
            gid_n = lane < nh ? hash_ctx(T, htab, ctx, pm.at(inext), lane) : 0;
            issue(inext, lane < nh ? pm.row(inext, lane, nh, gid_n) : 0, b ^ 1);
            if (inext + nw < n) ctx = load_ctx(T, tokens, seg_start, pm.at(inext + nw));
        } else {
            cp_async_commit_f();  // one group per iteration keeps the wait count uniform
        }
        if (lane < nh) {
            if (ids_out) ids_out[i * nh + lane] = gid;
            if (slots_out) slots_out[i * nh + lane] = slot;
        }
        hits += (unsigned long long)__popc(__ballot_sync(kFull, lane < nh && slot >= 0));
        cp_async_wait_f<1>();
        __syncwarp();
        const uint8_t* bb = wbuf + b * buf_bytes;
        __nv_bfloat16* orow = out + i * (int64_t)hpn * dim;
        for (int g = 0; g < hpn; g++) {
            const int32_t sa = __shfl_sync(kFull, slot, g);
            const int32_t sb = __shfl_sync(kFull, slot, hpn + g);
            const uint8_t* ra = bb + res_bytes + g * T.row_stride;
            const uint8_t* rb = bb + res_bytes + (hpn + g) * T.row_stride;
            const float* oa = sa >= 0 ? OV.rows + (int64_t)sa * dim : nullptr;
            const float* ob = sb >= 0 ? OV.rows + (int64_t)sb * dim : nullptr;
            for (int q = lane; q < (dim >> 3); q += 32) {
                float2 va[4], vb[4];
                row_pairs<FMT>(ra, oa, q, dim, pair_tab, va);
                row_pairs<FMT>(rb, ob, q, dim, pair_tab, vb);
                const int v0 = g * dim + 32 * (q >> 2) + 4 * (q & 3);
                const uint2 r0 = *reinterpret_cast<const uint2*>(bb + 2 * v0);
                const uint2 r1 = *reinterpret_cast<const uint2*>(bb + 2 * (v0 + 16));
                const uint32_t w0[2] = {r0.x, r0.y}, w1[2] = {r1.x, r1.y};
                uint32_t o0[2], o1[2];
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    // values v0+2k, v0+2k+1 (low halves) and v0+16+2k, v0+16+2k+1 (high halves)
                    const float2 s_lo = __fadd2_rn(va[2 * k], vb[2 * k]);          // (v0+2k, v0+16+2k)
                    const float2 s_hi = __fadd2_rn(va[2 * k + 1], vb[2 * k + 1]);  // (v0+2k+1, v0+16+2k+1)
                    const float2 x0 = __fadd2_rn(make_float2(bf16_lo(w0[k]), bf16_hi(w0[k])), make_float2(s_lo.x, s_hi.x));
                    const float2 x1 = __fadd2_rn(make_float2(bf16_lo(w1[k]), bf16_hi(w1[k])), make_float2(s_lo.y, s_hi.y));
                    o0[k] = pack_bf16x2(x0.x, x0.y);
                    o1[k] = pack_bf16x2(x1.x, x1.y);
                }
                __stcs(reinterpret_cast<uint2*>(orow + v0), make_uint2(o0[0], o0[1]));
                __stcs(reinterpret_cast<uint2*>(orow + v0 + 16), make_uint2(o1[0], o1[1]));
            }
        }
        __syncwarp();  // buffer b is refilled next iteration
        slot = -1;
        if (has_next && lane < nh) slot = overlay_slot(OV, gid_n);
        gid = gid_n;
        b ^= 1;
    }
    cp_async_wait_f<0>();
    flush_hits(hits, hit_count, lane);
}

template <int FMT>
__global__ void __launch_bounds__(256) k_gather_rows(engram_table T, const int32_t* __restrict__ ids, int64_t n,
                                                     float* __restrict__ out) {
    __shared__ float s_kv[16];
    __shared__ HeadTab htab;
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
    head_tab_fill(htab, T);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int cpr = T.dim >> 2;
    const uint8_t* rows = static_cast<const uint8_t*>(T.rows);
    for (int64_t k = warp0; k < n; k += nwarps) {
        const int32_t g = __ldg(ids + k);
        const bool ok = g >= 0 && (int64_t)g < T.n_rows;
        float4* dst = reinterpret_cast<float4*>(out + k * (int64_t)T.dim);
        for (int c = lane; c < cpr; c += 32)
            dst[c] = !ok ? make_float4(0.f, 0.f, 0.f, 0.f)
                         : FMT == ENGRAM_FMT_F32
                               ? __ldg(reinterpret_cast<const float4*>(rows + (int64_t)g * T.row_stride) + c)
                               : dq4<FMT>(raw4<FMT>(rows + (int64_t)g * T.row_stride, c, T.dim), c, s_kv);
    }
}

// ---- PAIRSUM_ADD specialised for the table geometries in use --------------------
//
// Same staging as k_forward_pairsum_staged, with the geometry fixed at compile
// time (8 bigram + 8 trigram heads, FMT, DIM), so every index is a constant or
// a shift, and with the position pipeline one step deeper: while position k is
// computed from its buffer, position k+1's rows are in flight, position k+1's
// first overlay-map probe is in flight, and position k+2's tokens are in
// flight.  Codes are decoded through a 16-float shared table (conflict-free:
// the 16 entries sit in 16 banks) and scaled with paired fp32 multiplies.
constexpr int kXsWarps = 4;

struct ProbeState {
    uint32_t pos;   // current probe position
    int32_t key;    // key loaded at pos
    int32_t slot;   // slot loaded at pos
};

__device__ __forceinline__ ProbeState probe_start(const engram_overlay& OV, int32_t gid) {
    ProbeState p{0u, -1, -1};
    if (OV.n_rows == 0) return p;
    p.pos = map_home(gid, OV.capacity);
    p.key = __ldg(OV.map_keys + p.pos);
    p.slot = __ldg(OV.map_slots + p.pos);
    return p;
}

__device__ __forceinline__ int32_t probe_finish(const engram_overlay& OV, int32_t gid, ProbeState p) {
    if (OV.n_rows == 0) return -1;
    const uint32_t mask = (uint32_t)OV.capacity - 1u;
    for (int64_t probe = 0; probe < OV.capacity; probe++) {
        if (p.key == gid) return p.slot;
        if (p.key == -1) return -1;
        p.pos = (p.pos + 1u) & mask;
        p.key = __ldg(OV.map_keys + p.pos);
        p.slot = __ldg(OV.map_slots + p.pos);
    }
    return -1;
}

template <int FMT, int DIM>
struct XsGeom {
    static constexpr int HPN = 8, NH = 16;
    static constexpr int ROW = FMT == ENGRAM_FMT_IQ4_XS ? 144 * (DIM / 256) : ((DIM / 32) * 18 + 15) / 16 * 16;
    static constexpr int RES = HPN * DIM * 2;
    static constexpr int BUF = RES + NH * ROW;
    static constexpr int PIECES = ROW / 16;
    static constexpr int NQ = (DIM / 8 + 31) / 32;  // 8-value lane chunks per row per lane
};

// Values [8q, 8q+8) of one row as four float pairs (v[k] = values 8q+2k, 8q+2k+1).
template <int FMT, int DIM>
// ov: the overlay serves this head, and ovv holds its values [8q, 8q+8) (loaded ahead by the caller).
__device__ __forceinline__ void xs_row(const uint8_t* row, bool ov, const float4* ovv, int q, const float* kv,
                                       float2* v) {
    if (ov) {
        const float4 a = ovv[0];
        const float4 b = ovv[1];
        v[0] = make_float2(a.x, a.y);
        v[1] = make_float2(a.z, a.w);
        v[2] = make_float2(b.x, b.y);
        v[3] = make_float2(b.z, b.w);
        return;
    }
    const int u = q >> 2, k = q & 3;  // 32-value sub-block u; k selects bytes (k&1)*8.. and the nibble half k>>1
    const int sh = (k >> 1) * 4;
    uint2 qs;
    float d;
    if (FMT == ENGRAM_FMT_IQ4_XS) {
        const uint8_t* sb = row + (u >> 3) * 144;
        const int ib = u & 7;
        qs = *reinterpret_cast<const uint2*>(sb + ib * 16 + (k & 1) * 8);
        const uint2 hdr = *reinterpret_cast<const uint2*>(sb + 128);
        d = block_scale<ENGRAM_FMT_IQ4_XS>(hdr.x, hdr.y, ib);
#pragma unroll
        for (int j = 0; j < 2; j++)
            v[j] = __fmul2_rn(f2(d), make_float2(kv[(qs.x >> (16 * j + sh)) & 15u], kv[(qs.x >> (16 * j + 8 + sh)) & 15u]));
#pragma unroll
        for (int j = 0; j < 2; j++)
            v[2 + j] = __fmul2_rn(f2(d), make_float2(kv[(qs.y >> (16 * j + sh)) & 15u], kv[(qs.y >> (16 * j + 8 + sh)) & 15u]));
    } else {
        qs = *reinterpret_cast<const uint2*>(row + u * 16 + (k & 1) * 8);
        d = half_bits_to_float(*reinterpret_cast<const unsigned short*>(row + 16 * (DIM / 32) + 2 * u));
#pragma unroll
        for (int j = 0; j < 2; j++)
            v[j] = __fmul2_rn(make_float2(kv[(qs.x >> (16 * j + sh)) & 15u], kv[(qs.x >> (16 * j + 8 + sh)) & 15u]), f2(d));
#pragma unroll
        for (int j = 0; j < 2; j++)
            v[2 + j] = __fmul2_rn(make_float2(kv[(qs.y >> (16 * j + sh)) & 15u], kv[(qs.y >> (16 * j + 8 + sh)) & 15u]), f2(d));
    }
}

template <int FMT, int DIM, bool SHARD>
__global__ void __launch_bounds__(kXsWarps * 32) k_forward_pairsum_fixed(
    engram_table T, engram_overlay OV, const int32_t* __restrict__ tokens, const int32_t* __restrict__ seg_start,
    PosMap pm, int64_t n, __nv_bfloat16* __restrict__ out, int32_t* ids_out, int32_t* slots_out,
    unsigned long long* hit_count) {
    using G = XsGeom<FMT, DIM>;
    extern __shared__ __align__(16) uint8_t smem[];
    float* kv = reinterpret_cast<float*>(smem);
    __shared__ HeadTab htab;
    if (threadIdx.x < 16) kv[threadIdx.x] = kKvIq4[threadIdx.x];
    head_tab_fill(htab, T);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* wbuf = smem + 64 + warp * 2 * G::BUF;
    const int64_t nw = (int64_t)gridDim.x * kXsWarps;
    const int64_t first = (int64_t)blockIdx.x * kXsWarps + warp;
    if (first >= n) return;  // no block-wide barrier follows
    const uint8_t* rows = static_cast<const uint8_t*>(T.rows);
    const bool head_lane = lane < G::NH;

    // Copies position pos's residual and the table rows of its heads that the
    // overlay does not serve (slot < 0; an overlay head reads its fp32 row instead).
    // gid: the head lane's row in T.rows; with SHARD, hp: the head lane's row address
    // (computed when the position was hashed, its row index loaded an iteration earlier).
    auto issue = [&](int64_t pos, int32_t gid, unsigned long long hp, int32_t slot, int b) {
        uint8_t* bb = wbuf + b * G::BUF;
        const uint4* src = reinterpret_cast<const uint4*>(out + pos * (G::HPN * DIM));
#pragma unroll
        for (int c = 0; c < G::RES / 16 / 32; c++) cp_async16_f(bb + (c * 32 + lane) * 16, src + c * 32 + lane);
#pragma unroll
        for (int j0 = 0; j0 < G::NH * G::PIECES; j0 += 32) {
            const int j = j0 + lane;
            const int h = j / G::PIECES;
            const int p = j - h * G::PIECES;
            const int32_t sl = __shfl_sync(kFull, slot, h < G::NH ? h : 0);
            const uint8_t* src;
            if (SHARD) {
                src = reinterpret_cast<const uint8_t*>(__shfl_sync(kFull, hp, h < G::NH ? h : 0));
            } else {
                const int32_t g = __shfl_sync(kFull, gid, h < G::NH ? h : 0);
                src = rows + (int64_t)g * G::ROW;
            }
            if (j < G::NH * G::PIECES && sl < 0) cp_async16_f(bb + G::RES + h * G::ROW + p * 16, src + p * 16);
        }
        cp_async_commit_f();
    };

    // pipeline state: position k (gid, slot), k+1 (gid, probe in flight), k+2 (tokens in flight)
    int64_t i = first;
    TokCtx c0 = load_ctx(T, tokens, seg_start, pm.at(i));
    int32_t gid = head_lane ? hash_ctx(T, htab, c0, pm.at(i), lane) : 0;
    int32_t slot = head_lane ? probe_finish(OV, gid, probe_start(OV, gid)) : -1;
    auto head_ptr = [&](int64_t pos, int32_t g, int32_t k_pre) -> unsigned long long {
        return SHARD && head_lane
                   ? reinterpret_cast<unsigned long long>(pm.row_ptr_pre(rows, G::ROW, g, k_pre, pos, lane, G::NH))
                   : 0ull;
    };
    auto srix_of = [&](int64_t pos) -> int32_t {
        return SHARD && pm.srix && head_lane ? __ldg(pm.srix + pos * G::NH + lane) : 0;
    };
    issue(i, head_lane ? pm.row(i, lane, G::NH, gid) : 0, head_ptr(i, gid, srix_of(i)), slot, 0);
    int64_t i1 = i + nw;
    int32_t gid1 = 0;
    ProbeState pr1{0u, -1, -1};
    if (i1 < n) {
        const TokCtx c1 = load_ctx(T, tokens, seg_start, pm.at(i1));
        gid1 = head_lane ? hash_ctx(T, htab, c1, pm.at(i1), lane) : 0;
        if (head_lane) pr1 = probe_start(OV, gid1);
    }
    int32_t row1 = head_lane && i1 < n ? pm.row(i1, lane, G::NH, gid1) : 0;
    unsigned long long hp1 = i1 < n ? head_ptr(i1, gid1, srix_of(i1)) : 0ull;
    // tokens (and gathered-row or exchanged-row indices) of position k+2 load one iteration ahead
    TokCtx c2{};
    int32_t r2 = 0, s2 = 0;
    if (i1 + nw < n) {
        c2 = load_ctx(T, tokens, seg_start, pm.at(i1 + nw));
        if (pm.rix && head_lane) r2 = __ldg(pm.rix + (i1 + nw) * G::NH + lane);
        s2 = srix_of(i1 + nw);
    }
    unsigned long long hits = 0;
    int b = 0;
    for (; i < n; i += nw) {
        const int64_t inext = i + nw;
        // the next position's probe (its key loads were issued an iteration ago) decides which rows to copy
        const int32_t slot1 = (inext < n && head_lane) ? probe_finish(OV, gid1, pr1) : -1;
        if (inext < n) issue(inext, row1, hp1, slot1, b ^ 1);
        else cp_async_commit_f();
        if (slot1 >= 0) {  // the next position's overlay row: pull it into L1 while this position computes
            const char* orow_p = reinterpret_cast<const char*>(OV.rows + (int64_t)slot1 * DIM);
#pragma unroll
            for (int l = 0; l < DIM * 4 / 128; l++)
                asm volatile("prefetch.global.L1 [%0];" ::"l"(orow_p + 128 * l));
        }
        if (head_lane) {
            if (ids_out) ids_out[i * G::NH + lane] = gid;
            if (slots_out) slots_out[i * G::NH + lane] = slot;
        }
        hits += (unsigned long long)__popc(__ballot_sync(kFull, head_lane && slot >= 0));
        cp_async_wait_f<1>();
        __syncwarp();
        const uint8_t* bb = wbuf + b * G::BUF;
        __nv_bfloat16* orow = out + i * (G::HPN * DIM);
        // The overlay rows of group g + 2's two heads load while group g computes: their L2 latency
        // overlaps two groups' dequantisation instead of stalling one.  A ring of 3 register slots.
        constexpr int kAhead = 2, kRing = kAhead + 1;
        float4 ova[kRing][G::NQ][2], ovb[kRing][G::NQ][2];
        bool oha[kRing], ohb[kRing];
        auto ov_fetch = [&](int g, float4 (&va)[G::NQ][2], float4 (&vb)[G::NQ][2], bool& ha, bool& hb) {
            const int32_t sa = __shfl_sync(kFull, slot, g);
            const int32_t sb = __shfl_sync(kFull, slot, G::HPN + g);
            ha = sa >= 0;
            hb = sb >= 0;
#pragma unroll
            for (int jq = 0; jq < G::NQ; jq++) {
                const int q = lane + 32 * jq;
                if (q < DIM / 8) {
                    if (ha) {
                        const float4* p = reinterpret_cast<const float4*>(OV.rows + (int64_t)sa * DIM + 8 * q);
                        va[jq][0] = __ldg(p);
                        va[jq][1] = __ldg(p + 1);
                    }
                    if (hb) {
                        const float4* p = reinterpret_cast<const float4*>(OV.rows + (int64_t)sb * DIM + 8 * q);
                        vb[jq][0] = __ldg(p);
                        vb[jq][1] = __ldg(p + 1);
                    }
                }
            }
        };
#pragma unroll
        for (int g = 0; g < kAhead && g < G::HPN; g++) ov_fetch(g, ova[g], ovb[g], oha[g], ohb[g]);
#pragma unroll
        for (int g = 0; g < G::HPN; g++) {
            const int r = g % kRing;
            if (g + kAhead < G::HPN) {
                const int rn = (g + kAhead) % kRing;
                ov_fetch(g + kAhead, ova[rn], ovb[rn], oha[rn], ohb[rn]);
            }
            const bool ha = oha[r], hb = ohb[r];
#pragma unroll
            for (int jq = 0; jq < G::NQ; jq++) {
                const int q = lane + 32 * jq;
                if (q < DIM / 8) {
                    float2 va[4], vb[4];
                    xs_row<FMT, DIM>(bb + G::RES + g * G::ROW, ha, ova[r][jq], q, kv, va);
                    xs_row<FMT, DIM>(bb + G::RES + (G::HPN + g) * G::ROW, hb, ovb[r][jq], q, kv, vb);
                    const int v0 = g * DIM + 8 * q;
                    const uint4 r = *reinterpret_cast<const uint4*>(bb + 2 * v0);
                    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
                    uint32_t o[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float2 x = __fadd2_rn(make_float2(bf16_lo(w[k]), bf16_hi(w[k])), __fadd2_rn(va[k], vb[k]));
                        o[k] = pack_bf16x2(x.x, x.y);
                    }
                    __stcs(reinterpret_cast<uint4*>(orow + v0), make_uint4(o[0], o[1], o[2], o[3]));
                }
            }
        }
        __syncwarp();  // buffer b is refilled next iteration
        // advance the pipeline: k+2 is hashed and probed, k+3's tokens load
        gid = gid1;
        slot = slot1;
        const int64_t i2 = inext + nw;
        if (i2 < n) {
            gid1 = head_lane ? hash_ctx(T, htab, c2, pm.at(i2), lane) : 0;
            if (head_lane) pr1 = probe_start(OV, gid1);
            row1 = pm.rix ? (r2 < 0 ? 0 : r2) : gid1;
            hp1 = head_ptr(i2, gid1, s2);
            if (i2 + nw < n) {
                c2 = load_ctx(T, tokens, seg_start, pm.at(i2 + nw));
                if (pm.rix && head_lane) r2 = __ldg(pm.rix + (i2 + nw) * G::NH + lane);
                s2 = srix_of(i2 + nw);
            }
        }
        b ^= 1;
    }
    cp_async_wait_f<0>();
    flush_hits(hits, hit_count, lane);
}

template <int FMT, int DIM, bool SHARD>
void launch_pairsum_fixed_k(const engram_table& T, const engram_overlay& OV, const int32_t* tokens,
                            const int32_t* seg_start, PosMap pm, int64_t n, __nv_bfloat16* out, int32_t* ids_out,
                            int32_t* slots_out, unsigned long long* hit_count, cudaStream_t s) {
    using G = XsGeom<FMT, DIM>;
    const int smem = 64 + kXsWarps * 2 * G::BUF;
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaFuncSetAttribute(k_forward_pairsum_fixed<FMT, DIM, SHARD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
        configured[dev] = true;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_forward_pairsum_fixed<FMT, DIM, SHARD>, kXsWarps * 32,
                                                  smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t want = (n + kXsWarps - 1) / kXsWarps;
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int blocks = (int)(want < cap ? want : cap);
    k_forward_pairsum_fixed<FMT, DIM, SHARD><<<blocks, kXsWarps * 32, smem, s>>>(T, OV, tokens, seg_start, pm, n,
                                                                                 out, ids_out, slots_out, hit_count);
}

// The row-sharded read is a separate instantiation, so the resident-table kernel carries no shard logic.
template <int FMT, int DIM>
void launch_pairsum_fixed(const engram_table& T, const engram_overlay& OV, const int32_t* tokens,
                          const int32_t* seg_start, PosMap pm, int64_t n, __nv_bfloat16* out, int32_t* ids_out,
                          int32_t* slots_out, unsigned long long* hit_count, cudaStream_t s) {
    if (pm.sharded()) launch_pairsum_fixed_k<FMT, DIM, true>(T, OV, tokens, seg_start, pm, n, out, ids_out, slots_out,
                                                         hit_count, s);
    else launch_pairsum_fixed_k<FMT, DIM, false>(T, OV, tokens, seg_start, pm, n, out, ids_out, slots_out,
                                                 hit_count, s);
}

// Runs the compile-time specialisation for this table if there is one.
template <int FMT>
bool launch_pairsum_specialised(const engram_table& T, const engram_overlay& OV, const int32_t* tokens,
                                const int32_t* seg_start, PosMap pm, int64_t n, __nv_bfloat16* out,
                                int32_t* ids_out, int32_t* slots_out, unsigned long long* hit_count, cudaStream_t s) {
    if (T.heads_per_ngram != 8 || T.n_heads != 16) return false;
    if (FMT == ENGRAM_FMT_IQ4_XS && T.dim == 256) {
        launch_pairsum_fixed<ENGRAM_FMT_IQ4_XS, 256>(T, OV, tokens, seg_start, pm, n, out, ids_out, slots_out, hit_count, s);
        return true;
    }
    if (FMT == ENGRAM_FMT_IQ4_XS && T.dim == 512) {
        launch_pairsum_fixed<ENGRAM_FMT_IQ4_XS, 512>(T, OV, tokens, seg_start, pm, n, out, ids_out, slots_out, hit_count, s);
        return true;
    }
    if (FMT == ENGRAM_FMT_IQ4_NL && T.dim == 160) {
        launch_pairsum_fixed<ENGRAM_FMT_IQ4_NL, 160>(T, OV, tokens, seg_start, pm, n, out, ids_out, slots_out, hit_count, s);
        return true;
    }
    return false;
}

constexpr int kMaxStagedSmem = 200 * 1024;

inline int staged_buf_bytes(const engram_table& T) {
    return (int)(T.heads_per_ngram * T.dim * 2 + T.n_heads * T.row_stride);
}
inline int staged_smem_bytes(const engram_table& T) {
    return kPairTableBytes + kStagedWarps * 2 * staged_buf_bytes(T);
}

template <int FMT>
void launch_pairsum_staged(const engram_table& T, const engram_overlay& OV, const int32_t* tokens,
                           const int32_t* seg_start, PosMap pm, int64_t n, __nv_bfloat16* out, int32_t* ids_out,
                           int32_t* slots_out, unsigned long long* hit_count, cudaStream_t s) {
    const int smem = staged_smem_bytes(T);
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured[dev] < smem) {
        cudaFuncSetAttribute(k_forward_pairsum_staged<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxStagedSmem);
        configured[dev] = kMaxStagedSmem;
    }
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_forward_pairsum_staged<FMT>, kStagedWarps * 32, smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t want = (n + kStagedWarps - 1) / kStagedWarps;
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int blocks = (int)(want < cap ? want : cap);
    k_forward_pairsum_staged<FMT><<<blocks, kStagedWarps * 32, smem, s>>>(T, OV, tokens, seg_start, pm, n, out, ids_out,
                                                                          slots_out, hit_count, staged_buf_bytes(T));
}

template <int FMT>
void launch_forward(const engram_table& T, const engram_overlay& OV, const int32_t* tokens, const int32_t* seg_start,
                    PosMap pm, int64_t n, int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                    unsigned long long* hit_count, cudaStream_t s) {
    const int threads = 256;
    const int64_t warps_needed = n;
    const int64_t blocks_needed = (warps_needed + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 2;  // persistent: the two blocks per SM that fit
    const int blocks = (int)(blocks_needed < cap ? blocks_needed : cap);
    if (mode == ENGRAM_MODE_CONCAT_F32)
        k_forward_concat<FMT, FMT == ENGRAM_FMT_F32 ? 16 : 8><<<blocks, threads, 0, s>>>(T, OV, tokens, seg_start, pm, n, (float*)out, ids_out,
                                                            slots_out, hit_count);
    else if (FMT != ENGRAM_FMT_F32 && launch_pairsum_specialised<FMT>(T, OV, tokens, seg_start, pm, n, (__nv_bfloat16*)out,
                                                                      ids_out, slots_out, hit_count, s)) {
    } else if (FMT != ENGRAM_FMT_F32 && staged_smem_bytes(T) <= kMaxStagedSmem)
        launch_pairsum_staged<FMT>(T, OV, tokens, seg_start, pm, n, (__nv_bfloat16*)out, ids_out, slots_out,
                                   hit_count, s);
    else
        k_forward_pairsum<FMT, 4><<<blocks, threads, 0, s>>>(T, OV, tokens, seg_start, pm, n, (__nv_bfloat16*)out,
                                                             ids_out, slots_out, hit_count);
}

}  // namespace

extern "C" int engram_hash(const engram_table* t, const int32_t* tokens, const int32_t* seg_start, int64_t t0,
                           int64_t n, int32_t* ids_out, void* stream) {
    if (!t || t0 < 0 || n < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!tokens || !ids_out) return ENGRAM_ERR_ARG;
    const int64_t total = n * t->n_heads;
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads, cap = (int64_t)sm_count() * 16;
    k_hash<<<(int)(want < cap ? want : cap), threads, 0, (cudaStream_t)stream>>>(*t, tokens, seg_start,
                                                                                PosMap{t0, nullptr, 0, nullptr}, n, ids_out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

namespace {
int forward_impl(const engram_table* t, const engram_overlay* ov, const int32_t* tokens, const int32_t* seg_start,
                 PosMap pm, int64_t n, int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                 int64_t* hit_count, void* stream) {
    if (!t || n < 0) return ENGRAM_ERR_ARG;
    if (mode != ENGRAM_MODE_CONCAT_F32 && mode != ENGRAM_MODE_PAIRSUM_ADD_BF16) return ENGRAM_ERR_ARG;
    if (mode == ENGRAM_MODE_PAIRSUM_ADD_BF16) {
        if (t->ngram_size != 3 || t->dim % 8) return ENGRAM_ERR_FORMAT;
    }
    engram_overlay OV;
    if (ov) {
        OV = *ov;
        if (OV.n_rows < 0) return ENGRAM_ERR_ARG;
        if (OV.n_rows > 0) {
            if (!OV.rows || !OV.map_keys || !OV.map_slots || !aligned16(OV.rows)) return ENGRAM_ERR_ARG;
            if ((OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows) return ENGRAM_ERR_RANGE;
        }
    } else {
        OV = engram_overlay{nullptr, 0, nullptr, nullptr, 0};
    }
    if (n == 0) return ENGRAM_OK;
    if (!tokens || !out || !aligned16(out)) return ENGRAM_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* hc = reinterpret_cast<unsigned long long*>(hit_count);
    switch (t->fmt) {
        case ENGRAM_FMT_F32: launch_forward<ENGRAM_FMT_F32>(*t, OV, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hc, s); break;
        case ENGRAM_FMT_IQ4_NL: launch_forward<ENGRAM_FMT_IQ4_NL>(*t, OV, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hc, s); break;
        case ENGRAM_FMT_IQ4_XS: launch_forward<ENGRAM_FMT_IQ4_XS>(*t, OV, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hc, s); break;
        default: return ENGRAM_ERR_FORMAT;
    }
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
}  // namespace

extern "C" int engram_forward(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                              const int32_t* seg_start, int64_t t0, int64_t n, int32_t mode, void* out,
                              int32_t* ids_out, int32_t* slots_out, int64_t* hit_count, void* stream) {
    if (t0 < 0) return ENGRAM_ERR_ARG;
    return forward_impl(t, ov, tokens, seg_start, PosMap{t0, nullptr, 0, nullptr}, n, mode, out, ids_out, slots_out, hit_count,
                        stream);
}

extern "C" int engram_forward_indirect(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                       const int32_t* seg_start, int64_t t0, int64_t n, const int32_t* row_index,
                                       int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                       int64_t* hit_count, void* stream) {
    if (t0 < 0 || (n > 0 && !row_index)) return ENGRAM_ERR_ARG;
    return forward_impl(t, ov, tokens, seg_start, PosMap{t0, nullptr, 0, row_index}, n, mode, out, ids_out, slots_out,
                        hit_count, stream);
}

namespace {
int sharded_map(PosMap& pm, const void* shard_rows, int32_t world, int32_t rank) {
    if (!shard_rows || world < 1 || world > 1024 || rank < 0 || rank >= world) return ENGRAM_ERR_ARG;
    pm.shard = static_cast<const uint8_t* const*>(shard_rows);
    pm.world = (uint32_t)world;
    pm.rank = (uint32_t)rank;
    pm.wshift = (world & (world - 1)) == 0 ? __builtin_ctz((unsigned)world) : -1;
    return ENGRAM_OK;
}
}  // namespace

extern "C" int64_t engram_stage_bytes(const engram_table* t, int64_t n) {
    if (!t || n < 0) return ENGRAM_ERR_ARG;
    return n * t->n_heads * t->row_stride;
}

extern "C" int engram_stage_sharded(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                    const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                    int32_t world, int32_t rank, void* stage, int32_t max_blocks, void* stream) {
    if (!t || t0 < 0 || n < 0 || max_blocks < 0) return ENGRAM_ERR_ARG;
    PosMap pm{t0, nullptr, 0, nullptr};
    const int st = sharded_map(pm, shard_rows, world, rank);
    if (st != ENGRAM_OK) return st;
    if (t->row_stride % 16 || t->n_heads < 1 || t->n_heads > 32) return ENGRAM_ERR_FORMAT;
    if (n == 0 || world == 1) return ENGRAM_OK;  // one rank: every row is local
    if (!tokens || !stage || !aligned16(stage)) return ENGRAM_ERR_ARG;
    engram_overlay OV{nullptr, 0, nullptr, nullptr, 0};
    if (ov && ov->n_rows > 0) {
        OV = *ov;
        if (!OV.map_keys || !OV.map_slots || (OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows)
            return ENGRAM_ERR_ARG;
    }
    const int64_t want = (n + 7) / 8;
    const int64_t cap = max_blocks > 0 ? max_blocks : (int64_t)sm_count() * 8;
    k_stage_sharded<<<(int)(want < cap ? want : cap), 256, 0, (cudaStream_t)stream>>>(*t, OV, tokens, seg_start, pm, n,
                                                                                       static_cast<uint8_t*>(stage));
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_forward_staged(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                     const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                     int32_t world, int32_t rank, const void* stage, int32_t mode, void* out,
                                     int32_t* ids_out, int32_t* slots_out, int64_t* hit_count, void* stream) {
    if (t0 < 0) return ENGRAM_ERR_ARG;
    PosMap pm{t0, nullptr, 0, nullptr};
    const int st = sharded_map(pm, shard_rows, world, rank);
    if (st != ENGRAM_OK) return st;
    if (world > 1 && n > 0 && (!stage || !aligned16(stage))) return ENGRAM_ERR_ARG;
    pm.stage = world > 1 ? static_cast<const uint8_t*>(stage) : nullptr;
    return forward_impl(t, ov, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hit_count, stream);
}

extern "C" int engram_forward_sharded(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                      const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                      int32_t world, int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                      int64_t* hit_count, void* stream) {
    if (t0 < 0) return ENGRAM_ERR_ARG;
    PosMap pm{t0, nullptr, 0, nullptr};
    const int st = sharded_map(pm, shard_rows, world, 0);
    if (st != ENGRAM_OK) return st;
    return forward_impl(t, ov, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hit_count, stream);
}

extern "C" int engram_forward_at(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                 int64_t n_tokens, const int32_t* seg_start, const int64_t* positions, int64_t n,
                                 int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out, int64_t* hit_count,
                                 void* stream) {
    if (n_tokens < 1 || (n > 0 && !positions)) return ENGRAM_ERR_ARG;
    return forward_impl(t, ov, tokens, seg_start, PosMap{0, positions, n_tokens, nullptr}, n, mode, out, ids_out, slots_out,
                        hit_count, stream);
}

extern "C" int engram_gather_rows(const engram_table* t, const int32_t* ids, int64_t n, float* out, void* stream) {
    if (!t || n < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!ids || !out || !aligned16(out)) return ENGRAM_ERR_ARG;
    const int64_t want = (n + 7) / 8, cap = (int64_t)sm_count() * 8;
    const int blocks = (int)(want < cap ? want : cap);
    cudaStream_t s = (cudaStream_t)stream;
    switch (t->fmt) {
        case ENGRAM_FMT_F32: k_gather_rows<ENGRAM_FMT_F32><<<blocks, 256, 0, s>>>(*t, ids, n, out); break;
        case ENGRAM_FMT_IQ4_NL: k_gather_rows<ENGRAM_FMT_IQ4_NL><<<blocks, 256, 0, s>>>(*t, ids, n, out); break;
        case ENGRAM_FMT_IQ4_XS: k_gather_rows<ENGRAM_FMT_IQ4_XS><<<blocks, 256, 0, s>>>(*t, ids, n, out); break;
        default: return ENGRAM_ERR_FORMAT;
    }
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_forward_exchanged(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                        const int32_t* seg_start, int64_t t0, int64_t n, const void* local_rows,
                                        int32_t world, int32_t rank, const void* recv_rows, const int32_t* row_index,
                                        int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                        int64_t* hit_count, void* stream) {
    if (!t || t0 < 0 || world < 1 || world > 1024 || rank < 0 || rank >= world) return ENGRAM_ERR_ARG;
    if (n > 0 && (!local_rows || !aligned16(local_rows))) return ENGRAM_ERR_ARG;
    if (n > 0 && world > 1 && (!recv_rows || !row_index || !aligned16(recv_rows))) return ENGRAM_ERR_ARG;
    if (t->row_stride % 16) return ENGRAM_ERR_FORMAT;
    PosMap pm{t0, nullptr, 0, nullptr};
    pm.world = (uint32_t)world;
    pm.rank = (uint32_t)rank;
    pm.wshift = (world & (world - 1)) == 0 ? __builtin_ctz((unsigned)world) : -1;
    pm.local = static_cast<const uint8_t*>(local_rows);
    if (world > 1) {
        pm.stage = static_cast<const uint8_t*>(recv_rows);
        pm.srix = row_index;
    }
    return forward_impl(t, ov, tokens, seg_start, pm, n, mode, out, ids_out, slots_out, hit_count, stream);
}
