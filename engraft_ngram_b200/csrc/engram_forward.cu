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
};

__device__ __forceinline__ PosHeads heads_of(const engram_table& T, const engram_overlay& OV, const TokCtx& c,
                                             int64_t t, int lane) {
    PosHeads r{0, -1};
    if (lane < T.n_heads) {
        r.gid = hash_ctx(T, c, t, lane);
        r.slot = overlay_slot(OV, r.gid);
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
                                              const int32_t* __restrict__ seg_start, int64_t t0, int64_t n,
                                              int32_t* __restrict__ ids_out) {
    const int nh = T.n_heads;
    const int64_t total = n * nh;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < total; k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = k / nh;
        const int h = (int)(k - i * nh);
        ids_out[k] = hash_row(T, tokens, seg_start, t0 + i, h);
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
                                                           const int32_t* __restrict__ seg_start, int64_t t0,
                                                           int64_t n, float* __restrict__ out, int32_t* ids_out,
                                                           int32_t* slots_out, unsigned long long* hit_count) {
    __shared__ float s_kv[16];
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
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
    if (warp0 < n) nxt = load_ctx(T, tokens, seg_start, t0 + warp0);
    for (int64_t i = warp0; i < n; i += nwarps) {
        const TokCtx cur = nxt;
        const PosHeads ph = heads_of(T, OV, cur, t0 + i, lane);
        write_heads(ph, i, nh, lane, ids_out, slots_out, hits);
        if (i + nwarps < n) nxt = load_ctx(T, tokens, seg_start, t0 + i + nwarps);
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
                const int32_t g = __shfl_sync(kFull, ph.gid, hs);
                const int32_t s = __shfl_sync(kFull, ph.slot, hs);
                sl[u] = s;
                if (c < cpp) {
                    if (FMT == ENGRAM_FMT_F32) {
                        const float* src = s >= 0 ? ovr + (int64_t)s * dim : reinterpret_cast<const float*>(rows + (int64_t)g * T.row_stride);
                        v[u] = __ldg(reinterpret_cast<const float4*>(src) + cc);
                    } else if (s < 0) {
                        raw[u] = raw4<FMT>(rows + (int64_t)g * T.row_stride, cc, dim);
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
                                                            const int32_t* __restrict__ seg_start, int64_t t0,
                                                            int64_t n, __nv_bfloat16* __restrict__ out,
                                                            int32_t* ids_out, int32_t* slots_out,
                                                            unsigned long long* hit_count) {
    __shared__ float s_kv[16];
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
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
    if (warp0 < n) nxt = load_ctx(T, tokens, seg_start, t0 + warp0);
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
                ph = heads_of(T, OV, cur, t0 + i, lane);
                write_heads(ph, i, nh, lane, ids_out, slots_out, hits);
                if (i + nwarps < n) nxt = load_ctx(T, tokens, seg_start, t0 + i + nwarps);
            }
            if constexpr (FMT == ENGRAM_FMT_F32) {
                float fa[U][8], fb[U][8];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int c = base + u * 32 + lane;
                    const int g = c / cpr;
                    const int cc = c - g * cpr;
                    const int gs = g < hpn ? g : 0;
                    const int32_t ga = __shfl_sync(kFull, ph.gid, gs);
                    const int32_t s0 = __shfl_sync(kFull, ph.slot, gs);
                    const int32_t gb = __shfl_sync(kFull, ph.gid, hpn + gs);
                    const int32_t s1 = __shfl_sync(kFull, ph.slot, hpn + gs);
                    if (c < cpp) {
                        ld_f8(s0 >= 0 ? ovr + (int64_t)s0 * dim + 8 * cc
                                      : reinterpret_cast<const float*>(rows + (int64_t)ga * T.row_stride) + 8 * cc, fa[u]);
                        ld_f8(s1 >= 0 ? ovr + (int64_t)s1 * dim + 8 * cc
                                      : reinterpret_cast<const float*>(rows + (int64_t)gb * T.row_stride) + 8 * cc, fb[u]);
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
                    const int32_t ga = __shfl_sync(kFull, ph.gid, gs);
                    const int32_t s0 = __shfl_sync(kFull, ph.slot, gs);
                    const int32_t gb = __shfl_sync(kFull, ph.gid, hpn + gs);
                    const int32_t s1 = __shfl_sync(kFull, ph.slot, hpn + gs);
                    if (c < cpp) {
                        if (s0 < 0) ra[u] = raw8<FMT>(rows + (int64_t)ga * T.row_stride, cc, dim);
                        if (s1 < 0) rb[u] = raw8<FMT>(rows + (int64_t)gb * T.row_stride, cc, dim);
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

template <int FMT>
__global__ void __launch_bounds__(256) k_gather_rows(engram_table T, const int32_t* __restrict__ ids, int64_t n,
                                                     float* __restrict__ out) {
    __shared__ float s_kv[16];
    if (threadIdx.x < 16) s_kv[threadIdx.x] = kKvIq4[threadIdx.x];
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

template <int FMT>
void launch_forward(const engram_table& T, const engram_overlay& OV, const int32_t* tokens, const int32_t* seg_start,
                    int64_t t0, int64_t n, int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                    unsigned long long* hit_count, cudaStream_t s) {
    const int threads = 256;
    const int64_t warps_needed = n;
    const int64_t blocks_needed = (warps_needed + 7) / 8;
    const int64_t cap = (int64_t)sm_count() * 2;  // persistent: the two blocks per SM that fit
    const int blocks = (int)(blocks_needed < cap ? blocks_needed : cap);
    if (mode == ENGRAM_MODE_CONCAT_F32)
        k_forward_concat<FMT, FMT == ENGRAM_FMT_F32 ? 16 : 8><<<blocks, threads, 0, s>>>(T, OV, tokens, seg_start, t0, n, (float*)out, ids_out,
                                                            slots_out, hit_count);
    else
        k_forward_pairsum<FMT, 4><<<blocks, threads, 0, s>>>(T, OV, tokens, seg_start, t0, n, (__nv_bfloat16*)out,
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
    k_hash<<<(int)(want < cap ? want : cap), threads, 0, (cudaStream_t)stream>>>(*t, tokens, seg_start, t0, n, ids_out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_forward(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                              const int32_t* seg_start, int64_t t0, int64_t n, int32_t mode, void* out,
                              int32_t* ids_out, int32_t* slots_out, int64_t* hit_count, void* stream) {
    if (!t || t0 < 0 || n < 0) return ENGRAM_ERR_ARG;
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
        case ENGRAM_FMT_F32: launch_forward<ENGRAM_FMT_F32>(*t, OV, tokens, seg_start, t0, n, mode, out, ids_out, slots_out, hc, s); break;
        case ENGRAM_FMT_IQ4_NL: launch_forward<ENGRAM_FMT_IQ4_NL>(*t, OV, tokens, seg_start, t0, n, mode, out, ids_out, slots_out, hc, s); break;
        case ENGRAM_FMT_IQ4_XS: launch_forward<ENGRAM_FMT_IQ4_XS>(*t, OV, tokens, seg_start, t0, n, mode, out, ids_out, slots_out, hc, s); break;
        default: return ENGRAM_ERR_FORMAT;
    }
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
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
