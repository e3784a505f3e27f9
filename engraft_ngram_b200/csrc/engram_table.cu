// engram_table.cu -- table descriptor, resident-layout packing and the overlay map.
#include <string.h>

#include <atomic>

#include "engram_common.cuh"

using namespace engram;

static std::atomic<int64_t> g_launches{0};

void engram::count_launches(int k) { g_launches.fetch_add(k, std::memory_order_relaxed); }

extern "C" int64_t engram_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int engram_version(void) { return 100; }

extern "C" int64_t engram_raw_row_bytes(int32_t fmt, int32_t dim) {
    if (dim <= 0 || dim > 1024) return ENGRAM_ERR_FORMAT;
    if (fmt == ENGRAM_FMT_F32) return (dim % 4) ? ENGRAM_ERR_FORMAT : (int64_t)dim * 4;
    if (fmt == ENGRAM_FMT_IQ4_NL) return (dim % 32) ? ENGRAM_ERR_FORMAT : (int64_t)(dim / 32) * 18;
    if (fmt == ENGRAM_FMT_IQ4_XS) return (dim % 256) ? ENGRAM_ERR_FORMAT : (int64_t)(dim / 256) * 136;
    return ENGRAM_ERR_FORMAT;
}

extern "C" int64_t engram_row_stride(int32_t fmt, int32_t dim) {
    const int64_t raw = engram_raw_row_bytes(fmt, dim);
    if (raw < 0) return raw;
    if (fmt == ENGRAM_FMT_F32) return raw;
    if (fmt == ENGRAM_FMT_IQ4_NL) return (raw + 15) / 16 * 16;
    return (int64_t)(dim / 256) * 144;
}

extern "C" int engram_table_init(engram_table* t, const void* rows, int64_t n_rows, int32_t fmt, int32_t dim,
                                 int32_t ngram_size, int32_t heads_per_ngram, const int64_t* head_sizes,
                                 const int64_t* head_offsets, const uint64_t* mult, int32_t n_mult,
                                 int64_t eos_token_id) {
    if (!t || !head_sizes || !head_offsets || !mult) return ENGRAM_ERR_ARG;
    if (ngram_size < 2 || ngram_size > ENGRAM_MAX_CTX || heads_per_ngram < 1) return ENGRAM_ERR_ARG;
    const int n_heads = (ngram_size - 1) * heads_per_ngram;
    if (n_heads > ENGRAM_MAX_HEADS || n_mult < ngram_size) return ENGRAM_ERR_ARG;
    const int64_t stride = engram_row_stride(fmt, dim);
    if (stride < 0) return ENGRAM_ERR_FORMAT;
    if (n_rows < 1 || n_rows > 2147483647LL) return ENGRAM_ERR_RANGE;
    if (!rows || !aligned16(rows)) return ENGRAM_ERR_ARG;
    memset(t, 0, sizeof(*t));
    t->rows = rows;
    t->n_rows = n_rows;
    t->row_stride = stride;
    t->fmt = fmt;
    t->dim = dim;
    t->ngram_size = ngram_size;
    t->heads_per_ngram = heads_per_ngram;
    t->n_heads = n_heads;
    t->eos_token_id = eos_token_id;
    for (int j = 0; j < ngram_size; j++) t->mult[j] = mult[j];
    for (int h = 0; h < n_heads; h++) {
        const int64_t p = head_sizes[h], off = head_offsets[h];
        if (p < 1 || p > 2147483647LL || off < 0 || off + p > n_rows) return ENGRAM_ERR_RANGE;
        t->head_size[h] = (uint32_t)p;
        t->head_offset[h] = off;
        magic_for((uint32_t)p, &t->head_magic[h], &t->head_shift[h]);
    }
    return ENGRAM_OK;
}

extern "C" int engram_selftest_mod(const uint64_t* x, int64_t count, uint32_t d, uint64_t* out) {
    if (!x || !out || count < 0 || d == 0) return ENGRAM_ERR_ARG;
    uint64_t magic;
    uint32_t l;
    magic_for(d, &magic, &l);
    for (int64_t i = 0; i < count; i++) out[i] = mod_by_magic(x[i], d, magic, l);
    return ENGRAM_OK;
}

// ---- packing: reference row bytes -> resident layout (one thread per 16-byte output word)
__global__ void k_pack(int32_t fmt, int32_t dim, const uint8_t* __restrict__ src, int64_t n_rows,
                       uint8_t* __restrict__ dst, int64_t raw_bytes, int64_t stride) {
    const int64_t words = stride / 16;
    const int64_t total = n_rows * words;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < total; w += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = w / words;
        const int wo = (int)(w - r * words) * 16;  // byte offset of this word inside the resident row
        const uint8_t* s = src + r * raw_bytes;
        uint8_t b[16];
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int o = wo + k;  // resident byte offset -> reference byte offset (or padding)
            int so = -1;
            if (fmt == ENGRAM_FMT_F32) {
                so = o;
            } else if (fmt == ENGRAM_FMT_IQ4_NL) {
                const int nb = dim / 32;
                if (o < 16 * nb) so = (o / 16) * 18 + 2 + (o % 16);
                else if (o < 18 * nb) so = ((o - 16 * nb) / 2) * 18 + ((o - 16 * nb) % 2);
            } else {
                const int sb = o / 144, q = o % 144;
                if (q < 128) so = sb * 136 + 8 + q;
                else if (q < 136) so = sb * 136 + (q - 128);
            }
            b[k] = (so >= 0) ? s[so] : (uint8_t)0;
        }
        uint4 v;
        memcpy(&v, b, 16);
        *reinterpret_cast<uint4*>(dst + r * stride + wo) = v;
    }
}

extern "C" int engram_table_pack(int32_t fmt, int32_t dim, const uint8_t* src, int64_t n_rows, void* dst,
                                 void* stream) {
    const int64_t raw = engram_raw_row_bytes(fmt, dim), stride = engram_row_stride(fmt, dim);
    if (raw < 0 || stride < 0) return ENGRAM_ERR_FORMAT;
    if (n_rows < 0) return ENGRAM_ERR_ARG;
    if (n_rows == 0) return ENGRAM_OK;
    if (!src || !dst || !aligned16(dst)) return ENGRAM_ERR_ARG;
    const int64_t total = n_rows * (stride / 16);
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    const int blocks = (int)(want < (int64_t)sm_count() * 32 ? want : (int64_t)sm_count() * 32);
    k_pack<<<blocks, threads, 0, (cudaStream_t)stream>>>(fmt, dim, src, n_rows, (uint8_t*)dst, raw, stride);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

// ---- overlay map ---------------------------------------------------------------
__global__ void k_map_clear(int32_t* keys, int64_t capacity) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < capacity; i += (int64_t)gridDim.x * blockDim.x)
        keys[i] = -1;
}

__global__ void k_map_insert(const int32_t* __restrict__ ids, int64_t R, int32_t* keys, int32_t* slots,
                             int64_t capacity) {
    const uint32_t mask = (uint32_t)capacity - 1u;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < R; k += (int64_t)gridDim.x * blockDim.x) {
        const int32_t gid = ids[k];
        uint32_t pos = map_home(gid, capacity);
        for (int64_t probe = 0; probe < capacity; probe++) {
            const int32_t prev = atomicCAS(keys + pos, -1, gid);
            if (prev == -1 || prev == gid) {
                slots[pos] = (int32_t)k;
                break;
            }
            pos = (pos + 1u) & mask;
        }
    }
}

extern "C" int engram_overlay_map_build(const int32_t* ids, int64_t R, int32_t* keys, int32_t* slots,
                                        int64_t capacity, void* stream) {
    if (R < 0 || capacity < 0) return ENGRAM_ERR_ARG;
    if (R == 0) return ENGRAM_OK;
    if (!ids || !keys || !slots) return ENGRAM_ERR_ARG;
    if ((capacity & (capacity - 1)) != 0 || capacity < 2 * R || capacity > (1LL << 31)) return ENGRAM_ERR_RANGE;
    cudaStream_t s = (cudaStream_t)stream;
    const int threads = 256;
    int64_t b1 = (capacity + threads - 1) / threads, b2 = (R + threads - 1) / threads;
    const int64_t cap_blocks = (int64_t)sm_count() * 16;
    k_map_clear<<<(int)(b1 < cap_blocks ? b1 : cap_blocks), threads, 0, s>>>(keys, capacity);
    k_map_insert<<<(int)(b2 < cap_blocks ? b2 : cap_blocks), threads, 0, s>>>(ids, R, keys, slots, capacity);
    count_launches(2);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

// ---- overlay lookup: slots of a batch of global ids (-1 when not an overlay row)
__global__ void k_overlay_lookup(engram_overlay OV, const int32_t* __restrict__ ids, int64_t n, int32_t* slots) {
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
        slots[k] = overlay_slot(OV, ids[k]);
}

extern "C" int engram_overlay_lookup(const engram_overlay* ov, const int32_t* ids, int64_t n, int32_t* slots_out,
                                     void* stream) {
    if (!ov || n < 0) return ENGRAM_ERR_ARG;
    if (n == 0) return ENGRAM_OK;
    if (!ids || !slots_out) return ENGRAM_ERR_ARG;
    const engram_overlay OV = *ov;
    if (OV.n_rows < 0 || (OV.n_rows > 0 && (!OV.map_keys || !OV.map_slots))) return ENGRAM_ERR_ARG;
    if (OV.n_rows > 0 && ((OV.capacity & (OV.capacity - 1)) != 0 || OV.capacity < 2 * OV.n_rows)) return ENGRAM_ERR_RANGE;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads, cap = (int64_t)sm_count() * 16;
    k_overlay_lookup<<<(int)(want < cap ? want : cap), threads, 0, (cudaStream_t)stream>>>(OV, ids, n, slots_out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
