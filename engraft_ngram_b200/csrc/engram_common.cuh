// engram_common.cuh -- device helpers shared by the Engram table kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "engram_b200.h"

namespace engram {

constexpr int kWarp = 32;

// ggml's kvalues_iq4nl codebook: the 16 levels of a 4-bit IQ4 code
// (engraft/table.py:26-29, engraft/replica/dequant.py:30).
__device__ __constant__ static const float kKvIq4[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f,
                                                           -22.f,  -10.f,  1.f,   13.f,  25.f,  38.f,
                                                           53.f,   69.f,   89.f,  113.f};

__host__ __device__ inline uint64_t mulhi64(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
    return __umul64hi(a, b);
#else
    return (uint64_t)(((unsigned __int128)a * b) >> 64);
#endif
}

// x mod d for a divisor fixed per head, by multiplication: Granlund & Montgomery,
// "Division by invariant integers using multiplication" (PLDI 1994), Fig. 4.1,
// unsigned N = 64.  With l = ceil(log2 d) and m = floor(2^64 (2^l - d) / d) + 1:
//   t1 = mulhi(m, x);  q = (t1 + ((x - t1) >> 1)) >> (l - 1)   (q = x when l = 0)
// is exact for every 64-bit x.  The remainder is x - q d.
__host__ __device__ inline uint64_t mod_by_magic(uint64_t x, uint32_t d, uint64_t magic, uint32_t l) {
    uint64_t q;
    if (l == 0) {
        q = x;
    } else {
        uint64_t t1 = mulhi64(magic, x);
        q = (t1 + ((x - t1) >> 1)) >> (l - 1);
    }
    return x - q * (uint64_t)d;
}

inline void magic_for(uint32_t d, uint64_t* magic, uint32_t* l) {
    uint32_t ll = 0;
    while (ll < 32 && (1ull << ll) < d) ll++;
    unsigned __int128 num = ((unsigned __int128)((1ull << ll) - d)) << 64;
    *magic = (uint64_t)(num / d) + 1;
    *l = ll;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

// The tokens one position's hash reads: x[s] = token at t-s (unread when t-s < 0)
// and lo = the first index of t's segment.  Loaded ahead of the hash so the
// loads of the next position overlap the current one's row reads.
struct TokCtx {
    int32_t x[ENGRAM_MAX_CTX];
    int32_t lo;
};

__device__ __forceinline__ TokCtx load_ctx(const engram_table& T, const int32_t* __restrict__ tokens,
                                           const int32_t* __restrict__ seg_start, int64_t t) {
    TokCtx c;
    c.lo = seg_start ? __ldg(seg_start + t) : 0;
#pragma unroll
    for (int s = 0; s < ENGRAM_MAX_CTX; s++) c.x[s] = (s < T.ngram_size && t - s >= 0) ? __ldg(tokens + t - s) : 0;
    return c;
}

// Flat (position, head) index k -> (k / nh, k % nh).  A 64-bit division is a
// long emulated sequence; 32-bit unsigned division is far shorter, so it is
// used whenever k fits (every batch this library sees; k < 2^32).
__device__ __forceinline__ void split_pair(int64_t k, int nh, int64_t& i, int& h) {
    if (nh == 16) {  // the reference's head count: shifts
        i = k >> 4;
        h = (int)(k & 15);
    } else if ((uint64_t)k <= 0xffffffffull) {
        const uint32_t q = (uint32_t)k / (uint32_t)nh;
        i = (int64_t)q;
        h = (int)((uint32_t)k - q * (uint32_t)nh);
    } else {
        i = k / nh;
        h = (int)(k - i * nh);
    }
}

// The per-head hash constants of a table, copied once per block into shared
// memory.  Read from the kernel's parameter block with a different head in
// every lane, they would be indexed constant-bank loads, which a warp
// serialises (one address at a time); from shared memory the heads of a warp
// hit distinct banks or the same word.
struct HeadTab {
    uint64_t magic[ENGRAM_MAX_HEADS];
    int64_t offset[ENGRAM_MAX_HEADS];
    uint32_t size[ENGRAM_MAX_HEADS];
    uint32_t shift[ENGRAM_MAX_HEADS];
    int32_t order[ENGRAM_MAX_HEADS];  // n of the n-gram head h hashes: 2 + h / heads_per_ngram
};

// Every thread of the block calls it; the caller then synchronises the block.
__device__ __forceinline__ void head_tab_fill(HeadTab& H, const engram_table& T) {
    for (int h = threadIdx.x; h < T.n_heads && h < ENGRAM_MAX_HEADS; h += blockDim.x) {
        H.magic[h] = T.head_magic[h];
        H.offset[h] = T.head_offset[h];
        H.size[h] = T.head_size[h];
        H.shift[h] = T.head_shift[h];
        H.order[h] = 2 + h / T.heads_per_ngram;
    }
}

// Global row id of head `h` at position t (engraft/table.py:111-144 + engraft/lens.py:108-110).
// ctx[0] = x_t; ctx[s] = x_{t-s}, or EOS once a predecessor is missing (before
// lo, the start of t's segment) or is itself EOS; the current token never cuts.
__device__ __forceinline__ int32_t hash_ctx(const engram_table& T, const HeadTab& H, const TokCtx& c, int64_t t,
                                            int h) {
    const int N = T.ngram_size;
    int64_t ctx[ENGRAM_MAX_CTX];
    ctx[0] = (int64_t)c.x[0];
    bool cut = false;
#pragma unroll
    for (int s = 1; s < ENGRAM_MAX_CTX; s++) {
        if (s < N) {
            const bool have = (t - s >= (int64_t)c.lo) && !cut;
            int64_t tok = have ? (int64_t)c.x[s] : T.eos_token_id;
            if (!have || tok == T.eos_token_id) {
                cut = true;
                tok = T.eos_token_id;
            }
            ctx[s] = tok;
        }
    }
    const int n = H.order[h];  // heads (n-2)*hpn .. hold the n-gram of order n
    uint64_t mixed = (uint64_t)ctx[0] * T.mult[0];
#pragma unroll
    for (int j = 1; j < ENGRAM_MAX_CTX; j++)
        if (j < n) mixed ^= (uint64_t)ctx[j] * T.mult[j];
    const uint64_t local = mod_by_magic(mixed, H.size[h], H.magic[h], H.shift[h]);
    return (int32_t)(H.offset[h] + (int64_t)local);
}

__device__ __forceinline__ int32_t hash_row(const engram_table& T, const HeadTab& H, const int32_t* __restrict__ tokens,
                                            const int32_t* __restrict__ seg_start, int64_t t, int h) {
    return hash_ctx(T, H, load_ctx(T, tokens, seg_start, t), t, h);
}

// Overlay map probe (open addressing, linear probing; built by
// engram_overlay_map_build).  Returns the slot of `gid` or -1.  The loop is
// bounded by the capacity, and the map always holds an empty key (load <= 1/2).
__device__ __forceinline__ uint32_t map_home(int32_t gid, int64_t capacity) {
    const int lg = 63 - __clzll((long long)capacity);
    const uint64_t hsh = (uint64_t)(uint32_t)gid * 0x9E3779B97F4A7C15ull;
    return lg == 0 ? 0u : (uint32_t)(hsh >> (64 - lg));
}

__device__ __forceinline__ int32_t overlay_slot(const engram_overlay& ov, int32_t gid) {
    if (ov.n_rows == 0) return -1;
    const uint32_t mask = (uint32_t)ov.capacity - 1u;
    uint32_t pos = map_home(gid, ov.capacity);
    for (int64_t probe = 0; probe < ov.capacity; probe++) {
        const int32_t k = __ldg(ov.map_keys + pos);
        if (k == gid) return __ldg(ov.map_slots + pos);
        if (k == -1) return -1;
        pos = (pos + 1u) & mask;
    }
    return -1;
}

inline int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Adds k to the process-wide count of kernels this library has launched
// (reported by engram_launch_count).
void count_launches(int k);

}  // namespace engram
