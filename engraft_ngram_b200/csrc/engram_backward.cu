// engram_backward.cu -- K3 (row gradients of the overlay) and K4 (Adam + the
// descent's regulariser).
//
// K3 reproduces the reference's accumulation order exactly.  The reference
// sums duplicate rows with index_put_(accumulate=True) over idx lists built in
// ascending (t, h) order (engraft/replica/seq.py:401-441): serially on one CPU
// thread, and after a stable sort of the indices on CUDA.  Here:
//   1. a stable LSD radix sort (8-bit digits) of the hit entries keyed by
//      overlay slot; entry values are flat indices t*n_heads+h, so each slot's
//      entries come out in ascending (t, h) order.  Ranks inside a tile come
//      from warp __match_any_sync groups plus per-warp digit counts, so no
//      comparison sort is needed;
//   2. segment starts per slot from the sorted keys;
//   3. one warp per slot adds its terms in that order, from +0, in fp32.
// The result is bit-identical to the reference and independent of scheduling.
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

inline int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct Workspace {
    int32_t* keys[2];
    int32_t* vals[2];
    uint32_t* block_hist;
    int32_t* seg_begin;
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
    w.seg_begin = reinterpret_cast<int32_t*>(take(4 * (R + 1)));
    w.counters = reinterpret_cast<int32_t*>(take(64));
    w.bytes = off;
    return w;
}

// Pass histogram: digit counts of this block's tile, stored digit-major.
__global__ void __launch_bounds__(kRsThreads) k_rs_hist(const int32_t* __restrict__ keys, const int32_t* n_dev,
                                                        int64_t n_static, int shift, uint32_t* block_hist, int nblk) {
    __shared__ uint32_t h[256];
    for (int d = threadIdx.x; d < 256; d += kRsThreads) h[d] = 0;
    __syncthreads();
    const int64_t n = n_dev ? (int64_t)*n_dev : n_static;
    const int64_t begin = (int64_t)blockIdx.x * kRsTile;
    for (int k = threadIdx.x; k < kRsTile; k += kRsThreads) {
        const int64_t i = begin + k;
        if (i < n) {
            const int32_t key = keys[i];
            if (key >= 0) atomicAdd(&h[(key >> shift) & 255], 1u);
        }
    }
    __syncthreads();
    for (int d = threadIdx.x; d < 256; d += kRsThreads) block_hist[(int64_t)d * nblk + blockIdx.x] = h[d];
}

// Exclusive scan in place over len entries (one block).  *total = sum.
__global__ void __launch_bounds__(kScanThreads) k_scan(uint32_t* a, int64_t len, int32_t* total) {
    __shared__ uint32_t part[kScanThreads];
    const int tid = threadIdx.x;
    const int64_t per = (len + kScanThreads - 1) / kScanThreads;
    const int64_t lo = tid * per, hi = (lo + per < len) ? lo + per : len;
    uint32_t s = 0;
    for (int64_t i = lo; i < hi; i++) s += a[i];
    part[tid] = s;
    __syncthreads();
    for (int off = 1; off < kScanThreads; off <<= 1) {
        const uint32_t v = tid >= off ? part[tid - off] : 0u;
        __syncthreads();
        part[tid] += v;
        __syncthreads();
    }
    uint32_t run = part[tid] - s;  // exclusive prefix of this thread's chunk
    for (int64_t i = lo; i < hi; i++) {
        const uint32_t x = a[i];
        a[i] = run;
        run += x;
    }
    if (tid == kScanThreads - 1 && total) *total = (int32_t)part[tid];
}

// Stable scatter of one pass.  vals_in == nullptr: the value is the index.
__global__ void __launch_bounds__(kRsThreads) k_rs_scatter(const int32_t* __restrict__ keys_in,
                                                           const int32_t* __restrict__ vals_in, const int32_t* n_dev,
                                                           int64_t n_static, int shift,
                                                           const uint32_t* __restrict__ block_off, int nblk,
                                                           int32_t* __restrict__ keys_out,
                                                           int32_t* __restrict__ vals_out) {
    __shared__ uint32_t wcnt[kRsWarps][256];
    __shared__ uint32_t run[256];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int d = tid; d < 256; d += kRsThreads) run[d] = block_off[(int64_t)d * nblk + blockIdx.x];
    const int64_t n = n_dev ? (int64_t)*n_dev : n_static;
    const int64_t begin = (int64_t)blockIdx.x * kRsTile;
    const unsigned lt = (1u << lane) - 1u;
    for (int sub = 0; sub < kRsItems; sub++) {
        for (int k = tid; k < kRsWarps * 256; k += kRsThreads) (&wcnt[0][0])[k] = 0;
        __syncthreads();
        const int64_t i = begin + (int64_t)sub * kRsThreads + tid;
        const int32_t key = (i < n) ? keys_in[i] : -1;
        const bool valid = key >= 0;
        const int digit = valid ? ((key >> shift) & 255) : (256 + lane);
        const unsigned peers = __match_any_sync(kFull, digit);
        const int rank = __popc(peers & lt);
        if (valid && rank == 0) wcnt[warp][digit] = (uint32_t)__popc(peers);
        __syncthreads();
        for (int d = tid; d < 256; d += kRsThreads) {
            uint32_t acc = run[d];
#pragma unroll
            for (int w = 0; w < kRsWarps; w++) {
                const uint32_t c = wcnt[w][d];
                wcnt[w][d] = acc;
                acc += c;
            }
            run[d] = acc;
        }
        __syncthreads();
        if (valid) {
            const uint32_t pos = wcnt[warp][digit] + (uint32_t)rank;
            keys_out[pos] = key;
            vals_out[pos] = vals_in ? vals_in[i] : (int32_t)i;
        }
        __syncthreads();
    }
}

// seg_begin[s] = number of sorted entries with key < s, for s in [0, R].
__global__ void k_seg_begin(const int32_t* __restrict__ keys, const int32_t* n_dev, int64_t R,
                            int32_t* __restrict__ seg_begin) {
    const int64_t n = *n_dev;
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

// One warp per slot: grad_rows[s] = sum of its terms in sorted (ascending) order.
// CONCAT: term = grad[i, :] (fp32, i = t*n_heads+h); CPL = float4 chunks per lane.
template <int CPL>
__global__ void __launch_bounds__(256) k_reduce_concat(const int32_t* __restrict__ seg_begin,
                                                       const int32_t* __restrict__ vals, int64_t R, int dim,
                                                       const float* __restrict__ grad, float* __restrict__ grad_rows) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int cpr = dim >> 2;
    const float4* g4 = reinterpret_cast<const float4*>(grad);
    for (int64_t s = warp0; s < R; s += nwarps) {
        const int b = __ldg(seg_begin + s), e = __ldg(seg_begin + s + 1);
        float4 acc[CPL];
#pragma unroll
        for (int j = 0; j < CPL; j++) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        constexpr int P = 4;
        for (int k = b; k < e; k += P) {
            float4 x[P][CPL];
#pragma unroll
            for (int p = 0; p < P; p++) {
                if (k + p < e) {
                    const int64_t i = __ldg(vals + k + p);
#pragma unroll
                    for (int j = 0; j < CPL; j++) {
                        const int c = lane + 32 * j;
                        if (c < cpr) x[p][j] = __ldg(g4 + i * cpr + c);
                    }
                }
            }
#pragma unroll
            for (int p = 0; p < P; p++) {
                if (k + p < e) {
#pragma unroll
                    for (int j = 0; j < CPL; j++) {
                        acc[j].x = __fadd_rn(acc[j].x, x[p][j].x);
                        acc[j].y = __fadd_rn(acc[j].y, x[p][j].y);
                        acc[j].z = __fadd_rn(acc[j].z, x[p][j].z);
                        acc[j].w = __fadd_rn(acc[j].w, x[p][j].w);
                    }
                }
            }
        }
        float4* dst = reinterpret_cast<float4*>(grad_rows + s * (int64_t)dim);
#pragma unroll
        for (int j = 0; j < CPL; j++) {
            const int c = lane + 32 * j;
            if (c < cpr) dst[c] = acc[j];
        }
    }
}

// PAIRSUM: term of (t,h) = bf16 grad[t, (h%hpn)*dim : +dim]; CPL = 8-value chunks per lane.
template <int CPL>
__global__ void __launch_bounds__(256) k_reduce_pairsum(const int32_t* __restrict__ seg_begin,
                                                        const int32_t* __restrict__ vals, int64_t R, int dim,
                                                        int n_heads, int hpn, const uint16_t* __restrict__ grad,
                                                        float* __restrict__ grad_rows) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int cpr = dim >> 3;
    const int64_t row_elems = (int64_t)hpn * dim;
    for (int64_t s = warp0; s < R; s += nwarps) {
        const int b = __ldg(seg_begin + s), e = __ldg(seg_begin + s + 1);
        float acc[CPL][8];
#pragma unroll
        for (int j = 0; j < CPL; j++)
#pragma unroll
            for (int q = 0; q < 8; q++) acc[j][q] = 0.f;
        constexpr int P = 4;
        for (int k = b; k < e; k += P) {
            uint4 x[P][CPL];
#pragma unroll
            for (int p = 0; p < P; p++) {
                if (k + p < e) {
                    const int32_t i = __ldg(vals + k + p);
                    const int64_t t = i / n_heads;
                    const int h = i - (int)(t * n_heads);
                    const uint4* src = reinterpret_cast<const uint4*>(grad + t * row_elems + (int64_t)(h % hpn) * dim);
#pragma unroll
                    for (int j = 0; j < CPL; j++) {
                        const int c = lane + 32 * j;
                        if (c < cpr) x[p][j] = __ldg(src + c);
                    }
                }
            }
#pragma unroll
            for (int p = 0; p < P; p++) {
                if (k + p < e) {
#pragma unroll
                    for (int j = 0; j < CPL; j++) {
                        const uint32_t w[4] = {x[p][j].x, x[p][j].y, x[p][j].z, x[p][j].w};
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            acc[j][2 * q] = __fadd_rn(acc[j][2 * q], __uint_as_float(w[q] << 16));
                            acc[j][2 * q + 1] = __fadd_rn(acc[j][2 * q + 1], __uint_as_float(w[q] & 0xffff0000u));
                        }
                    }
                }
            }
        }
        float4* dst = reinterpret_cast<float4*>(grad_rows + s * (int64_t)dim);
#pragma unroll
        for (int j = 0; j < CPL; j++) {
            const int c = lane + 32 * j;
            if (c < cpr) {
                dst[2 * c] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
                dst[2 * c + 1] = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
            }
        }
    }
}

struct AdamScalars {
    float w1, b2, w2, eps, neg_step_size, bc2_sqrt, reg_scale;
};

__device__ __forceinline__ float adam_elem(float& p, float g, float& m, float& v, float p0, bool reg,
                                           const AdamScalars& a) {
    if (reg) g = __fadd_rn(g, __fmul_rn(a.reg_scale, __fmul_rn(2.0f, __fsub_rn(p, p0))));
    const float mi = __fmaf_rn(a.w1, __fsub_rn(g, m), m);
    const float vi = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(__fmul_rn(a.w2, g), g));
    const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), a.bc2_sqrt), a.eps);
    p = __fadd_rn(p, __fdiv_rn(__fmul_rn(a.neg_step_size, mi), den));
    m = mi;
    v = vi;
    return p;
}

__global__ void __launch_bounds__(256) k_adam_vec4(float4* __restrict__ p, const float4* __restrict__ g,
                                                   float4* __restrict__ m, float4* __restrict__ v,
                                                   const float4* __restrict__ p0, int64_t n4, AdamScalars a) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 pp = p[i], mm = m[i], vv = v[i];
        const float4 gg = __ldcs(g + i);
        const float4 q = p0 ? __ldg(p0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const bool reg = p0 != nullptr;
        adam_elem(pp.x, gg.x, mm.x, vv.x, q.x, reg, a);
        adam_elem(pp.y, gg.y, mm.y, vv.y, q.y, reg, a);
        adam_elem(pp.z, gg.z, mm.z, vv.z, q.z, reg, a);
        adam_elem(pp.w, gg.w, mm.w, vv.w, q.w, reg, a);
        p[i] = pp;
        m[i] = mm;
        v[i] = vv;
    }
}

__global__ void k_adam_scalar(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                              float* __restrict__ v, const float* __restrict__ p0, int64_t lo, int64_t n,
                              AdamScalars a) {
    for (int64_t i = lo + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float pp = p[i], mm = m[i], vv = v[i];
        adam_elem(pp, g[i], mm, vv, p0 ? p0[i] : 0.f, p0 != nullptr, a);
        p[i] = pp;
        m[i] = mm;
        v[i] = vv;
    }
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

extern "C" int engram_backward(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                               int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                               void* workspace, int64_t workspace_bytes, void* stream) {
    if (n < 0 || R < 0 || n_heads < 1 || n_heads > ENGRAM_MAX_HEADS || heads_per_ngram < 1) return ENGRAM_ERR_ARG;
    if (mode != ENGRAM_MODE_CONCAT_F32 && mode != ENGRAM_MODE_PAIRSUM_ADD_BF16) return ENGRAM_ERR_ARG;
    if (dim <= 0 || dim > 1024 || (mode == ENGRAM_MODE_CONCAT_F32 ? dim % 4 : dim % 8)) return ENGRAM_ERR_FORMAT;
    if (mode == ENGRAM_MODE_PAIRSUM_ADD_BF16 && n_heads != 2 * heads_per_ngram) return ENGRAM_ERR_FORMAT;
    if (R >= (1LL << 24) || n * n_heads >= (1LL << 31)) return ENGRAM_ERR_RANGE;
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
    const int64_t hist_len = 256LL * w.nblk;
    int cur = 0;
    for (int pass = 0; pass < passes; pass++) {
        const int shift = 8 * pass;
        const int32_t* kin = pass == 0 ? slots : w.keys[cur];
        const int32_t* vin = pass == 0 ? nullptr : w.vals[cur];
        const int32_t* n_dev = pass == 0 ? nullptr : w.counters;
        const int out = pass == 0 ? 0 : 1 - cur;
        k_rs_hist<<<w.nblk, kRsThreads, 0, s>>>(kin, n_dev, N, shift, w.block_hist, w.nblk);
        k_scan<<<1, kScanThreads, 0, s>>>(w.block_hist, hist_len, pass == 0 ? w.counters : w.counters + 1);
        k_rs_scatter<<<w.nblk, kRsThreads, 0, s>>>(kin, vin, n_dev, N, shift, w.block_hist, w.nblk, w.keys[out],
                                                     w.vals[out]);
        cur = out;
    }
    count_launches(3 * passes + 2);
    k_seg_begin<<<grid_for(N, 256, 8), 256, 0, s>>>(w.keys[cur], w.counters, R, w.seg_begin);
    const int rblocks = grid_for(R * 32, 256, 8);
    if (mode == ENGRAM_MODE_CONCAT_F32) {
        const int cpl = (dim / 4 + 31) / 32;
        const float* g = static_cast<const float*>(grad);
        if (cpl <= 1) k_reduce_concat<1><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, g, grad_rows);
        else if (cpl <= 2) k_reduce_concat<2><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, g, grad_rows);
        else if (cpl <= 4) k_reduce_concat<4><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, g, grad_rows);
        else k_reduce_concat<8><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, g, grad_rows);
    } else {
        const int cpl = (dim / 8 + 31) / 32;
        const uint16_t* g = static_cast<const uint16_t*>(grad);
        if (cpl <= 1) k_reduce_pairsum<1><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, n_heads, heads_per_ngram, g, grad_rows);
        else if (cpl <= 2) k_reduce_pairsum<2><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, n_heads, heads_per_ngram, g, grad_rows);
        else k_reduce_pairsum<4><<<rblocks, 256, 0, s>>>(w.seg_begin, w.vals[cur], R, dim, n_heads, heads_per_ngram, g, grad_rows);
    }
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_adam_step(float* p, const float* g, float* m, float* v, const float* p0, int64_t numel,
                                int64_t step, double lr, double beta1, double beta2, double eps, float reg_scale,
                                void* stream) {
    if (numel < 0 || step < 1) return ENGRAM_ERR_ARG;
    if (numel == 0) return ENGRAM_OK;
    if (!p || !g || !m || !v) return ENGRAM_ERR_ARG;
    AdamScalars a;
    const double bc1 = 1.0 - pow(beta1, (double)step);
    const double bc2 = 1.0 - pow(beta2, (double)step);
    a.w1 = (float)(1.0 - beta1);
    a.b2 = (float)beta2;
    a.w2 = (float)(1.0 - beta2);
    a.eps = (float)eps;
    a.neg_step_size = -(float)(lr / bc1);
    a.bc2_sqrt = (float)sqrt(bc2);
    a.reg_scale = reg_scale;
    cudaStream_t s = (cudaStream_t)stream;
    const bool vec = aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v) && (!p0 || aligned16(p0));
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = numel / 4;
        if (n4 > 0)
        {
            k_adam_vec4<<<grid_for(n4, 256, 8), 256, 0, s>>>((float4*)p, (const float4*)g, (float4*)m, (float4*)v,
                                                             (const float4*)p0, n4, a);
            count_launches(1);
        }
        done = n4 * 4;
    }
    if (done < numel) {
        k_adam_scalar<<<grid_for(numel - done, 256, 8), 256, 0, s>>>(p, g, m, v, p0, done, numel, a);
        count_launches(1);
    }
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
