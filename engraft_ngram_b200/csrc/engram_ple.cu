// engram_ple.cu -- the PLE block that consumes the gathered rows
// (engraft/replica/layers.py:565-626, ple_forward), minus its two projections:
//   key   = emb @ w_key.T    [T, hc, n]     value = emb @ w_value.T  [T, n]
// are plain GEMMs the caller runs (cuBLAS); the rest is two HBM-bound kernels.
//
// k_ple_gate, one block per position t:
//   s_j    = <rmsnorm(key_j) * norm_key_j, rmsnorm(hidden_j) * norm_query_j> / sqrt(n)
//   gate_j = sigmoid(sign(s_j) * sqrt(max(|s_j|, 1e-6)))
//   normed_j = rmsnorm(value * gate_j) * norm_conv_j           (the conv input)
// k_ple_conv, one thread per 4 channels of one position:
//   conv = sum_k w[c, k] * normed[t - (K-1-k) * dilation, c]   (history rows
//          before position 0, zero before the history; layers.py:257-293)
//   out  = hidden + value * gate_j + silu(conv)
// rmsnorm(x) = x * rsqrt(mean(x^2) + eps) (layers.py:23-34).  Reductions run in
// fp32 in a different order from torch's, so results agree to fp32 rounding,
// not bit for bit.
#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kPleMaxHc = 8;
constexpr int kGateThreads = 256;

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void __launch_bounds__(kGateThreads) k_ple_gate(const float* __restrict__ key, int64_t key_stride,
                                                           const float* __restrict__ value, int64_t value_stride,
                                                           const float* __restrict__ hidden,
                                                           const float* __restrict__ norm_key,
                                                           const float* __restrict__ norm_query,
                                                           const float* __restrict__ norm_conv, int64_t T, int hc,
                                                           int n, float eps, float* __restrict__ gate_out,
                                                           float* __restrict__ s_out, float* __restrict__ normed) {
    // per stream j: sum key^2, sum hidden^2, sum (key*nk)(hidden*nq); then sum value^2
    constexpr int kSums = 3 * kPleMaxHc + 1;
    __shared__ float part[kGateThreads / 32][kSums];
    __shared__ float coef[2 * kPleMaxHc];  // per stream: gate, rsqrt of the gated mean square
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n4 = n >> 2;
    for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
        const float4* k4 = reinterpret_cast<const float4*>(key + t * key_stride);
        const float4* v4 = reinterpret_cast<const float4*>(value + t * value_stride);
        const float4* h4 = reinterpret_cast<const float4*>(hidden + t * (int64_t)hc * n);
        float acc[kSums];
#pragma unroll
        for (int q = 0; q < kSums; q++) acc[q] = 0.f;
        for (int c = tid; c < n4; c += kGateThreads) {
            const float4 v = __ldg(v4 + c);
            acc[3 * kPleMaxHc] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
            for (int j = 0; j < kPleMaxHc; j++) {
                if (j < hc) {
                    const float4 k = __ldg(k4 + j * n4 + c), h = __ldg(h4 + j * n4 + c);
                    const float4 a = __ldg(reinterpret_cast<const float4*>(norm_key + (int64_t)j * n) + c);
                    const float4 b = __ldg(reinterpret_cast<const float4*>(norm_query + (int64_t)j * n) + c);
                    acc[3 * j] += k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w;
                    acc[3 * j + 1] += h.x * h.x + h.y * h.y + h.z * h.z + h.w * h.w;
                    acc[3 * j + 2] += (k.x * a.x) * (h.x * b.x) + (k.y * a.y) * (h.y * b.y) +
                                      (k.z * a.z) * (h.z * b.z) + (k.w * a.w) * (h.w * b.w);
                }
            }
        }
        // one block reduction for all the sums: shuffles within warps, then thread q adds the warps' q-th sum
#pragma unroll
        for (int q = 0; q < kSums; q++) {
            float x = acc[q];
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) x += __shfl_xor_sync(kFull, x, d);
            if (lane == 0) part[warp][q] = x;
        }
        __syncthreads();
        if (tid < hc) {
            const int j = tid;
            float ssk = 0.f, ssq = 0.f, dot = 0.f, ssv = 0.f;
#pragma unroll
            for (int w = 0; w < kGateThreads / 32; w++) {
                ssk += part[w][3 * j];
                ssq += part[w][3 * j + 1];
                dot += part[w][3 * j + 2];
                ssv += part[w][3 * kPleMaxHc];
            }
            const float rk = 1.0f / sqrtf(ssk / (float)n + eps);
            const float rq = 1.0f / sqrtf(ssq / (float)n + eps);
            const float s = dot * rk * rq / sqrtf((float)n);
            const float mag = sqrtf(fmaxf(fabsf(s), 1e-6f));
            const float sg = s > 0.f ? 1.f : (s < 0.f ? -1.f : 0.f);
            const float g = sigmoidf_(sg * mag);
            gate_out[t * hc + j] = g;
            if (s_out) s_out[t * hc + j] = s;
            coef[2 * j] = g;
            coef[2 * j + 1] = 1.0f / sqrtf(g * g * (ssv / (float)n) + eps);
        }
        __syncthreads();
        for (int j = 0; j < hc; j++) {
            const float g = coef[2 * j], r = coef[2 * j + 1];
            const float4* nc4 = reinterpret_cast<const float4*>(norm_conv + (int64_t)j * n);
            float4* o4 = reinterpret_cast<float4*>(normed + (t * hc + j) * (int64_t)n);
            for (int c = tid; c < n4; c += kGateThreads) {
                const float4 v = __ldg(v4 + c), w = __ldg(nc4 + c);
                o4[c] = make_float4(v.x * g * r * w.x, v.y * g * r * w.y, v.z * g * r * w.z, v.w * g * r * w.w);
            }
        }
        __syncthreads();  // part and coef are rewritten by the next position
    }
}

// Grid: x over 4-channel groups of one position, y over positions (strided),
// so a thread keeps its channels' conv taps in registers across positions.
// KT = 4: the reference's 4 taps, unrolled, two positions per iteration (t and
// t + gridDim.y) so that their loads are in flight together; KT = 0: any K.
template <int KT>
__global__ void __launch_bounds__(256) k_ple_conv(const float* __restrict__ value, int64_t value_stride,
                                                  const float* __restrict__ hidden, const float* __restrict__ gate,
                                                  const float* __restrict__ normed, const float* __restrict__ hist,
                                                  int64_t hist_len, const float* __restrict__ conv_w, int K,
                                                  int dilation, int64_t T, int hc, int n, float* __restrict__ out) {
    constexpr int P = KT > 0 ? 2 : 1;
    constexpr int KR = KT > 0 ? KT : 1;  // taps held in registers
    const int C = hc * n, C4 = C >> 2;
    const int c4 = blockIdx.x * blockDim.x + threadIdx.x;
    if (c4 >= C4) return;
    const int c = c4 * 4;
    const int j = c4 / (n >> 2);
    const int cv = c - j * n;
    float w[4][KR];
    if (KT > 0) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float4 wq = __ldg(reinterpret_cast<const float4*>(conv_w + (int64_t)(c + q) * 4));
            w[q][0] = wq.x;
            if (KR > 1) w[q][KR > 1 ? 1 : 0] = wq.y;
            if (KR > 2) w[q][KR > 2 ? 2 : 0] = wq.z;
            if (KR > 3) w[q][KR > 3 ? 3 : 0] = wq.w;
        }
    }
    auto tap_row = [&](int64_t t, int k) -> const float* {
        const int64_t src = t - (int64_t)(K - 1 - k) * dilation;
        return src >= 0 ? normed + src * C : (hist_len + src >= 0 ? hist + (hist_len + src) * C : nullptr);
    };
    for (int64_t tb = blockIdx.y; tb < T; tb += P * (int64_t)gridDim.y) {
        float4 x[P][KR], v[P], h[P];
        float g[P];
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int64_t t = tb + p * (int64_t)gridDim.y;
            if (t < T) {
                if (KT > 0) {
#pragma unroll
                    for (int k = 0; k < KR; k++) {
                        const float* row = tap_row(t, k);
                        x[p][k] = row ? __ldg(reinterpret_cast<const float4*>(row + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
                g[p] = __ldg(gate + t * hc + j);
                v[p] = __ldg(reinterpret_cast<const float4*>(value + t * value_stride + cv));
                h[p] = __ldg(reinterpret_cast<const float4*>(hidden + t * C + c));
            }
        }
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int64_t t = tb + p * (int64_t)gridDim.y;
            if (t >= T) break;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if (KT > 0) {
#pragma unroll
                for (int k = 0; k < KR; k++) {
                    if (tap_row(t, k) == nullptr) continue;  // before the history: no term, as in the reference
                    const float xs[4] = {x[p][k].x, x[p][k].y, x[p][k].z, x[p][k].w};
#pragma unroll
                    for (int q = 0; q < 4; q++) acc[q] = __fadd_rn(acc[q], __fmul_rn(xs[q], w[q][k]));
                }
            } else {
                for (int k = 0; k < K; k++) {
                    const float* row = tap_row(t, k);
                    if (row == nullptr) continue;
                    const float4 xv = __ldg(reinterpret_cast<const float4*>(row + c));
                    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        acc[q] = __fadd_rn(acc[q], __fmul_rn(xs[q], __ldg(conv_w + (int64_t)(c + q) * K + k)));
                }
            }
            const float vs[4] = {v[p].x, v[p].y, v[p].z, v[p].w}, hs[4] = {h[p].x, h[p].y, h[p].z, h[p].w};
            float o[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float silu = acc[q] * sigmoidf_(acc[q]);
                o[q] = __fadd_rn(__fadd_rn(hs[q], __fmul_rn(vs[q], g[p])), silu);
            }
            reinterpret_cast<float4*>(out + t * C)[c4] = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

}  // namespace

extern "C" int engram_ple_gate(const float* key, int64_t key_stride, const float* value, int64_t value_stride,
                               const float* hidden, const float* norm_key, const float* norm_query,
                               const float* norm_conv, int64_t T, int32_t hc, int32_t n_embd, float eps,
                               float* gate, float* s_out, float* normed, void* stream) {
    if (T < 0 || hc < 1 || hc > kPleMaxHc || n_embd < 4 || (n_embd & 3)) return ENGRAM_ERR_ARG;
    if (key_stride < (int64_t)hc * n_embd || value_stride < n_embd || (key_stride & 3) || (value_stride & 3))
        return ENGRAM_ERR_ARG;
    if (T == 0) return ENGRAM_OK;
    if (!key || !value || !hidden || !norm_key || !norm_query || !norm_conv || !gate || !normed) return ENGRAM_ERR_ARG;
    if (!aligned16(key) || !aligned16(value) || !aligned16(hidden) || !aligned16(norm_key) || !aligned16(norm_query) ||
        !aligned16(norm_conv) || !aligned16(normed))
        return ENGRAM_ERR_ARG;
    const int64_t cap = (int64_t)sm_count() * 8;
    const int blocks = (int)(T < cap ? T : cap);
    k_ple_gate<<<blocks, kGateThreads, 0, (cudaStream_t)stream>>>(key, key_stride, value, value_stride, hidden,
                                                                   norm_key, norm_query, norm_conv, T, hc, n_embd, eps,
                                                                   gate, s_out, normed);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_ple_conv(const float* value, int64_t value_stride, const float* hidden, const float* gate,
                               const float* normed, const float* hist, int64_t hist_len, const float* conv_w,
                               int32_t K, int32_t dilation, int64_t T, int32_t hc, int32_t n_embd, float* out,
                               void* stream) {
    if (T < 0 || hc < 1 || hc > kPleMaxHc || n_embd < 4 || (n_embd & 3) || K < 1 || dilation < 1 || hist_len < 0)
        return ENGRAM_ERR_ARG;
    if (value_stride < n_embd || (value_stride & 3)) return ENGRAM_ERR_ARG;
    if (T == 0) return ENGRAM_OK;
    if (!value || !hidden || !gate || !normed || !conv_w || !out || (hist_len > 0 && !hist)) return ENGRAM_ERR_ARG;
    if (!aligned16(value) || !aligned16(hidden) || !aligned16(normed) || !aligned16(out) || (hist && !aligned16(hist)) ||
        (K == 4 && !aligned16(conv_w)))
        return ENGRAM_ERR_ARG;
    if ((int64_t)hc * n_embd >= ((int64_t)1 << 30)) return ENGRAM_ERR_RANGE;
    const int C4 = hc * n_embd / 4;
    const int gx = (C4 + 255) / 256;
    const int64_t want_y = ((int64_t)sm_count() * 8 + gx - 1) / gx;
    const int64_t gy = T < want_y ? T : (want_y < 65535 ? want_y : 65535);
    const dim3 grid(gx, (unsigned)(gy > 0 ? gy : 1));
    if (K == 4)
        k_ple_conv<4><<<grid, 256, 0, (cudaStream_t)stream>>>(value, value_stride, hidden, gate, normed, hist,
                                                              hist_len, conv_w, K, dilation, T, hc, n_embd, out);
    else
        k_ple_conv<0><<<grid, 256, 0, (cudaStream_t)stream>>>(value, value_stride, hidden, gate, normed, hist,
                                                              hist_len, conv_w, K, dilation, T, hc, n_embd, out);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
