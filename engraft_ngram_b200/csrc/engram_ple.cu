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

template <int MAXHC>
__global__ void __launch_bounds__(kGateThreads) k_ple_gate(const float* __restrict__ key, int64_t key_stride,
                                                           const float* __restrict__ value, int64_t value_stride,
                                                           const float* __restrict__ hidden,
                                                           const float* __restrict__ norm_key,
                                                           const float* __restrict__ norm_query,
                                                           const float* __restrict__ norm_conv, int64_t T, int hc,
                                                           int n, float eps, float* __restrict__ gate_out,
                                                           float* __restrict__ s_out, float* __restrict__ normed) {
    // per stream j: sum key^2, sum hidden^2, sum (key*nk)(hidden*nq); then sum value^2
    constexpr int kSums = 3 * MAXHC + 1;
    __shared__ float part[kGateThreads / 32][kSums];
    __shared__ float coef[2 * MAXHC];  // per stream: gate, rsqrt of the gated mean square
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
            acc[3 * MAXHC] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
            for (int j = 0; j < MAXHC; j++) {
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
                ssv += part[w][3 * MAXHC];
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
__global__ void __launch_bounds__(256, KT == 4 ? 3 : 1) k_ple_conv(const float* __restrict__ value, int64_t value_stride,
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

// ---- backward of the block (autograd of layers.py:565-626) -----------------------
//
// k_ple_gate_bwd, one block per position t.  With, per stream j, the sums
//   A = sum key^2, B = sum hidden^2, Cq = sum (key*nk)(hidden*nq),
//   E = sum value*nc*dn, F = sum dout*value, and V = sum value^2
// (key = emb @ w_key.T before its norm, dn = the gradient of normed, dout the
// gradient of out), every gradient is elementwise in closed form:
//   rk = rsqrt(A/n + eps), rq = rsqrt(B/n + eps), rg = rsqrt(g^2 V/n + eps)
//   d_gated_c = dout_c + rg*nc_c*dn_c - (g^2 rg^3 E / n) * value_c
//   d_gate    = sum_c d_gated_c value_c = F + rg E - (g^2 rg^3 E / n) V
//   ds        = d_gate * g (1 - g) * [|s| >= 1e-6] * 0.5 / sqrt(max(|s|, 1e-6))
//   u = ds / sqrt(n)
//   d_key_c    = u rq rk nk_c nq_c hidden_c - (u rq rk^3 Cq / n) key_c
//   d_hidden_c = dout_c + u rq rk nq_c nk_c key_c - (u rk rq^3 Cq / n) hidden_c
//   d_value_c  = sum_j d_gated_jc g_j
// (rmsnorm's backward: d x = r w dy - x r^3 sum(x w dy) / n).  detach_gate
// zeroes d_gate (gated = value * gate.detach()), detach_value zeroes d_value.
template <int MAXHC>
__global__ void __launch_bounds__(kGateThreads) k_ple_gate_bwd(
    const float* __restrict__ key, int64_t key_stride, const float* __restrict__ value, int64_t value_stride,
    const float* __restrict__ hidden, const float* __restrict__ norm_key, const float* __restrict__ norm_query,
    const float* __restrict__ norm_conv, const float* __restrict__ gate, const float* __restrict__ s_in,
    const float* __restrict__ dout, const float* __restrict__ dnormed, int64_t T, int hc, int n, float eps,
    int detach_value, int detach_gate, float* __restrict__ dkey, int64_t dkey_stride, float* __restrict__ dvalue,
    int64_t dvalue_stride, float* __restrict__ dhidden) {
    constexpr int kSums = 5 * MAXHC + 1;
    __shared__ float part[kGateThreads / 32][kSums];
    __shared__ float coef[8 * MAXHC];  // per stream: g, rg, cg, ck1, ck2, ch1, ch2
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n4 = n >> 2;
    const float fn = (float)n;
    for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
        const float4* k4 = reinterpret_cast<const float4*>(key + t * key_stride);
        const float4* v4 = reinterpret_cast<const float4*>(value + t * value_stride);
        const float4* h4 = reinterpret_cast<const float4*>(hidden + t * (int64_t)hc * n);
        const float4* o4 = reinterpret_cast<const float4*>(dout + t * (int64_t)hc * n);
        const float4* d4 = reinterpret_cast<const float4*>(dnormed + t * (int64_t)hc * n);
        float acc[kSums];
#pragma unroll
        for (int q = 0; q < kSums; q++) acc[q] = 0.f;
        for (int c = tid; c < n4; c += kGateThreads) {
            const float4 v = __ldg(v4 + c);
            acc[5 * MAXHC] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
            for (int j = 0; j < MAXHC; j++) {
                if (j < hc) {
                    const float4 k = __ldg(k4 + j * n4 + c), h = __ldg(h4 + j * n4 + c);
                    const float4 a = __ldg(reinterpret_cast<const float4*>(norm_key + (int64_t)j * n) + c);
                    const float4 b = __ldg(reinterpret_cast<const float4*>(norm_query + (int64_t)j * n) + c);
                    const float4 w = __ldg(reinterpret_cast<const float4*>(norm_conv + (int64_t)j * n) + c);
                    const float4 dn = __ldg(d4 + j * n4 + c), dy = __ldg(o4 + j * n4 + c);
                    acc[5 * j] += k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w;
                    acc[5 * j + 1] += h.x * h.x + h.y * h.y + h.z * h.z + h.w * h.w;
                    acc[5 * j + 2] += (k.x * a.x) * (h.x * b.x) + (k.y * a.y) * (h.y * b.y) +
                                      (k.z * a.z) * (h.z * b.z) + (k.w * a.w) * (h.w * b.w);
                    acc[5 * j + 3] += v.x * w.x * dn.x + v.y * w.y * dn.y + v.z * w.z * dn.z + v.w * w.w * dn.w;
                    acc[5 * j + 4] += dy.x * v.x + dy.y * v.y + dy.z * v.z + dy.w * v.w;
                }
            }
        }
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
            float A = 0.f, B = 0.f, Cq = 0.f, E = 0.f, F = 0.f, V = 0.f;
#pragma unroll
            for (int w = 0; w < kGateThreads / 32; w++) {
                A += part[w][5 * j];
                B += part[w][5 * j + 1];
                Cq += part[w][5 * j + 2];
                E += part[w][5 * j + 3];
                F += part[w][5 * j + 4];
                V += part[w][5 * MAXHC];
            }
            const float rk = 1.0f / sqrtf(A / fn + eps);
            const float rq = 1.0f / sqrtf(B / fn + eps);
            const float g = gate[t * hc + j];
            const float s = s_in[t * hc + j];
            const float rg = 1.0f / sqrtf(g * g * (V / fn) + eps);
            const float cg = g * g * rg * rg * rg * E / fn;
            float dgate = detach_gate ? 0.f : F + rg * E - cg * V;
            const float as = fabsf(s);
            const float ds = as >= 1e-6f ? dgate * g * (1.0f - g) * 0.5f / sqrtf(as) : 0.f;
            const float u = ds / sqrtf(fn);
            coef[8 * j] = g;
            coef[8 * j + 1] = rg;
            coef[8 * j + 2] = cg;
            coef[8 * j + 3] = u * rq * rk;
            coef[8 * j + 4] = u * rq * rk * rk * rk * Cq / fn;
            coef[8 * j + 5] = u * rk * rq;
            coef[8 * j + 6] = u * rk * rq * rq * rq * Cq / fn;
        }
        __syncthreads();
        for (int c = tid; c < n4; c += kGateThreads) {
            const float4 v = __ldg(v4 + c);
            float dv[4] = {0.f, 0.f, 0.f, 0.f};
            const float vs[4] = {v.x, v.y, v.z, v.w};
            for (int j = 0; j < hc; j++) {
                const float g = coef[8 * j], rg = coef[8 * j + 1], cg = coef[8 * j + 2];
                const float ck1 = coef[8 * j + 3], ck2 = coef[8 * j + 4], ch1 = coef[8 * j + 5], ch2 = coef[8 * j + 6];
                const float4 k = __ldg(k4 + j * n4 + c), h = __ldg(h4 + j * n4 + c);
                const float4 a = __ldg(reinterpret_cast<const float4*>(norm_key + (int64_t)j * n) + c);
                const float4 b = __ldg(reinterpret_cast<const float4*>(norm_query + (int64_t)j * n) + c);
                const float4 w = __ldg(reinterpret_cast<const float4*>(norm_conv + (int64_t)j * n) + c);
                const float4 dn = __ldg(d4 + j * n4 + c), dy = __ldg(o4 + j * n4 + c);
                const float ks[4] = {k.x, k.y, k.z, k.w}, hs[4] = {h.x, h.y, h.z, h.w};
                const float as[4] = {a.x, a.y, a.z, a.w}, bs[4] = {b.x, b.y, b.z, b.w};
                const float ws[4] = {w.x, w.y, w.z, w.w}, dns[4] = {dn.x, dn.y, dn.z, dn.w};
                const float dys[4] = {dy.x, dy.y, dy.z, dy.w};
                float dk[4], dh[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float dgated = dys[q] + rg * ws[q] * dns[q] - cg * vs[q];
                    dv[q] += dgated * g;
                    dk[q] = ck1 * as[q] * bs[q] * hs[q] - ck2 * ks[q];
                    dh[q] = dys[q] + ch1 * bs[q] * as[q] * ks[q] - ch2 * hs[q];
                }
                reinterpret_cast<float4*>(dkey + t * dkey_stride + (int64_t)j * n)[c] =
                    make_float4(dk[0], dk[1], dk[2], dk[3]);
                reinterpret_cast<float4*>(dhidden + (t * hc + j) * (int64_t)n)[c] =
                    make_float4(dh[0], dh[1], dh[2], dh[3]);
            }
            if (detach_value) dv[0] = dv[1] = dv[2] = dv[3] = 0.f;
            reinterpret_cast<float4*>(dvalue + t * dvalue_stride)[c] = make_float4(dv[0], dv[1], dv[2], dv[3]);
        }
        __syncthreads();  // part and coef are rewritten by the next position
    }
}

// Backward of the conv + silu, step 1: dconv[t, c] = dout[t, c] * silu'(conv[t, c])
// with conv recomputed as k_ple_conv forms it; silu'(x) = sig(x) (1 + x (1 - sig(x))).
__global__ void __launch_bounds__(256) k_ple_dconv(const float* __restrict__ normed, const float* __restrict__ hist,
                                                   int64_t hist_len, const float* __restrict__ conv_w, int K,
                                                   int dilation, int64_t T, int C, const float* __restrict__ dout,
                                                   float* __restrict__ dconv) {
    const int64_t total = T * (int64_t)C;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / C;
        const int c = (int)(e - t * C);
        float acc = 0.f;
        for (int k = 0; k < K; k++) {
            const int64_t src = t - (int64_t)(K - 1 - k) * dilation;
            const float* row = src >= 0 ? normed + src * C : (hist_len + src >= 0 ? hist + (hist_len + src) * C : nullptr);
            if (row == nullptr) continue;
            acc = __fadd_rn(acc, __fmul_rn(__ldg(row + c), __ldg(conv_w + (int64_t)c * K + k)));
        }
        const float sg = sigmoidf_(acc);
        dconv[e] = __ldg(dout + e) * (sg * (1.0f + acc * (1.0f - sg)));
    }
}

// Step 2: the transposed (anti-causal) conv.  Row u of [hist; normed] (u from
// -hist_len to T-1) feeds output t = u + (K-1-k) * dilation through tap k, so
// its gradient is sum_k w[c, k] * dconv[u + (K-1-k) * dilation, c] over the
// outputs that exist, plus the gradient of the new history tail when row u is
// one of its rows (dtail [tail_len, C]: rows hist_len + T - tail_len.. of the
// concatenation).  Rows u >= 0 go to dnormed, rows u < 0 to dhist (nullable).
__global__ void __launch_bounds__(256) k_ple_dx(const float* __restrict__ dconv, const float* __restrict__ conv_w,
                                                int K, int dilation, int64_t T, int C, int64_t hist_len,
                                                const float* __restrict__ dtail, int64_t tail_len,
                                                float* __restrict__ dnormed, float* __restrict__ dhist) {
    const int64_t rows = hist_len + T;
    const int64_t total = rows * (int64_t)C;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / C;  // row of the concatenation
        const int c = (int)(e - r * C);
        const int64_t u = r - hist_len;
        float acc = 0.f;
        for (int k = K - 1; k >= 0; k--) {
            const int64_t t = u + (int64_t)(K - 1 - k) * dilation;
            if (t < 0 || t >= T) continue;
            acc = __fadd_rn(acc, __fmul_rn(__ldg(conv_w + (int64_t)c * K + k), __ldg(dconv + t * C + c)));
        }
        const int64_t tr = r - (rows - tail_len);
        if (dtail && tr >= 0) acc = __fadd_rn(acc, __ldg(dtail + tr * C + c));
        if (u >= 0) dnormed[u * C + c] = acc;
        else if (dhist) dhist[r * C + c] = acc;
    }
}

// The two steps above for the reference's K = 4 with 16-byte aligned rows: a
// thread owns a channel quad (its 16 tap weights stay in registers) and walks
// positions with a grid stride, so every row access is one float4 load and no
// index needs a division.  The per-channel arithmetic and its order are those
// of the scalar kernels.
__global__ void __launch_bounds__(256) k_ple_dconv4(const float* __restrict__ normed, const float* __restrict__ hist,
                                                    int64_t hist_len, const float* __restrict__ conv_w, int dilation,
                                                    int64_t T, int C, const float* __restrict__ dout,
                                                    float* __restrict__ dconv) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;  // channel quad: channels 4q..4q+3
    if (q >= (C >> 2)) return;
    float w[4][4];  // w[channel][tap]
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(conv_w) + (4 * q + ch));
        w[ch][0] = v.x, w[ch][1] = v.y, w[ch][2] = v.z, w[ch][3] = v.w;
    }
    for (int64_t t = blockIdx.y; t < T; t += gridDim.y) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t src = t - (int64_t)(3 - k) * dilation;
            const float* row = src >= 0 ? normed + src * C : (hist_len + src >= 0 ? hist + (hist_len + src) * C : nullptr);
            if (row == nullptr) continue;
            const float4 x = __ldg(reinterpret_cast<const float4*>(row) + q);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(x.x, w[0][k]));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(x.y, w[1][k]));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(x.z, w[2][k]));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(x.w, w[3][k]));
        }
        const float4 d = __ldg(reinterpret_cast<const float4*>(dout + t * C) + q);
        const float dd[4] = {d.x, d.y, d.z, d.w};
        float o[4];
#pragma unroll
        for (int ch = 0; ch < 4; ch++) {
            const float sg = sigmoidf_(acc[ch]);
            o[ch] = dd[ch] * (sg * (1.0f + acc[ch] * (1.0f - sg)));
        }
        reinterpret_cast<float4*>(dconv + t * C)[q] = make_float4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void __launch_bounds__(256) k_ple_dx4(const float* __restrict__ dconv, const float* __restrict__ conv_w,
                                                 int dilation, int64_t T, int C, int64_t hist_len,
                                                 const float* __restrict__ dtail, int64_t tail_len,
                                                 float* __restrict__ dnormed, float* __restrict__ dhist) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (C >> 2)) return;
    float w[4][4];
#pragma unroll
    for (int ch = 0; ch < 4; ch++) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(conv_w) + (4 * q + ch));
        w[ch][0] = v.x, w[ch][1] = v.y, w[ch][2] = v.z, w[ch][3] = v.w;
    }
    const int64_t rows = hist_len + T;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const int64_t u = r - hist_len;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 3; k >= 0; k--) {
            const int64_t t = u + (int64_t)(3 - k) * dilation;
            if (t < 0 || t >= T) continue;
            const float4 g = __ldg(reinterpret_cast<const float4*>(dconv + t * C) + q);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(w[0][k], g.x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(w[1][k], g.y));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(w[2][k], g.z));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(w[3][k], g.w));
        }
        const int64_t tr = r - (rows - tail_len);
        if (dtail && tr >= 0) {
            const float4 d = __ldg(reinterpret_cast<const float4*>(dtail + tr * C) + q);
            acc[0] = __fadd_rn(acc[0], d.x);
            acc[1] = __fadd_rn(acc[1], d.y);
            acc[2] = __fadd_rn(acc[2], d.z);
            acc[3] = __fadd_rn(acc[3], d.w);
        }
        const float4 o = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (u >= 0) reinterpret_cast<float4*>(dnormed + u * C)[q] = o;
        else if (dhist) reinterpret_cast<float4*>(dhist + r * C)[q] = o;
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
    if (hc <= 4)  // the reference's hc: fewer sums live and no skipped streams in the unrolled loops
        k_ple_gate<4><<<blocks, kGateThreads, 0, (cudaStream_t)stream>>>(key, key_stride, value, value_stride, hidden,
                                                                   norm_key, norm_query, norm_conv, T, hc, n_embd, eps,
                                                                   gate, s_out, normed);
    else
        k_ple_gate<kPleMaxHc><<<blocks, kGateThreads, 0, (cudaStream_t)stream>>>(key, key_stride, value, value_stride, hidden,
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

extern "C" int engram_ple_gate_backward(const float* key, int64_t key_stride, const float* value, int64_t value_stride,
                                        const float* hidden, const float* norm_key, const float* norm_query,
                                        const float* norm_conv, const float* gate, const float* s, const float* dout,
                                        const float* dnormed, int64_t T, int32_t hc, int32_t n_embd, float eps,
                                        int32_t detach_value, int32_t detach_gate, float* dkey, int64_t dkey_stride,
                                        float* dvalue, int64_t dvalue_stride, float* dhidden, void* stream) {
    if (T < 0 || hc < 1 || hc > kPleMaxHc || n_embd < 4 || (n_embd & 3)) return ENGRAM_ERR_ARG;
    if (key_stride < (int64_t)hc * n_embd || value_stride < n_embd || (key_stride & 3) || (value_stride & 3) ||
        dkey_stride < (int64_t)hc * n_embd || dvalue_stride < n_embd || (dkey_stride & 3) || (dvalue_stride & 3))
        return ENGRAM_ERR_ARG;
    if (T == 0) return ENGRAM_OK;
    if (!key || !value || !hidden || !norm_key || !norm_query || !norm_conv || !gate || !s || !dout || !dnormed ||
        !dkey || !dvalue || !dhidden)
        return ENGRAM_ERR_ARG;
    if (!aligned16(key) || !aligned16(value) || !aligned16(hidden) || !aligned16(norm_key) || !aligned16(norm_query) ||
        !aligned16(norm_conv) || !aligned16(dout) || !aligned16(dnormed) || !aligned16(dkey) || !aligned16(dvalue) ||
        !aligned16(dhidden))
        return ENGRAM_ERR_ARG;
    const int64_t cap = (int64_t)sm_count() * 8;
    const int blocks = (int)(T < cap ? T : cap);
    if (hc <= 4)  // the reference's hc: a quarter of the accumulators live, twice the resident blocks
        k_ple_gate_bwd<4><<<blocks, kGateThreads, 0, (cudaStream_t)stream>>>(
        key, key_stride, value, value_stride, hidden, norm_key, norm_query, norm_conv, gate, s, dout, dnormed, T, hc,
        n_embd, eps, detach_value, detach_gate, dkey, dkey_stride, dvalue, dvalue_stride, dhidden);
    else
        k_ple_gate_bwd<kPleMaxHc><<<blocks, kGateThreads, 0, (cudaStream_t)stream>>>(
        key, key_stride, value, value_stride, hidden, norm_key, norm_query, norm_conv, gate, s, dout, dnormed, T, hc,
        n_embd, eps, detach_value, detach_gate, dkey, dkey_stride, dvalue, dvalue_stride, dhidden);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

extern "C" int engram_ple_conv_backward(const float* normed, const float* hist, int64_t hist_len, const float* conv_w,
                                        int32_t K, int32_t dilation, int64_t T, int32_t hc, int32_t n_embd,
                                        const float* dout, const float* dtail, int64_t tail_len, float* dconv,
                                        float* dnormed, float* dhist, void* stream) {
    if (T < 0 || hc < 1 || hc > kPleMaxHc || n_embd < 4 || (n_embd & 3) || K < 1 || dilation < 1 || hist_len < 0 ||
        tail_len < 0 || tail_len > hist_len + T)
        return ENGRAM_ERR_ARG;
    if (T == 0 && hist_len == 0) return ENGRAM_OK;
    if ((int64_t)hc * n_embd >= ((int64_t)1 << 30)) return ENGRAM_ERR_RANGE;
    if ((T > 0 && (!normed || !dout || !dconv || !dnormed)) || !conv_w || (hist_len > 0 && !hist) ||
        (tail_len > 0 && !dtail))
        return ENGRAM_ERR_ARG;
    const int C = hc * n_embd;
    const int64_t cap = (int64_t)sm_count() * 8;
    cudaStream_t st = (cudaStream_t)stream;
    int launched = 0;
    const bool vec = K == 4 && aligned16(conv_w) && (T == 0 || (aligned16(normed) && aligned16(dout) &&
                                                              aligned16(dconv) && aligned16(dnormed))) &&
                     (hist_len == 0 || aligned16(hist)) && (!dhist || aligned16(dhist)) &&
                     (tail_len == 0 || aligned16(dtail));
    if (vec) {  // channel quads x strided positions, as k_ple_conv<4>
        const int gx = (C / 4 + 255) / 256;
        const int64_t want_y = ((int64_t)sm_count() * 8 + gx - 1) / gx;
        if (T > 0) {
            const int64_t gy = T < want_y ? T : (want_y < 65535 ? want_y : 65535);
            k_ple_dconv4<<<dim3(gx, (unsigned)gy), 256, 0, st>>>(normed, hist, hist_len, conv_w, dilation, T, C, dout,
                                                                 dconv);
            launched++;
        }
        const int64_t rows = hist_len + T;
        const int64_t gy = rows < want_y ? rows : (want_y < 65535 ? want_y : 65535);
        k_ple_dx4<<<dim3(gx, (unsigned)gy), 256, 0, st>>>(dconv, conv_w, dilation, T, C, hist_len, dtail, tail_len,
                                                          dnormed, dhist);
        launched++;
        count_launches(launched);
        return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
    }
    if (T > 0) {
        const int64_t want = (T * (int64_t)C + 255) / 256;
        k_ple_dconv<<<(int)(want < cap ? want : cap), 256, 0, st>>>(normed, hist, hist_len, conv_w, K, dilation, T, C,
                                                                  dout, dconv);
        launched++;
    }
    const int64_t want = ((hist_len + T) * (int64_t)C + 255) / 256;
    k_ple_dx<<<(int)(want < cap ? want : cap), 256, 0, st>>>(dconv, conv_w, K, dilation, T, C, hist_len, dtail,
                                                           tail_len, dnormed, dhist);
    launched++;
    count_launches(launched);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
