// engram_adam.cu -- K4: the optimizer step over the overlay rows, fused with the
// gradient of the descent's regulariser (engraft/descend_corpus.py:921-947).
// The update follows torch.optim.Adam's single-tensor rule op for op (lerp as
// one fma, then v*b2 + ((1-b2)*g)*g, sqrt(v)/sqrt(bc2) + eps, p + (-ss*m)/den)
// with IEEE-rounded sqrt and division, so it matches the CPU oracle bit for bit.
#include "engram_common.cuh"

using namespace engram;

namespace {

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

// Data-parallel optimizer step over peer memory, owner side.  recv is this
// rank's receive buffer [world, size, dim]: block k holds rank k's row
// gradients of the rows this rank owns (written there by the backward,
// engram_backward_to_owners).  For each owned element: the sum of the blocks
// in rank order, the Adam update of this rank's copy of the parameter (m, v,
// p0 hold the owned rows only), and a store of the result into every rank's
// rows_var (rows[k], mapped over NVLink).  No waits inside: the caller orders
// the ranks around the launch.
template <int W>  // W > 0: world size known at compile time; 0: any
__global__ void __launch_bounds__(256) k_adam_owner_vec4(const float4* __restrict__ recv, int64_t shard4,
                                                         float4* const* __restrict__ rows, int world, int rank,
                                                         int64_t lo4, float4* __restrict__ m, float4* __restrict__ v,
                                                         const float4* __restrict__ p0, AdamScalars a) {
    const int nw = W > 0 ? W : world;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < shard4;
         i += (int64_t)gridDim.x * blockDim.x) {
        float4 gg;
        if (W > 0) {
            float4 x[W > 0 ? W : 1];
#pragma unroll
            for (int k = 0; k < W; k++) x[k] = __ldcs(recv + k * shard4 + i);
            gg = x[0];
#pragma unroll
            for (int k = 1; k < W; k++) {
                gg.x = __fadd_rn(gg.x, x[k].x);
                gg.y = __fadd_rn(gg.y, x[k].y);
                gg.z = __fadd_rn(gg.z, x[k].z);
                gg.w = __fadd_rn(gg.w, x[k].w);
            }
        } else {
            gg = __ldcs(recv + i);
            for (int k = 1; k < nw; k++) {
                const float4 x = __ldcs(recv + k * shard4 + i);
                gg.x = __fadd_rn(gg.x, x.x);
                gg.y = __fadd_rn(gg.y, x.y);
                gg.z = __fadd_rn(gg.z, x.z);
                gg.w = __fadd_rn(gg.w, x.w);
            }
        }
        float4 pp = rows[rank][lo4 + i], mm = m[i], vv = v[i];
        const float4 q = p0 ? __ldg(p0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const bool reg = p0 != nullptr;
        adam_elem(pp.x, gg.x, mm.x, vv.x, q.x, reg, a);
        adam_elem(pp.y, gg.y, mm.y, vv.y, q.y, reg, a);
        adam_elem(pp.z, gg.z, mm.z, vv.z, q.z, reg, a);
        adam_elem(pp.w, gg.w, mm.w, vv.w, q.w, reg, a);
        m[i] = mm;
        v[i] = vv;
        for (int k = 0; k < nw; k++) __stcg(rows[k] + lo4 + i, pp);
    }
}

AdamScalars adam_scalars(int64_t step, double lr, double beta1, double beta2, double eps, float reg_scale) {
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
    return a;
}

int grid_for(int64_t work, int threads, int per_sm) {
    const int64_t want = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int64_t g = want < cap ? want : cap;
    return (int)(g > 0 ? g : 1);
}

}  // namespace

extern "C" int engram_adam_step(float* p, const float* g, float* m, float* v, const float* p0, int64_t numel,
                                int64_t step, double lr, double beta1, double beta2, double eps, float reg_scale,
                                void* stream) {
    if (numel < 0 || step < 1) return ENGRAM_ERR_ARG;
    if (numel == 0) return ENGRAM_OK;
    if (!p || !g || !m || !v) return ENGRAM_ERR_ARG;
    const AdamScalars a = adam_scalars(step, lr, beta1, beta2, eps, reg_scale);
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


extern "C" int engram_adam_owner_step(const float* recv, const void* rows_ptrs, int32_t world, int32_t rank,
                                      int64_t R, int32_t dim, float* m, float* v, const float* p0, int64_t step,
                                      double lr, double beta1, double beta2, double eps, float reg_scale,
                                      void* stream) {
    if (world < 1 || rank < 0 || rank >= world || R < 0 || dim <= 0 || step < 1) return ENGRAM_ERR_ARG;
    if (dim & 3) return ENGRAM_ERR_FORMAT;  // float4 pieces
    const int64_t base = R / world, extra = R % world;
    const int64_t lo = rank * base + (rank < extra ? rank : extra);
    const int64_t size = base + (rank < extra ? 1 : 0);
    if (size == 0) return ENGRAM_OK;
    if (!recv || !rows_ptrs || !m || !v) return ENGRAM_ERR_ARG;
    if (!aligned16(recv) || !aligned16(m) || !aligned16(v) || (p0 && !aligned16(p0))) return ENGRAM_ERR_ARG;
    const AdamScalars a = adam_scalars(step, lr, beta1, beta2, eps, reg_scale);
    const int64_t shard4 = size * dim / 4, lo4 = lo * dim / 4;
    const int grid = grid_for(shard4, 256, 8);
    cudaStream_t s = (cudaStream_t)stream;
    const float4* r4 = reinterpret_cast<const float4*>(recv);
    float4* const* rows4 = static_cast<float4* const*>(rows_ptrs);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    const float4* q4 = reinterpret_cast<const float4*>(p0);
    switch (world) {
        case 1: k_adam_owner_vec4<1><<<grid, 256, 0, s>>>(r4, shard4, rows4, world, rank, lo4, m4, v4, q4, a); break;
        case 2: k_adam_owner_vec4<2><<<grid, 256, 0, s>>>(r4, shard4, rows4, world, rank, lo4, m4, v4, q4, a); break;
        case 4: k_adam_owner_vec4<4><<<grid, 256, 0, s>>>(r4, shard4, rows4, world, rank, lo4, m4, v4, q4, a); break;
        case 8: k_adam_owner_vec4<8><<<grid, 256, 0, s>>>(r4, shard4, rows4, world, rank, lo4, m4, v4, q4, a); break;
        default: k_adam_owner_vec4<0><<<grid, 256, 0, s>>>(r4, shard4, rows4, world, rank, lo4, m4, v4, q4, a);
    }
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}
