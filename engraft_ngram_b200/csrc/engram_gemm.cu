// engram_gemm.cu -- the PLE block's projections on the tensor cores (sm_100a
// tcgen05): C[M, N] = sum over terms p of A_p[M, K] @ B_p[N, K]^T, every operand
// K-major fp32 read as TF32, fp32 accumulation in tensor memory.  With the
// three terms (A_lo, B_hi), (A_hi, B_lo), (A_hi, B_hi) of the split x = hi + lo
// (hi = x with its low 13 mantissa bits cleared) this is the 3xTF32 product,
// accurate to fp32 level; one term (A, B) is a plain TF32 GEMM.
//
// One CTA per 128 x 256 output tile, 192 threads:
//   warp 0, one lane: the producer.  For every 32-wide K slice of every term it
//     waits until a shared-memory stage is free, arms the stage's "full"
//     barrier with the slice's byte count and issues two TMA tile loads
//     (cp.async.bulk.tensor, 128-byte swizzle; no multicast): A rows m0..m0+127
//     and B rows n0..n0+255, columns k..k+31;
//   warp 1: allocates 256 TMEM columns (the fp32 accumulator, 128 lanes x 256),
//     and one lane issues the MMAs: per stage, 4 tcgen05.mma kind::tf32 of
//     128 x 256 x 8 from shared-memory descriptors, then tcgen05.commit to the
//     stage's "empty" barrier (the stage is refilled once those MMAs have read
//     it); after the last slice, tcgen05.commit to the accumulator barrier;
//   warps 2..5 (TMEM lanes 32*(w%4)..+31): wait for the accumulator, read it
//     with tcgen05.ld (32 columns at a time) and store the rows of C.
// engram_gemm_3xtf32 runs the fused form: per 16-wide K slice the stage holds
// A_hi, A_lo, B_hi and B_lo (64-byte swizzle) and the MMA lane issues the three
// products from them, so the shared operands are loaded once (a third less
// traffic than three separate terms).  The grid runs M tiles fastest: the CTAs
// resident together share B tiles, which are then read from DRAM about once.
// STAGES stages of 48 KB.  Every wait on a barrier is bounded: after
// kSpinLimit polls the thread records the failure in *err (nullable) and
// stops its loop; the CTA still drains its TMA loads and MMAs (bounded waits
// again) and frees its TMEM before it returns.  Rows, columns and K beyond the
// operands are zero-filled by the TMA unit and never stored.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "engram_common.cuh"

using namespace engram;

namespace {

constexpr int BM = 128, BN = 256;
constexpr int STAGES = 4;
// Plain terms: per stage A [128 x 32] and B [256 x 32] (32 fp32 = one 128-byte swizzle row).
// Fused 3xTF32: per stage A_hi, A_lo [128 x 16] and B_hi, B_lo [256 x 16] (64-byte swizzle rows),
// so the operands the three products share are loaded once.  Both are 48 KB per stage.
template <bool FUSED>
struct Cfg {
    static constexpr int BK = FUSED ? 16 : 32;
    static constexpr int ROW_BYTES = BK * 4;
    static constexpr int A_BYTES = BM * ROW_BYTES, B_BYTES = BN * ROW_BYTES;
    static constexpr int STAGE_BYTES = FUSED ? 2 * (A_BYTES + B_BYTES) : A_BYTES + B_BYTES;
    static constexpr uint32_t SWIZZLE = FUSED ? 4u : 2u;      // descriptor layout type: 64-byte / 128-byte
    static constexpr uint32_t SBO = 8 * ROW_BYTES;            // 8-row groups
};
constexpr int BK = 32;  // the plain kernel's K slice (used by the host's tensor maps)
constexpr int SMEM_BYTES = STAGES * Cfg<false>::STAGE_BYTES + 1024 /* alignment */ + 256 /* barriers */;
static_assert(Cfg<true>::STAGE_BYTES == Cfg<false>::STAGE_BYTES, "one shared-memory size for both kernels");
constexpr int kThreads = 192;
constexpr int kMaxTerms = 3;
constexpr uint32_t kTmemCols = 256;
constexpr long long kSpinLimit = 1ll << 24;

struct GemmMaps {
    CUtensorMap a[kMaxTerms];  // fused: a[0] = A_hi, a[1] = A_lo
    CUtensorMap b[kMaxTerms];  // fused: b[0] = B_hi, b[1] = B_lo
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity; false (and *err raised) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
    for (long long it = 0; it < kSpinLimit; it++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicAdd(err, 1);
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with a
// 128-byte (layout type 2) or 64-byte (type 4) swizzle: rows of 128 or 64
// bytes, 8-row groups sbo bytes apart.
template <bool FUSED>
__device__ __forceinline__ uint64_t smem_desc_k(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);                       // start address
    d |= (uint64_t)1u << 16;                                      // leading byte offset (unused when swizzled)
    d |= (uint64_t)((Cfg<FUSED>::SBO >> 4) & 0x3FFFu) << 32;      // stride byte offset: 8-row groups
    d |= (uint64_t)1u << 46;                                      // descriptor version for sm_100
    d |= (uint64_t)Cfg<FUSED>::SWIZZLE << 61;                     // swizzle mode
    return d;
}

// Instruction descriptor: A and B TF32, K-major; D fp32; M = 128, N = 256.
constexpr uint32_t kInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kInstrDesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

template <bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_tf32(const __grid_constant__ GemmMaps maps, int n_terms,
                                                           int64_t M, int64_t N, int64_t K, float* __restrict__ c,
                                                           int64_t ldc, int* err) {
    using G = Cfg<FUSED>;
    constexpr int SK = G::BK;
    constexpr int STAGE_BYTES = G::STAGE_BYTES, A_BYTES = G::A_BYTES, B_BYTES = G::B_BYTES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), acc_bar = smem_u32(bars + 2 * STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // M tiles vary fastest across the grid, so the CTAs resident together share B tiles (the large operand)
    const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
    const int k_slices = (int)((K + SK - 1) / SK);
    const int total = FUSED ? k_slices : k_slices * n_terms;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {  // the accumulator: 256 TMEM columns of 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued[STAGES] = {0, 0, 0, 0};  // loads issued per stage (its last phase is issued - 1)
            bool ok = true;
            for (int i = 0; i < total && ok; i++) {
                const int s = i % STAGES, round = i / STAGES;
                if (round > 0) ok = mbar_wait(empty0 + 8 * s, (uint32_t)((round - 1) & 1), err);
                if (!ok) break;
                const int term = FUSED ? 0 : i / k_slices, kk = (i % k_slices) * SK;
                const uint32_t bar = full0 + 8 * s;
                mbar_expect_tx(bar, STAGE_BYTES);
                uint8_t* st = smem + s * STAGE_BYTES;
                tma_load_2d(smem_u32(st), &maps.a[term], kk, (int)m0, bar);
                tma_load_2d(smem_u32(st + A_BYTES), &maps.b[term], kk, (int)n0, bar);
                if (FUSED) {  // the remainders: A_lo, B_lo
                    tma_load_2d(smem_u32(st + A_BYTES + B_BYTES), &maps.a[1], kk, (int)m0, bar);
                    tma_load_2d(smem_u32(st + 2 * A_BYTES + B_BYTES), &maps.b[1], kk, (int)n0, bar);
                }
                issued[s]++;
            }
            // drain: every load issued into this CTA's shared memory has landed
            for (int s = 0; s < STAGES; s++)
                if (issued[s] > 0) mbar_wait(full0 + 8 * s, (uint32_t)((issued[s] - 1) & 1), err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int done = 0;
            for (int i = 0; i < total && ok; i++) {
                const int s = i % STAGES, round = i / STAGES;
                ok = mbar_wait(full0 + 8 * s, (uint32_t)(round & 1), err);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES), b_addr = a_addr + A_BYTES;
#pragma unroll
                for (int k = 0; k < SK / 8; k++) {  // 8 TF32 = 32 bytes per MMA along the swizzled row
                    const uint32_t first = (i > 0 || k > 0) ? 1u : 0u;
                    if (FUSED) {  // the small terms first: A_lo B_hi, A_hi B_lo, then A_hi B_hi
                        const uint32_t alo = b_addr + B_BYTES, blo = alo + A_BYTES;
                        umma_tf32(tmem, smem_desc_k<FUSED>(alo + 32 * k), smem_desc_k<FUSED>(b_addr + 32 * k), first);
                        umma_tf32(tmem, smem_desc_k<FUSED>(a_addr + 32 * k), smem_desc_k<FUSED>(blo + 32 * k), 1u);
                        umma_tf32(tmem, smem_desc_k<FUSED>(a_addr + 32 * k), smem_desc_k<FUSED>(b_addr + 32 * k), 1u);
                    } else {
                        umma_tf32(tmem, smem_desc_k<FUSED>(a_addr + 32 * k), smem_desc_k<FUSED>(b_addr + 32 * k),
                                  first);
                    }
                }
                umma_commit(empty0 + 8 * s);  // the stage is free once these MMAs have read it
                done++;
            }
            umma_commit(acc_bar);  // arrives when every MMA issued above has completed
            (void)done;
        }
        __syncwarp();
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4)..+31, i.e. rows m0 + 32*(w%4) + lane
        const int q = warp & 3;
        const bool ok = mbar_wait(acc_bar, 0u, err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int64_t row = m0 + 32 * q + lane;
        const bool vec = (ldc & 3) == 0 && ((reinterpret_cast<uintptr_t>(c) & 15) == 0);
        for (int col = 0; col < BN; col += 32) {
            uint32_t r[32];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                  "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                  "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (!ok || row >= M) continue;
            float* dst = c + row * ldc + n0 + col;
            const int64_t left = N - (n0 + col);
            if (vec && left >= 32) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(dst + j) =
                        make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                    __uint_as_float(r[j + 3]));
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (j < left) dst[j] = __uint_as_float(r[j]);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D map of a row-major fp32 matrix [rows, K] (row stride ld floats), boxes of
// box_rows x box_k columns, 128-byte (box_k 32) or 64-byte (box_k 16) swizzle.
bool make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t K, int64_t ld, int box_rows, int box_k) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    const cuuint32_t box[2] = {(cuuint32_t)box_k, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, box_k == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool FUSED>
int launch_gemm(const GemmMaps& maps, int n_terms, int64_t M, int64_t N, int64_t K, float* c, int64_t ldc, int32_t* err,
                cudaStream_t stream) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(k_gemm_tf32<FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return ENGRAM_ERR_CUDA;
        configured[dev] = true;
    }
    const dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)((N + BN - 1) / BN));
    if (grid.y > 65535) return ENGRAM_ERR_RANGE;
    k_gemm_tf32<FUSED><<<grid, kThreads, SMEM_BYTES, stream>>>(maps, n_terms, M, N, K, c, ldc, err);
    count_launches(1);
    return cudaGetLastError() == cudaSuccess ? ENGRAM_OK : ENGRAM_ERR_CUDA;
}

int check_shape(int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc) {
    if (M < 0 || N < 0 || K < 0) return ENGRAM_ERR_ARG;
    if (M == 0 || N == 0) return 1;
    if (K == 0 || (K & 3) || lda < K || ldb < K || ldc < N || (lda & 3) || (ldb & 3)) return ENGRAM_ERR_ARG;
    if (M > INT32_MAX - BM || N > INT32_MAX - BN || K > INT32_MAX - BK) return ENGRAM_ERR_RANGE;
    return 0;
}

}  // namespace

extern "C" int engram_gemm_tf32(int32_t n_terms, const float* const* a, const float* const* b, int64_t M, int64_t N,
                                int64_t K, int64_t lda, int64_t ldb, float* c, int64_t ldc, int32_t* err,
                                void* stream) {
    if (n_terms < 1 || n_terms > kMaxTerms || !a || !b || !c) return ENGRAM_ERR_ARG;
    const int sh = check_shape(M, N, K, lda, ldb, ldc);
    if (sh != 0) return sh > 0 ? ENGRAM_OK : sh;
    for (int p = 0; p < n_terms; p++)
        if (!a[p] || !b[p] || !aligned16(a[p]) || !aligned16(b[p])) return ENGRAM_ERR_ARG;
    GemmMaps maps;
    memset(&maps, 0, sizeof(maps));
    for (int p = 0; p < n_terms; p++)
        if (!make_map(&maps.a[p], a[p], M, K, lda, BM, 32) || !make_map(&maps.b[p], b[p], N, K, ldb, BN, 32))
            return ENGRAM_ERR_CUDA;
    return launch_gemm<false>(maps, n_terms, M, N, K, c, ldc, err, (cudaStream_t)stream);
}

extern "C" int engram_gemm_3xtf32(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, float* c, int64_t ldc,
                                  int32_t* err, void* stream) {
    if (!c) return ENGRAM_ERR_ARG;
    const int sh = check_shape(M, N, K, lda, ldb, ldc);
    if (sh != 0) return sh > 0 ? ENGRAM_OK : sh;
    const float* ops[4] = {a_hi, a_lo, b_hi, b_lo};
    for (const float* x : ops)
        if (!x || !aligned16(x)) return ENGRAM_ERR_ARG;
    GemmMaps maps;
    memset(&maps, 0, sizeof(maps));
    if (!make_map(&maps.a[0], a_hi, M, K, lda, BM, 16) || !make_map(&maps.a[1], a_lo, M, K, lda, BM, 16) ||
        !make_map(&maps.b[0], b_hi, N, K, ldb, BN, 16) || !make_map(&maps.b[1], b_lo, N, K, ldb, BN, 16))
        return ENGRAM_ERR_CUDA;
    return launch_gemm<true>(maps, 3, M, N, K, c, ldc, err, (cudaStream_t)stream);
}
