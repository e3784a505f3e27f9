/*
 * engram_oracle.c -- CPU restatement of the reference's Engram/PLE table path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (engraft_ngram_b200/) links,
 * loads or calls this file.  It is the checker for the CUDA path: tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg are
 * the only callers.
 *
 * Every function cites the reference code it restates (paths are inside the
 * fulvian/engraft-ngram project).  Parity of this file with the reference is
 * pinned by tests/test_oracle_golden.py against fixtures produced by running
 * the reference itself (tests/golden/make_golden.py).
 *
 * Floating point: compiled with -ffp-contract=off so that every a*b+c below is
 * two roundings unless fmaf() is written out, exactly as the reference's
 * numpy/torch element-wise ops are.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { FMT_F32 = 0, FMT_IQ4_NL = 1, FMT_IQ4_XS = 2 };
enum { MODE_CONCAT_F32 = 0, MODE_PAIRSUM_ADD_BF16 = 1 };

/* engraft/table.py:26-29 (kvalues_iq4nl), same list at engraft/replica/dequant.py:30 */
static const float KV_IQ4NL[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f,
                                   1.f,    13.f,   25.f,  38.f,  53.f,  69.f,  89.f,  113.f};

/* IEEE binary16 -> binary32, exact (numpy .view(float16).astype(float32)). */
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_float(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> bfloat16, round to nearest even; NaN stays a quiet NaN. */
static uint16_t float_to_bf16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u);
    uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7fffu + lsb;
    return (uint16_t)(bits >> 16);
}

/*
 * The n-gram hash, engraft/table.py:111-144 (identical in
 * engraft/testing/fake_table.py:41-66, vectorised in engraft/damage.py:68-104).
 *
 * ctx = [x_t, x_{t-1}, ..., x_{t-N+1}].  A predecessor that is missing (before
 * the start of the sequence or, with segments, before the start of t's
 * segment -- engraft/replica/seq.py:393-399 passes tokens[s_t:]) or equal to
 * EOS cuts the context: it and every older slot read EOS.  The current token's
 * own EOS does not cut.  For n = 2..N: mixed = XOR_{j<n} (ctx[j]*mult[j] mod
 * 2^64); head (n-2)*hpn+g reads row mixed % p_h.  Output: global row ids
 * (head_offsets[h] + local, engraft/lens.py:108-110).
 *
 * tokens: the whole token list; positions t0 .. t0+n-1 are hashed.
 * seg_start: NULL, or [len] with seg_start[t] = first index of t's segment.
 */
void orc_hash(const int32_t* tokens, const int32_t* seg_start, int64_t t0, int64_t n,
              int32_t ngram_size, int32_t hpn, const uint64_t* mult,
              const int64_t* head_sizes, const int64_t* head_offsets, int64_t eos,
              int32_t* ids_out) {
    const int n_heads = (ngram_size - 1) * hpn;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int64_t t = t0 + i;
        int64_t lo = seg_start ? (int64_t)seg_start[t] : 0;
        int64_t ctx[8];
        ctx[0] = tokens[t];
        int cut = 0;
        for (int s = 1; s < ngram_size; s++) {
            int64_t pos = t - s;
            int64_t tok = eos;
            int have = (pos >= lo) && !cut;
            if (have) tok = tokens[pos];
            if (!have || tok == eos) {
                cut = 1;
                tok = eos;
            }
            ctx[s] = tok;
        }
        for (int nn = 2; nn <= ngram_size; nn++) {
            uint64_t mixed = (uint64_t)ctx[0] * mult[0];
            for (int j = 1; j < nn; j++) mixed ^= (uint64_t)ctx[j] * mult[j];
            int base = (nn - 2) * hpn;
            for (int g = 0; g < hpn; g++) {
                int h = base + g;
                uint64_t local = mixed % (uint64_t)head_sizes[h];
                ids_out[i * n_heads + h] = (int32_t)(head_offsets[h] + (int64_t)local);
            }
        }
    }
}

/*
 * Dequantise one row from the reference's raw byte layout.
 *   F32:    dim little-endian floats.
 *   IQ4_NL: dim/32 blocks of 18 B = fp16 d, qs[16]; y[j] = d*kv[qs[j]&15],
 *           y[j+16] = d*kv[qs[j]>>4]  (engraft/table.py:147-169,
 *           engraft/replica/dequant.py:127-147).
 *   IQ4_XS: dim/256 superblocks of 136 B = fp16 d, u16 scales_h, u8 scales_l[4],
 *           qs[128]; sub-block ib: ls = ((scales_l[ib/2] >> 4*(ib%2)) & 15) |
 *           (((scales_h >> 2*ib) & 3) << 4); dl = d*(ls-32); then the IQ4_NL
 *           rule on qs[16*ib..16*ib+15]  (engraft/replica/dequant.py:150-189).
 */
static void dequant_row(int fmt, int dim, const uint8_t* src, float* out) {
    if (fmt == FMT_F32) {
        memcpy(out, src, (size_t)dim * 4);
    } else if (fmt == FMT_IQ4_NL) {
        for (int b = 0; b < dim / 32; b++) {
            const uint8_t* blk = src + 18 * b;
            float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 16; j++) {
                out[32 * b + j] = KV_IQ4NL[blk[2 + j] & 15] * d;
                out[32 * b + 16 + j] = KV_IQ4NL[blk[2 + j] >> 4] * d;
            }
        }
    } else {
        for (int sb = 0; sb < dim / 256; sb++) {
            const uint8_t* blk = src + 136 * sb;
            float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
            uint32_t sh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8);
            const uint8_t* sl = blk + 4;
            const uint8_t* qs = blk + 8;
            for (int ib = 0; ib < 8; ib++) {
                int ls = ((sl[ib / 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
                float dl = d * (float)(ls - 32);
                for (int j = 0; j < 16; j++) {
                    out[256 * sb + 32 * ib + j] = dl * KV_IQ4NL[qs[16 * ib + j] & 15];
                    out[256 * sb + 32 * ib + 16 + j] = dl * KV_IQ4NL[qs[16 * ib + j] >> 4];
                }
            }
        }
    }
}

int64_t orc_raw_row_bytes(int32_t fmt, int32_t dim) {
    if (fmt == FMT_F32) return (int64_t)dim * 4;
    if (fmt == FMT_IQ4_NL) return (dim % 32) ? -1 : (int64_t)(dim / 32) * 18;
    if (fmt == FMT_IQ4_XS) return (dim % 256) ? -1 : (int64_t)(dim / 256) * 136;
    return -1;
}

void orc_dequant(int32_t fmt, int32_t dim, const uint8_t* raw, int64_t n, float* out) {
    int64_t rb = orc_raw_row_bytes(fmt, dim);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) dequant_row(fmt, dim, raw + i * rb, out + i * dim);
}

/* Membership of a global id in the overlay: the reference's `g in row_map`
 * (engraft/replica/seq.py:411-417), restated as a binary search over the
 * overlay ids sorted ascending; returns row_map[g] or -1. */
static int32_t overlay_slot(const int32_t* keys_sorted, const int32_t* vals, int64_t R, int32_t g) {
    int64_t lo = 0, hi = R;
    while (lo < hi) {
        int64_t mid = (lo + hi) / 2;
        if (keys_sorted[mid] < g) lo = mid + 1; else hi = mid;
    }
    return (lo < R && keys_sorted[lo] == g) ? vals[lo] : -1;
}

/*
 * Forward: OverlayEmb.build (engraft/replica/seq.py:372-444) on resident rows.
 * base[t,h] = dequantised true row of ids[t,h]; where ids[t,h] is an overlay
 * row, the value is rows_var[row_map[id]] instead (index_put, :433-441).
 *
 * mode CONCAT_F32:        out float [n, n_heads, dim]  (the reference's emb).
 * mode PAIRSUM_ADD_BF16:  out bf16 [n, hpn*dim] updated in place:
 *     out[t, g*dim+c] = bf16_rne( float(out[t,g*dim+c]) + (v[g][c] + v[hpn+g][c]) )
 *   (a builder-defined epilogue; the reference has no residual add).
 * slots_out (nullable): [n, n_heads] overlay slot or -1.
 */
void orc_forward(int32_t fmt, int32_t dim, const uint8_t* table_raw, int64_t n_rows,
                 const int32_t* ids, int64_t n, int32_t n_heads, int32_t hpn,
                 const float* ov_rows, const int32_t* ov_keys_sorted, const int32_t* ov_vals,
                 int64_t R, int32_t mode, void* out, int32_t* slots_out) {
    int64_t rb = orc_raw_row_bytes(fmt, dim);
    (void)n_rows;
#pragma omp parallel
    {
        float* tmp = (float*)malloc(sizeof(float) * (size_t)dim * (size_t)n_heads);
#pragma omp for schedule(static)
        for (int64_t t = 0; t < n; t++) {
            for (int h = 0; h < n_heads; h++) {
                int32_t g = ids[t * n_heads + h];
                int32_t slot = overlay_slot(ov_keys_sorted, ov_vals, R, g);
                if (slots_out) slots_out[t * n_heads + h] = slot;
                float* dst = tmp + (size_t)h * dim;
                if (slot >= 0)
                    memcpy(dst, ov_rows + (int64_t)slot * dim, (size_t)dim * 4);
                else
                    dequant_row(fmt, dim, table_raw + (int64_t)g * rb, dst);
            }
            if (mode == MODE_CONCAT_F32) {
                memcpy((float*)out + t * (int64_t)n_heads * dim, tmp, (size_t)n_heads * dim * 4);
            } else {
                uint16_t* res = (uint16_t*)out + t * (int64_t)hpn * dim;
                for (int g = 0; g < hpn; g++)
                    for (int c = 0; c < dim; c++) {
                        float s = tmp[(size_t)g * dim + c] + tmp[(size_t)(hpn + g) * dim + c];
                        float r = bf16_to_float(res[g * dim + c]) + s;
                        res[g * dim + c] = float_to_bf16(r);
                    }
            }
        }
        free(tmp);
    }
}

/*
 * Backward of the overlay substitution: autograd of rows_var[idx_r] through
 * index_put (engraft/replica/seq.py:433-441).  grad_rows[r] = sum over the
 * (t,h) with slot(t,h) = r of the upstream gradient at (t,h), accumulated
 * from +0 in ascending flat order t*n_heads+h -- the order of the reference's
 * idx lists (:401-417) and the order in which index_put_(accumulate=True)
 * adds duplicates (serially on one CPU thread; stable sort on CUDA).
 *
 * mode CONCAT_F32:       grad float [n, n_heads, dim], term = grad[t,h,:].
 * mode PAIRSUM_ADD_BF16: grad bf16 [n, hpn*dim], term = float(grad[t, (h%hpn)*dim : +dim]).
 *
 * Threads own disjoint slot ranges and each scans all hits in order, so the
 * per-slot order is the sequential one whatever the thread count.
 */
void orc_backward(const int32_t* slots, int64_t n, int32_t n_heads, int32_t hpn, int32_t mode,
                  const void* grad, int32_t dim, int64_t R, float* grad_rows) {
    memset(grad_rows, 0, sizeof(float) * (size_t)R * dim);
    int64_t nh = n * n_heads;
#pragma omp parallel
    {
        int nt = 1, me = 0;
#ifdef _OPENMP
        nt = omp_get_num_threads();
        me = omp_get_thread_num();
#endif
        int64_t lo = R * me / nt, hi = R * (me + 1) / nt;
        for (int64_t i = 0; i < nh; i++) {
            int32_t s = slots[i];
            if (s < lo || s >= hi) continue;
            float* acc = grad_rows + (int64_t)s * dim;
            if (mode == MODE_CONCAT_F32) {
                const float* src = (const float*)grad + i * dim;
                for (int c = 0; c < dim; c++) acc[c] = acc[c] + src[c];
            } else {
                int64_t t = i / n_heads;
                int h = (int)(i % n_heads);
                const uint16_t* src = (const uint16_t*)grad + t * (int64_t)hpn * dim + (int64_t)(h % hpn) * dim;
                for (int c = 0; c < dim; c++) acc[c] = acc[c] + bf16_to_float(src[c]);
            }
        }
    }
}

/*
 * One optimizer step over the overlay, engraft/descend_corpus.py:921-947:
 *   g   = g_kd + reg_scale * (2*(p - p0))     reg = mu*sum((p-p0)^2)/max(sum(p0^2),1e-12),
 *                                              reg_scale = float(mu)/max(S,1e-12) (autograd of :936)
 *   torch.optim.Adam (betas, eps, no weight decay, single-tensor rule):
 *   m   = lerp(m, g, 1-beta1)                 = fma(1-beta1, g-m, m)
 *   v   = v*beta2 + ((1-beta2)*g)*g
 *   den = sqrt(v)/sqrt(1-beta2^step) + eps
 *   p   = p + (-(lr/(1-beta1^step))*m)/den
 * p0 == NULL: no regulariser.
 */
void orc_adam(float* p, const float* g, float* m, float* v, const float* p0, int64_t numel,
              int64_t step, double lr, double beta1, double beta2, double eps, float reg_scale) {
    double bc1 = 1.0 - pow(beta1, (double)step);
    double bc2 = 1.0 - pow(beta2, (double)step);
    float step_size = (float)(lr / bc1);
    float bc2_sqrt = (float)sqrt(bc2);
    float w1 = (float)(1.0 - beta1);
    float b2 = (float)beta2;
    float w2 = (float)(1.0 - beta2);
    float epsf = (float)eps;
    float neg_ss = -step_size;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < numel; i++) {
        float gi = g[i];
        if (p0) {
            float d = p[i] - p0[i];
            float r = reg_scale * (2.0f * d);
            gi = gi + r;
        }
        float mi = fmaf(w1, gi - m[i], m[i]);
        float vi = v[i] * b2;
        vi = vi + (w2 * gi) * gi;
        float den = sqrtf(vi) / bc2_sqrt + epsf;
        p[i] = p[i] + (neg_ss * mi) / den;
        m[i] = mi;
        v[i] = vi;
    }
}

/* Repack the reference's raw rows into the device-resident layout used by the
 * CUDA path (the layout is documented with engram_table_pack in the C ABI
 * header).  Used by tests to check the device pack kernel byte for byte. */
void orc_pack(int32_t fmt, int32_t dim, const uint8_t* raw, int64_t n, uint8_t* dst, int64_t stride) {
    int64_t rb = orc_raw_row_bytes(fmt, dim);
    for (int64_t i = 0; i < n; i++) {
        const uint8_t* s = raw + i * rb;
        uint8_t* d = dst + i * stride;
        memset(d, 0, (size_t)stride);
        if (fmt == FMT_F32) {
            memcpy(d, s, (size_t)rb);
        } else if (fmt == FMT_IQ4_NL) {
            int nb = dim / 32;
            for (int b = 0; b < nb; b++) {
                memcpy(d + 16 * b, s + 18 * b + 2, 16);
                memcpy(d + 16 * nb + 2 * b, s + 18 * b, 2);
            }
        } else {
            for (int sb = 0; sb < dim / 256; sb++) {
                memcpy(d + 144 * sb, s + 136 * sb + 8, 128);
                memcpy(d + 144 * sb + 128, s + 136 * sb, 8);
            }
        }
    }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* numpy's float32 pairwise sum of a short row (the reduction of
 * `matched_dnorm.sum(axis=1)`): fewer than 8 terms are added in order from 0;
 * otherwise 8 running partial sums over strides of 8, combined as
 * ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the remaining terms in order. */
static float np_pairwise_sum_f32(const float* a, int n) {
    if (n < 8) {
        float res = 0.0f;
        for (int i = 0; i < n; i++) res = res + a[i];
        return res;
    }
    float r[8];
    for (int k = 0; k < 8; k++) r[k] = a[k];
    int i = 8;
    for (; i + 8 <= n; i += 8)
        for (int k = 0; k < 8; k++) r[k] = r[k] + a[i + k];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) res = res + a[i];
    return res;
}

/*
 * Bulk hash + overlay hit scan, engraft/damage.py:168-224 (with ngram_rows
 * :68-104 over the whole token array: the reference's 8M-token blocks carry 2
 * tokens of overlap, iter_blocks :107-121, so the ids are those of one pass).
 * For every position: its n_heads global rows; matched = row in the sorted
 * overlay; read_count[overlay index] += 1 for every match (all positions);
 * positions with >= 1 match, except the last one (t = n-1), are listed with
 * n_hit_rows, dnorm_max = max over heads of (matched ? dnorm : 0) and
 * dnorm_sum = numpy's pairwise float32 sum of the same row.  Returns the number
 * of listed positions.
 */
int64_t orc_scan_hits(const int32_t* tokens, int64_t n, int32_t ngram_size, int32_t hpn, const uint64_t* mult,
                      const int64_t* head_sizes, const int64_t* head_offsets, int64_t eos,
                      const int32_t* ov_sorted, const float* dnorm_sorted, int64_t R, int64_t* pos_out,
                      int32_t* nhit_out, float* dmax_out, float* dsum_out, int64_t* read_count) {
    const int n_heads = (ngram_size - 1) * hpn;
    int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1) * n_heads);
    orc_hash(tokens, NULL, 0, n, ngram_size, hpn, mult, head_sizes, head_offsets, eos, ids);
    memset(read_count, 0, sizeof(int64_t) * (size_t)R);
    int64_t m = 0;
    float v[32];
    for (int64_t t = 0; t < n; t++) {
        int nh = 0;
        float dmax = 0.0f;
        for (int h = 0; h < n_heads; h++) {
            const int32_t g = ids[t * n_heads + h];
            int64_t lo = 0, hi = R;
            while (lo < hi) {
                int64_t mid = (lo + hi) / 2;
                if (ov_sorted[mid] < g) lo = mid + 1; else hi = mid;
            }
            const int match = lo < R && ov_sorted[lo] == g;
            v[h] = match ? dnorm_sorted[lo] : 0.0f;
            if (match) {
                read_count[lo] += 1;
                nh++;
            }
            if (v[h] > dmax || h == 0) dmax = (h == 0) ? v[h] : (v[h] > dmax ? v[h] : dmax);
        }
        if (nh > 0 && t < n - 1) {
            pos_out[m] = t;
            nhit_out[m] = nh;
            dmax_out[m] = dmax;
            dsum_out[m] = np_pairwise_sum_f32(v, n_heads);
            m++;
        }
    }
    free(ids);
    return m;
}
