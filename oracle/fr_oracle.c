/*
 * fr_oracle.c -- CPU restatement of the NVFP4 x q8_1 matmul hot path of
 * FlashRT-llama.cpp (reference paths are relative to that project).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels and the CPU
 * baseline that bench.py reports beside them.  The product never links it.
 *
 * Compile with -ffp-contract=off: the q8_1 quantizer must reproduce the
 * reference's float arithmetic bit for bit.
 */
#include "fr_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* number formats                                                      */
/* ------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even (what __float2half_rn and
 * the GGML_FP32_TO_FP16 of a q8_1 scale do). */
uint16_t or_f32_to_f16(float f) {
    const uint32_t x = f2u(f);
    const uint16_t sign = (uint16_t) ((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u);
    if (a >= 0x477ff000u) return sign | 0x7c00u;              /* >= 65520 -> inf */
    const uint32_t e = a >> 23;
    if (e < 113) {                                            /* f16 subnormal range */
        if (e < 102) return sign;
        const uint32_t m = (a & 0x7fffffu) | 0x800000u;
        const uint32_t sh = 126 - e;                          /* 14..24 */
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return sign | (uint16_t) q;
    }
    const uint32_t m = a & 0x7fffffu;
    uint32_t q = ((e - 112) << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return sign | (uint16_t) q;
}

float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    if (e == 0) {
        const float v = (float) m * 0x1p-24f;
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112) << 23) | (m << 13));
}

/* ggml's UE4M3 decode with the 1/2 that pairs with the doubled E2M1 table:
 * codes 0, 0x7F and 0xFF are zero and the sign bit is ignored.
 * Follows src/fr_win_flint_batched.cuh:442-447 (frt_h_ue4m3). */
float or_ue4m3_half(uint8_t x) {
    if (x == 0 || x == 0x7F || x == 0xFF) return 0.0f;
    const int e = (x >> 3) & 0xF, m = x & 7;
    const float raw = e == 0 ? ldexpf((float) m, -9) : ldexpf(1.0f + (float) m / 8.0f, e - 7);
    return raw / 2;
}

/* OCP e4m3 ("fn": no infinities, S.1111.111 is NaN) */
float or_e4m3_to_f32(uint8_t x) {
    const int s = x >> 7, e = (x >> 3) & 0xF, m = x & 7;
    float v;
    if (e == 15 && m == 7) v = NAN;
    else if (e == 0) v = ldexpf((float) m, -9);
    else v = ldexpf(1.0f + (float) m / 8.0f, e - 7);
    return s ? -v : v;
}

/* float -> e4m3, round to nearest even, saturating to +-448, NaN -> 0x7F:
 * the conversion __nv_fp8_e4m3(float) performs in src/fr_quant_act.cu:64. */
uint8_t or_f32_to_e4m3_satfinite(float f) {
    if (f != f) return 0x7F;
    const uint32_t x = f2u(f);
    const uint8_t sign = (uint8_t) ((x >> 24) & 0x80u);
    const uint32_t a = x & 0x7fffffffu;
    if (u2f(a) > 448.0f) return sign | 0x7E;
    const uint32_t e = a >> 23;
    if (e < 121) {                                 /* below 2^-6: subnormal grid 2^-9 */
        if (e < 117) return sign;                  /* < 2^-10 rounds to 0 (2^-10 ties to 0) */
        const uint32_t m = (a & 0x7fffffu) | 0x800000u;
        const uint32_t sh = 141 - e;               /* 21..24 */
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return sign | (uint8_t) q;
    }
    const uint32_t m = a & 0x7fffffu;
    uint32_t q = ((e - 120) << 3) | (m >> 20);
    const uint32_t rem = m & 0xfffffu;
    if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) q++;
    if (q > 0x7E) q = 0x7E;
    return sign | (uint8_t) q;
}

/* activation E2M1 rounding with `<=` boundaries (src/fr_quant_act.cu:23-36) */
uint8_t or_f32_to_e2m1_act(float x) {
    const uint8_t sign = (x < 0.f) ? 0x8u : 0x0u;
    const float ax = fabsf(x);
    uint8_t m;
    if      (ax <= 0.25f) m = 0u;
    else if (ax <= 0.75f) m = 1u;
    else if (ax <= 1.25f) m = 2u;
    else if (ax <= 1.75f) m = 3u;
    else if (ax <= 2.5f)  m = 4u;
    else if (ax <= 3.5f)  m = 5u;
    else if (ax <= 5.0f)  m = 6u;
    else                  m = 7u;
    return sign | m;
}

float or_e2m1_to_f32(uint8_t code) {
    static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float v = mag[code & 7];
    return (code & 8) ? -v : v;
}

/* doubled E2M1 values, ggml's kvalues_mxfp4 (include/fr_kernels.h:13-15) */
static const int kv16[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* block_nvfp4: d[4] (one UE4M3 per 16), qs[32]; sub-block s in qs[8s..8s+7],
 * byte j = elem j (low nibble) and elem j+8 (high nibble)
 * (src/fr_repack.cu:4-10, src/fr_win_flint_batched.cuh:449-466). */
void or_nvfp4_dequant(const uint8_t *blocks, int64_t nb, float *out) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *blk = blocks + b * 36;
        for (int s = 0; s < 4; ++s) {
            const float d = or_ue4m3_half(blk[s]);
            for (int e = 0; e < 16; ++e) {
                const uint8_t q = blk[4 + 8 * s + (e & 7)];
                const int nib = e < 8 ? (q & 0xF) : (q >> 4);
                out[b * 64 + s * 16 + e] = d * (float) kv16[nib];
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* quantize_q8_1                                                       */
/* ------------------------------------------------------------------ */

/* One 32-element chunk exactly as frt_q8_1_chunk (src/fr_win_flint_sm120.cu:
 * 289-300) computes it: amax and the xor-butterfly sum (lane i adds lane
 * i^16, then i^8, ...), d = amax/127, q = roundf(x/d) with IEEE division
 * (the host form src/fr_win_flint_batched.cuh:389-398), ds = half2(d, sum). */
static void q8_1_chunk(const float *x, uint8_t *blk) {
    float amax = 0.0f;
    float v[32];
    for (int j = 0; j < 32; ++j) {
        v[j] = x[j];
        const float a = fabsf(x[j]);
        if (a > amax) amax = a;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float nv[32];
        for (int j = 0; j < 32; ++j) nv[j] = v[j] + v[j ^ off];
        memcpy(v, nv, sizeof(v));
    }
    const float sum = v[0];
    const float d = amax / 127.0f;
    const uint16_t dh = or_f32_to_f16(d), sh = or_f32_to_f16(sum);
    memcpy(blk + 0, &dh, 2);
    memcpy(blk + 2, &sh, 2);
    for (int j = 0; j < 32; ++j) {
        const int8_t q = amax == 0.0f ? 0 : (int8_t) roundf(x[j] / d);
        blk[4 + j] = (uint8_t) q;
    }
}

void or_quantize_q8_1(const float *x, int64_t ldx, int T, int K, uint8_t *q8) {
    const int nc = K / 32;
    for (int t = 0; t < T; ++t)
        for (int c = 0; c < nc; ++c)
            q8_1_chunk(x + (int64_t) t * ldx + (int64_t) c * 32, q8 + ((int64_t) t * nc + c) * 36);
}

/* ggml's CPU reference form: id = 1/d, q = roundf(x * id) (the same as
 * gguf-py's Q8_0.quantize_blocks); used only to count and classify flips
 * against the x/d form, as src/fr_win_flint_batched.cuh:410-441 does. */
void or_quantize_q8_ggml_cpu(const float *x, int64_t n, int8_t *q, uint16_t *d16) {
    for (int64_t c = 0; c < n / 32; ++c) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) { const float a = fabsf(x[c * 32 + j]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        d16[c] = or_f32_to_f16(d);
        for (int j = 0; j < 32; ++j) q[c * 32 + j] = (int8_t) roundf(x[c * 32 + j] * id);
    }
}

/* ------------------------------------------------------------------ */
/* NVFP4 x q8_1 dot (reference: src/fr_win_flint_batched.cuh:449-466)  */
/* ------------------------------------------------------------------ */

static inline float q8_d(const uint8_t *blk) { uint16_t h; memcpy(&h, blk, 2); return or_f16_to_f32(h); }

double or_dot_nvfp4_q8_1(const uint8_t *row, const uint8_t *q8, int K) {
    double acc = 0.0;
    for (int b = 0; b < K / 64; ++b) {
        const uint8_t *blk = row + (int64_t) b * 36;
        for (int sb = 0; sb < 4; ++sb) {
            const uint8_t *qs = blk + 4 + 8 * sb;
            const int elem0 = b * 64 + sb * 16;
            const uint8_t *yb = q8 + (int64_t) (elem0 / 32) * 36;
            const int8_t *yq = (const int8_t *) (yb + 4) + (elem0 % 32);
            int sumi = 0;
            for (int e = 0; e < 16; ++e) {
                const int nib = e < 8 ? (qs[e] & 0xF) : (qs[e - 8] >> 4);
                sumi += kv16[nib] * (int) yq[e];
            }
            acc += (double) or_ue4m3_half(blk[sb]) * (double) q8_d(yb) * (double) sumi;
        }
    }
    return acc;
}

void or_gemv_q8_1(const uint8_t *w, int64_t w_ld, const uint8_t *q8, int64_t q8_ld_blocks,
                  float scale, int N, int K, int T, double *y, int64_t ldy, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int n = 0; n < N; ++n)
        for (int t = 0; t < T; ++t)
            y[(int64_t) t * ldy + n] = (double) scale *
                or_dot_nvfp4_q8_1(w + (int64_t) n * w_ld, q8 + (int64_t) t * q8_ld_blocks * 36, K);
    (void) nthreads;
}

/* fp32 form of the same op (exact int32 sub-block sums, fp32 scaling and
 * accumulation, the order ggml's vec_dot uses per block): the CPU baseline. */
void or_gemv_q8_1_f32(const uint8_t *w, int64_t w_ld, const uint8_t *q8, int64_t q8_ld_blocks,
                      float scale, int N, int K, int T, float *y, int64_t ldy, int nthreads) {
    const int nb = K / 64;
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = or_ue4m3_half((uint8_t) i);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int n = 0; n < N; ++n) {
        const uint8_t *row = w + (int64_t) n * w_ld;
        for (int t = 0; t < T; ++t) {
            const uint8_t *yt = q8 + (int64_t) t * q8_ld_blocks * 36;
            float acc = 0.0f;
            for (int b = 0; b < nb; ++b) {
                const uint8_t *blk = row + (int64_t) b * 36;
                for (int sb = 0; sb < 4; ++sb) {
                    const uint8_t *qs = blk + 4 + 8 * sb;
                    const uint8_t *yb = yt + (int64_t) ((b * 64 + sb * 16) / 32) * 36;
                    const int8_t *yq = (const int8_t *) (yb + 4) + ((sb & 1) * 16);
                    int sumi = 0;
                    for (int e = 0; e < 8; ++e) {
                        sumi += kv16[qs[e] & 0xF] * (int) yq[e];
                        sumi += kv16[qs[e] >> 4] * (int) yq[e + 8];
                    }
                    acc += (lut[blk[sb]] * q8_d(yb)) * (float) sumi;
                }
            }
            y[(int64_t) t * ldy + n] = acc * scale;
        }
    }
    (void) nthreads;
}

/* ggml_cuda_op_silu_single: x / (1 + exp(-x)) */
float or_silu(float x) { return x / (1.0f + expf(-x)); }

/* ------------------------------------------------------------------ */
/* MoE routing                                                         */
/* ------------------------------------------------------------------ */

void or_router_logits(const float *x, const float *wr, int T, int K, int E, double *logits) {
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += (double) wr[(int64_t) e * K + k] * (double) x[(int64_t) t * K + k];
            logits[(int64_t) t * E + e] = s;
        }
}

/* Softmax over E experts, n_used rounds of arg-max with the lower expert id
 * winning ties, then w_k = p_k / max(sum of the selected p, clamp)
 * (frt_router_fused phase 2, src/fr_win_qwen36_sm120.cu:1826-1870). */
/* fp32 sum over 32 lanes with the xor butterfly (lane 0's result) */
static float butterfly_sum(const float *lanes) {
    float v[32];
    memcpy(v, lanes, sizeof(v));
    for (int off = 16; off > 0; off >>= 1) {
        float nv[32];
        for (int j = 0; j < 32; ++j) nv[j] = v[j] + v[j ^ off];
        memcpy(v, nv, sizeof(v));
    }
    return v[0];
}

/* E must be a multiple of 32 (one warp; expert e lives in lane e % 32).
 * Every float operation is in the order the warp performs it. */
void or_topk_softmax(const float *logits, int T, int E, int n_used, float clamp_val,
                     int32_t *ids, float *wts) {
    float *p = (float *) malloc(sizeof(float) * (size_t) E);
    const int per = E / 32;
    for (int t = 0; t < T; ++t) {
        const float *l = logits + (int64_t) t * E;
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) mx = fmaxf(mx, l[e]);
        float part[32];
        for (int lane = 0; lane < 32; ++lane) {
            float s = 0.0f;
            for (int i = 0; i < per; ++i) {
                const int e = lane + 32 * i;
                p[e] = expf(l[e] - mx);
                s += p[e];
            }
            part[lane] = s;
        }
        const float inv = 1.0f / butterfly_sum(part);
        for (int e = 0; e < E; ++e) { p[e] *= inv; if (p[e] != p[e]) p[e] = -3.402823466e+38f; }
        float lane_sum[32] = {0};
        for (int k = 0; k < n_used; ++k) {
            int best = 0;
            for (int e = 1; e < E; ++e) if (p[e] > p[best]) best = e;
            ids[(int64_t) t * n_used + k] = best;
            wts[(int64_t) t * n_used + k] = p[best];
            lane_sum[best & 31] += p[best];
            p[best] = -INFINITY;
        }
        float ws = butterfly_sum(lane_sum);
        if (ws < clamp_val) ws = clamp_val;
        const float invs = 1.0f / ws;
        for (int k = 0; k < n_used; ++k) wts[(int64_t) t * n_used + k] *= invs;
    }
    free(p);
}

/* Expert grouping (the token permute of frt_b_topk_group,
 * src/fr_win_flint_batched_moe.cuh:100-165, and ggml's mm_ids_helper,
 * hosts/llama.cpp-flint/patches/0004-...:27-113): histogram over experts,
 * exclusive scan into eoff, slots grouped by expert.  The order inside an
 * expert is the slot order (a stable counting sort); the reference's atomic
 * placement leaves it unspecified. */
void or_group_by_expert(const int32_t *ids, int T, int n_used, int E,
                        int32_t *eoff, int32_t *slots, int32_t *act) {
    int32_t *cnt = (int32_t *) calloc((size_t) E, sizeof(int32_t));
    const int ns = T * n_used;
    for (int s = 0; s < ns; ++s) cnt[ids[s]]++;
    int run = 0, na = 0;
    for (int e = 0; e < E; ++e) {
        eoff[e] = run;
        run += cnt[e];
        if (cnt[e] > 0) act[na++] = e;
    }
    eoff[E] = run;
    for (int e = na; e < E; ++e) act[e] = -1;
    act[E] = na;
    int32_t *cur = (int32_t *) malloc(sizeof(int32_t) * (size_t) E);
    for (int e = 0; e < E; ++e) cur[e] = eoff[e];
    for (int s = 0; s < ns; ++s) slots[cur[ids[s]]++] = s;
    free(cnt);
    free(cur);
}

/* ------------------------------------------------------------------ */
/* W4A4 (the Thor tcgen05 path)                                        */
/* ------------------------------------------------------------------ */

/* Byte offset of the scale for (row, k) in the block-scaled atom layout:
 * rows in chunks of 128, K/16 scale columns in chunks of 4, one 512 B atom
 * per (128 rows, 64 k) with the K atoms of a row block contiguous
 * (vendor/csrc/quantize/f32_act_to_nvfp4_swizzled_mrows_sm120.cuh:19-28;
 * sizes include/fr_kernels.h:25-33). */
int64_t or_sf_offset(int64_t row, int64_t k, int64_t K) {
    const int64_t kb = (K + 63) >> 6;
    const int64_t r = row & 127;
    return (row >> 7) * kb * 512 + (k >> 6) * 512 + (r & 31) * 16 + (r >> 5) * 4 + ((k & 63) >> 4);
}

int64_t or_sf_bytes(int64_t rows, int64_t K) {
    return ((rows + 127) / 128 * 128) * (((K / 16) + 3) / 4 * 4);
}

/* quantize_act_f32 (src/fr_quant_act.cu:38-84): per 16 elements
 * s = e4m3(max(amax/6, 1e-12)), codes e2m1(x * (1/float(s))), adjacent-pair
 * nibbles (elem 2i low, 2i+1 high). */
void or_quantize_act_f32(const float *x, int M, int K, uint8_t *packed, uint8_t *sf) {
    for (int m = 0; m < M; ++m)
        for (int b = 0; b < K / 16; ++b) {
            const float *v = x + (int64_t) m * K + b * 16;
            float amax = 0.f;
            for (int i = 0; i < 16; ++i) { const float a = fabsf(v[i]); if (a > amax) amax = a; }
            float desired = amax / 6.f;
            if (desired < 1e-12f) desired = 1e-12f;
            const uint8_t sc = or_f32_to_e4m3_satfinite(desired);
            sf[or_sf_offset(m, (int64_t) b * 16, K)] = sc;
            const float inv = 1.f / or_e4m3_to_f32(sc);
            uint8_t *o = packed + (int64_t) m * (K / 2) + b * 8;
            for (int p = 0; p < 8; ++p)
                o[p] = (uint8_t) (or_f32_to_e2m1_act(v[2 * p] * inv) | (or_f32_to_e2m1_act(v[2 * p + 1] * inv) << 4));
        }
}

/* repack_weight (src/fr_repack.cu:33-59): split nibbles -> adjacent pairs,
 * scale bytes passed through to the atom layout. */
void or_repack_weight(const uint8_t *blocks, int N, int K, uint8_t *packed, uint8_t *sf) {
    for (int n = 0; n < N; ++n)
        for (int t = 0; t < K / 16; ++t) {
            const uint8_t *b = blocks + ((int64_t) n * (K / 64) + t / 4) * 36;
            const int sub = t & 3;
            const uint8_t *qs = b + 4 + sub * 8;
            uint8_t *o = packed + (int64_t) n * (K / 2) + t * 8;
            for (int p = 0; p < 4; ++p) {
                o[p]     = (uint8_t) ((qs[2 * p] & 0x0F) | ((qs[2 * p + 1] & 0x0F) << 4));
                o[p + 4] = (uint8_t) ((qs[2 * p] >> 4) | (qs[2 * p + 1] & 0xF0));
            }
            sf[or_sf_offset(n, (int64_t) t * 16, K)] = b[sub];
        }
}

/* D = alpha * A . B^T over e2m1 x e4m3 blocks, fp64 accumulation
 * (the semantics of gemm_f32out, src/fr_gemm_f32out.cu:122-187). */
void or_gemm_f32out(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                    double *D, int M, int N, int K, float alpha, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int m = 0; m < M; ++m) {
        double *arow = (double *) malloc(sizeof(double) * (size_t) K);
        for (int k = 0; k < K; ++k) {
            const uint8_t byte = A[(int64_t) m * (K / 2) + k / 2];
            const uint8_t code = (k & 1) ? (byte >> 4) : (byte & 0xF);
            arow[k] = (double) or_e2m1_to_f32(code) * (double) or_e4m3_to_f32(SFA[or_sf_offset(m, k, K)]);
        }
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; k += 16) {
                const double sb = (double) or_e4m3_to_f32(SFB[or_sf_offset(n, k, K)]);
                double part = 0.0;
                for (int i = 0; i < 16; ++i) {
                    const uint8_t byte = B[(int64_t) n * (K / 2) + (k + i) / 2];
                    const uint8_t code = ((k + i) & 1) ? (byte >> 4) : (byte & 0xF);
                    part += arow[k + i] * (double) or_e2m1_to_f32(code);
                }
                acc += part * sb;
            }
            D[(int64_t) m * N + n] = (double) alpha * acc;
        }
        free(arow);
    }
    (void) nthreads;
}
