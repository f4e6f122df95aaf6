/*
 * fr_oracle.h -- CPU restatement of FlashRT-llama.cpp's NVFP4-weight x
 * q8_1-activation matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and the cpu_baseline / --impl reference
 * legs of bench.py may load it.  Nothing in the product links or calls it.
 *
 * Parity pins (see oracle/README.md for the full list):
 *   - NVFP4 block decode and the UE4M3 scale decode are pinned against
 *     gguf-py 0.19.0 (`gguf.quants.NVFP4`), the Python restatement of ggml's
 *     reference CPU code, through tests/golden/nvfp4_decode.npz.
 *   - The e4m3 RNE encoder is pinned against torch.float8_e4m3fn
 *     (tests/golden/e4m3_encode.npz).
 *   - q8_1 is pinned against gguf-py's Q8_0 quantizer for the int8 values
 *     (ggml CPU form x * (1/d)); every flip between that and the
 *     reference's x / d form must be a proven one-LSB tie.
 *   The remaining arithmetic (dot, routing, combine, W4A4) follows the
 *   reference's own restatements cited per function in fr_oracle.c; the
 *   reference ships no stored vectors for them.
 */
#ifndef FR_ORACLE_H
#define FR_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* number formats */
uint16_t or_f32_to_f16(float f);
float    or_f16_to_f32(uint16_t h);
float    or_ue4m3_half(uint8_t x);          /* ggml UE4M3 decode, halved   */
float    or_e4m3_to_f32(uint8_t x);         /* OCP e4m3 (fn) decode        */
uint8_t  or_f32_to_e4m3_satfinite(float f); /* RNE, saturate to +-448      */
uint8_t  or_f32_to_e2m1_act(float x);       /* activation rule, <= bounds  */
float    or_e2m1_to_f32(uint8_t code);

/* block_nvfp4 decode: nb blocks of 36 B -> nb*64 floats */
void or_nvfp4_dequant(const uint8_t *blocks, int64_t nb, float *out);

/* quantize_q8_1: x [T, ldx] f32 -> T * (K/32) blocks of 36 B (half d, half s, int8[32]) */
void or_quantize_q8_1(const float *x, int64_t ldx, int T, int K, uint8_t *q8);
/* the ggml CPU form (q = roundf(x * (1/d))) for the flip analysis */
void or_quantize_q8_ggml_cpu(const float *x, int64_t n, int8_t *q, uint16_t *d16);

/* NVFP4 x q8_1 dot of one row in fp64 (reference frt_h_dot) */
double or_dot_nvfp4_q8_1(const uint8_t *row, const uint8_t *q8, int K);

/* y[t, n] = s * dot(W[n], q8[t]) in fp64, rows strided by w_ld bytes */
void or_gemv_q8_1(const uint8_t *w, int64_t w_ld, const uint8_t *q8, int64_t q8_ld_blocks,
                  float scale, int N, int K, int T, double *y, int64_t ldy, int nthreads);
/* same, fp32 accumulation per sub-block order (CPU baseline arm) */
void or_gemv_q8_1_f32(const uint8_t *w, int64_t w_ld, const uint8_t *q8, int64_t q8_ld_blocks,
                      float scale, int N, int K, int T, float *y, int64_t ldy, int nthreads);

float or_silu(float x);

/* MoE routing (softmax, top-k with lower-index ties, clamp-normalise) on given logits */
void or_topk_softmax(const float *logits, int T, int E, int n_used, float clamp_val,
                     int32_t *ids, float *wts);
/* router logits in fp64: x [T, K] . W_r [E, K]^T */
void or_router_logits(const float *x, const float *wr, int T, int K, int E, double *logits);
/* stable expert grouping: eoff[E+1], slots[T*n_used] (= t*n_used + k), act[E+1] (count at act[E]) */
void or_group_by_expert(const int32_t *ids, int T, int n_used, int E,
                        int32_t *eoff, int32_t *slots, int32_t *act);

/* W4A4 (Thor path) */
int64_t or_sf_offset(int64_t row, int64_t k, int64_t K);
int64_t or_sf_bytes(int64_t rows, int64_t K);
void or_quantize_act_f32(const float *x, int M, int K, uint8_t *packed, uint8_t *sf);
void or_repack_weight(const uint8_t *blocks, int N, int K, uint8_t *packed, uint8_t *sf);
void or_gemm_f32out(const uint8_t *A, const uint8_t *SFA, const uint8_t *B, const uint8_t *SFB,
                    double *D, int M, int N, int K, float alpha, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
