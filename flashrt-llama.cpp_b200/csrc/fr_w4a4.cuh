// fr_w4a4.cuh -- the W4A4 (Thor) half of the path on sm_100a:
//   k_quantize_act : f32 [M, K] -> packed E2M1 [M, K/2] + UE4M3 scales in the
//                    block-scaled atom layout (src/fr_quant_act.cu:23-84)
//   k_repack       : ggml block_nvfp4 -> packed adjacent-pair nibbles + scales
//                    in the atom layout (src/fr_repack.cu:33-59)
//   (the GEMM itself, D = alpha * A . B^T on tcgen05 kind::mxf4nvf4, is the
//    persistent stream-K kernel of fr_gemm.cuh)
//
// Scale atom layout: rows in blocks of 128, K in blocks of 64; one 512-byte
// atom per (row block, K block), the K atoms of a row block contiguous; inside
// an atom, row r and scale column k (of 4) at (r % 32) * 16 + (r / 32) * 4 + k
// (vendor/csrc/quantize/f32_act_to_nvfp4_swizzled_mrows_sm120.cuh:19-28).
#pragma once

#include <cuda_fp8.h>

#include "fr_tc.cuh"

namespace frb {

__host__ __device__ __forceinline__ int64_t sf_offset(int64_t row, int64_t k, int64_t K) {
    const int64_t kb = (K + 63) >> 6;
    const int64_t r = row & 127;
    return (row >> 7) * kb * 512 + (k >> 6) * 512 + (r & 31) * 16 + (r >> 5) * 4 + ((k & 63) >> 4);
}

// activation rule with `<=` boundaries (src/fr_quant_act.cu:23-36)
__device__ __forceinline__ uint32_t e2m1_act(float x) {
    const uint32_t sign = (x < 0.f) ? 0x8u : 0x0u;
    const float ax = fabsf(x);
    uint32_t m;
    if (ax <= 0.25f) m = 0u;
    else if (ax <= 0.75f) m = 1u;
    else if (ax <= 1.25f) m = 2u;
    else if (ax <= 1.75f) m = 3u;
    else if (ax <= 2.5f) m = 4u;
    else if (ax <= 3.5f) m = 5u;
    else if (ax <= 5.0f) m = 6u;
    else m = 7u;
    return sign | m;
}

// one thread per 16-value block; grid (ceil(K/16/128), M)
__global__ void __launch_bounds__(128) k_quantize_act(const float4 *__restrict__ src, uint2 *__restrict__ dst,
                                                      uint8_t *__restrict__ sf, int M, int K) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = blockIdx.y;
    const int nb = K / 16;
    if (row >= M || b >= nb) return;
    float v[16];
    const float4 *s = src + static_cast<int64_t>(row) * (K / 4) + 4 * b;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 f = s[c];
        v[4 * c] = f.x; v[4 * c + 1] = f.y; v[4 * c + 2] = f.z; v[4 * c + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    float desired = __fdiv_rn(amax, 6.f);
    if (desired < 1e-12f) desired = 1e-12f;
    const __nv_fp8_storage_t code = __nv_cvt_float_to_fp8(desired, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
    const float dq = __half2float(__half(hr));
    sf[sf_offset(row, static_cast<int64_t>(b) * 16, K)] = static_cast<uint8_t>(code);
    const float inv = __fdiv_rn(1.f, dq);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) lo |= (e2m1_act(v[2 * p] * inv) | (e2m1_act(v[2 * p + 1] * inv) << 4)) << (8 * p);
#pragma unroll
    for (int p = 0; p < 4; ++p)
        hi |= (e2m1_act(v[8 + 2 * p] * inv) | (e2m1_act(v[8 + 2 * p + 1] * inv) << 4)) << (8 * p);
    dst[static_cast<int64_t>(row) * nb + b] = make_uint2(lo, hi);
}

// one thread per 16-value sub-block; grid (ceil(K/16/128), N).  Source row
// `row` lands in destination row row * dst_step + dst_row0 (1, 0 for a plain
// repack; 2, 0 and 2, 1 interleave a gate and an up matrix row by row, the
// reference's repack_weight_pair_interleaved, src/fr_repack.cu:66-136)
__global__ void __launch_bounds__(128) k_repack(const uint8_t *__restrict__ src, uint2 *__restrict__ dst,
                                                uint8_t *__restrict__ sf, int N, int K, int dst_step,
                                                int dst_row0) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int src_row = blockIdx.y;
    const int K16 = K / 16;
    if (src_row >= N || t >= K16) return;
    const int row = src_row * dst_step + dst_row0;
    const uint8_t *b = src + (static_cast<int64_t>(src_row) * (K16 >> 2) + (t >> 2)) * NV_BYTES;
    const int sub = t & 3;
    const uint8_t *qs = b + 4 + sub * 8;
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t c0 = qs[2 * p], c1 = qs[2 * p + 1];
        w0 |= ((c0 & 0x0Fu) | ((c1 & 0x0Fu) << 4)) << (8 * p);   // elements 2p, 2p+1
        w1 |= ((c0 >> 4) | (c1 & 0xF0u)) << (8 * p);            // elements 8+2p, 8+2p+1
    }
    dst[static_cast<int64_t>(row) * K16 + t] = make_uint2(w0, w1);
    sf[sf_offset(row, static_cast<int64_t>(t) * 16, K)] = b[sub];
}

} // namespace frb
