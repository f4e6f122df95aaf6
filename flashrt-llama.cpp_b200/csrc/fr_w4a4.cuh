// fr_w4a4.cuh -- the W4A4 (Thor) half of the path on sm_100a:
//   k_quantize_act : f32 [M, K] -> packed E2M1 [M, K/2] + UE4M3 scales in the
//                    block-scaled atom layout (src/fr_quant_act.cu:23-84)
//   k_repack       : ggml block_nvfp4 -> packed adjacent-pair nibbles + scales
//                    in the atom layout (src/fr_repack.cu:33-59)
//   k_gemm_nvf4    : D = alpha * A . B^T on tcgen05 kind::mxf4nvf4 with the
//                    accumulator in TMEM (replaces the CUTLASS Sm100 GEMM of
//                    src/fr_gemm_f32out.cu:122-205)
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

// one thread per 16-value sub-block; grid (ceil(K/16/128), N)
__global__ void __launch_bounds__(128) k_repack(const uint8_t *__restrict__ src, uint2 *__restrict__ dst,
                                                uint8_t *__restrict__ sf, int N, int K) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = blockIdx.y;
    const int K16 = K / 16;
    if (row >= N || t >= K16) return;
    const uint8_t *b = src + (static_cast<int64_t>(row) * (K16 >> 2) + (t >> 2)) * NV_BYTES;
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

// ------------------------------------------------------------ tcgen05 GEMM
constexpr int G_BM = 128, G_BN = 128, G_BK = 256;      // K tile = 128 bytes per row
constexpr int G_STAGES = 4;
constexpr int G_A_BYTES = G_BM * G_BK / 2;             // 16 KB
constexpr int G_B_BYTES = G_BN * G_BK / 2;             // 16 KB
constexpr int G_SF_BYTES = 4 * 512;                    // 4 atoms (K blocks of 64) per operand
constexpr int G_STAGE_BYTES = G_A_BYTES + G_B_BYTES + 2 * G_SF_BYTES;
constexpr int G_THREADS = 192;                         // producer, MMA, 4 epilogue warps
constexpr int G_TMEM_COLS = 256;                       // 128 accumulator + 4 stages x 32 scale columns
constexpr size_t G_SMEM = 1024 + static_cast<size_t>(G_STAGES) * G_STAGE_BYTES + 256;

struct GemmArgs {
    const uint8_t *sfa, *sfb;
    float *D;
    int M, N, K;
    float alpha;
};

__global__ void __launch_bounds__(G_THREADS, 1) k_gemm_nvf4(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           const GemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned stage area (128-byte swizzle atoms)
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stage0 = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + G_STAGES * G_STAGE_BYTES);
    uint64_t *empty = full + G_STAGES;
    uint64_t *acc_full = empty + G_STAGES;
    uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * G_BN, m0 = blockIdx.y * G_BM;
    const int nkb = (g.K + 63) / 64;                   // K blocks of 64
    const int nkt = (nkb + 3) / 4;                     // K tiles of 256
    const int kb_total = (g.K + 63) >> 6;              // atoms per row block in the SF buffers

    if (threadIdx.x == 0) {
        for (int s = 0; s < G_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_base_s, G_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_base_s;
    const uint32_t t_acc = tbase;                      // columns [0, 128)

    fr_pdl_wait();
    if (warp == 0 && lane == 0) {
        // ---------------- producer
        const uint8_t *sfa_blk = g.sfa + static_cast<int64_t>(m0 / 128) * kb_total * 512;
        const uint8_t *sfb_blk = g.sfb + static_cast<int64_t>(n0 / 128) * kb_total * 512;
        for (int kt = 0; kt < nkt; ++kt) {
            const int s = kt % G_STAGES;
            if (kt >= G_STAGES && !mbar_wait(&empty[s], ((kt / G_STAGES) - 1) & 1, 10)) break;
            const int kbs = min(4, nkb - 4 * kt);
            uint8_t *st = stage0 + s * G_STAGE_BYTES;
            mbar_expect_tx(&full[s], G_A_BYTES + G_B_BYTES + 2 * kbs * 512);
            tma_load_2d(st, &tmA, kt * (G_BK / 2), m0, &full[s]);
            tma_load_2d(st + G_A_BYTES, &tmB, kt * (G_BK / 2), n0, &full[s]);
            bulk_g2s(st + G_A_BYTES + G_B_BYTES, sfa_blk + static_cast<int64_t>(4 * kt) * 512, kbs * 512, &full[s]);
            bulk_g2s(st + G_A_BYTES + G_B_BYTES + G_SF_BYTES, sfb_blk + static_cast<int64_t>(4 * kt) * 512, kbs * 512,
                     &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer
        const uint32_t idesc = idesc_nvf4(G_BM, G_BN);
        for (int kt = 0; kt < nkt; ++kt) {
            const int s = kt % G_STAGES;
            if (!mbar_wait(&full[s], (kt / G_STAGES) & 1, 11)) break;
            tc_fence_after();
            const int kbs = min(4, nkb - 4 * kt);
            uint8_t *st = stage0 + s * G_STAGE_BYTES;
            const uint32_t a_addr = smem_u32(st), b_addr = smem_u32(st + G_A_BYTES);
            const uint32_t sfa_addr = smem_u32(st + G_A_BYTES + G_B_BYTES);
            const uint32_t sfb_addr = sfa_addr + G_SF_BYTES;
            const uint32_t t_sfa = tbase + 128 + s * 32, t_sfb = t_sfa + 16;
            for (int j = 0; j < kbs; ++j) {
                tc_cp_sf(t_sfa + 4 * j, sdesc_plain(sfa_addr + 512 * j, 128));
                tc_cp_sf(t_sfb + 4 * j, sdesc_plain(sfb_addr + 512 * j, 128));
            }
            for (int j = 0; j < kbs; ++j) {
                tc_mma_nvf4(t_acc, sdesc_sw128(a_addr + 32 * j), sdesc_sw128(b_addr + 32 * j), idesc, t_sfa + 4 * j,
                            t_sfb + 4 * j, (kt > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(acc_full);
    } else if (warp >= 2) {
        // ---------------- epilogue: TMEM -> registers -> D
        const int q = warp & 3;                        // lane quadrant this warp may access
        const bool ok = mbar_wait(acc_full, 0, 12);
        tc_fence_after();
        if (ok) {
            const int row = m0 + 32 * q + lane;
#pragma unroll 1
            for (int c = 0; c < G_BN; c += 32) {
                uint32_t r[32];
                tmem_ld32(t_acc + (static_cast<uint32_t>(32 * q) << 16) + c, r);
                if (row < g.M) {
                    float *dst = g.D + static_cast<int64_t>(row) * g.N + n0 + c;
                    if (n0 + c + 32 <= g.N && (g.N & 3) == 0) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(dst + i) =
                                make_float4(__uint_as_float(r[i]) * g.alpha, __uint_as_float(r[i + 1]) * g.alpha,
                                            __uint_as_float(r[i + 2]) * g.alpha, __uint_as_float(r[i + 3]) * g.alpha);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (n0 + c + i < g.N) dst[i] = __uint_as_float(r[i]) * g.alpha;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    fr_pdl_trigger();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, G_TMEM_COLS);
    }
}

} // namespace frb
