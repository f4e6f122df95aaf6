// fr_fp4mv.cuh -- NVFP4 x q8_1 matvec on the tcgen05 block-scaled FP4 tensor
// cores (kind::mxf4nvf4): the weights go to the tensor core as they are stored
// (E2M1 codes with their UE4M3 sub-block scales), with no per-value decode.
//
// Arithmetic.  ggml's nvfp4 . q8_1 dot (src/fr_win_flint_sm120.cu:320-342)
// is  sum_k w_k * x_k  with  w_k = e2m1(code) * e4m3(scale & 0x7F)  (0x7F -> 0)
// and  x_k = q_k * d_b  (q_k int8, d_b the f16-rounded q8_1 block scale).
// Write d_b = m_b * 2^E_b (m_b an integer < 2^11) and take per token
// E0 = E_max - 6 (E_max the largest block exponent): then
//     x_k = r_k * 2^E0,   r_k = q_k * m_b * 2^(E_b - E0)
// is an integer, |r_k| < 2^24, for every block with E_b >= E0 -- exactly; a
// block more than six binades below the token's largest has r_k rounded to
// the nearest integer (an absolute error below 2^(E0-1), under 2^-24 of the
// token's largest activation).  In balanced base 9,
//     r_k = sum_{p<8} c_{p,k} 9^p,   c in {-4..4},
// and c/2 is an E2M1 value.  So the activation becomes eight E2M1 columns
// B_p[k] = c_{p,k}/2, all with the scale 1.0, and the column factor
// 9^p * 2^(E0+1):
//     sum_k w_k x_k = sum_p 9^p 2^(E0+1) * sum_k (e2m1 * sfa) * B_p[k].
// The tensor core forms every product exactly and accumulates in fp32, so the
// result equals ggml's up to fp32 summation order (and the rounding above).
// One constant activation scale means one scale-factor copy per kernel for
// the B operand instead of one per 64-value block.
//
// K order.  ggml packs sub-block byte j as values (j, j+8); the MMA reads a
// byte as K positions (2j, 2j+1).  The activation columns are packed the same
// way, so both operands see the same permutation of K inside each 16-value
// sub-block and the scale groups stay aligned.
//
// Data flow per CTA (rows [r0, r0+R), K stages [kt0, kt1) of 256 values):
//   weight producer : TMA box of the raw block_nvfp4 rows (R x 144 B: four
//                     36-byte blocks per row, rows 144 B apart), ahead of
//                     the previous kernel's end (weights need no PDL wait);
//   column producer : bulk copies of the stage's activation columns and their
//                     scale atoms (prepared by k_act_fp4) into their own ring;
//   4 warps/matrix  : thread = row: nine 128-bit loads of the row's stage
//                     segment (conflict-free: rows are nine 16-byte units
//                     apart), eight 128-bit stores of its codes into a
//                     128-byte-swizzled K-major tile and four stores of its
//                     scale words into the scale-factor atoms;
//   MMA lane        : tcgen05.cp of the scale atoms into TMEM, four
//                     tcgen05.mma (K = 64 each) per matrix per stage;
//   epilogue        : tcgen05.ld of the column sums, y = sum_p 9^p 2^g D_p,
//                     SwiGLU / scale / residual; split-K partials are added
//                     in split order by the last CTA of the row tile.
#pragma once

#include "fr_tc.cuh"

namespace frb {

constexpr int FM_WBOX = 144;                   // bytes per row per stage (4 blocks)
constexpr int FM_KS = 256;                     // K values per stage
constexpr int FM_DIGITS = 8;                   // E2M1 columns per token
constexpr int FM_BIAS = 21523360;              // 4 * (9^8 - 1) / 8: makes r + bias a base-9 number
constexpr int FM_SPAN = 6;                     // binades below the largest block kept exactly
constexpr uint32_t FM_SFB = 0x38u;             // ue4m3 1.0: the activation columns' scale
constexpr int FM_GSTRIDE = 8;                  // floats per token in the column-factor table

// ------------------------------------------------------------ activation
// f16 value h = m * 2^E (m integer); E of a zero is reported as -1000
__device__ __forceinline__ void f16_split(__half h, int &m, int &E) {
    const uint32_t bits = __half_as_ushort(h) & 0x7FFFu;
    const uint32_t ex = bits >> 10, fr = bits & 0x3FFu;
    if (bits == 0) { m = 0; E = -1000; return; }
    if (ex == 0) { m = static_cast<int>(fr); E = -24; return; }
    m = static_cast<int>(1024u + fr);
    E = static_cast<int>(ex) - 25;
}

// Activation columns for T tokens.  bimg: per K stage kq, NCOL rows x 128 B
// in the 128-byte-swizzled K-major layout (row n = 8t + p); sfb: per 64-block
// one 512-byte scale atom, every entry of rows n < 8T set to 1.0 (consumers
// that keep one constant atom ignore it); gtab[t * 8 + p] = 9^p * 2^(E0_t+1).
// Rows n >= 8T are left as they are (their MMA columns are never read).  With
// t_stride > 0 (and NCOL = 8) every token gets its own image instead, at
// bimg + t * t_stride: per K stage one 1024-byte swizzle atom of its eight
// rows, so a consumer can gather any set of tokens atom by atom (the MoE
// expert windows); sfb may then be null.  x_k follows quantize_q8_1 exactly
// (d = f16(amax / 127), q = roundf(x / d)); the input is f32 rows or q8_1
// blocks.  Grid (slices, T), 256 threads; warp per q8_1 block.
// The eight E2M1 digit nibbles of this lane's value of one q8_1 block (q,
// f16 scale hd) against the token's reference exponent e0:
// r = q * m * 2^(E - e0) exact for E >= e0, rounded half away from zero below.
__device__ __forceinline__ void fp4_digits(int q, __half hd, int e0, uint32_t (&nib)[FM_DIGITS]) {
    int m, E;
    f16_split(hd, m, E);
    const int v = q * m;
    int r = 0;
    if (m != 0) {
        const int sh = E - e0;
        if (sh >= 0) {
            r = v * (1 << sh);
        } else if (sh > -31) {
            const int s2 = -sh;
            const int a = (v < 0 ? -v : v);
            const int ra = (a + (1 << (s2 - 1))) >> s2;
            r = v < 0 ? -ra : ra;
        }
    }
    int R = r + FM_BIAS;                             // 0 <= R < 9^8
#pragma unroll
    for (int p = 0; p < FM_DIGITS; ++p) {
        const int dgt = R % 9;
        R /= 9;
        const int c = dgt - 4;
        nib[p] = c < 0 ? (8u | static_cast<uint32_t>(-c)) : static_cast<uint32_t>(c);
    }
}

// Store a warp's digits of q8_1 block `c` (0..7) of a 256-value K stage into
// the stage's column tile (rows n0 .. n0+7, 128-byte-swizzled K-major):
// lanes j and j+8 of a sub-block share a byte, as ggml packs the weights.
__device__ __forceinline__ void fp4_digits_store(const uint32_t (&nib)[FM_DIGITS], uint8_t *tile, int n0, int c) {
    const int lane = threadIdx.x & 31;
    const int kbl = c >> 1;
    const int sbk = (c & 1) * 2 + (lane >> 4);       // sub-block inside the 64-block
    const int j = lane & 15;
#pragma unroll
    for (int p = 0; p < FM_DIGITS; ++p) {
        const uint32_t hi = __shfl_xor_sync(0xffffffffu, nib[p], 8);
        if (j < 8) {
            const int n = n0 + p;
            const int idx = kbl * 32 + sbk * 8 + j;
            const int c16 = idx >> 4;
            tile[n * 128 + ((c16 ^ (n & 7)) << 4) + (idx & 15)] = static_cast<uint8_t>(nib[p] | (hi << 4));
        }
    }
}

// f16 exponent of amax / 127 (the q8_1 scale of the row's largest block),
// -1000 for a zero row
__device__ __forceinline__ int fp4_row_emax(float amax) {
    int m, E;
    f16_split(__float2half_rn(__fdiv_rn(amax, 127.0f)), m, E);
    return E;
}

// One CTA's share (slice `slice` of `nslices`) of token t's columns; every
// thread of the 256-thread CTA calls it.
__device__ __forceinline__ void act_fp4_row(const float *__restrict__ x, int64_t ldx,
                                            const uint8_t *__restrict__ q8, int64_t ldq, int K, int NCOL,
                                            uint8_t *__restrict__ bimg, uint8_t *__restrict__ sfb,
                                            float *__restrict__ gtab, int64_t t_stride, int t, int slice,
                                            int nslices, const float *__restrict__ amax_in = nullptr,
                                            int n_amax = 0) {
    const int nq = K / Q8_ELEMS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ int s_e[8];
    // this CTA's q8_1 blocks, one warp each; the first block's value is
    // loaded before the row scan so both loads are in flight together
    const int per = (nq + nslices - 1) / nslices;
    const int b_lo = slice * per, b_hi = min(nq, b_lo + per);
    const int b_first = b_lo + warp;
    float x_first = 0.0f;
    if (x != nullptr && b_first < b_hi)
        x_first = x[static_cast<int64_t>(t) * ldx + static_cast<int64_t>(b_first) * Q8_ELEMS + lane];

    // 1. the token's largest block-scale exponent (each CTA scans the row, or
    // the producer of x left the maxima of its row groups in amax_in)
    int emax = -1000;
    if (x != nullptr && amax_in != nullptr) {
        float amax = 0.0f;
        for (int i = threadIdx.x; i < n_amax; i += blockDim.x) amax = fmaxf(amax, amax_in[static_cast<int64_t>(t) * n_amax + i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        emax = fp4_row_emax(amax);
    } else if (x != nullptr) {
        // many independent loads in flight per thread, 16-byte loads when the
        // row allows them
        float am[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        const float *row = x + static_cast<int64_t>(t) * ldx;
        if ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && (K & 3) == 0) {
            const float4 *r4 = reinterpret_cast<const float4 *>(row);
            const int K4 = K >> 2;
            int k = threadIdx.x;
            for (; k + 7 * 256 < K4; k += 8 * 256) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = r4[k + u * 256];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    am[u] = fmaxf(fmaxf(am[u], fmaxf(fabsf(v[u].x), fabsf(v[u].y))), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
            }
            for (; k < K4; k += 256) {
                const float4 v = r4[k];
                am[0] = fmaxf(fmaxf(am[0], fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
            }
        } else {
            int k = threadIdx.x;
            for (; k + 7 * 256 < K; k += 8 * 256) {
#pragma unroll
                for (int u = 0; u < 8; ++u) am[u] = fmaxf(am[u], fabsf(row[k + u * 256]));
            }
            for (; k < K; k += 256) am[0] = fmaxf(am[0], fabsf(row[k]));
        }
        float amax = am[0];
#pragma unroll
        for (int u = 1; u < 8; ++u) amax = fmaxf(amax, am[u]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        int m, E;
        f16_split(__float2half_rn(__fdiv_rn(amax, 127.0f)), m, E);
        emax = E;
    } else {
        for (int b = threadIdx.x; b < nq; b += blockDim.x) {
            const uint8_t *blk = q8 + (static_cast<int64_t>(t) * ldq + b) * Q8_BYTES;
            int m, E;
            f16_split(__low2half(*reinterpret_cast<const __half2 *>(blk)), m, E);
            emax = max(emax, E);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, off));
    }
    if (lane == 0) s_e[warp] = emax;
    __syncthreads();
    emax = s_e[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) emax = max(emax, s_e[w]);
    const int e0 = emax > -1000 ? emax - FM_SPAN : 0;
    if (slice == 0 && threadIdx.x < FM_GSTRIDE) {
        float v = 1.0f;
        for (int p = 0; p < static_cast<int>(threadIdx.x); ++p) v *= 9.0f;
        gtab[t * FM_GSTRIDE + threadIdx.x] = ldexpf(v, e0 + 1);
    }

    // 2. this CTA's q8_1 blocks, one warp each
    for (int b = b_first; b < b_hi; b += 8) {
        int q;
        __half hd;
        if (x != nullptr) {
            const q8_lane r = q8_1_chunk(
                b == b_first ? x_first : x[static_cast<int64_t>(t) * ldx + static_cast<int64_t>(b) * Q8_ELEMS + lane]);
            q = r.q;
            hd = __float2half_rn(r.d);
        } else {
            const uint8_t *blk = q8 + (static_cast<int64_t>(t) * ldq + b) * Q8_BYTES;
            q = static_cast<int8_t>(blk[4 + lane]);
            hd = __low2half(*reinterpret_cast<const __half2 *>(blk));
        }
        uint32_t nib[FM_DIGITS];
        fp4_digits(q, hd, e0, nib);
        const int kb = b >> 1, kq = kb >> 2;
        const int sbk = (b & 1) * 2 + (lane >> 4);   // sub-block inside the 64-block
        const int j = lane & 15;
        uint8_t *img = bimg + t * t_stride + static_cast<int64_t>(kq) * NCOL * 128;
        const int n0 = t_stride > 0 ? 0 : FM_DIGITS * t;
        fp4_digits_store(nib, img, n0, b & 7);
        if (j == 0 && sfb != nullptr) {
#pragma unroll
            for (int p = 0; p < FM_DIGITS; ++p) {
                const int n = n0 + p;
                sfb[static_cast<int64_t>(kb) * 512 + (n & 31) * 16 + (n >> 5) * 4 + sbk] = static_cast<uint8_t>(FM_SFB);
            }
        }
    }
}

__global__ void __launch_bounds__(256) k_act_fp4(const float *__restrict__ x, int64_t ldx,
                                                 const uint8_t *__restrict__ q8, int64_t ldq, int K, int NCOL,
                                                 uint8_t *__restrict__ bimg, uint8_t *__restrict__ sfb,
                                                 float *__restrict__ gtab, int64_t t_stride,
                                                 const float *__restrict__ amax_in, int n_amax) {
    // Dependents may launch at once: the matvec that follows streams its
    // weights (which need nothing from here) as soon as SMs free up, and
    // waits for this grid's completion before it reads the columns.
    fr_pdl_trigger();
    fr_pdl_wait();
    act_fp4_row(x, ldx, q8, ldq, K, NCOL, bimg, sfb, gtab, t_stride, blockIdx.y, blockIdx.x, gridDim.x, amax_in,
                n_amax);
}

// ------------------------------------------------------------ matvec
enum FmEpi : int { FM_PLAIN = 0, FM_SWIGLU = 1 };

struct FmArgs {
    int N, K, T;                 // rows, row length, tokens in this launch (6T <= NCOL)
    int t0;                      // first output token index
    int R;                       // rows per tile (<= 128)
    int n_kt;                    // K stages of 256
    int ksplit;                  // K splits per row tile
    int kt_per_split;
    const uint8_t *bimg;         // activation columns [n_kt][NCOL x 128 B]
    const uint8_t *sfb;          // their scale atoms [n_kt * 4][512 B]
    const float *gtab;           // column factors [T][8]
    const float *s0, *s1;        // per-tensor scales (nullable)
    const float *resid;          // [.., ldr] (nullable)
    int64_t ldr;
    float *y;                    // [.., ldy]
    int64_t ldy;
    float *part;                 // split-K partials [n_rt][ksplit][2][TMAX][128]
    unsigned int *counter;       // [n_rt][4 quadrants], zero on entry, reset by the last split
    int n_raw, n_can, n_b;       // ring depths: raw weight, MMA-ready weight, activation stages
};

template <int NCOL, int EPI>
struct FmShape {
    static constexpr int NM = EPI == FM_SWIGLU ? 2 : 1;
    static constexpr int RAW = NM * 128 * FM_WBOX;                 // raw weight stage (R <= 128 rows)
    static constexpr int A_BYTES = 128 * 128;                      // one 128 x 256 FP4 tile
    static constexpr int SF_BYTES = 4 * 512;                       // four scale atoms per operand
    static constexpr int CAN = NM * (A_BYTES + SF_BYTES);          // MMA-ready weight stage
    static constexpr int B_BYTES = NCOL * 128;
    static constexpr int BST = B_BYTES + SF_BYTES;                 // activation stage
    static constexpr int TMAX = NCOL / FM_DIGITS;                  // tokens per launch
    static constexpr int THREADS = (3 + 4 * NM) * 32;
};

template <int NCOL, int EPI>
__global__ void __launch_bounds__(FmShape<NCOL, EPI>::THREADS, 1)
k_fp4mv(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1, const FmArgs g) {
    using S = FmShape<NCOL, EPI>;
    constexpr int NM = S::NM;
    constexpr bool DUAL = NM == 2;
    constexpr int TMAX = S::TMAX;
    constexpr uint32_t TMEM_COLS = 512;
    static_assert(2 * NCOL <= 256, "accumulators live in TMEM columns [0, 256)");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NR = g.n_raw, NC = g.n_can, NB = g.n_b;
    uint8_t *can0 = smem;                                    // NC MMA-ready weight stages (1024-aligned)
    uint8_t *b0 = can0 + static_cast<size_t>(NC) * S::CAN;  // NB activation stages
    uint8_t *raw0 = b0 + static_cast<size_t>(NB) * S::BST;  // NR raw weight stages
    uint64_t *rfull = reinterpret_cast<uint64_t *>(raw0 + static_cast<size_t>(NR) * S::RAW);
    uint64_t *rempty = rfull + NR;
    uint64_t *cfull = rempty + NR;
    uint64_t *cempty = cfull + NC;
    uint64_t *bfull = cempty + NC;
    uint64_t *bempty = bfull + NB;
    uint64_t *accfull = bempty + NB;
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(accfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x / g.ksplit, ks = blockIdx.x % g.ksplit;
    const int r0 = rt * g.R;
    const int kt0 = ks * g.kt_per_split;
    const int kt1 = min(g.n_kt, kt0 + g.kt_per_split);
    const int n_st = kt1 - kt0;
    const int RW = 4 * NM;                                   // row warps

    if (threadIdx.x == 0) {
        for (int s = 0; s < NR; ++s) {
            mbar_init(&rfull[s], 1);
            mbar_init(&rempty[s], RW);
        }
        for (int s = 0; s < NC; ++s) {
            mbar_init(&cfull[s], RW);
            mbar_init(&cempty[s], 1);
        }
        for (int s = 0; s < NB; ++s) {
            mbar_init(&bfull[s], 1);
            mbar_init(&bempty[s], 1);
        }
        mbar_init(accfull, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmW0);
        if (DUAL) tma_prefetch_desc(&tmW1);
    }
    if (warp == 1) tmem_alloc(tmem_s, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    const uint32_t tD = tbase;                               // matrix m: + m * NCOL
    fr_pdl_trigger();

    if (warp == 0) {
        // ---------------- weight producer: no PDL wait
        if (lane == 0) {
            for (int i = 0; i < n_st; ++i) {
                const int s = i % NR;
                if (i >= NR && !mbar_wait(&rempty[s], ((i / NR) - 1) & 1, 40)) break;
                uint8_t *st = raw0 + static_cast<size_t>(s) * S::RAW;
                const int kt = kt0 + i;
                mbar_expect_tx(&rfull[s], NM * g.R * FM_WBOX);
                tma_load_2d(st, &tmW0, kt * FM_WBOX, r0, &rfull[s]);
                if (DUAL) tma_load_2d(st + 128 * FM_WBOX, &tmW1, kt * FM_WBOX, r0, &rfull[s]);
            }
        }
    } else if (warp == 2) {
        // ---------------- activation-column producer (after the PDL wait)
        if (lane == 0) {
            fr_pdl_wait();
            for (int i = 0; i < n_st; ++i) {
                const int s = i % NB;
                if (i >= NB && !mbar_wait(&bempty[s], ((i / NB) - 1) & 1, 45)) break;
                uint8_t *bs = b0 + static_cast<size_t>(s) * S::BST;
                const int kt = kt0 + i;
                mbar_expect_tx(&bfull[s], S::BST);
                bulk_g2s(bs, g.bimg + static_cast<int64_t>(kt) * S::B_BYTES, S::B_BYTES, &bfull[s]);
                bulk_g2s(bs + S::B_BYTES, g.sfb + static_cast<int64_t>(kt) * S::SF_BYTES, S::SF_BYTES, &bfull[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_nvf4(128, NCOL);
            for (int i = 0; i < n_st; ++i) {
                const int sc = i % NC, sb = i % NB;
                if (!mbar_wait(&bfull[sb], (i / NB) & 1, 46)) break;
                if (!mbar_wait(&cfull[sc], (i / NC) & 1, 41)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(can0 + static_cast<size_t>(sc) * S::CAN);
                const uint32_t sfa_addr = a_addr + NM * S::A_BYTES;        // SFA m at + m * SF_BYTES
                const uint32_t b_addr = smem_u32(b0 + static_cast<size_t>(sb) * S::BST);
                const uint32_t sfb_addr = b_addr + S::B_BYTES;
                const uint32_t t_sf = tbase + 256 + sc * 48;                // SFA m at + 16 m, SFB at + 32
#pragma unroll
                for (int j = 0; j < 4; ++j) {
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                        tc_cp_sf(t_sf + 16 * m + 4 * j, sdesc_plain(sfa_addr + m * S::SF_BYTES + 512 * j, 128));
                    tc_cp_sf(t_sf + 32 + 4 * j, sdesc_plain(sfb_addr + 512 * j, 128));
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                        tc_mma_nvf4(tD + m * NCOL, sdesc_sw128(a_addr + m * S::A_BYTES + 32 * j),
                                    sdesc_sw128(b_addr + 32 * j), idesc, t_sf + 16 * m + 4 * j, t_sf + 32 + 4 * j,
                                    (i > 0 || j > 0) ? 1u : 0u);
                }
                tc_commit(&cempty[sc]);
                tc_commit(&bempty[sb]);
            }
            tc_commit(accfull);
        }
    } else {
        // ---------------- row warps: raw rows -> swizzled code tiles + scale atoms
        const int rw = warp - 3;
        const int m = rw >> 2;                               // matrix
        const int q = warp & 3;                              // TMEM lane quadrant (for the epilogue)
        const int row = 32 * (rw & 3) + lane;                // tile row this thread moves
        const bool live_row = row < g.R;
        bool ok = true;
        for (int i = 0; i < n_st; ++i) {
            const int sr = i % NR, sc = i % NC;
            if (!mbar_wait(&rfull[sr], (i / NR) & 1, 42)) { ok = false; break; }
            uint4 u[9];
            if (live_row) {
                const uint4 *src = reinterpret_cast<const uint4 *>(raw0 + static_cast<size_t>(sr) * S::RAW +
                                                                  m * 128 * FM_WBOX + row * FM_WBOX);
#pragma unroll
                for (int k = 0; k < 9; ++k) u[k] = src[k];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[sr]);
            if (i >= NC && !mbar_wait(&cempty[sc], ((i / NC) - 1) & 1, 43)) { ok = false; break; }
            uint8_t *cs = can0 + static_cast<size_t>(sc) * S::CAN;
            if (live_row) {
                const uint32_t w[36] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y, u[1].z, u[1].w,
                                        u[2].x, u[2].y, u[2].z, u[2].w, u[3].x, u[3].y, u[3].z, u[3].w,
                                        u[4].x, u[4].y, u[4].z, u[4].w, u[5].x, u[5].y, u[5].z, u[5].w,
                                        u[6].x, u[6].y, u[6].z, u[6].w, u[7].x, u[7].y, u[7].z, u[7].w,
                                        u[8].x, u[8].y, u[8].z, u[8].w};
                uint8_t *a = cs + m * S::A_BYTES + row * 128;
                uint8_t *sfa = cs + NM * S::A_BYTES + m * S::SF_BYTES + (row & 31) * 16 + (row >> 5) * 4;
                const int sw = row & 7;
#pragma unroll
                for (int kb = 0; kb < 4; ++kb) {
                    // scale word: ggml ignores the sign bits; code 0x7F (NaN
                    // in e4m3) is zero for ggml
                    uint32_t sv = w[9 * kb] & 0x7F7F7F7Fu;
                    const uint32_t nan = (sv + 0x01010101u) & 0x80808080u;
                    sv &= ~((nan >> 7) * 0xFFu);
                    *reinterpret_cast<uint32_t *>(sfa + kb * 512) = sv;
                    *reinterpret_cast<uint4 *>(a + (((2 * kb) ^ sw) << 4)) =
                        make_uint4(w[9 * kb + 1], w[9 * kb + 2], w[9 * kb + 3], w[9 * kb + 4]);
                    *reinterpret_cast<uint4 *>(a + (((2 * kb + 1) ^ sw) << 4)) =
                        make_uint4(w[9 * kb + 5], w[9 * kb + 6], w[9 * kb + 7], w[9 * kb + 8]);
                }
            }
            // generic-proxy stores -> visible to the tensor core's async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&cfull[sc]);
        }
        // ---------------- epilogue: the row warps of matrix 0, one per quadrant
        if (m == 0 && ok && mbar_wait(accfull, 0, 44)) {
            tc_fence_after();
            fr_pdl_wait();
            const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
            const int erow = 32 * q + lane;                  // TMEM lane = tile row
            const bool split = g.ksplit > 1;
            const int n = r0 + erow;
            const bool live = erow < g.R && n < g.N;
            const float sc0 = g.s0 ? *g.s0 : 1.0f;
            const float sc1 = (DUAL && g.s1) ? *g.s1 : 1.0f;
            float *pp = g.part + ((static_cast<int64_t>(rt) * g.ksplit + ks) * 2) * TMAX * 128;
            auto finish = [&](int t, float a0, float a1) {
                if (!live || t >= g.T) return;
                const int64_t tt = g.t0 + t;
                float v;
                if (DUAL) {
                    float result = a1;
                    result *= sc1;
                    float gate = a0;
                    gate *= sc0;
                    result *= silu_f(gate);
                    v = result;
                } else {
                    v = a0 * sc0;
                    if (g.resid) v += g.resid[tt * g.ldr + n];
                }
                g.y[tt * g.ldy + n] = v;
            };
            // column sums -> per-token values, 16 columns at a time
            float acc0[TMAX], acc1[TMAX];
#pragma unroll
            for (int t = 0; t < TMAX; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }
#pragma unroll
            for (int c = 0; c < NCOL; c += 16) {
                uint32_t d0[16], d1[16];
                tmem_ld16(tD + lane_off + c, d0);
                if (DUAL) tmem_ld16(tD + NCOL + lane_off + c, d1);
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int col = c + u, t = col / FM_DIGITS, p = col % FM_DIGITS;
                    if (t < TMAX && t < g.T) {
                        const float gf = g.gtab[t * FM_GSTRIDE + p];
                        acc0[t] = fmaf(gf, __uint_as_float(d0[u]), acc0[t]);
                        if (DUAL) acc1[t] = fmaf(gf, __uint_as_float(d1[u]), acc1[t]);
                    }
                }
            }
            if (!split) {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) finish(t, acc0[t], acc1[t]);
            } else {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    pp[t * 128 + erow] = acc0[t];
                    if (DUAL) pp[TMAX * 128 + t * 128 + erow] = acc1[t];
                }
                __threadfence();
                __syncwarp();
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&g.counter[rt * 4 + q], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == static_cast<unsigned>(g.ksplit - 1)) {
                    __threadfence();
                    const float *pb = g.part + (static_cast<int64_t>(rt) * g.ksplit * 2) * TMAX * 128;
#pragma unroll 1
                    for (int t = 0; t < TMAX && t < g.T; ++t) {
                        float a0 = 0.0f, a1 = 0.0f;
                        for (int k2 = 0; k2 < g.ksplit; ++k2) {
                            a0 += __ldcg(pb + (k2 * 2) * TMAX * 128 + t * 128 + erow);
                            if (DUAL) a1 += __ldcg(pb + (k2 * 2 + 1) * TMAX * 128 + t * 128 + erow);
                        }
                        finish(t, a0, a1);
                    }
                    if (lane == 0) g.counter[rt * 4 + q] = 0;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

} // namespace frb
