// fr_tcgemv.cuh -- NVFP4 x q8_1 matvec / batched GEMM on the tcgen05 tensor
// cores (T = 1..64 tokens per launch, weights read once per launch).
//
// Arithmetic (exact restatement of vec_dot_nvfp4_q8_1 up to fp32 summation
// order, src/fr_win_flint_sm120.cu:320-342):
//   * weight w = e2m1(code) * e4m3(scale) is exact in f16 (<= 6 significant
//     bits, 2^-10 .. 2688), and equals ggml's kvalues * ue4m3 / 4 ... / 2 pair;
//   * the q8_1 activation x_q = q * d (d the f16-rounded block scale) has at
//     most 18 significant bits and splits exactly into f16 hi + lo;
//   * D = W . [hi | lo] accumulates in fp32 in TMEM; y = D_hi + D_lo.
// So the only difference from ggml's int32 sub-block sums with fp32 scaling is
// the fp32 summation order.
//
// Data flow per CTA (rows [r0, r0+R), K stages [kt0, kt1) of 256 values):
//   producer warp  : TMA 2-D box of the raw block_nvfp4 rows (R rows x 144 B:
//                    four 36-byte blocks per row, rows 144 B apart in shared
//                    memory so thread-per-row 128-bit reads are conflict-free)
//                    and four 128-byte-swizzled boxes of the hi/lo activation;
//   16 decode warps: thread = weight row = TMEM lane; warp (quadrant q,
//                    phase p) decodes block p of each stage: cvt e2m1x2 ->
//                    f16x2, times the sub-block scale, tcgen05.st into a ring
//                    of TMEM A slots (one 64-value block each), so decoding
//                    block g + NA overlaps the MMAs of block g;
//   MMA lane       : tcgen05.mma kind::f16, A from TMEM, B from shared memory,
//                    D (R x 2T, f32) in TMEM;
//   epilogue       : tcgen05.ld of D, y = D_hi + D_lo, SwiGLU / scale /
//                    residual; with split-K the partial goes to a workspace
//                    and the last CTA of the row tile adds the K splits in
//                    order (deterministic) and applies the epilogue.
#pragma once

#include "fr_tc.cuh"

namespace frb {

constexpr int TG_DW = 16;                          // decode warps (4 per TMEM lane quadrant)
constexpr int TG_THREADS = (2 + TG_DW) * 32;       // + producer warp + MMA warp
constexpr int TG_KS = 256;                         // K values per stage
constexpr int TG_WBOX = 144;                       // bytes per row per stage (4 blocks)
constexpr int TG_WBYTES = 128 * TG_WBOX;           // 18 KB per matrix per stage

__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    // c_format F32 (bit 4), A/B f16, K-major, N >> 3, M >> 4
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        :: "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
           "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
           "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
           "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// four codes-bytes of one word -> four f16x2 (low nibble in the low half),
// each times the sub-block scale pair `s2`
__device__ __forceinline__ void e2m1x8_scaled(uint32_t w, uint32_t s2, uint32_t *out) {
    uint32_t h0, h1, h2, h3;
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h0) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h1) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h2) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(h3) : "r"(s2));
    out[0] = h0; out[1] = h1; out[2] = h2; out[3] = h3;
}

// One 64-value block (9 words) -> 32 TMEM columns of f16x2 (exact weights).
// Column 8s + j holds values (j, j+8) of sub-block s: the K order the
// activation operand is written in (k_act_hilo).
__device__ __forceinline__ void decode_block_f16(const uint32_t (&w)[9], uint32_t (&col)[32]) {
    const uint32_t m = w[0] & 0x7F7F7F7Fu;          // ggml ignores the scale's sign bit
    uint32_t s01, s23;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s01) : "h"(static_cast<unsigned short>(m & 0xFFFFu)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s23) : "h"(static_cast<unsigned short>(m >> 16)));
    // code 0x7F is NaN in e4m3 and zero for ggml: max(x, 0) maps NaN to 0
    asm("max.f16x2 %0, %0, %1;" : "+r"(s01) : "r"(0u));
    asm("max.f16x2 %0, %0, %1;" : "+r"(s23) : "r"(0u));
    const uint32_t sp[4] = {prmt(s01, 0, 0x1010), prmt(s01, 0, 0x3232), prmt(s23, 0, 0x1010), prmt(s23, 0, 0x3232)};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        e2m1x8_scaled(w[1 + 2 * s], sp[s], &col[8 * s]);
        e2m1x8_scaled(w[2 + 2 * s], sp[s], &col[8 * s + 4]);
    }
}

// The 9 words of block `ph` (0..3) of a row's 144-byte stage segment, read as
// three aligned 128-bit loads (rows are 144 B apart: eight lanes of a quarter
// warp hit eight different 16-byte bank groups).
__device__ __forceinline__ void load_block(const uint8_t *rowseg, int ph, uint32_t (&w)[9]) {
    const uint4 *p = reinterpret_cast<const uint4 *>(rowseg + ((ph * 36) & ~15));
    const uint4 a = p[0], b = p[1], c = p[2];
    const uint32_t u[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
    switch (ph) {
    case 0:
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = u[k];
        break;
    case 1:
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = u[k + 1];
        break;
    case 2:
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = u[k + 2];
        break;
    default:
#pragma unroll
        for (int k = 0; k < 9; ++k) w[k] = u[k + 3];
        break;
    }
}

// ------------------------------------------------------------ activation
// B operand [NP rows, Kp] f16: row 2t = hi(x_q[t]), row 2t+1 = lo, zero rows
// for t >= T and zero columns past K.  Value j of a 16-value sub-block sits at
// position 2j (j < 8) or 2(j-8)+1 (j >= 8).  x_q follows quantize_q8_1
// exactly (d = f16(amax/127), q = roundf(x/d)).  Input either q8_1 blocks or
// f32 rows.  One warp per (token, 32-value chunk).
__global__ void __launch_bounds__(256) k_act_hilo(const float *__restrict__ x, int64_t ldx,
                                                  const uint8_t *__restrict__ q8, int64_t ldq, int T, int K, int Kp,
                                                  int NP, __half *__restrict__ B) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int ncp = Kp / 32;
    const int64_t c = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (c >= static_cast<int64_t>(NP / 2) * ncp) return;
    const int t = static_cast<int>(c / ncp), ch = static_cast<int>(c % ncp);
    float xq = 0.0f;
    if (t < T && ch * 32 < K) {
        if (x != nullptr) {
            const q8_lane r = q8_1_chunk(x[t * ldx + static_cast<int64_t>(ch) * 32 + lane]);
            xq = static_cast<float>(r.q) * __half2float(__float2half_rn(r.d));
        } else {
            const uint8_t *blk = q8 + (t * ldq + ch) * Q8_BYTES;
            xq = static_cast<float>(static_cast<int8_t>(blk[4 + lane])) * __low2float(*reinterpret_cast<const __half2 *>(blk));
        }
    }
    const __half hi = __float2half_rn(xq);
    const __half lo = __float2half_rn(xq - __half2float(hi));
    const int j = lane & 15;
    const int pos = ch * 32 + (lane & 16) + (j < 8 ? 2 * j : 2 * (j - 8) + 1);
    B[static_cast<int64_t>(2 * t) * Kp + pos] = hi;
    B[static_cast<int64_t>(2 * t + 1) * Kp + pos] = lo;
}

// ------------------------------------------------------------ matvec
enum TgEpi : int { TG_PLAIN = 0, TG_SWIGLU = 1 };

struct TgArgs {
    int N, K, T;                 // rows, row length, tokens in this launch (<= NP/2)
    int t0;                      // first output token index
    int R;                       // rows per tile (<= 128)
    int n_kt;                    // K stages of 256
    int ksplit;                  // K splits per row tile
    int kt_per_split;
    const float *s0, *s1;        // per-tensor scales (nullable)
    const float *resid;          // [.., ldr] (nullable)
    int64_t ldr;
    float *y;                    // [.., ldy]
    int64_t ldy;
    float *part;                 // split-K partials [n_rt][ksplit][2][NP/2][128]
    unsigned int *counter;       // [n_rt][4 quadrants][4 column ranges], zero on entry, reset by the last split
    int n_stages;                // shared-memory ring depth
};

template <int NP, int EPI>
__global__ void __launch_bounds__(TG_THREADS, 1) k_tcgemv(const __grid_constant__ CUtensorMap tmW0,
                                                        const __grid_constant__ CUtensorMap tmW1,
                                                        const __grid_constant__ CUtensorMap tmB, const TgArgs g) {
    constexpr bool DUAL = EPI == TG_SWIGLU;
    constexpr int NM = DUAL ? 2 : 1;
    constexpr int BBYTES = 4 * NP * 128;                    // activation tiles per stage
    constexpr int STAGE = NM * TG_WBYTES + BBYTES;
    constexpr int NT = NP / 2;                              // tokens
    // A ring: NA slots of one 64-value block (32 columns) per matrix, so the
    // decode of block g+NA overlaps the MMAs of block g
    constexpr int NA = !DUAL ? 8 : (NP <= 64 ? 6 : 4);
    constexpr uint32_t A_COLS = NA * 32;                    // per matrix
    constexpr uint32_t TMEM_COLS = (NM * A_COLS + NM * NP) <= 256 ? 256 : 512;
    static_assert(NM * A_COLS + NM * NP <= 512, "TMEM budget");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = g.n_stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * STAGE);
    uint64_t *wfree = full + S;
    uint64_t *bfree = wfree + S;
    uint64_t *afull = bfree + S;                            // [NA]
    uint64_t *aempty = afull + NA;                          // [NA]
    uint64_t *accfull = aempty + NA;
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(accfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = blockIdx.x / g.ksplit, ks = blockIdx.x % g.ksplit;
    const int r0 = rt * g.R;
    const int kt0 = ks * g.kt_per_split;
    const int kt1 = min(g.n_kt, kt0 + g.kt_per_split);
    const int n_st = kt1 - kt0;
    const int nkb_total = g.K / 64;                         // 64-blocks in a row

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&wfree[s], TG_DW);
            mbar_init(&bfree[s], 1);
        }
        for (int a = 0; a < NA; ++a) {
            mbar_init(&afull[a], 4);
            mbar_init(&aempty[a], 1);
        }
        mbar_init(accfull, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmW0);
        if (DUAL) tma_prefetch_desc(&tmW1);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_s, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    const uint32_t tA = tbase;                               // matrix m: + m * 128
    const uint32_t tD = tbase + NM * A_COLS;                 // matrix m: + m * NP

    if (warp == 0) {
        // ---------------- producer: weights need no PDL wait, the activation does
        if (lane == 0) {
            bool waited_pdl = false;
            // ring slot s and its use count as counters (no runtime division
            // on this thread's critical path)
            for (int i = 0, s = 0, use = 0; i < n_st; ++i, use += (++s == S), s = (s == S) ? 0 : s) {
                if (use > 0) {
                    if (!mbar_wait(&wfree[s], (use - 1) & 1, 20)) break;
                    if (!mbar_wait(&bfree[s], (use - 1) & 1, 21)) break;
                }
                uint8_t *st = smem + s * STAGE;
                const int kt = kt0 + i;
                mbar_expect_tx(&full[s], NM * g.R * TG_WBOX + BBYTES);
                tma_load_2d(st, &tmW0, kt * TG_WBOX, r0, &full[s]);
                if (DUAL) tma_load_2d(st + TG_WBYTES, &tmW1, kt * TG_WBOX, r0, &full[s]);
                if (!waited_pdl) { fr_pdl_wait(); waited_pdl = true; }
                uint8_t *bs = st + NM * TG_WBYTES;
#pragma unroll
                for (int c = 0; c < 4; ++c) tma_load_2d(bs + c * NP * 128, &tmB, kt * TG_KS + 64 * c, 0, &full[s]);
            }
            if (!waited_pdl) fr_pdl_wait();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(128, NP);
            bool ok = true;
            for (int i = 0, s = 0, use = 0; i < n_st && ok; ++i, use += (++s == S), s = (s == S) ? 0 : s) {
                if (!mbar_wait(&full[s], use & 1, 22)) { ok = false; break; }
                const int kb0 = (kt0 + i) * 4;
                const uint32_t b_addr = smem_u32(smem + s * STAGE + NM * TG_WBYTES);
                for (int blk = 0; blk < 4; ++blk) {
                    if (kb0 + blk >= nkb_total) break;
                    const int gb = 4 * i + blk, slot = gb % NA, use = gb / NA;
                    if (!mbar_wait(&afull[slot], use & 1, 23)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            tc_mma_f16_ts(tD + m * NP, tA + m * A_COLS + slot * 32 + 8 * j,
                                          sdesc_sw128(b_addr + blk * NP * 128 + 32 * j), idesc,
                                          (i > 0 || blk > 0 || j > 0) ? 1u : 0u);
                        }
                    }
                    tc_commit(&aempty[slot]);
                }
                tc_commit(&bfree[s]);
            }
            tc_commit(accfull);
        }
    } else {
        // ---------------- decoders (and the epilogue)
        const int q = warp & 3;                              // TMEM lane quadrant
        const int ph = (warp - 2) >> 2;                      // block of the stage this warp decodes
        const int row = 32 * q + lane;                       // tile row = TMEM lane
        const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
        bool ok = true;
        for (int i = 0, s = 0, su = 0; i < n_st; ++i, su += (++s == S), s = (s == S) ? 0 : s) {
            if (!mbar_wait(&full[s], su & 1, 24)) { ok = false; break; }
            const bool has_blk = (kt0 + i) * 4 + ph < nkb_total;
            uint32_t w0[9], w1[9];
            if (has_blk) {
                const uint8_t *src = smem + s * STAGE + row * TG_WBOX;
                load_block(src, ph, w0);
                if (DUAL) load_block(src + TG_WBYTES, ph, w1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&wfree[s]);
            if (!has_blk) continue;
            const int gb = 4 * i + ph, slot = gb % NA, use = gb / NA;
            uint32_t col[32];
            decode_block_f16(w0, col);                      // decode before waiting for the slot
            if (use > 0 && !mbar_wait(&aempty[slot], (use - 1) & 1, 25)) { ok = false; break; }
            tc_fence_after();
            tmem_st32(tA + lane_off + slot * 32, col);
            if (DUAL) {
                decode_block_f16(w1, col);
                tmem_st32(tA + A_COLS + lane_off + slot * 32, col);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[slot]);
        }
        // ---------------- epilogue: EW warps per quadrant (EW = NP / 16, at
        // most 4), warp ph for the columns [ph CW, ph CW + CW) (tokens
        // [ph CW / 2, ...)) of its quadrant's 32 rows.  With split-K it
        // publishes its partial and the last of the K splits for that
        // (row tile, quadrant, column range) adds them in split order, its
        // partial loads batched so their latencies overlap -- no CTA-wide
        // barrier, so a timed-out warp cannot hang it.
        constexpr int EW = NP / 16 < 4 ? NP / 16 : 4;
        constexpr int CW = NP / EW;                          // columns per epilogue warp
        constexpr int TWW = CW / 2;                          // tokens per epilogue warp
        if (ph < EW && ok && mbar_wait(accfull, 0, 26)) {
            tc_fence_after();
            fr_pdl_wait();
            const bool split = g.ksplit > 1;
            const int n = r0 + row;
            const bool live = row < g.R && n < g.N;
            const float sc0 = g.s0 ? *g.s0 : 1.0f;
            const float sc1 = (DUAL && g.s1) ? *g.s1 : 1.0f;
            const int tw0 = ph * TWW;
            float *pp = g.part + ((static_cast<int64_t>(rt) * g.ksplit + ks) * 2) * NT * 128;
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
#pragma unroll
            for (int c = 0; c < CW; c += 16) {
                uint32_t r0v[16], r1v[16];
                tmem_ld16(tD + lane_off + ph * CW + c, r0v);
                if (DUAL) tmem_ld16(tD + NP + lane_off + ph * CW + c, r1v);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = tw0 + c / 2 + u;
                    const float a0 = __uint_as_float(r0v[2 * u]) + __uint_as_float(r0v[2 * u + 1]);
                    const float a1 = DUAL ? __uint_as_float(r1v[2 * u]) + __uint_as_float(r1v[2 * u + 1]) : 0.0f;
                    if (split) {
                        pp[t * 128 + row] = a0;
                        if (DUAL) pp[NT * 128 + t * 128 + row] = a1;
                    } else {
                        finish(t, a0, a1);
                    }
                }
            }
            if (split) {
                __threadfence();
                __syncwarp();
                unsigned int *cnt = &g.counter[(rt * 4 + q) * 4 + ph];
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(cnt, 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == static_cast<unsigned>(g.ksplit - 1)) {
                    __threadfence();
                    const float *pb = g.part + (static_cast<int64_t>(rt) * g.ksplit * 2) * NT * 128 + tw0 * 128 + row;
                    constexpr int KU = DUAL ? 2 : 4;         // splits whose loads go out together
                    float acc0[TWW], acc1[TWW];
#pragma unroll
                    for (int u = 0; u < TWW; ++u) {
                        acc0[u] = 0.0f;
                        acc1[u] = 0.0f;
                    }
                    int k2 = 0;
#pragma unroll 1
                    for (; k2 + KU <= g.ksplit; k2 += KU) {
                        float v0[KU][TWW], v1[KU][TWW];
#pragma unroll
                        for (int j = 0; j < KU; ++j)
#pragma unroll
                            for (int u = 0; u < TWW; ++u) {
                                v0[j][u] = __ldcg(pb + ((k2 + j) * 2) * NT * 128 + u * 128);
                                if (DUAL) v1[j][u] = __ldcg(pb + ((k2 + j) * 2 + 1) * NT * 128 + u * 128);
                            }
#pragma unroll
                        for (int j = 0; j < KU; ++j)
#pragma unroll
                            for (int u = 0; u < TWW; ++u) {
                                acc0[u] += v0[j][u];
                                if (DUAL) acc1[u] += v1[j][u];
                            }
                    }
#pragma unroll 1
                    for (; k2 < g.ksplit; ++k2) {
                        float v0[TWW], v1[TWW];
#pragma unroll
                        for (int u = 0; u < TWW; ++u) {
                            v0[u] = __ldcg(pb + (k2 * 2) * NT * 128 + u * 128);
                            if (DUAL) v1[u] = __ldcg(pb + (k2 * 2 + 1) * NT * 128 + u * 128);
                        }
#pragma unroll
                        for (int u = 0; u < TWW; ++u) {
                            acc0[u] += v0[u];
                            if (DUAL) acc1[u] += v1[u];
                        }
                    }
#pragma unroll
                    for (int u = 0; u < TWW; ++u) finish(tw0 + u, acc0[u], acc1[u]);
                    if (lane == 0) *cnt = 0;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    fr_pdl_trigger();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

} // namespace frb
