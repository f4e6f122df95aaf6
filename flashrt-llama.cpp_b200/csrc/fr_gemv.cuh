// fr_gemv.cuh -- q8_1 quantizer and the NVFP4 x q8_1 matvec for B200.
//
// Matvec design (HBM-bound; one pass over the weight rows per launch):
//   * Each CTA owns a contiguous range of weight rows.  Because ggml's
//     block_nvfp4 rows are contiguous, that range is one contiguous byte
//     stream, which a single producer lane moves into a shared-memory ring with
//     1-D bulk copies (cp.async.bulk, the TMA engine, no multicast) completing
//     on mbarriers.  No register or LSU cost for the stream itself.
//   * A "stage" is the rows one consumer warp finishes in one pass
//     (32 / LG rows, LG lanes per row); stage i goes to ring slot i % NS and
//     consumer warp i % 8, so every slot has exactly one consumer.
//   * The activations (T tokens of q8_1) are staged once per CTA into shared
//     memory, byte-permuted to the order the weight decode produces and
//     swizzled for conflict-free 128-bit reads.  The f32 entry points quantize
//     into that staging area directly (the reference fuses quantize_q8_1 into
//     its GEMV prologues the same way, src/fr_win_flint_sm120.cu:1047-1049).
//   * Weight decode: two prmt per 4 codes against the table |kvalues| with the
//     sign bit selecting 0 (prmt sign-replicate of a positive byte), once for
//     the code and once for the code with bit 3 flipped, so
//     sum kv*q = dp4a(pos, q) - dp4a(neg, q) exactly in int32 per 16-value
//     sub-block, as vec_dot_nvfp4_q8_1 computes it
//     (src/fr_win_flint_sm120.cu:320-342); then fp32 (d_w * d_q8) * sumi.
//   * Weight bytes are fetched before griddepcontrol.wait (they do not depend
//     on the previous kernel), so under PDL the stream starts while the
//     producer of the activations is still finishing.
#pragma once

#include "fr_common.cuh"

namespace frb {

// ------------------------------------------------------------ quantize_q8_1
// Row r of the output is x row (r / n_in) * ldx + (r % n_in) * ldx_in, so one
// launch also covers [T, n_used, K] activations with two strides.
__global__ void __launch_bounds__(256) k_quantize_q8_1(const float *__restrict__ x, int64_t ldx, int n_in,
                                                       int64_t ldx_in, uint8_t *__restrict__ q8, int64_t ldq,
                                                       int T, int K) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int nc = K / Q8_ELEMS;
    const int64_t c = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (c >= static_cast<int64_t>(T) * nc) return;
    const int t = static_cast<int>(c / nc), ch = static_cast<int>(c % nc);
    const int64_t xrow = static_cast<int64_t>(t / n_in) * ldx + static_cast<int64_t>(t % n_in) * ldx_in;
    const float xi = x[xrow + static_cast<int64_t>(ch) * Q8_ELEMS + lane];
    const q8_lane r = q8_1_chunk(xi);
    uint8_t *blk = q8 + (t * ldq + ch) * Q8_BYTES;
    blk[4 + lane] = static_cast<uint8_t>(r.q);
    if (lane == 0) {
        const __half2 ds = __halves2half2(__float2half_rn(r.d), __float2half_rn(r.sum));
        *reinterpret_cast<__half2 *>(blk) = ds;
    }
}

// ------------------------------------------------------------ matvec
constexpr int GV_CWARPS = 8;                        // consumer warps (MoE kernel)
#ifndef FR_GV_CW
#define FR_GV_CW 16
#endif
constexpr int GV_MAIN_CW = FR_GV_CW;                // consumer warps of the dense matvec
constexpr int GV_THREADS = (GV_CWARPS + 1) * 32;    // + one producer warp

enum GvEpi : int { GV_PLAIN = 0, GV_SWIGLU = 1 };

struct GvParams {
    const uint8_t *w0;      // rows [N, w_ld]
    const uint8_t *w1;      // up rows for the SwiGLU pair (else null)
    int64_t w_ld;           // bytes per row (multiple of 16 on the bulk path)
    const uint8_t *q8;      // q8_1 activations [T, ldq blocks] (if x == null)
    int64_t ldq;
    const float *x;         // f32 activations [T, ldx] (fused quantize)
    int64_t ldx;
    const float *s0, *s1;   // per-tensor scales (nullable)
    const float *resid;     // [T, ldr] added to the output (nullable)
    int64_t ldr;
    float *y;
    int64_t ldy;
    int N, K;
    int t0, nt;             // token window of this launch
    int rows_per_cta;
    int rows_per_stage;     // 32 / LG
    int n_slots;            // ring slots (multiple of GV_CWARPS)
    int slot_bytes;         // bytes per slot (both operands)
    int word_mode;          // rows not 16-byte aligned: producer warp copies words
    // tensor-parallel epilogue (npeers > 0): every output value is also stored
    // into each rank's copy of the output (peer_base[p] + peer_off bytes, row
    // offset col_off), and when the CTA is done it adds 1 to its rank's slot
    // of every peer's flag array (peer_base[p] + flag_off bytes)
    uint8_t *const *peer_base;
    int npeers, rank;
    int64_t peer_off, flag_off, col_off;
    // step parity of the receiving slots: the values go to peer_off +
    // (epoch[0] & 1) * par_bytes (the reduce's step count, final by the time
    // the epilogue runs; null = parity 0)
    const unsigned int *epoch;
    int64_t par_bytes;
    // q8 input in a double-buffered exchange buffer: q8 + (q8_epoch[0] & 1) *
    // q8_par (null = q8 as given)
    const unsigned int *q8_epoch;
    int64_t q8_par;
};

// Bounded wait of one lane for flags[r] to reach seen + expect (counters only
// grow; the difference is compared signed so the counters may wrap).
__device__ __forceinline__ void tp_flag_wait(const unsigned int *flags, unsigned int *seen, int r,
                                             unsigned int expect) {
    const unsigned int target = *seen + expect;
    const uint64_t t0 = fr_now_ns();
    for (;;) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
        if (static_cast<int>(v - target) >= 0) break;
        if (fr_now_ns() - t0 > g_fr_wait_ns) {
            fr_flag(FR_ST_TIMEOUT | (30u << FR_ST_SITE_SHIFT));
            break;
        }
    }
    *seen = target;
}

// Byte position inside a sub-block's 16 activation bytes of value j (0..15),
// matching the order nv_decode emits: words (j,j+8,j+1,j+9), (j+2,..), ...
__device__ __forceinline__ int act_perm(int j) {
    const int jj = j & 7, hi = j >> 3;
    return (jj >> 1) * 4 + (jj & 1) * 2 + hi;
}

// Stage the activation of tokens [t0, t0+nt) into shared memory:
// act_q: int4 per (token, 64-block, sub-block), swizzled by (b >> 1) & 3;
// act_d: float2 per (token, 64-block) = 0.5 * f16-rounded q8_1 scales.
// Loads are batched so that each thread has up to 8 in flight: the staging
// costs about one L2 round trip per batch instead of one per chunk.
__device__ __forceinline__ void act_put(uint8_t *aq, float *ad, int NB, int t, int ch, int j, int8_t q) {
    const int b = ch >> 1;
    const int s = ((ch & 1) << 1) | (j >> 4);
    const int slot = (t * NB + b) * 4 + (s ^ ((b >> 1) & 3));
    aq[slot * 16 + act_perm(j & 15)] = static_cast<uint8_t>(q);
    (void) ad;
}

template <int CW>
__device__ __forceinline__ void gv_stage_act(const GvParams &p, int4 *act_q, float2 *act_d, int warp, int lane) {
    const int nc = p.K / Q8_ELEMS, NB = p.K / NV_ELEMS;
    uint8_t *aq = reinterpret_cast<uint8_t *>(act_q);
    float *ad = reinterpret_cast<float *>(act_d);
    constexpr int BATCH = 8;
    if (p.x != nullptr) {
        // f32 input: one warp per 32-value chunk (the butterfly needs the warp)
        const int total = p.nt * nc;
        for (int base = warp; base < total; base += CW * BATCH) {
            float v[BATCH];
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const int c = base + CW * u;
                v[u] = 0.0f;
                if (c < total) {
                    const int t = c / nc, ch = c % nc;
                    v[u] = p.x[(p.t0 + t) * p.ldx + static_cast<int64_t>(ch) * Q8_ELEMS + lane];
                }
            }
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const int c = base + CW * u;
                if (c < total) {
                    const int t = c / nc, ch = c % nc;
                    const q8_lane r = q8_1_chunk(v[u]);
                    act_put(aq, ad, NB, t, ch, lane, r.q);
                    if (lane == 0) ad[(t * NB + (ch >> 1)) * 2 + (ch & 1)] = 0.5f * __half2float(__float2half_rn(r.d));
                }
            }
        }
    } else {
        // q8_1 input: every consumer thread moves 4-byte words of the blocks
        // (from the step-parity half of an exchange buffer when q8_epoch is set)
        const uint8_t *q8 = p.q8 + (p.q8_epoch ? static_cast<int64_t>(*p.q8_epoch & 1u) * p.q8_par : 0);
        const int tid = warp * 32 + lane;
        const int total = p.nt * nc * 9;
        for (int base = tid; base < total; base += CW * 32 * BATCH) {
            uint32_t w[BATCH];
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const int wi = base + CW * 32 * u;
                w[u] = 0;
                if (wi < total) {
                    const int c = wi / 9, k = wi % 9;
                    const int t = c / nc, ch = c % nc;
                    w[u] = *reinterpret_cast<const uint32_t *>(q8 + ((p.t0 + t) * p.ldq + ch) * Q8_BYTES + 4 * k);
                }
            }
#pragma unroll
            for (int u = 0; u < BATCH; ++u) {
                const int wi = base + CW * 32 * u;
                if (wi < total) {
                    const int c = wi / 9, k = wi % 9;
                    const int t = c / nc, ch = c % nc;
                    if (k == 0) {
                        const __half2 ds = *reinterpret_cast<const __half2 *>(&w[u]);
                        ad[(t * NB + (ch >> 1)) * 2 + (ch & 1)] = 0.5f * __low2float(ds);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            act_put(aq, ad, NB, t, ch, 4 * (k - 1) + i, static_cast<int8_t>((w[u] >> (8 * i)) & 0xFF));
                    }
                }
            }
        }
    }
}

// dot of one 64-block (9 words at `blk`) with TT tokens' staged activations
template <int TT>
__device__ __forceinline__ void gv_block(const uint32_t *blk, int b, int NB, int nt,
                                         const int4 *act_q, const float2 *act_d, float (&acc)[TT]) {
    const uint32_t dw = blk[0];
    nv_word dec[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) dec[i] = nv_decode(blk[1 + i]);
    float sc[4];
    ue4m3x4(dw, sc);
    const int swz = (b >> 1) & 3;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        if (t < nt) {
            const int4 *aq = act_q + (t * NB + b) * 4;
            const float2 dd = act_d[t * NB + b];
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int4 a = aq[s ^ swz];
                int ip = dp4a(dec[2 * s].p0, a.x, 0);
                ip = dp4a(dec[2 * s].p1, a.y, ip);
                ip = dp4a(dec[2 * s + 1].p0, a.z, ip);
                ip = dp4a(dec[2 * s + 1].p1, a.w, ip);
                int in = dp4a(dec[2 * s].n0, a.x, 0);
                in = dp4a(dec[2 * s].n1, a.y, in);
                in = dp4a(dec[2 * s + 1].n0, a.z, in);
                in = dp4a(dec[2 * s + 1].n1, a.w, in);
                const float dsc = sc[s] * (s < 2 ? dd.x : dd.y);
                acc[t] += dsc * static_cast<float>(ip - in);
            }
        }
    }
}

// Activation of one 64-block for up to TT tokens, held in registers while
// the lane walks several weight rows (TT <= 2) -- one shared-memory read of
// the activation per block instead of one per row.
template <int TT>
struct ActBlk {
    int4 q[TT][4];
    float2 d[TT];
};

template <int TT>
__device__ __forceinline__ void act_load(ActBlk<TT> &a, const int4 *act_q, const float2 *act_d, int b, int NB, int nt) {
    const int swz = (b >> 1) & 3;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        if (t < nt) {
#pragma unroll
            for (int s = 0; s < 4; ++s) a.q[t][s] = act_q[(t * NB + b) * 4 + (s ^ swz)];
            a.d[t] = act_d[t * NB + b];
        }
    }
}

// dot of one 64-block (9 words at `blk`) with register-held activations
template <int TT>
__device__ __forceinline__ void gv_block_reg(const uint32_t *blk, const ActBlk<TT> &a, int nt, float (&acc)[TT]) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = blk[i];
    float sc[4];
    ue4m3x4(w[0], sc);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const nv_word d0 = nv_decode(w[1 + 2 * s]);
        const nv_word d1 = nv_decode(w[2 + 2 * s]);
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            if (t < nt) {
                const int4 q = a.q[t][s];
                int ip = dp4a(d0.p0, q.x, 0);
                ip = dp4a(d0.p1, q.y, ip);
                ip = dp4a(d1.p0, q.z, ip);
                ip = dp4a(d1.p1, q.w, ip);
                int in = dp4a(d0.n0, q.x, 0);
                in = dp4a(d0.n1, q.y, in);
                in = dp4a(d1.n0, q.z, in);
                in = dp4a(d1.n1, q.w, in);
                acc[t] += (sc[s] * (s < 2 ? a.d[t].x : a.d[t].y)) * static_cast<float>(ip - in);
            }
        }
    }
}

// The matvec.  A stage is SR = 8 warps x (32/LG) lane groups x R2 rows; all
// eight consumer warps work on every stage (warp w takes rows
// [(w*(32/LG) + g) * R2, +R2) with lane group g), so each ring slot is waited
// on by every warp in phase order and freed by eight arrivals.  Stages are
// 16-74 KB: large enough that one bulk copy per operand keeps HBM busy.
// One-row-group, one-token forms (small matvecs: the decode step's QKV / O,
// configs[0]) are compiled for two CTAs per SM, so the next launch's CTAs can
// start streaming their weights while this one's finish.
template <int LG, int TT, int EPI, int R2, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, (TT == 1 && R2 == 1) ? 2 : 1) k_gemv(const GvParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NS = p.n_slots;
    const int NB = p.K / NV_ELEMS;
    constexpr bool DUAL = EPI == GV_SWIGLU;
    constexpr int GPW = 32 / LG;                         // lane groups per warp
    constexpr int SR = CW * GPW * R2;             // rows per stage
    constexpr bool HOLD = TT <= 2;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + NS;
    uint8_t *ring = smem + 2048;
    int4 *act_q = reinterpret_cast<int4 *>(ring + static_cast<size_t>(NS) * p.slot_bytes);
    float2 *act_d = reinterpret_cast<float2 *>(act_q + static_cast<size_t>(p.nt) * NB * 4);

    const int r_begin = blockIdx.x * p.rows_per_cta;
    const int n_rows = min(p.N, r_begin + p.rows_per_cta) - r_begin;
    const int n_st = n_rows > 0 ? (n_rows + SR - 1) / SR : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], p.word_mode ? 32 : 1);
            mbar_init(&empty[s], CW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer: stream the CTA's weight rows, before the
        // PDL wait (weights do not depend on the previous kernel)
        const int64_t dual_off = static_cast<int64_t>(SR) * p.w_ld;
        // ring slot s and its use count as counters (no runtime division per stage)
        for (int i = 0, s = 0, use = 0; i < n_st; ++i, use += (++s == NS), s = (s == NS) ? 0 : s) {
            if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, 1)) break;
            const int rows = min(SR, n_rows - i * SR);
            const int64_t off = static_cast<int64_t>(r_begin + i * SR) * p.w_ld;
            uint8_t *dst = ring + static_cast<size_t>(s) * p.slot_bytes;
            if (p.word_mode) {
                const int nw = static_cast<int>(rows * p.w_ld / 4);
                uint32_t *d32 = reinterpret_cast<uint32_t *>(dst);
                const uint32_t *a0 = reinterpret_cast<const uint32_t *>(p.w0 + off);
                for (int k = lane; k < nw; k += 32) d32[k] = __ldg(a0 + k);
                if (DUAL) {
                    const uint32_t *a1 = reinterpret_cast<const uint32_t *>(p.w1 + off);
                    for (int k = lane; k < nw; k += 32) d32[dual_off / 4 + k] = __ldg(a1 + k);
                }
                mbar_arrive(&full[s]);
            } else if (lane == 0) {
                const uint32_t bytes = static_cast<uint32_t>(rows * p.w_ld);
                mbar_expect_tx(&full[s], DUAL ? 2 * bytes : bytes);
                bulk_g2s(dst, p.w0 + off, bytes, &full[s]);
                if (DUAL) bulk_g2s(dst + dual_off, p.w1 + off, bytes, &full[s]);
            }
        }
        return;
    }

    // ---------------- consumers
    fr_pdl_wait();
    gv_stage_act<CW>(p, act_q, act_d, warp, lane);
    named_bar(1, CW * 32);
    fr_pdl_trigger();

    const float sc0 = p.s0 ? *p.s0 : 1.0f;
    const float sc1 = (DUAL && p.s1) ? *p.s1 : 1.0f;
    const int64_t peer_off = p.peer_off + (p.epoch ? static_cast<int64_t>(*p.epoch & 1u) * p.par_bytes : 0);
    const int g = lane / LG, j = lane % LG;
    const int rg0 = (warp * GPW + g) * R2;              // first stage row of this lane group

    for (int i = 0, s = 0, use = 0; i < n_st; ++i, use += (++s == NS), s = (s == NS) ? 0 : s) {
        if (!mbar_wait(&full[s], use & 1, 2)) break;
        const int rows = min(SR, n_rows - i * SR);
        const uint8_t *st = ring + static_cast<size_t>(s) * p.slot_bytes;
        float acc0[R2][TT], acc1[R2][TT];
#pragma unroll
        for (int r = 0; r < R2; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t) { acc0[r][t] = 0.0f; acc1[r][t] = 0.0f; }
        if (rg0 < rows) {
#pragma unroll 2
            for (int b = j; b < NB; b += LG) {
                if constexpr (HOLD) {
                    ActBlk<TT> a;
                    act_load<TT>(a, act_q, act_d, b, NB, p.nt);
#pragma unroll
                    for (int r = 0; r < R2; ++r) {
                        if (rg0 + r < rows) {
                            const uint8_t *row = st + static_cast<size_t>(rg0 + r) * p.w_ld + b * NV_BYTES;
                            gv_block_reg<TT>(reinterpret_cast<const uint32_t *>(row), a, p.nt, acc0[r]);
                            if (DUAL)
                                gv_block_reg<TT>(reinterpret_cast<const uint32_t *>(row + SR * p.w_ld), a, p.nt, acc1[r]);
                        }
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < R2; ++r) {
                        if (rg0 + r < rows) {
                            const uint8_t *row = st + static_cast<size_t>(rg0 + r) * p.w_ld + b * NV_BYTES;
                            gv_block<TT>(reinterpret_cast<const uint32_t *>(row), b, NB, p.nt, act_q, act_d, acc0[r]);
                            if (DUAL)
                                gv_block<TT>(reinterpret_cast<const uint32_t *>(row + SR * p.w_ld), b, NB, p.nt, act_q,
                                             act_d, acc1[r]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int r = 0; r < R2; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t) {
#pragma unroll
                for (int off = LG / 2; off > 0; off >>= 1) {
                    acc0[r][t] += __shfl_xor_sync(0xffffffffu, acc0[r][t], off);
                    if (DUAL) acc1[r][t] += __shfl_xor_sync(0xffffffffu, acc1[r][t], off);
                }
            }
        if (j == 0) {
#pragma unroll
            for (int r = 0; r < R2; ++r) {
                if (rg0 + r < rows) {
                    const int row = r_begin + i * SR + rg0 + r;
#pragma unroll
                    for (int t = 0; t < TT; ++t) {
                        if (t < p.nt) {
                            const int64_t tt = p.t0 + t;
                            float v;
                            if (DUAL) {
                                // fused mmvq epilogue: x = up, gate = gate, SwiGLU
                                float result = acc1[r][t];
                                result *= sc1;
                                float gate = acc0[r][t];
                                gate *= sc0;
                                result *= silu_f(gate);
                                v = result;
                            } else {
                                v = acc0[r][t] * sc0;
                                if (p.resid) v += p.resid[tt * p.ldr + row];
                            }
                            if (p.npeers > 0) {
                                for (int q = 0; q < p.npeers; ++q) {
                                    float *py = reinterpret_cast<float *>(p.peer_base[q] + peer_off);
                                    py[tt * p.ldy + p.col_off + row] = v;
                                }
                            } else {
                                p.y[tt * p.ldy + row] = v;
                            }
                        }
                    }
                }
            }
        }
    }
    if (p.npeers > 0) {
        // publish this CTA's rows to every rank: the consumer warps meet (the
        // barrier orders their stores before thread 0's), then one system-scope
        // fence and one flag increment per peer
        named_bar(2, CW * 32);
        if (warp == 0 && lane == 0) {
            __threadfence_system();
            for (int q = 0; q < p.npeers; ++q) {
                unsigned int *fl = reinterpret_cast<unsigned int *>(p.peer_base[q] + p.flag_off);
                atomicAdd_system(fl + p.rank, 1u);
            }
        }
    }
}

// Tensor-parallel push: copy this rank's [T, cols] block (row stride ld) from
// its local staging area (byte offset src_off of its own buffer) into its slot
// of every rank's buffer, this rank's included (byte offset dst_off, plus
// par_bytes when the step parity epoch[0] is odd), then count the CTA into
// every rank's flag[rank] (same publication protocol as the matvec epilogue).
__global__ void __launch_bounds__(256) k_tp_push(uint8_t *const *peer_base, int npeers, int rank, int64_t src_off,
                                                 int64_t dst_off, int64_t par_bytes, const unsigned int *epoch,
                                                 int64_t ld, int T, int cols, int64_t flag_off) {
    fr_pdl_wait();
    const float *src = reinterpret_cast<const float *>(peer_base[rank] + src_off);
    const int64_t off = dst_off + static_cast<int64_t>(*epoch & 1u) * par_bytes;
    const int64_t n = static_cast<int64_t>(T) * cols;
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t lo = blockIdx.x * per, hi = min(n, lo + per);
    for (int q = 0; q < npeers; ++q) {
        float *dst = reinterpret_cast<float *>(peer_base[q] + off);
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const int64_t t = i / cols, c = i % cols;
            dst[t * ld + c] = src[t * ld + c];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < npeers; ++q)
            atomicAdd_system(reinterpret_cast<unsigned int *>(peer_base[q] + flag_off) + rank, 1u);
    }
    fr_pdl_trigger();
}

// Row-sharded tensor parallelism: quantize this rank's GLU columns [T, cols]
// (f32, row stride ldg) to q8_1 and store the blocks into every rank's copy
// of the full q8_1 GLU (at byte offset dst_off + (epoch[0] & 1) * par_bytes,
// rows ldq blocks apart, this rank's blocks from block col0 / 32 on), then
// count the CTA into every rank's flag[rank] at flag_off.  q8_1 blocks are
// local to 32 values and shard boundaries are multiples of 64, so the blocks
// are the ones one GPU quantizing the whole GLU makes.  One warp per block.
__global__ void __launch_bounds__(256) k_q8_push(const float *__restrict__ glu, int64_t ldg, int T, int cols,
                                                 int col0, uint8_t *const *peer_base, int npeers, int rank,
                                                 int64_t dst_off, int64_t par_bytes, const unsigned int *epoch,
                                                 int64_t ldq, int64_t flag_off) {
    fr_pdl_wait();
    const int lane = threadIdx.x & 31;
    const int nc = cols / Q8_ELEMS;
    const int64_t off = dst_off + static_cast<int64_t>(*epoch & 1u) * par_bytes;
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5); c < static_cast<int64_t>(T) * nc;
         c += static_cast<int64_t>(gridDim.x) * 8) {
        const int t = static_cast<int>(c / nc), ch = static_cast<int>(c % nc);
        const q8_lane r = q8_1_chunk(glu[t * ldg + static_cast<int64_t>(ch) * Q8_ELEMS + lane]);
        const __half2 ds = __halves2half2(__float2half_rn(r.d), __float2half_rn(r.sum));
        const int64_t boff = off + (t * ldq + col0 / Q8_ELEMS + ch) * Q8_BYTES;
        for (int q = 0; q < npeers; ++q) {
            uint8_t *blk = peer_base[q] + boff;
            blk[4 + lane] = static_cast<uint8_t>(r.q);
            if (lane == 0) *reinterpret_cast<__half2 *>(blk) = ds;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < npeers; ++q)
            atomicAdd_system(reinterpret_cast<unsigned int *>(peer_base[q] + flag_off) + rank, 1u);
    }
    fr_pdl_trigger();
}

// Tensor-parallel completion wait and reduction: in every CTA, lane r waits
// until rank r's flag counter reached this CTA's consumed count plus `expect`
// (the producer kernels' CTA count) and records the new count in the CTA's
// own row of `seen` (seen[blockIdx.x * 32 + r]; counters only grow, so
// CUDA-graph replays need no reset).  Then the CTA sums its slice of the
// ranks' partial outputs in rank order (identical on every rank), adds the
// residual and writes `out` (nsum slots are summed: nranks for the partial
// sums of the n_ff-sharded form, 1 for an output the ranks assembled by
// columns).  The wait is bounded (status bit 0, site 30).
//
// Step parity (epoch non-null): the partial outputs are double-buffered.
// epoch[blockIdx.x] counts this CTA's completed steps; a step reads the half
// `parts + (epoch & 1) * par_floats` and then advances the count.  The
// producers of the next step read epoch[0] to pick the other half, so a fast
// rank's next partials never land in the half a slower rank is still summing:
// a rank can only be one step ahead, because its step s+1 needs every rank's
// step-s+1 partials, which each rank produces only after its own step-s
// reduce completed.  (epoch null: a single buffer, wait only.)
//
// The kernel releases its dependents at once, then waits for its predecessor
// in the stream to complete: the consumed counts and the step count it reads
// are the previous step's final values, whatever the depth of the launch
// chain ahead of it.
__global__ void __launch_bounds__(256) k_tp_reduce(const unsigned int *flags, unsigned int *seen, int nranks,
                                                   unsigned int expect, const float *parts, int64_t n,
                                                   const float *resid, int64_t ldr, int64_t width, float *out,
                                                   int64_t ldo, unsigned int *epoch, int64_t par_floats, int nsum) {
    fr_pdl_trigger();
    fr_pdl_wait();
    const unsigned int e = epoch ? epoch[blockIdx.x] : 0u;
    if (threadIdx.x < static_cast<unsigned>(nranks))
        tp_flag_wait(flags, seen + blockIdx.x * 32 + threadIdx.x, threadIdx.x, expect);
    __syncthreads();
    parts += static_cast<int64_t>(e & 1u) * par_floats;
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t lo = blockIdx.x * per, hi = min(n, lo + per);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float v = parts[i];
        for (int r = 1; r < nsum; ++r) v += parts[r * n + i];
        const int64_t t = i / width, c = i % width;
        if (resid) v += resid[t * ldr + c];
        out[t * ldo + c] = v;
    }
    if (epoch) {
        __syncthreads();
        if (threadIdx.x == 0) epoch[blockIdx.x] = e + 1u;
    }
}

} // namespace frb
