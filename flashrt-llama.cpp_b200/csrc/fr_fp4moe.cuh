// fr_fp4moe.cuh -- the MoE expert matvecs (the per-expert GEMV/GEMM of
// mul_mat_id, src/fr_win_flint_batched_moe.cuh:180-340 in the reference) on
// the FP4 tensor cores, with every expert's matrix in the tile-major NVFP4
// layout of fr_fp4tile.cuh (the stacked [E * N, K] matrix repacked at once:
// expert e's tiles start at e * e_stride).
//
// Work.  The routing's grouping (eoff / slots / act) lists each active
// expert's slots in slot order.  They are cut into windows of at most TMAX
// tokens (8 * TMAX = NCOL activation columns, the MMA's N); a unit is
// (window, row block of 128, K stage of 256), and the units are divided evenly
// over the CTAs in that order (stream-K, as k_fp4t), so every row block of
// every used expert is streamed from HBM once per window -- once per call
// unless more than TMAX tokens chose the expert.  The windows are counted on
// the device from the grouping, so the launch needs no host sync and can be
// captured in a CUDA graph.
//
// Activation.  k_act_fp4 writes one image per source row (a token for the
// gate/up pair, a slot for the down projection): per K stage one 1024-byte
// 128-byte-swizzled atom of its eight E2M1 digit columns.  The activation
// producer gathers the window's atoms into the stage buffer (token i at rows
// [8i, 8i+8)); rows past the window keep stale bytes, which are valid E2M1
// codes and only reach accumulator columns that are never read.
//
// Epilogue.  Column factors (9^p 2^(E0+1), per source row) and output rows are
// staged per window in each epilogue warp's own shared-memory copy (no barrier
// between warps inside the loop, so a warp whose wait timed out holds no one).
// SwiGLU with per-expert scales writes the GLU row of each slot; the plain
// form writes each slot's projected row.  Row blocks shared by several CTAs
// are finished by the last to arrive, adding the partials in CTA order.
#pragma once

#include "fr_fp4tile.cuh"

namespace frb {

constexpr int FE_MAX_E = 256;                  // experts (one scan entry per thread)
constexpr int FE_TAB = 32;                     // windows of one CTA kept in its shared-memory table

struct FeArgs {
    int N, K;                    // rows per expert, row length
    int n_kq, n_rb;              // K stages of 256, row blocks of 128 per expert
    int E, n_used, bcast;        // source row of slot s: bcast ? s / n_used : s
    const int32_t *eoff, *slots, *act;
    const uint8_t *w0, *w1;      // tiled expert matrices; w1 = up for the SwiGLU pair
    int64_t e_stride;            // bytes per expert
    const uint8_t *img;          // per source row: n_kq atoms of 1024 B (k_act_fp4, t_stride = n_kq * 1024)
    const float *gtab;           // per source row: 8 column factors
    const float *s0, *s1;        // per-expert scales [E] (nullable)
    float *y;                    // output row of slot s = t * n_used + k at y + t * ld_tok + k * ld_slot
    int64_t ld_tok, ld_slot;
    float *part;                 // [grid][2: first / last segment][2: matrix][TMAX][128]
    unsigned int *counter;       // [max_rbg][4 quadrants], zero on entry, reset by the last arrival
    int max_rbg;                 // window row blocks the counters cover
    int n_w, n_b;                // ring depth (stages of weights + activation atoms); n_b = n_w
};

// Issue groups.  Each tcgen05 step of an issuing thread (barrier wait, scale
// copy, MMA, commit) costs it ~0.1-0.2 us, so one thread issuing a whole
// 18 KB tile (two waits, four scale copies, four MMAs, two commits) moves
// only ~15 GB/s.  Stages therefore alternate between P issue groups (one
// thread per matrix in each; group p takes the stages i with i % P == p), each
// with its own TMEM accumulators, which the epilogue adds.  The ring depth is
// a multiple of P, so a group owns its ring slots and waits on every phase of
// them in order (a parity wait that skipped a phase could pass on a later
// one).  Where TMEM allows, the accumulators are double-buffered across
// row-block segments (D = 2), so the MMAs of a segment need not wait for the
// epilogue to drain the previous one.  Weights and activation atoms of a stage
// share one full / empty barrier pair (one wait and one commit per stage).
template <int NCOL, int EPI>
struct FeShape {
    static constexpr int NM = EPI == FM_SWIGLU ? 2 : 1;           // matrices per stage
    static constexpr int P = 2 * NM * NCOL <= 256 ? 2 : 1;        // issue groups
    static constexpr int D = 2 * P * NM * NCOL <= 256 ? 2 : 1;    // accumulator sets (segments in flight)
    static constexpr int NISS = P * NM;                           // issuer threads
    // weight producer, issuers (warps 1, 2, then 8, 9), epilogue 3..6, activation producer 7
    static constexpr int THREADS = 32 * (8 + (NISS > 2 ? NISS - 2 : 0));
};

// shared-memory bytes past the two rings
__host__ __device__ constexpr int fe_extra_bytes() {
    return 512 + 4 * (16 * FM_GSTRIDE * 4) + 4 * 16 * 8 + (FE_MAX_E + 1) * 4 + 64 +
           FE_TAB * (3 + 16) * 4 + 32 * 4 + 64 * 8 + 16;
}

template <int NCOL, int EPI>
__global__ void __launch_bounds__(FeShape<NCOL, EPI>::THREADS, 1) k_fp4e(const FeArgs g) {
    using S = FtShape<NCOL, EPI, 1>;
    using H = FeShape<NCOL, EPI>;
    constexpr int NM = H::NM, P = H::P, D = H::D, NISS = H::NISS;
    constexpr bool DUAL = NM == 2;
    constexpr int TMAX = S::TMAX;
    constexpr uint32_t TMEM_COLS = 512;
    static_assert(D * NISS * NCOL <= 256, "accumulators live in TMEM columns [0, 256)");
    static_assert(TMAX <= 16, "window factor tables hold 16 tokens");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NW = g.n_w;                                   // stages in the ring (weights + activations)
    uint8_t *w_ring = smem;
    uint8_t *b_ring = w_ring + static_cast<size_t>(NW) * S::WST;
    uint8_t *sfb_const = b_ring + static_cast<size_t>(NW) * S::BST;      // 512 B
    float *gtab_w = reinterpret_cast<float *>(sfb_const + 512);            // [4 warps][16 * 8]
    int64_t *orow_w = reinterpret_cast<int64_t *>(gtab_w + 4 * 16 * FM_GSTRIDE); // [4 warps][16]
    int *win_off = reinterpret_cast<int *>(orow_w + 4 * 16);                       // [FE_MAX_E + 1]
    int *wsum = win_off + FE_MAX_E + 1;                                    // [8] warp sums of the scan
    int *tab_e = wsum + 16;                                                // this CTA's windows: expert,
    int *tab_sb = tab_e + FE_TAB;                                          //   first slot,
    int *tab_nt = tab_sb + FE_TAB;                                         //   tokens,
    int *tab_row = tab_nt + FE_TAB;                                        //   source rows [FE_TAB][16]
    int *stage_n = tab_row + FE_TAB * 16;                                  // MMA N of each activation stage
    uint64_t *full = reinterpret_cast<uint64_t *>(
        (reinterpret_cast<uintptr_t>(stage_n + 32) + 7) & ~uintptr_t(7));
    uint64_t *empty = full + NW;
    uint64_t *accfull = empty + NW;                          // [D]
    uint64_t *accempty = accfull + D;                        // [D]
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(accempty + D);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NW; ++s) {
            mbar_init(&full[s], 2);                          // weight and activation producers
            mbar_init(&empty[s], NM);                        // the owning group's issuers
        }
        for (int d = 0; d < D; ++d) {
            mbar_init(&accfull[d], NISS);                    // every issuer, once per segment
            mbar_init(&accempty[d], 4);                      // the four epilogue warps
        }
        fence_mbar_init();
    }
    if (warp == 3) {
        reinterpret_cast<uint4 *>(sfb_const)[lane] = make_uint4(FM_SFB * 0x01010101u, FM_SFB * 0x01010101u,
                                                                FM_SFB * 0x01010101u, FM_SFB * 0x01010101u);
        fence_proxy_async();
    }
    if (warp == 1) tmem_alloc(tmem_s, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    const uint32_t tD = tbase;
    fr_pdl_trigger();
    fr_pdl_wait();                                           // the grouping and the activation images

    // windows per active expert -> exclusive prefix win_off, one entry per
    // thread of the first FE_MAX_E (the block may have more threads)
    const int n_act = min(max(g.act[g.E], 0), g.E);
    {
        const int i = threadIdx.x;
        int nw = 0;
        if (i < n_act) {
            const int e = g.act[i];
            if (e >= 0 && e < g.E) nw = (g.eoff[e + 1] - g.eoff[e] + TMAX - 1) / TMAX;
        }
        int inc = nw;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += v;
        }
        if (i < FE_MAX_E && lane == 31) wsum[warp] = inc;
        __syncthreads();
        if (i < FE_MAX_E) {
            int base = 0;
            for (int w = 0; w < warp; ++w) base += wsum[w];
            win_off[i + 1] = base + inc;
            if (i == 0) win_off[0] = 0;
        }
        __syncthreads();
    }
    const int W = win_off[n_act];
    const int nsr = g.n_kq;
    int U = W * g.n_rb * nsr;
    if (W * g.n_rb > g.max_rbg) {
        if (threadIdx.x == 0) fr_flag(FR_ST_BADINPUT);
        U = 0;
    }
    const int G = min(static_cast<int>(gridDim.x), U);
    const bool active = static_cast<int>(blockIdx.x) < G;
    const int u_lo = active ? ft_lo(blockIdx.x, U, G) : 0;
    const int u_hi = active ? ft_lo(blockIdx.x + 1, U, G) : 0;
    const int n_st = u_hi - u_lo;

    // window w -> expert e, first slot sb, tokens nt (from the grouping)
    auto window = [&](int w, int &e, int &sb, int &nt) {
        int lo = 0, hi = n_act;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (win_off[mid] <= w) lo = mid; else hi = mid;
        }
        e = g.act[lo];
        if (e < 0 || e >= g.E) {                             // never from a valid grouping
            fr_flag(FR_ST_BADINPUT);
            e = 0;
            sb = 0;
            nt = 0;
            return;
        }
        sb = g.eoff[e] + (w - win_off[lo]) * TMAX;
        nt = max(0, min(TMAX, g.eoff[e + 1] - sb));
    };
    // The windows this CTA touches, with their source rows, looked up once
    // here (two rounds of loads for the whole CTA) so that no role waits on a
    // global load inside its loop.  A CTA spanning more than FE_TAB windows
    // looks the rest up as it reaches them.
    const int wpu = g.n_rb * nsr;                            // units per window
    const int w_first = n_st > 0 ? u_lo / wpu : 0;
    const int n_tab = n_st > 0 ? min(FE_TAB, (u_hi - 1) / wpu - w_first + 1) : 0;
    if (static_cast<int>(threadIdx.x) < n_tab) {
        int e, sb, nt;
        window(w_first + threadIdx.x, e, sb, nt);
        tab_e[threadIdx.x] = e;
        tab_sb[threadIdx.x] = sb;
        tab_nt[threadIdx.x] = nt;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < n_tab * 16; idx += blockDim.x) {
        const int j = idx >> 4, t = idx & 15;
        if (t < tab_nt[j]) {
            const int sl = g.slots[tab_sb[j] + t];
            tab_row[idx] = g.bcast ? sl / g.n_used : sl;
        }
    }
    __syncthreads();
    auto win_at = [&](int w, int &e, int &sb, int &nt) {
        const int j = w - w_first;
        if (j < n_tab) {
            e = tab_e[j];
            sb = tab_sb[j];
            nt = tab_nt[j];
        } else {
            window(w, e, sb, nt);
        }
    };
    auto row_at = [&](int w, int sb, int t) -> int {
        const int j = w - w_first;
        if (j < n_tab) return tab_row[j * 16 + t];
        const int sl = g.slots[sb + t];
        return g.bcast ? sl / g.n_used : sl;
    };
    const int64_t img_row = static_cast<int64_t>(g.n_kq) * 1024;

    if (warp == 0) {
        // ---------------- weight producer
        if (lane == 0) {
            int cur_w = -1, e = 0, sb = 0, nt = 0;
            // unit u = (window u / wpu, row block (u % wpu) / nsr, K stage
            // u % nsr), ring slot s and its use count, all as counters: a
            // runtime division per stage is a dependent chain this lone
            // thread pays
            int w = u_lo / wpu, rb = (u_lo % wpu) / nsr, kq = u_lo % nsr, s = 0, use = 0;
            for (int i = 0; i < n_st; ++i) {
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, 60)) break;
                if (w != cur_w) {
                    win_at(w, e, sb, nt);
                    cur_w = w;
                }
                const int64_t off = static_cast<int64_t>(e) * g.e_stride +
                                    (static_cast<int64_t>(rb) * g.n_kq + kq) * FT_TILE;
                uint8_t *st = w_ring + static_cast<size_t>(s) * S::WST;
                mbar_expect_tx(&full[s], S::WST);
                bulk_g2s(st, g.w0 + off, FT_TILE, &full[s]);
                if (DUAL) bulk_g2s(st + FT_TILE, g.w1 + off, FT_TILE, &full[s]);
                if (++s == NW) {
                    s = 0;
                    ++use;
                }
                if (++kq == nsr) {
                    kq = 0;
                    if (++rb == g.n_rb) {
                        rb = 0;
                        ++w;
                    }
                }
            }
        }
    } else if (warp == 7) {
        // ---------------- activation producer: lane t copies token t's atom
        // of the stage; the stage records the MMA width its tokens need
        int cur_w = -1, nt = 0, ncol = 16;
        const uint8_t *src = g.img;
        int w = u_lo / wpu, rb = (u_lo % wpu) / nsr, kq = u_lo % nsr, s = 0, use = 0;
        for (int i = 0; i < n_st; ++i) {
            if (w != cur_w) {
                int e, sb;
                win_at(w, e, sb, nt);
                if (lane < nt) src = g.img + static_cast<int64_t>(row_at(w, sb, lane)) * img_row;
                const int need = nt * FM_DIGITS;
                ncol = need <= 16 ? 16 : need <= 32 ? 32 : need <= 64 ? 64 : 128;
                cur_w = w;
            }
            bool ok = true;
            if (lane == 0 && use > 0) ok = mbar_wait(&empty[s], (use - 1) & 1, 61);
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            uint8_t *st = b_ring + static_cast<size_t>(s) * S::BST;
            if (lane == 0) {
                stage_n[s] = min(ncol, NCOL);
                mbar_expect_tx(&full[s], static_cast<uint32_t>(nt) * 1024u);
            }
            __syncwarp();
            if (lane < nt) bulk_g2s(st + lane * 1024, src + kq * 1024, 1024, &full[s]);
            if (++s == NW) {
                s = 0;
                ++use;
            }
            if (++kq == nsr) {
                kq = 0;
                if (++rb == g.n_rb) {
                    rb = 0;
                    ++w;
                }
            }
        }
    } else if (warp == 1 || warp == 2 || warp >= 8) {
        // ---------------- MMA issuers: thread (group p, matrix m) issues the
        // stages i with i % P == p into accumulator (set seg % D, p, m)
        const int ii = warp <= 2 ? warp - 1 : warp - 6;
        if (lane == 0 && ii < NISS) {
            const int p = ii / NM, m = ii % NM;
            const uint32_t t_sfb = tbase + 256 + NW * 16 * NM + 4 * ii;
            tc_cp_sf(t_sfb, sdesc_plain(smem_u32(sfb_const), 128));
            int seg = 0;
            bool started = false;
            // K stage within the row block, ring slot and its use count as
            // counters (no runtime division on this thread's critical path)
            int kq = u_lo % nsr, sw = 0, use = 0;
            for (int i = 0; i < n_st; ++i) {
                const bool first = i == 0 || kq == 0;
                const bool last = i == n_st - 1 || kq == nsr - 1;
                const int d = seg % D;
                if (first) {
                    started = false;
                    // every issuer waits for each drain of its set, in order
                    if (seg >= D && !mbar_wait(&accempty[d], ((seg / D) - 1) & 1, 62)) break;
                }
                if (i % P == p) {
                    if (!mbar_wait(&full[sw], use & 1, 63)) break;
                    tc_fence_after();
                    const uint32_t idesc = idesc_nvf4(128, stage_n[sw]);
                    const uint32_t a_addr = smem_u32(w_ring + static_cast<size_t>(sw) * S::WST) + m * FT_TILE;
                    const uint32_t b_addr = smem_u32(b_ring + static_cast<size_t>(sw) * S::BST);
                    const uint32_t t_sfa = tbase + 256 + (sw * NM + m) * 16;
                    const uint32_t t_acc = tD + ((d * P + p) * NM + m) * NCOL;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc_cp_sf(t_sfa + 4 * j, sdesc_plain(a_addr + FT_CODES + 512 * j, 128));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc_mma_nvf4(t_acc, sdesc_sw128(a_addr + 32 * j), sdesc_sw128(b_addr + 32 * j), idesc,
                                    t_sfa + 4 * j, t_sfb, (started || j > 0) ? 1u : 0u);
                    tc_commit(&empty[sw]);
                    started = true;
                }
                if (last) {
                    tc_commit(&accfull[d]);
                    ++seg;
                }
                if (++kq == nsr) kq = 0;
                if (++sw == NW) {
                    sw = 0;
                    ++use;
                }
            }
        }
    } else if (warp >= 3 && warp <= 6) {
        // ---------------- epilogue warps (3..6), one TMEM lane quadrant each
        const int q = warp & 3;
        const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
        const int erow = 32 * q + lane;
        float *gt = gtab_w + q * 16 * FM_GSTRIDE;
        int64_t *orow = orow_w + q * 16;
        float *part_cta = g.part + static_cast<int64_t>(blockIdx.x) * 2 * 2 * TMAX * 128;
        int seg = 0;
        int cur_w = -1, e = 0, sb = 0, nt = 0;
        float sc0 = 1.0f, sc1 = 1.0f;
        // row-block group rbg (window w, row block rb) of each segment kept as
        // counters: one segment per row block, in order
        int rbg = u_lo / nsr, w = rbg / g.n_rb, rb = rbg % g.n_rb;
        for (int s0u = u_lo; s0u < u_hi; ++seg, ++rbg, (++rb == g.n_rb) ? (rb = 0, ++w) : 0) {
            const int s1u = min(u_hi, (rbg + 1) * nsr);
            if (w != cur_w) {
                // this warp's copy of the window's factors, output rows and
                // scales, loaded once per window (its row blocks follow)
                win_at(w, e, sb, nt);
                __syncwarp();
#pragma unroll
                for (int c = lane; c < TMAX * FM_GSTRIDE; c += 32) {
                    const int t = c / FM_GSTRIDE;
                    float v = 0.0f;
                    if (t < nt) v = g.gtab[static_cast<int64_t>(row_at(w, sb, t)) * FM_GSTRIDE + (c % FM_GSTRIDE)];
                    gt[c] = v;
                }
                if (lane < TMAX) {
                    const int slot = lane < nt ? g.slots[sb + lane] : 0;
                    orow[lane] = static_cast<int64_t>(slot / g.n_used) * g.ld_tok +
                                 static_cast<int64_t>(slot % g.n_used) * g.ld_slot;
                }
                __syncwarp();
                sc0 = g.s0 ? g.s0[e] : 1.0f;
                sc1 = (DUAL && g.s1) ? g.s1[e] : 1.0f;
                cur_w = w;
            }
            auto finish = [&](int t, float a0, float a1) {
                const int n = rb * 128 + erow;
                if (n >= g.N || t >= nt) return;
                float val;
                if (DUAL) {
                    float result = a1;
                    result *= sc1;
                    float gate = a0;
                    gate *= sc0;
                    result *= silu_f(gate);
                    val = result;
                } else {
                    val = a0 * sc0;
                }
                g.y[orow[t] + n] = val;
            };

            const int d = seg % D;                           // this segment's accumulator set
            if (!mbar_wait(&accfull[d], (seg / D) & 1, 65)) break;
            tc_fence_after();
            float acc0[TMAX], acc1[TMAX];
#pragma unroll
            for (int t = 0; t < TMAX; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }
            const int ncol_used = nt * FM_DIGITS;
            // groups that issued a stage of this segment
            const int i0 = s0u - u_lo, n_seg = s1u - s0u;
#pragma unroll
            for (int p = 0; p < P; ++p) {
                if (n_seg < P && (i0 + n_seg - 1) % P != p && i0 % P != p) continue;
                const uint32_t t_acc = tD + ((d * P + p) * NM) * NCOL + lane_off;
#pragma unroll
                for (int c = 0; c < NCOL; c += 16) {
                    if (c >= ncol_used) break;
                    uint32_t d0[16], d1[16];
                    tmem_ld16(t_acc + c, d0);
                    if (DUAL) tmem_ld16(t_acc + NCOL + c, d1);
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const int col = c + v, t = col / FM_DIGITS;
                        const float gf = gt[col];
                        acc0[t] = fmaf(gf, __uint_as_float(d0[v]), acc0[t]);
                        if (DUAL) acc1[t] = fmaf(gf, __uint_as_float(d1[v]), acc1[t]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[d]);
            if (s0u == rbg * nsr && s1u == (rbg + 1) * nsr) {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) finish(t, acc0[t], acc1[t]);
            } else {
                const int c_first = ft_owner(rbg * nsr, U, G);
                const int c_last = ft_owner((rbg + 1) * nsr - 1, U, G);
                const int which = s0u == u_lo ? 0 : 1;
                float *pp = part_cta + which * 2 * TMAX * 128;
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    if (t < nt) {
                        pp[t * 128 + erow] = acc0[t];
                        if (DUAL) pp[TMAX * 128 + t * 128 + erow] = acc1[t];
                    }
                }
                fence_acq_rel_gpu();
                __syncwarp();
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&g.counter[rbg * 4 + q], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == static_cast<unsigned>(c_last - c_first)) {
                    fence_acq_rel_gpu();
                    float s0[TMAX], s1[TMAX];
                    ft_sum_parts<TMAX, DUAL>(
                        [&](int k2) {
                            const int c = c_first + k2;
                            const int wc = (ft_lo(c, U, G) / nsr == rbg) ? 0 : 1;
                            return g.part + (static_cast<int64_t>(c) * 2 + wc) * 2 * TMAX * 128;
                        },
                        c_last - c_first + 1, nt, erow, s0, s1);
#pragma unroll
                    for (int t = 0; t < TMAX; ++t) finish(t, s0[t], s1[t]);
                    if (lane == 0) g.counter[rbg * 4 + q] = 0;
                }
            }
            s0u = s1u;
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
