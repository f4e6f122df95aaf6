// fr_fp4tile.cuh -- the FP4 tensor-core matvec on tile-major weights.
//
// Tile-major NVFP4 ("tiled") layout.  A one-time repack (k_tile_nvfp4, in the
// spirit of the reference's load-time repack_weight for its tensor-core path,
// src/fr_repack.cu:1-13) rewrites a ggml block_nvfp4 matrix [N, K] as tiles
// of 128 rows x 256 values, tile (rb, kq) at ((rb * n_kq) + kq) * 18432 bytes:
//   * 16384 B of codes, 128-byte-swizzled K-major: row r at r * 128, its
//     16-byte unit c (block c >> 1 of the tile, half c & 1 of that block's 32
//     code bytes) at ((c ^ (r & 7)) << 4); bytes keep ggml's order (byte j of
//     a sub-block = values j, j+8), which the activation columns share;
//   * 2048 B of scale atoms, block j of the tile at 16384 + 512 j, row r's
//     four sub-block scales at (r & 31) * 16 + (r >> 5) * 4, with ggml's
//     reading applied (sign bit dropped, 0x7F -> 0).
// Rows past N and blocks past K are zero.  The byte count equals ggml's when
// N % 128 == 0 and K % 256 == 0.
//
// Because a tile is one contiguous 18 KB block and a row block's tiles follow
// each other along K, every CTA streams one contiguous byte range per matrix
// with 1-D bulk copies that land MMA-ready in shared memory: no per-value
// work on the SMs at all.  Work split: stream-K -- the (row block, K stage)
// units are divided evenly over the CTAs in row-block-major order; a CTA
// finishes each row block it touches; when several CTAs share a row block,
// each writes its partial sums and the last to arrive adds them in CTA order
// (deterministic) and applies the epilogue.  Arithmetic: as k_fp4mv (exact
// products, fp32 accumulation, activation as six E2M1 digit columns).
#pragma once

#include "fr_fp4mv.cuh"

namespace frb {

constexpr int FT_TILE = 18432;                 // bytes per 128 x 256 tile
constexpr int FT_CODES = 16384;

// ------------------------------------------------------------ repack
// one thread per (row, 64-block) of the padded matrix
__global__ void __launch_bounds__(256) k_tile_nvfp4(const uint8_t *__restrict__ src, int64_t w_ld, int N, int K,
                                                    int n_kq, uint8_t *__restrict__ dst, int64_t total) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= total) return;
    const int nkb_p = n_kq * 4;                          // padded blocks per row
    const int64_t row = id / nkb_p;
    const int kb = static_cast<int>(id % nkb_p);
    uint32_t w[9];
    if (row < N && kb < K / 64) {
        const uint8_t *b = src + row * w_ld + static_cast<int64_t>(kb) * NV_BYTES;
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = *reinterpret_cast<const uint32_t *>(b + 4 * i);
    } else {
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = 0u;
    }
    uint32_t sv = w[0] & 0x7F7F7F7Fu;
    const uint32_t nan = (sv + 0x01010101u) & 0x80808080u;
    sv &= ~((nan >> 7) * 0xFFu);
    const int64_t rb = row >> 7;
    const int r = static_cast<int>(row & 127);
    const int kq = kb >> 2, j = kb & 3;
    uint8_t *tile = dst + (rb * n_kq + kq) * FT_TILE;
    uint8_t *a = tile + r * 128;
    const int sw = r & 7;
    *reinterpret_cast<uint4 *>(a + (((2 * j) ^ sw) << 4)) = make_uint4(w[1], w[2], w[3], w[4]);
    *reinterpret_cast<uint4 *>(a + (((2 * j + 1) ^ sw) << 4)) = make_uint4(w[5], w[6], w[7], w[8]);
    *reinterpret_cast<uint32_t *>(tile + FT_CODES + j * 512 + (r & 31) * 16 + (r >> 5) * 4) = sv;
}

// ------------------------------------------------------------ matvec
struct FtArgs {
    int N, K, T;                 // rows, row length, tokens in this launch (8T <= NCOL)
    int t0;                      // first output token index
    int n_kq;                    // K stages of 256 (tiles per row block)
    int n_units;                 // row blocks x (n_kq / NT)
    int maxp;                    // partial slots per row block
    const uint8_t *w0, *w1;      // tiled matrices
    const uint8_t *bimg;         // activation columns (k_act_fp4) [n_kq][NCOL x 128 B]
    const float *gtab;           // column factors (k_act_fp4) [T][8]
    const float *s0, *s1;        // per-tensor scales (nullable)
    const float *resid;          // [.., ldr] (nullable)
    int64_t ldr;
    float *y;                    // [.., ldy]
    int64_t ldy;
    float *part;                 // partials [row blocks][maxp][2][TMAX][128]
    float *amax_out;             // nullable: max |y| of each token's 32-row groups, [t][amax_ld]
    // tensor-parallel output (plain form; peer_base null otherwise): every
    // finished row is stored into this rank's slot of every rank's buffer
    // (peer_base[q] + peer_off, row stride ldy), and each CTA counts itself
    // into every rank's flag[rank] (at flag_off) when it ends
    uint8_t *const *peer_base;
    int npeers, rank;
    int64_t peer_off, flag_off;
    const unsigned int *epoch;   // step parity of the receiving slots (as GvParams::epoch)
    int64_t par_bytes;
    unsigned int *counter;       // [row blocks][4 quadrants], zero on entry, reset by the last arrival
    int n_w, n_b;                // ring depth (stages of weights + activation columns); n_b = n_w
    int amax_ld;
};

// A pipeline stage is two 18 KB weight tiles -- the gate and up tiles of one
// K stage (SwiGLU, NT = 1), or two consecutive K stages of one matrix
// (NT = 2) -- so that every step of the rings moves ~37 KB: each step costs
// a fixed hand-off latency (barrier wake-up, MMA issue) of about half a
// microsecond, and 18 KB steps would halve the stream rate.  Each tile has
// its own MMA issuer and TMEM accumulator.  Each tcgen05 step of an issuing
// thread costs it ~0.1-0.2 us, so where TMEM allows the stages alternate
// between two issue groups (P = 2; four issuer threads, each with its own
// accumulator, added by the epilogue); the ring depth is then even, so a group
// owns its slots and waits on every phase of them in order.  Weights and
// activation columns of a stage share one full / empty barrier pair.
template <int NCOL, int EPI, int NT>
struct FtShape {
    static constexpr int NM = EPI == FM_SWIGLU ? 2 : 1;
    static_assert(NM * NT <= 2, "at most two tiles per stage");
    static constexpr int NI = NM * NT;                             // tiles (issuers, accumulators) per stage
    static constexpr int WST = NI * FT_TILE;                       // weight stage
    static constexpr int B_BYTES = NCOL * 128;                     // activation tile (columns only)
    static constexpr int BST = NT * B_BYTES;                       // activation stage
    static constexpr int TMAX = NCOL / FM_DIGITS;
    static constexpr int P = 2 * NI * NCOL <= 256 ? 2 : 1;         // issue groups
    static constexpr int NISS = P * NI;                            // issuer threads = accumulators
    // weight producer, issuers (warps 1, 2, then 8, 9), four epilogue warps
    // (3..6), activation producer (7)
    static constexpr int THREADS = 32 * (8 + (NISS > 2 ? NISS - 2 : 0));
};

// first unit of CTA c when U units go to G CTAs, and the CTA owning unit u
__device__ __forceinline__ int ft_lo(int c, int U, int G) {
    return static_cast<int>((static_cast<int64_t>(c) * U) / G);
}
__device__ __forceinline__ int ft_owner(int u, int U, int G) {
    return static_cast<int>(((static_cast<int64_t>(u) + 1) * G - 1) / U);
}

// a[t] (and b[t]) = sum over the n partial slices k = 0..n-1, in k order, of
// this thread's row; slice k's [2][TMAX][128] block at part(k).  The loads of
// several slices are issued together so that their latencies overlap.
template <int TMAX, bool DUAL, typename F>
__device__ __forceinline__ void ft_sum_parts(F part, int n, int T, int erow, float (&a)[TMAX], float (&b)[TMAX]) {
    constexpr int CH = 32 / (TMAX * (DUAL ? 2 : 1)) > 0 ? 32 / (TMAX * (DUAL ? 2 : 1)) : 1;
#pragma unroll
    for (int t = 0; t < TMAX; ++t) { a[t] = 0.0f; b[t] = 0.0f; }
    for (int k0 = 0; k0 < n; k0 += CH) {
        float va[CH][TMAX], vb[CH][TMAX];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const float *pc = part(min(k0 + c, n - 1));
#pragma unroll
            for (int t = 0; t < TMAX; ++t) {
                va[c][t] = t < T ? __ldcg(pc + t * 128 + erow) : 0.0f;
                vb[c][t] = (DUAL && t < T) ? __ldcg(pc + TMAX * 128 + t * 128 + erow) : 0.0f;
            }
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            if (k0 + c < n) {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    a[t] += va[c][t];
                    if (DUAL) b[t] += vb[c][t];
                }
            }
        }
    }
}

// a[t] (and b[t]) += the partial slices k = 1..n-1 of this thread's row, in
// k order (the owner's own slice 0 is already in a / b); the loads of
// several slices are issued together
template <int TMAX, bool DUAL, typename F>
__device__ __forceinline__ void ft_add_parts(F part, int n, int T, int erow, float (&a)[TMAX], float (&b)[TMAX]) {
    constexpr int CH = 32 / (TMAX * (DUAL ? 2 : 1)) > 0 ? 32 / (TMAX * (DUAL ? 2 : 1)) : 1;
    for (int k0 = 1; k0 < n; k0 += CH) {
        float va[CH][TMAX], vb[CH][TMAX];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const float *pc = part(min(k0 + c, n - 1));
#pragma unroll
            for (int t = 0; t < TMAX; ++t) {
                va[c][t] = t < T ? __ldcg(pc + t * 128 + erow) : 0.0f;
                vb[c][t] = (DUAL && t < T) ? __ldcg(pc + TMAX * 128 + t * 128 + erow) : 0.0f;
            }
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            if (k0 + c < n) {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    a[t] += va[c][t];
                    if (DUAL) b[t] += vb[c][t];
                }
            }
        }
    }
}

template <int NCOL, int EPI, int NT>
__global__ void __launch_bounds__(FtShape<NCOL, EPI, NT>::THREADS, 1) k_fp4t(const FtArgs g) {
    using S = FtShape<NCOL, EPI, NT>;
    constexpr int NI = S::NI, P = S::P, NISS = S::NISS;
    constexpr bool DUAL = S::NM == 2;
    constexpr int TMAX = S::TMAX;
    constexpr uint32_t TMEM_COLS = 512;
    static_assert(NISS * NCOL <= 256, "accumulators live in TMEM columns [0, 256)");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NW = g.n_w;                                   // ring stages (weights + activation columns)
    uint8_t *w_ring = smem;
    uint8_t *b_ring = w_ring + static_cast<size_t>(NW) * S::WST;
    uint8_t *sfb_const = b_ring + static_cast<size_t>(NW) * S::BST;   // 512 B: the activation scale atom
    float *gtab = reinterpret_cast<float *>(sfb_const + 512);             // [TMAX][8] column factors
    uint64_t *full = reinterpret_cast<uint64_t *>(gtab + TMAX * FM_GSTRIDE);
    uint64_t *empty = full + NW;
    uint64_t *accfull = empty + NW;
    uint64_t *accempty = accfull + 1;
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(accempty + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, U = g.n_units;
    const int nsr = g.n_kq / NT;                             // stages per row block
    const int u_lo = ft_lo(blockIdx.x, U, G), u_hi = ft_lo(blockIdx.x + 1, U, G);
    const int n_st = u_hi - u_lo;
    const int T = g.T;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NW; ++s) {
            mbar_init(&full[s], 2);                          // weight and activation producers
            mbar_init(&empty[s], NI);                        // the owning group's issuers
        }
        mbar_init(accfull, NISS);                            // every issuer, once per segment
        mbar_init(accempty, 4);
        fence_mbar_init();
    }
    if (warp == 3) {
        // every activation column has scale 1.0
        reinterpret_cast<uint4 *>(sfb_const)[lane] = make_uint4(FM_SFB * 0x01010101u, FM_SFB * 0x01010101u,
                                                                FM_SFB * 0x01010101u, FM_SFB * 0x01010101u);
        fence_proxy_async();
    }
    if (warp == 1) tmem_alloc(tmem_s, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    const uint32_t tD = tbase;                               // tile k's accumulator: + k * NCOL
    fr_pdl_trigger();

    if (warp == 0) {
        // ---------------- weight producer: contiguous tiles, no PDL wait
        if (lane == 0) {
            // ring slot s and its use count kept as counters: a runtime
            // division per stage is a dependent chain this lone thread pays
            int s = 0, use = 0;
            for (int i = 0; i < n_st; ++i) {
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, 50)) break;
                uint8_t *st = w_ring + static_cast<size_t>(s) * S::WST;
                // unit u = row block u / nsr, K stage (u % nsr) * NT: tiles
                // are stored row block by row block, n_kq = nsr * NT per block,
                // so its first tile is tile u * NT
                const int64_t off = static_cast<int64_t>(u_lo + i) * NT * FT_TILE;
                mbar_expect_tx(&full[s], S::WST);
                bulk_g2s(st, g.w0 + off, NT * FT_TILE, &full[s]);
                if (DUAL) bulk_g2s(st + FT_TILE, g.w1 + off, FT_TILE, &full[s]);
                if (++s == NW) {
                    s = 0;
                    ++use;
                }
            }
        }
    } else if (warp == 7) {
        // ---------------- activation producer (after the PDL wait)
        if (lane == 0) {
            fr_pdl_wait();
            int s = 0, use = 0, kq = u_lo % nsr;
            for (int i = 0; i < n_st; ++i) {
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, 51)) break;
                const int kq0 = kq * NT;
                mbar_expect_tx(&full[s], S::BST);
                bulk_g2s(b_ring + static_cast<size_t>(s) * S::BST, g.bimg + static_cast<int64_t>(kq0) * S::B_BYTES,
                         S::BST, &full[s]);
                if (++s == NW) {
                    s = 0;
                    ++use;
                }
                if (++kq == nsr) kq = 0;
            }
        }
    } else if (warp == 1 || warp == 2 || warp >= 8) {
        // ---------------- MMA issuers: thread (group p, tile k) issues tile k
        // of the stages i with i % P == p into accumulator p * NI + k
        const int ii = warp <= 2 ? warp - 1 : warp - 6;
        if (lane == 0 && ii < NISS) {
            const int p = ii / NI, k = ii % NI;
            const uint32_t idesc = idesc_nvf4(128, NCOL);
            // scale columns: [256, 256 + 16 NI NW) weights by ring slot and
            // tile, then four per issuer for the constant activation atom
            const uint32_t t_sfb = tbase + 256 + NW * 16 * NI + 4 * ii;
            const uint32_t t_acc = tD + ii * NCOL;
            tc_cp_sf(t_sfb, sdesc_plain(smem_u32(sfb_const), 128));
            int seg = 0;
            bool started = false;
            // K stage within the row block, ring slot and its use count as
            // counters (no runtime division on this thread's critical path)
            int kq = u_lo % nsr, sw = 0, use = 0;
            for (int i = 0; i < n_st; ++i) {
                const bool first = i == 0 || kq == 0;             // first stage of a row-block segment
                const bool last = i == n_st - 1 || kq == nsr - 1;
                if (first) {
                    started = false;
                    // every issuer waits for each drain, in order
                    if (seg > 0 && !mbar_wait(accempty, (seg - 1) & 1, 52)) break;
                }
                if (i % P == p) {
                    if (!mbar_wait(&full[sw], use & 1, 53)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(w_ring + static_cast<size_t>(sw) * S::WST) + k * FT_TILE;
                    const uint32_t b_addr = smem_u32(b_ring + static_cast<size_t>(sw) * S::BST) +
                                            (NT == 2 ? k : 0) * S::B_BYTES;
                    const uint32_t t_sfa = tbase + 256 + (sw * NI + k) * 16;
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
                    tc_commit(accfull);
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
        const int at = threadIdx.x - 96;                  // 0..127
        const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
        const int erow = 32 * q + lane;
        fr_pdl_wait();
        if (at < TMAX * FM_GSTRIDE) gtab[at] = at / FM_GSTRIDE < T ? g.gtab[at] : 0.0f;
        named_bar(1, 128);
        const float sc0 = g.s0 ? *g.s0 : 1.0f;
        const float sc1 = (DUAL && g.s1) ? *g.s1 : 1.0f;
        const int64_t peer_off = g.peer_off + (g.epoch ? static_cast<int64_t>(*g.epoch & 1u) * g.par_bytes : 0);

        // writes one output value; returns |value| (0 for rows past N)
        auto finish = [&](int rb, int t, float a0, float a1) -> float {
            const int n = rb * 128 + erow;
            if (n >= g.N || t >= T) return 0.0f;
            const int64_t tt = g.t0 + t;
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
                if (g.resid) val += g.resid[tt * g.ldr + n];
            }
            if (!DUAL && g.peer_base != nullptr) {
                for (int q2 = 0; q2 < g.npeers; ++q2)
                    reinterpret_cast<float *>(g.peer_base[q2] + peer_off)[tt * g.ldy + n] = val;
            } else {
                g.y[tt * g.ldy + n] = val;
            }
            return fabsf(val);
        };
        // this warp's 32 rows of row block rb, token t: their largest |value|
        // for the next activation kernel (it then needs no scan of the row)
        auto publish = [&](int rb, int t, float am) {
            if (g.amax_out == nullptr || t >= T) return;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
            if (lane == 0) g.amax_out[(g.t0 + t) * static_cast<int64_t>(g.amax_ld) + rb * 4 + q] = am;
        };
        // every row-block segment: drain the accumulators, then either finish
        // the rows or publish the partial; the last of the CTAs sharing a row
        // block adds the partials in CTA order (per quadrant, so a warp that
        // timed out cannot hold the others)
        int seg = 0;
        int rb = u_lo / nsr;                               // one segment per row block, in order
        for (int s0u = u_lo; s0u < u_hi; ++seg, ++rb) {
            const int s1u = min(u_hi, (rb + 1) * nsr);
            if (!mbar_wait(accfull, seg & 1, 55)) break;
            tc_fence_after();
            float acc0[TMAX], acc1[TMAX];
#pragma unroll
            for (int t = 0; t < TMAX; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }
            // groups that issued a stage of this segment
            const int i0 = s0u - u_lo, n_seg = s1u - s0u;
#pragma unroll
            for (int p = 0; p < P; ++p) {
                if (n_seg < P && i0 % P != p) continue;
                const uint32_t t_acc = tD + (p * NI) * NCOL + lane_off;
#pragma unroll
                for (int c = 0; c < NCOL; c += 16) {
                    uint32_t d0[16], d1[16];
                    tmem_ld16(t_acc + c, d0);
                    if (NI == 2) tmem_ld16(t_acc + NCOL + c, d1);
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const int col = c + v, t = col / FM_DIGITS;
                        if (t < TMAX) {
                            const float gf = gtab[col];
                            acc0[t] = fmaf(gf, __uint_as_float(d0[v]), acc0[t]);
                            if (NI == 2) acc1[t] = fmaf(gf, __uint_as_float(d1[v]), acc1[t]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accempty);        // the accumulators may be overwritten now
            if (!DUAL && NI == 2) {
                // two K stages per step: the two accumulators are two halves of the sum
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    acc0[t] += acc1[t];
                    acc1[t] = 0.0f;
                }
            }
            if (s0u == rb * nsr && s1u == (rb + 1) * nsr) {
#pragma unroll
                for (int t = 0; t < TMAX; ++t) publish(rb, t, finish(rb, t, acc0[t], acc1[t]));
            } else {
                // a row block shared with neighbouring CTAs.  Its owner is the
                // CTA holding its first unit, for which it is the last
                // segment; the others hold its later units at the start of
                // their ranges (or all of their range), so their parts are
                // usually in before the owner's.  They publish; the owner
                // waits (bounded) for them and adds them after its own, in CTA
                // order -- the sum the last-arriver form made, without the
                // owner's own store, fence and atomic on the critical path.
                const int c_first = ft_owner(rb * nsr, U, G);
                const int nparts = ft_owner((rb + 1) * nsr - 1, U, G) - c_first + 1;
                const int slot = static_cast<int>(blockIdx.x) - c_first;
                unsigned int *cnt = &g.counter[rb * 4 + q];
                if (slot > 0) {
                    float *pp = g.part + ((static_cast<int64_t>(rb) * g.maxp + slot) * 2) * TMAX * 128;
#pragma unroll
                    for (int t = 0; t < TMAX; ++t) {
                        pp[t * 128 + erow] = acc0[t];
                        if (DUAL) pp[TMAX * 128 + t * 128 + erow] = acc1[t];
                    }
                    fence_acq_rel_gpu();
                    __syncwarp();
                    if (lane == 0) atomicAdd(cnt, 1u);
                } else {
                    int got = 1;
                    if (lane == 0) {
                        const uint64_t t0w = fr_now_ns();
                        for (;;) {
                            unsigned int fv;
                            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(fv) : "l"(cnt) : "memory");
                            if (fv >= static_cast<unsigned>(nparts - 1)) break;
                            if (fr_now_ns() - t0w > g_fr_wait_ns) {
                                fr_flag(FR_ST_TIMEOUT | (58u << FR_ST_SITE_SHIFT));
                                got = 0;
                                break;
                            }
                        }
                        if (got) *cnt = 0u;                  // nobody touches it again before the next launch
                    }
                    got = __shfl_sync(0xffffffffu, got, 0);
                    if (got) {
                        fence_acq_rel_gpu();
                        const float *pb = g.part + (static_cast<int64_t>(rb) * g.maxp * 2) * TMAX * 128;
                        float s0[TMAX], s1[TMAX];
#pragma unroll
                        for (int t = 0; t < TMAX; ++t) {
                            s0[t] = 0.0f + acc0[t];
                            s1[t] = 0.0f + acc1[t];
                        }
                        ft_add_parts<TMAX, DUAL>([&](int k2) { return pb + (k2 * 2) * TMAX * 128; }, nparts, T, erow,
                                                 s0, s1);
#pragma unroll
                        for (int t = 0; t < TMAX; ++t) publish(rb, t, finish(rb, t, s0[t], s1[t]));
                    }
                }
            }
            s0u = s1u;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (!DUAL && g.peer_base != nullptr && threadIdx.x == 0) {
        // this CTA's rows are stored everywhere: count it into every rank
        __threadfence_system();
        for (int q2 = 0; q2 < g.npeers; ++q2)
            atomicAdd_system(reinterpret_cast<unsigned int *>(g.peer_base[q2] + g.flag_off) + g.rank, 1u);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, TMEM_COLS);
    }
}

} // namespace frb
