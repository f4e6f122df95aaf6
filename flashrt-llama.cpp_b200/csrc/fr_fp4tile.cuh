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
    int n_w, n_b;                // ring depth (stages of weights + activation columns); n_b = n_w,
                                 // or 0 when the kernel builds the columns itself (x below)
    int amax_ld;
    // in-kernel activation columns (T <= 2, NCOL = 16): with x set, bimg and
    // gtab are unused; the CTA copies the x values of its K stages into
    // shared memory and builds their digit columns there.  amax_in
    // (nullable): per token the maxima of x's 32-value groups ([T][n_amax]),
    // else the row is scanned.  n_slots: K-stage groups a CTA holds at most.
    const float *x;
    int64_t ldx;
    const float *amax_in;
    int n_amax;
    int n_slots;
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
    // (3..6), activation producer (7), then four more column-building warps
    // (WB..WB+3; with warp 7 the builders of the in-kernel form)
    static constexpr int WB = 8 + (NISS > 2 ? NISS - 2 : 0);
    static constexpr int NBW = 5;
    static constexpr int THREADS = 32 * (WB + NBW - 1);
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

// The eight digit planes of one q8_1 block (32 values, lane = value) as
// 32-bit words: W holds this lane's digit nibbles (plane p at bits 4p).  Byte
// b of plane p's 16-byte unit packs values b and b + 8 of its sub-block
// (ggml's order, as fp4_digits_store); lane L writes bytes 4(L&3)..+3 of
// plane L>>2, so the warp stores 128 bytes in one conflict-free instruction
// (eight rows, each in its own 16-byte swizzle position).
__device__ __forceinline__ void fp4_words_store(uint32_t W, uint8_t *tile, int n0, int c) {
    const int lane = threadIdx.x & 31;
    const uint32_t hiW = __shfl_xor_sync(0xffffffffu, W, 8);
    // valid on lanes j < 8 of each half: even planes' bytes, odd planes' bytes
    const uint32_t E = (W & 0x0F0F0F0Fu) | ((hiW & 0x0F0F0F0Fu) << 4);
    const uint32_t O = ((W >> 4) & 0x0F0F0F0Fu) | (hiW & 0xF0F0F0F0u);
    const int p = lane >> 2, qd = lane & 3;
    const int src = 4 * (qd & 1) + 16 * (qd >> 1);
    uint32_t v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t e = __shfl_sync(0xffffffffu, E, src + i);
        const uint32_t o = __shfl_sync(0xffffffffu, O, src + i);
        v[i] = (p & 1) ? o : e;
    }
    const uint32_t k = static_cast<uint32_t>(p >> 1);
    const uint32_t sel = k | ((k + 4u) << 4);
    const uint32_t word = __byte_perm(__byte_perm(v[0], v[1], sel), __byte_perm(v[2], v[3], sel), 0x5410);
    const int n = n0 + p;
    *reinterpret_cast<uint32_t *>(tile + n * 128 + ((c ^ (n & 7)) << 4) + 4 * qd) = word;
}

// The activation columns of this CTA's K stages, built in shared memory by
// five warps (bw = 0..4) instead of by a separate kernel (T <= 2).  Slot j
// holds the K-stage group (u_lo + j) mod nsr, the group of the CTA's unit j
// (and of every unit j + m nsr): its NT column tiles and, per token, its
// NT x 256 x values.  The arithmetic is act_fp4_row's, value for value:
// the token's reference exponent from the row's largest |x| (or from the
// producer's 32-value-group maxima), q8_1 per 32 values, the eight balanced
// base-9 digits as E2M1 codes in the 128-byte-swizzled K-major tiles.
// The x values (and the row scan) arrive by plain vector loads, all in
// flight at once; each warp then builds up to four q8_1 blocks together,
// and every slot is released to the MMA issuers as soon as it is built.
template <int NCOL, int NT>
__device__ __forceinline__ void ft_build_columns(const FtArgs &g, int bw, int u_lo, int n_st, int nsr, uint8_t *act,
                                                 float *xbuf, float *gtab, int *scr, uint64_t *gready,
                                                 uint64_t *act_ready) {
    constexpr int NBW = 5, NTH = NBW * 32;
    constexpr int SV = NT * 256;                      // x values of one slot per token
    constexpr int B_BYTES = NCOL * 128;
    constexpr int LD = 8;                             // float4 loads in flight per thread and batch
    const int lane = threadIdx.x & 31;
    const int bt = bw * 32 + lane;
    const int T = g.T;
    const int nsl = min(n_st, nsr);
    const int xt = g.n_slots * SV;                    // floats per token in xbuf
    const int ga = u_lo % nsr;
    const int n1 = min(nsl, nsr - ga);                // slots before the wrap at the row's end
    fr_pdl_wait();
    // 1. the slots' x values into xbuf (slot order) and each token's largest
    // |x| (from the row, or from the producer's group maxima)
    const int span4 = nsl * SV / 4;                   // float4 per token
    const int K4 = g.K / 4;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        float am = 0.0f;
        if (t < T) {
            const float4 *r4 = reinterpret_cast<const float4 *>(g.x + static_cast<int64_t>(t) * g.ldx);
            float4 *dst = reinterpret_cast<float4 *>(xbuf + t * xt);
            for (int k0 = 0; k0 < span4; k0 += LD * NTH) {
                float4 v[LD];
#pragma unroll
                for (int u = 0; u < LD; ++u) {
                    const int k = k0 + u * NTH + bt;
                    // slot-order index k -> row position (one wrap at most)
                    const int sl = k / (SV / 4);
                    const int src = (sl < n1 ? (ga + sl) : (sl - n1)) * (SV / 4) + k % (SV / 4);
                    v[u] = k < span4 ? r4[src] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int u = 0; u < LD; ++u) {
                    const int k = k0 + u * NTH + bt;
                    if (k < span4) dst[k] = v[u];
                }
            }
            if (g.amax_in != nullptr) {
                const float *ai = g.amax_in + static_cast<int64_t>(t) * g.n_amax;
                for (int i0 = 0; i0 < g.n_amax; i0 += LD * NTH) {
                    float v[LD];
#pragma unroll
                    for (int u = 0; u < LD; ++u) {
                        const int i = i0 + u * NTH + bt;
                        v[u] = i < g.n_amax ? ai[i] : 0.0f;
                    }
#pragma unroll
                    for (int u = 0; u < LD; ++u) am = fmaxf(am, v[u]);
                }
            } else {
                for (int k0 = 0; k0 < K4; k0 += LD * NTH) {
                    float4 v[LD];
#pragma unroll
                    for (int u = 0; u < LD; ++u) {
                        const int k = k0 + u * NTH + bt;
                        v[u] = k < K4 ? r4[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
#pragma unroll
                    for (int u = 0; u < LD; ++u)
                        am = fmaxf(am, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
        if (lane == 0) scr[t * NBW + bw] = __float_as_int(am);
    }
    named_bar(2, NTH);                                // xbuf and the maxima are complete
    int e0v[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        float am = __int_as_float(scr[t * NBW]);
#pragma unroll
        for (int w = 1; w < NBW; ++w) am = fmaxf(am, __int_as_float(scr[t * NBW + w]));
        const int emax = fp4_row_emax(am);
        e0v[t] = emax > -1000 ? emax - FM_SPAN : 0;
    }
    if (bt < (NCOL / FM_DIGITS) * FM_GSTRIDE) {
        const int t = bt / FM_GSTRIDE, p = bt % FM_GSTRIDE;
        float v = 1.0f;
        for (int i = 0; i < p; ++i) v *= 9.0f;
        gtab[bt] = t < T ? ldexpf(v, (t == 0 ? e0v[0] : e0v[1]) + 1) : 0.0f;
    }
    // 2. the slots, in the order the issuers use them; the q8_1 blocks of
    // all slots are dealt round-robin over the five warps, four at a time
    const int NB = NT * 8 * T;                        // q8_1 blocks per slot
    for (int j = 0; j < nsl; ++j) {
        const int b0 = ((bw - (j * NB) % NBW) % NBW + NBW) % NBW;
        for (int b = b0; b < NB; b += 4 * NBW) {
            float xv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int bb = b + k * NBW;
                const int t = bb / (NT * 8), c8 = bb % (NT * 8);
                xv[k] = bb < NB ? xbuf[t * xt + j * SV + c8 * 32 + lane] : 0.0f;
            }
            uint32_t W[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int bb = b + k * NBW;
                const q8_lane r = q8_1_chunk(xv[k]);
                uint32_t nib[FM_DIGITS];
                fp4_digits(r.q, __float2half_rn(r.d), bb / (NT * 8) == 0 ? e0v[0] : e0v[1], nib);
                uint32_t w = 0;
#pragma unroll
                for (int p = 0; p < FM_DIGITS; ++p) w |= nib[p] << (4 * p);
                W[k] = w;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int bb = b + k * NBW;
                if (bb < NB) {
                    const int t = bb / (NT * 8), c8 = bb % (NT * 8);
                    fp4_words_store(W[k], act + (j * NT + (c8 >> 3)) * B_BYTES, FM_DIGITS * t, c8 & 7);
                }
            }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&act_ready[j]);
        if (j == 0 && bt == 0) mbar_arrive(gready);   // gtab was written before the first slot
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
    const bool build = g.x != nullptr;                      // columns built here (T <= 2, NCOL = 16)
    const int NSL = build ? g.n_slots : 0;
    uint8_t *w_ring = smem;
    uint8_t *b_ring = w_ring + static_cast<size_t>(NW) * S::WST;
    uint8_t *act = b_ring + static_cast<size_t>(g.n_b) * S::BST;        // [NSL][NT] column tiles (built)
    float *xbuf = reinterpret_cast<float *>(act + static_cast<size_t>(NSL) * S::BST);  // [T][NSL * NT * 256]
    uint8_t *sfb_const = reinterpret_cast<uint8_t *>(xbuf + static_cast<size_t>(NSL) * NT * 256 * (build ? g.T : 0));
    float *gtab = reinterpret_cast<float *>(sfb_const + 512);             // [TMAX][8] column factors
    uint64_t *full = reinterpret_cast<uint64_t *>(gtab + TMAX * FM_GSTRIDE);
    uint64_t *empty = full + NW;
    uint64_t *accfull = empty + NW;
    uint64_t *accempty = accfull + 1;
    uint64_t *gready = accempty + 1;                         // column factors written (built form)
    uint64_t *act_ready = gready + 1;                        // [NSL] column tiles built
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(act_ready + NSL);
    int *bscr = reinterpret_cast<int *>(tmem_s + 1);         // [2][5] builder scratch

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, U = g.n_units;
    const int nsr = g.n_kq / NT;                             // stages per row block
    const int u_lo = ft_lo(blockIdx.x, U, G), u_hi = ft_lo(blockIdx.x + 1, U, G);
    const int n_st = u_hi - u_lo;
    const int T = g.T;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NW; ++s) {
            mbar_init(&full[s], build ? 1 : 2);              // weight (and activation) producers
            mbar_init(&empty[s], NI);                        // the owning group's issuers
        }
        mbar_init(accfull, NISS);                            // every issuer, once per segment
        mbar_init(accempty, 4);
        mbar_init(gready, 1);
        for (int j = 0; j < NSL; ++j) mbar_init(&act_ready[j], S::NBW);
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
            for (int i = 0; i < n_st; ++i) {
                const int s = i % NW;
                if (i >= NW && !mbar_wait(&empty[s], ((i / NW) - 1) & 1, 50)) break;
                uint8_t *st = w_ring + static_cast<size_t>(s) * S::WST;
                const int u = u_lo + i;
                // first tile of the stage: row block u / nsr, K stage (u % nsr) * NT
                const int64_t off = (static_cast<int64_t>(u / nsr) * g.n_kq + (u % nsr) * NT) * FT_TILE;
                mbar_expect_tx(&full[s], S::WST);
                bulk_g2s(st, g.w0 + off, NT * FT_TILE, &full[s]);
                if (DUAL) bulk_g2s(st + FT_TILE, g.w1 + off, FT_TILE, &full[s]);
            }
        }
    } else if (build && (warp == 7 || warp >= S::WB)) {
        // ---------------- column builders (five warps; the host selects
        // this form only for NCOL = 16)
        if constexpr (NCOL == 16)
            ft_build_columns<NCOL, NT>(g, warp == 7 ? 0 : warp - S::WB + 1, u_lo, n_st, nsr, act, xbuf, gtab, bscr,
                                       gready, act_ready);
    } else if (warp == 7) {
        // ---------------- activation producer (after the PDL wait)
        if (lane == 0) {
            fr_pdl_wait();
            for (int i = 0; i < n_st; ++i) {
                const int s = i % NW;
                if (i >= NW && !mbar_wait(&empty[s], ((i / NW) - 1) & 1, 51)) break;
                const int kq0 = ((u_lo + i) % nsr) * NT;
                mbar_expect_tx(&full[s], S::BST);
                bulk_g2s(b_ring + static_cast<size_t>(s) * S::BST, g.bimg + static_cast<int64_t>(kq0) * S::B_BYTES,
                         S::BST, &full[s]);
            }
        }
    } else if (warp == 1 || warp == 2 || (warp >= 8 && warp < S::WB)) {
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
            for (int i = 0; i < n_st; ++i) {
                const int u = u_lo + i;
                const bool first = i == 0 || u % nsr == 0;       // first stage of a row-block segment
                const bool last = i == n_st - 1 || (u + 1) % nsr == 0;
                if (first) {
                    started = false;
                    // every issuer waits for each drain, in order
                    if (seg > 0 && !mbar_wait(accempty, (seg - 1) & 1, 52)) break;
                }
                if (i % P == p) {
                    const int sw = i % NW;
                    if (!mbar_wait(&full[sw], (i / NW) & 1, 53)) break;
                    // built columns: unit i's K-stage group sits in slot i mod nsr
                    if (build && !mbar_wait(&act_ready[i % nsr], 0, 54)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(w_ring + static_cast<size_t>(sw) * S::WST) + k * FT_TILE;
                    const uint32_t b_addr = (build ? smem_u32(act + static_cast<size_t>(i % nsr) * S::BST)
                                                   : smem_u32(b_ring + static_cast<size_t>(sw) * S::BST)) +
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
            }
        }
    } else if (warp >= 3 && warp <= 6) {
        // ---------------- epilogue warps (3..6), one TMEM lane quadrant each
        const int q = warp & 3;
        const int at = threadIdx.x - 96;                  // 0..127
        const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
        const int erow = 32 * q + lane;
        fr_pdl_wait();
        if (build) {
            mbar_wait(gready, 0, 57);                     // the builders wrote gtab
        } else if (at < TMAX * FM_GSTRIDE) {
            gtab[at] = at / FM_GSTRIDE < T ? g.gtab[at] : 0.0f;
        }
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
        for (int s0u = u_lo; s0u < u_hi; ++seg) {
            const int rb = s0u / nsr;
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
                const int c_first = ft_owner(rb * nsr, U, G);
                const int nparts = ft_owner((rb + 1) * nsr - 1, U, G) - c_first + 1;
                const int slot = static_cast<int>(blockIdx.x) - c_first;
                float *pp = g.part + ((static_cast<int64_t>(rb) * g.maxp + slot) * 2) * TMAX * 128;
#pragma unroll
                for (int t = 0; t < TMAX; ++t) {
                    pp[t * 128 + erow] = acc0[t];
                    if (DUAL) pp[TMAX * 128 + t * 128 + erow] = acc1[t];
                }
                fence_acq_rel_gpu();
                __syncwarp();
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&g.counter[rb * 4 + q], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == static_cast<unsigned>(nparts - 1)) {
                    fence_acq_rel_gpu();
                    const float *pb = g.part + (static_cast<int64_t>(rb) * g.maxp * 2) * TMAX * 128;
                    float s0[TMAX], s1[TMAX];
                    ft_sum_parts<TMAX, DUAL>([&](int k2) { return pb + (k2 * 2) * TMAX * 128; }, nparts, T, erow,
                                             s0, s1);
#pragma unroll
                    for (int t = 0; t < TMAX; ++t) publish(rb, t, finish(rb, t, s0[t], s1[t]));
                    if (lane == 0) g.counter[rb * 4 + q] = 0;
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
