// fr_gemm.cuh -- persistent stream-K W4A4 GEMM on the tcgen05 tensor cores
// (kind::mxf4nvf4.block_scale.block16, fp32 accumulation in TMEM).
//
// D[M, N] = alpha * A[M, K] . B[N, K]^T with A, B in the reference's wire
// format (include/fr_kernels.h:35-57 of the reference: packed E2M1 rows,
// adjacent-pair nibbles, UE4M3 scales per 16 values in the 128x4 atom
// layout), f32 out -- the semantics of the reference's gemm_f32out
// (src/fr_gemm_f32out.cu:122-205, a CUTLASS Sm100 collective).  The SwiGLU
// form takes B from repack_weight_pair_interleaved (row 2j = gate row j, row
// 2j+1 = up row j) and writes D[M, N/2] = silu(alpha g) * (alpha u), so the
// prefill FFN never writes the gate/up product.
//
// Design (B200):
//   * tile 128 x 256 (one block-scaled MMA of N = 256 per 64-value K block:
//     half the MMA issues and a third less operand traffic per FLOP than a
//     128 x 128 tile), K stage 256 values, 4-stage TMA ring of 54 KB stages;
//   * schedule: with at least as many tiles as SMs, one CTA per SM takes whole
//     tiles c, c + grid, ... (no partial sum is ever written); with fewer,
//     every tile is split into S = SMs / tiles equal K ranges on S CTAs: for
//     S = 2 the two CTAs exchange halves (each finishes 64 rows, bounded
//     wait on its partner's flag, site 47), for S > 2 the last to arrive
//     adds the S partials in K-range order (deterministic); each CTA owns one
//     partial slot.  (A stream-K
//     division of the units over the SMs was measured and dropped: the
//     partial traffic at the end of the kernel cost 15-20 us on configs[3]'s
//     shapes);
//   * warp roles: warpgroup 0 = warp 0 TMA producer, warp 1 MMA issuer (and
//     TMEM owner), warps 2-3 idle; warpgroups 1-2 = epilogue warps 4..11
//     (lane quadrant = warp % 4, 128-column half = (warp - 4) / 4), which
//     drain the accumulator into registers and release it at once, so the
//     next segment's MMAs overlap their stores.  setmaxnreg moves registers
//     from warpgroup 0 (40 each) to the epilogue (232 each): 4 x 32 x 40 +
//     8 x 32 x 232 = 64,512 = 384 threads x 168 at launch (ptxas -v);
//   * scale factors: per stage one 512-byte atom per 64-value K block for A
//     and two for B (rows 0..127 and 128..255 of the tile), tcgen05.cp'd into
//     TMEM columns of that stage (SFA: 4 columns, SFB: 8 columns per block) by
//     two copier threads (warps 2 and 3, alternate stages), which hand the
//     stage to the MMA thread through an mbarrier: twelve copies cost an
//     issuing thread more than the stage's four MMAs;
//   * every wait is bounded (status word, sites 40..45) and a CTA that gave up
//     waits for its own copies in flight before it exits.
#pragma once

#include "fr_tc.cuh"

namespace frb {

constexpr int P_BM = 128, P_BN = 256, P_BK = 256;
constexpr int P_STAGES = 4;
constexpr int P_A_BYTES = P_BM * P_BK / 2;                 // 16 KB
constexpr int P_B_BYTES = P_BN * P_BK / 2;                 // 32 KB
constexpr int P_SFA_BYTES = 4 * 512;                       // 4 K blocks x 1 atom
constexpr int P_SFB_BYTES = 8 * 512;                       // 2 row halves x 4 K blocks
constexpr int P_STAGE = P_A_BYTES + P_B_BYTES + P_SFA_BYTES + P_SFB_BYTES;   // 54 KB (1024-aligned)
constexpr int P_EPI_WARPS = 8;
constexpr int P_CW = P_BN / (P_EPI_WARPS / 4);               // accumulator columns per epilogue thread
constexpr int P_THREADS = (4 + P_EPI_WARPS) * 32;             // warpgroup 0: producer, MMA, 2 idle
constexpr uint32_t P_TMEM_COLS = 512;                      // acc [0,256) + 4 stages x 48 SF columns
constexpr int P_STG_FLOATS = 32 * 9;                       // per epilogue warp: 32 rows x 8 columns (+1 pad)
constexpr size_t P_SMEM = 1024 + static_cast<size_t>(P_STAGES) * P_STAGE + 256 +
                          static_cast<size_t>(P_EPI_WARPS) * P_STG_FLOATS * sizeof(float);
constexpr int P_SLOT_FLOATS = P_BM * P_BN;                 // one partial accumulator

enum PEpi : int { P_PLAIN = 0, P_SWIGLU = 1 };

struct PGemmArgs {
    const uint8_t *sfa, *sfb;
    float *D;
    int64_t ldd;                 // row stride of D (floats)
    int M, N, K;                 // N = rows of B (the SwiGLU output has N/2 columns)
    int nkt;                     // K stages of 256
    int n_m, n_n;                // tiles along M and N
    int tiles;
    int split;                   // 0: whole tiles (CTA c takes tiles c, c + grid, ...);
                                 // S > 0: grid = tiles * S, CTA c takes K range c % S of tile c / S
    float alpha;
    float *part;                 // [grid][128 x 256] partial accumulators (split mode)
    unsigned int *counter;       // [2 * tiles], zero on entry, reset by the last arrival / the finisher
};

// The (tile, K range) segments of one CTA, in order.  Whole tiles when there
// are at least as many tiles as CTAs (no partial ever written); otherwise
// every tile split into S equal K ranges on S consecutive CTAs.
struct PSegIter {
    int c, G, nkt, tiles, S, i;
    __device__ __forceinline__ bool next(int &t, int &kt0, int &kt1) {
        if (S == 0) {
            t = c + i * G;
            if (t >= tiles) return false;
            kt0 = 0;
            kt1 = nkt;
            ++i;
            return true;
        }
        if (i > 0) return false;
        ++i;
        t = c / S;
        const int s = c % S;
        kt0 = static_cast<int>(static_cast<int64_t>(s) * nkt / S);
        kt1 = static_cast<int>(static_cast<int64_t>(s + 1) * nkt / S);
        return t < tiles && kt1 > kt0;
    }
};

// tile t -> (m block, n block): consecutive tiles share their B tile, so the
// CTAs working on them at the same time read it from HBM once
__device__ __forceinline__ void p_tile_mn(const PGemmArgs &g, int t, int &mb, int &nb) {
    mb = t % g.n_m;
    nb = t / g.n_m;
}

// 32 columns of this warp's TMEM lanes into r (no wait)
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// tcgen05.wait::ld with the loaded registers as operands, so that no use of
// them can be scheduled before the wait
__device__ __forceinline__ void tmem_ld_wait_dep(uint32_t *r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :: "memory");
}

// Stores the finished values of one epilogue warp: v[i] is column c0 + i of
// tile row rbase + lane (i < ncols, ncols % 8 == 0).  Plain: D[m, n0 + c] =
// alpha v; SwiGLU: v holds (gate, up) pairs, output column (n0 + c) / 2.  The
// values go through a 32 x 8 shared-memory tile per warp so that each store
// instruction writes whole 32-byte sectors of 16 rows instead of 16 bytes of
// 32 rows.
template <int EPI, int NC>
__device__ __forceinline__ void p_store_rows(const PGemmArgs &g, int rbase, int n0, int c0, const float *v,
                                             float *stg, int lane) {
    if (EPI == P_SWIGLU) {
        float o[NC / 2];
#pragma unroll
        for (int i = 0; i < NC / 2; ++i) {
            float up = v[2 * i + 1] * g.alpha;
            const float gate = v[2 * i] * g.alpha;
            up *= silu_f(gate);
            o[i] = up;
        }
        const int nout = g.N / 2;
#pragma unroll
        for (int cc = 0; cc < NC / 2; cc += 8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) stg[lane * 9 + i] = o[cc + i];
            __syncwarp();
#pragma unroll
            for (int rep = 0; rep < 2; ++rep) {
                const int rr = (lane >> 1) + 16 * rep, hf = lane & 1;
                const int m = rbase + rr, col = (n0 + c0) / 2 + cc + 4 * hf;
                if (m < g.M && col < nout)
                    *reinterpret_cast<float4 *>(g.D + static_cast<int64_t>(m) * g.ldd + col) =
                        make_float4(stg[rr * 9 + 4 * hf], stg[rr * 9 + 4 * hf + 1], stg[rr * 9 + 4 * hf + 2],
                                    stg[rr * 9 + 4 * hf + 3]);
            }
            __syncwarp();
        }
    } else {
#pragma unroll
        for (int cc = 0; cc < NC; cc += 8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) stg[lane * 9 + i] = v[cc + i];
            __syncwarp();
#pragma unroll
            for (int rep = 0; rep < 2; ++rep) {
                const int rr = (lane >> 1) + 16 * rep, hf = lane & 1;
                const int m = rbase + rr, col = n0 + c0 + cc + 4 * hf;
                if (m < g.M && col < g.N)
                    *reinterpret_cast<float4 *>(g.D + static_cast<int64_t>(m) * g.ldd + col) =
                        make_float4(stg[rr * 9 + 4 * hf] * g.alpha, stg[rr * 9 + 4 * hf + 1] * g.alpha,
                                    stg[rr * 9 + 4 * hf + 2] * g.alpha, stg[rr * 9 + 4 * hf + 3] * g.alpha);
            }
            __syncwarp();
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(P_THREADS, 1) k_gemm_p(const __grid_constant__ CUtensorMap tmA,
                                                        const __grid_constant__ CUtensorMap tmB,
                                                        const PGemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P_STAGES * P_STAGE);
    uint64_t *empty = full + P_STAGES;
    uint64_t *sf_ready = empty + P_STAGES;              // the stage's scale factors are in TMEM
    uint64_t *acc_full = sf_ready + P_STAGES;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *epi_done = acc_empty + 1;                // every epilogue warp is past its last TMEM read
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(epi_done + 1);
    volatile int *bcast = reinterpret_cast<volatile int *>(tmem_s + 1);     // [4]: last arrival, lo, hi, abort

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkt = g.nkt;
    const int kb_total = g.K >> 6;
    const int n_rb_b = (g.N + 127) >> 7;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&sf_ready[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, P_EPI_WARPS);
        mbar_init(epi_done, P_EPI_WARPS);
        bcast[3] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_s, P_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    // A comes from the previous kernel; the tile counters and partial slots
    // may have been touched by the previous launch of this kernel
    fr_pdl_wait();

    if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 40;" ::: "memory");
    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer: A / B tiles by TMA, scale atoms by bulk copies
            int64_t it = 0;
            bool ok = true;
            PSegIter sg{static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), nkt, g.tiles, g.split, 0};
            int t, kt0, kt1;
            while (ok && sg.next(t, kt0, kt1)) {
                int mb, nb;
                p_tile_mn(g, t, mb, nb);
                const uint8_t *sfa_blk = g.sfa + static_cast<int64_t>(mb) * kb_total * 512;
                const uint8_t *sfb0 = g.sfb + static_cast<int64_t>(2 * nb) * kb_total * 512;
                // a ragged last tile has no second row block: its B rows are
                // zero-filled, any finite scales serve
                const uint8_t *sfb1 = g.sfb + static_cast<int64_t>(min(2 * nb + 1, n_rb_b - 1)) * kb_total * 512;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = static_cast<int>(it % P_STAGES);
                    if (it >= P_STAGES && !mbar_wait(&empty[s], static_cast<uint32_t>((it / P_STAGES) - 1) & 1u, 40)) {
                        ok = false;
                        break;
                    }
                    const int kbs = min(4, kb_total - 4 * kt);
                    uint8_t *st = smem + s * P_STAGE;
                    mbar_expect_tx(&full[s], P_A_BYTES + P_B_BYTES + 3 * kbs * 512);
                    tma_load_2d(st, &tmA, kt * (P_BK / 2), mb * P_BM, &full[s]);
                    tma_load_2d(st + P_A_BYTES, &tmB, kt * (P_BK / 2), nb * P_BN, &full[s]);
                    uint8_t *sf = st + P_A_BYTES + P_B_BYTES;
                    bulk_g2s(sf, sfa_blk + static_cast<int64_t>(4 * kt) * 512, kbs * 512, &full[s]);
                    bulk_g2s(sf + P_SFA_BYTES, sfb0 + static_cast<int64_t>(4 * kt) * 512, kbs * 512, &full[s]);
                    bulk_g2s(sf + P_SFA_BYTES + 2048, sfb1 + static_cast<int64_t>(4 * kt) * 512, kbs * 512, &full[s]);
                }
            }
            // nothing of this CTA's may still be landing when it exits: wait
            // (bounded) for the last stages issued
            for (int64_t j = it > P_STAGES ? it - P_STAGES : 0; j < it; ++j)
                mbar_wait(&full[j % P_STAGES], static_cast<uint32_t>(j / P_STAGES) & 1u, 41);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            const uint32_t idesc = idesc_nvf4(P_BM, P_BN);
            int64_t it = 0;
            int seg = 0;
            bool ok = true;
            PSegIter sg{static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), nkt, g.tiles, g.split, 0};
            int t, kt0, kt1;
            for (; sg.next(t, kt0, kt1); ++seg) {
                if (seg > 0 && ok) {
                    ok = mbar_wait(acc_empty, static_cast<uint32_t>(seg - 1) & 1u, 42);
                    tc_fence_after();
                }
                for (int kt = kt0; kt < kt1 && ok; ++kt, ++it) {
                    const int s = static_cast<int>(it % P_STAGES);
                    // the stage's operands landed and a copier thread put
                    // its scale factors into TMEM
                    if (!mbar_wait(&sf_ready[s], static_cast<uint32_t>(it / P_STAGES) & 1u, 43)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int kbs = min(4, kb_total - 4 * kt);
                    uint8_t *st = smem + s * P_STAGE;
                    const uint32_t a_addr = smem_u32(st), b_addr = smem_u32(st + P_A_BYTES);
                    const uint32_t t_sfa = tbase + 256 + static_cast<uint32_t>(s) * 48, t_sfb = t_sfa + 16;
                    for (int j = 0; j < kbs; ++j)
                        tc_mma_nvf4(tbase, sdesc_sw128(a_addr + 32 * j), sdesc_sw128(b_addr + 32 * j), idesc,
                                    t_sfa + 4 * j, t_sfb + 8 * j, (kt > kt0 || j > 0) ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                // always signal the segment, so the epilogue never waits on a
                // producer or issuer that gave up (the status word says so)
                tc_commit(acc_full);
            }
        }
    } else if (warp == 2 || warp == 3) {
        if (lane == 0) {
            // ---------------- scale-factor copiers: each tcgen05.cp costs its
            // issuing thread ~45 ns, twelve per stage -- more than the
            // stage's four MMAs -- so two threads copy alternate stages'
            // atoms into that stage's TMEM columns while the MMA thread
            // issues, and signal it through sf_ready
            const int cid = warp - 2;
            int64_t it = 0;
            bool ok = true;
            PSegIter sg{static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), nkt, g.tiles, g.split, 0};
            int t, kt0, kt1;
            while (ok && sg.next(t, kt0, kt1)) {
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    if ((it & 1) != cid) continue;
                    const int s = static_cast<int>(it % P_STAGES);
                    if (!mbar_wait(&full[s], static_cast<uint32_t>(it / P_STAGES) & 1u, 46)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int kbs = min(4, kb_total - 4 * kt);
                    uint8_t *st = smem + s * P_STAGE;
                    const uint32_t sfa_addr = smem_u32(st + P_A_BYTES + P_B_BYTES);
                    const uint32_t sfb_addr = sfa_addr + P_SFA_BYTES;
                    const uint32_t t_sfa = tbase + 256 + static_cast<uint32_t>(s) * 48, t_sfb = t_sfa + 16;
                    for (int j = 0; j < kbs; ++j) {
                        tc_cp_sf(t_sfa + 4 * j, sdesc_plain(sfa_addr + 512 * j, 128));
                        tc_cp_sf(t_sfb + 8 * j, sdesc_plain(sfb_addr + 512 * j, 128));
                        tc_cp_sf(t_sfb + 8 * j + 4, sdesc_plain(sfb_addr + 2048 + 512 * j, 128));
                    }
                    tc_commit(&sf_ready[s]);
                }
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue warps 4..11
        asm volatile("setmaxnreg.inc.sync.aligned.u32 232;" ::: "memory");
        const int q = warp & 3;                             // TMEM lane quadrant this warp may access
        const int cw0 = ((warp - 4) >> 2) * P_CW;           // first accumulator column of this warp
        const int wb = q + 4 * ((warp - 4) >> 2);           // this warp's block of a partial slot
        float *stg = reinterpret_cast<float *>(smem + P_STAGES * P_STAGE + 256) + (warp - 4) * P_STG_FLOATS;
        const bool leader = threadIdx.x == 128;
        int seg = 0;
        PSegIter sg{static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), nkt, g.tiles, g.split, 0};
        int t, kt0, kt1;
        for (; sg.next(t, kt0, kt1); ++seg) {
            int mb, nb;
            p_tile_mn(g, t, mb, nb);
            const int n0 = nb * P_BN;
            const bool ok = mbar_wait(acc_full, static_cast<uint32_t>(seg) & 1u, 44);
            tc_fence_after();
            uint32_t r[P_CW];
            if (ok) {
                const uint32_t ta = tbase + (static_cast<uint32_t>(32 * q) << 16) + cw0;
#pragma unroll
                for (int c = 0; c < P_CW / 32; ++c) tmem_ld32_async(ta + 32 * c, r + 32 * c);
#pragma unroll
                for (int c = 0; c < P_CW / 32; ++c) tmem_ld_wait_dep(r + 32 * c);
            } else {
                bcast[3] = 1;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);          // the accumulator is free for the next segment
            named_bar(1, P_EPI_WARPS * 32);
            if (bcast[3]) break;                            // a wait gave up (flagged): all epilogue warps stop
            const float *v = reinterpret_cast<const float *>(r);
            if (kt0 == 0 && kt1 == nkt) {
                p_store_rows<EPI, P_CW>(g, mb * P_BM + 32 * q, n0, cw0, v, stg, lane);
            } else if (g.split == 2) {
                // two CTAs share the tile (K ranges 0 and 1): CTA s finishes
                // rows [64 s, 64 s + 64) (lane quadrants 2s, 2s+1) and hands
                // its other rows to its partner through its slot, so each
                // moves half a tile each way instead of one CTA merging all
                const int sh = static_cast<int>(blockIdx.x) & 1;
                const bool mine = (q >> 1) == sh;
                if (!mine) {
                    float4 *blk = reinterpret_cast<float4 *>(g.part + static_cast<int64_t>(blockIdx.x) * P_SLOT_FLOATS +
                                                             wb * (32 * P_CW)) + lane;
#pragma unroll
                    for (int i = 0; i < P_CW / 4; ++i)
                        blk[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    fence_acq_rel_gpu();
                }
                named_bar(1, P_EPI_WARPS * 32);
                if (leader) {
                    __threadfence();
                    atomicAdd(&g.counter[2 * t + (1 - sh)], 1u);           // the partner's half is out
                    unsigned int *f = &g.counter[2 * t + sh];
                    const uint64_t t0 = fr_now_ns();
                    int got = 0;
                    for (;;) {
                        unsigned int fv;
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(fv) : "l"(f) : "memory");
                        if (fv != 0u) { got = 1; break; }
                        if (fr_now_ns() - t0 > g_fr_wait_ns) {
                            fr_flag(FR_ST_TIMEOUT | (47u << FR_ST_SITE_SHIFT));
                            break;
                        }
                    }
                    if (got) *f = 0u;                       // nobody else touches it before the next launch
                    bcast[0] = got;
                }
                named_bar(1, P_EPI_WARPS * 32);
                if (mine && bcast[0]) {
                    fence_acq_rel_gpu();
                    const float4 *src = reinterpret_cast<const float4 *>(
                                            g.part + static_cast<int64_t>(blockIdx.x ^ 1u) * P_SLOT_FLOATS +
                                            wb * (32 * P_CW)) + lane;
#pragma unroll
                    for (int ch = 0; ch < P_CW; ch += 32) {
                        float acc[32];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 w = __ldcg(src + (ch / 4 + i) * 32);
                            acc[4 * i] = v[ch + 4 * i] + w.x;          // two terms: the order is immaterial
                            acc[4 * i + 1] = v[ch + 4 * i + 1] + w.y;
                            acc[4 * i + 2] = v[ch + 4 * i + 2] + w.z;
                            acc[4 * i + 3] = v[ch + 4 * i + 3] + w.w;
                        }
                        p_store_rows<EPI, 32>(g, mb * P_BM + 32 * q, n0, cw0 + ch, acc, stg, lane);
                    }
                }
            } else {
                // part of a tile shared with neighbouring CTAs: publish this
                // CTA's partial in its slot (0: first segment, 1: last one),
                // laid out [warp block][column / 4][row][4] so that the
                // warp's stores (and the merging loads) are 512-byte lines
                float *slot = g.part + static_cast<int64_t>(blockIdx.x) * P_SLOT_FLOATS;
                float4 *blk = reinterpret_cast<float4 *>(slot + wb * (32 * P_CW)) + lane;
#pragma unroll
                for (int i = 0; i < P_CW / 4; ++i)
                    blk[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                fence_acq_rel_gpu();
                named_bar(1, P_EPI_WARPS * 32);
                if (leader) {
                    const int c_lo = t * g.split, c_hi = t * g.split + g.split - 1;
                    const unsigned prev = atomicAdd(&g.counter[t], 1u);
                    const bool last = prev == static_cast<unsigned>(c_hi - c_lo);
                    if (last) g.counter[t] = 0u;            // every contributor has arrived: ready for the next call
                    bcast[0] = last ? 1 : 0;
                    bcast[1] = c_lo;
                    bcast[2] = c_hi;
                }
                named_bar(1, P_EPI_WARPS * 32);
                if (bcast[0]) {
                    fence_acq_rel_gpu();
                    const int c_lo = bcast[1], c_hi = bcast[2];
                    // the tile's partials (this CTA's own included, from its
                    // slot) added in CTA order, whoever arrived last; 32
                    // columns at a time
#pragma unroll 1
                    for (int ch = 0; ch < P_CW; ch += 32) {
                        float acc[32];
                        // two contributors' loads in flight at a time, then
                        // their sums in CTA order
#pragma unroll 1
                        for (int c0 = c_lo; c0 <= c_hi; c0 += 2) {
                            float4 w[2][8];
#pragma unroll
                            for (int j = 0; j < 2; ++j) {
                                const int c = min(c0 + j, c_hi);           // a spare slot re-reads the last
                                const float4 *src = reinterpret_cast<const float4 *>(
                                                        g.part + static_cast<int64_t>(c) * P_SLOT_FLOATS +
                                                        wb * (32 * P_CW)) + (ch / 4) * 32 + lane;
#pragma unroll
                                for (int i = 0; i < 8; ++i) w[j][i] = __ldcg(src + i * 32);
                            }
#pragma unroll
                            for (int j = 0; j < 2; ++j) {
                                if (c0 + j > c_hi) continue;
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    if (c0 + j == c_lo) {
                                        acc[4 * i] = w[j][i].x; acc[4 * i + 1] = w[j][i].y;
                                        acc[4 * i + 2] = w[j][i].z; acc[4 * i + 3] = w[j][i].w;
                                    } else {
                                        acc[4 * i] += w[j][i].x; acc[4 * i + 1] += w[j][i].y;
                                        acc[4 * i + 2] += w[j][i].z; acc[4 * i + 3] += w[j][i].w;
                                    }
                                }
                            }
                        }
                        p_store_rows<EPI, 32>(g, mb * P_BM + 32 * q, n0, cw0 + ch, acc, stg, lane);
                    }
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_done);
    }
    // the role branches ran on one lane of warps 0 and 1: reconverge every
    // warp before the block-wide barrier
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    fr_pdl_trigger();
    if (warp == 1) {
        // free TMEM only once every epilogue warp has read its last
        // accumulator (bounded; the status word says if it gave up)
        if (lane == 0) mbar_wait(epi_done, 0, 45);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, P_TMEM_COLS);
    }
}

} // namespace frb
