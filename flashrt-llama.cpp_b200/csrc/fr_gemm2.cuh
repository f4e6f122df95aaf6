// fr_gemm2.cuh -- the W4A4 prefill GEMM on SM pairs (tcgen05 cta_group::2).
//
// Same product as k_gemm_p (fr_gemm.cuh; the reference's gemm_f32out,
// src/fr_gemm_f32out.cu:189-205, whose large-M configuration is also a 2-SM
// tile): D = alpha * A . B^T with A [M, K] and B [N, K] in the packed E2M1
// layout and UE4M3 scale atoms of fr_repack_weight / fr_quantize_act_f32.
//
// A cluster of two CTAs computes one 256 x 256 tile.  CTA r (rank in the
// pair) loads rows [128 r, 128 r + 128) of the tile's A panel and of its B
// panel, its A rows' scale atoms and all 256 B rows' scale atoms; one thread
// of CTA 0 issues `tcgen05.mma.cta_group::2` (M = 256, N = 256, K = 64), which
// reads A and B from both CTAs' shared memory and accumulates rows
// [128 r, 128 r + 128) x 256 columns in CTA r's TMEM.  Against the one-SM
// 128 x 256 tile each SM streams a third fewer operand bytes per MMA
// (16 + 16 KB per K stage instead of 16 + 32 KB), and the 38 KB stages leave
// room for the epilogue's store buffers.
//
// Pipeline per K stage (5 stages: a stage's loads take ~1.5 us to land while
// every SM streams, and four stages left the MMA waiting):
//   producer (warp 0 of each CTA): waits its own `empty`, then five TMA loads
//     (A rows, B rows, A scales, B scales x 2) whose completion counts on
//     CTA 0's `full` barrier (the `.cta_group::2` form of the tensor load
//     signals the pair's barrier); CTA 0's producer arms it with both CTAs'
//     bytes;
//   scale copiers (warps 2, 3 of CTA 0, six atoms each per stage, so a
//     stage's scales reach TMEM in half the time one thread takes):
//     `tcgen05.cp.cta_group::2` of the stage's scale atoms into both CTAs'
//     TMEM columns for the stage, then `sf_ready` (two arrivals);
//   MMA (warp 1 of CTA 0): four MMAs, then a commit that arrives on `empty`
//     in both CTAs; after a tile's last stage a commit to both `acc_full`.
// Epilogue (warps 4..11 of each CTA): TMEM -> registers, the accumulator is
// released to CTA 0's MMA thread (`acc_empty` counts the 16 epilogue warps
// of the pair), then the rows leave through a 32 x 32 f32 box in shared
// memory per warp (128-byte swizzle) with TMA tensor stores, whole 128-byte
// lines and no per-thread global stores.
//
// Every wait is bounded (status word + site on expiry).  The cluster is
// synchronised after barrier initialisation (the peer signals CTA 0's
// barriers) and before TMEM is freed.  Each CTA loads only its own operands
// from this GPU's memory; the tcgen05.commit that releases a stage is the
// one operation that reaches both CTAs' barriers.
#pragma once

#include "fr_gemm.cuh"

namespace frb {

constexpr int C2_STAGES = 5;
constexpr int C2_A = 128 * 128;                              // 128 rows x 256 values, E2M1
constexpr int C2_B = 128 * 128;
constexpr int C2_SFA = 4 * 512;                              // 4 K blocks x 1 atom (this CTA's rows)
constexpr int C2_SFB = 8 * 512;                              // 2 row halves x 4 K blocks (all 256 B rows)
constexpr int C2_STAGE = C2_A + C2_B + C2_SFA + C2_SFB;      // 38 KB (1024-aligned)
constexpr int C2_STG = 32 * 32 * 4;                          // per epilogue warp: one 32 x 32 f32 box
constexpr size_t C2_SMEM = 1024 + static_cast<size_t>(C2_STAGES) * C2_STAGE +
                           static_cast<size_t>(P_EPI_WARPS) * C2_STG + 256;

struct C2Args {
    int M, N, K;
    int nkt;                     // K stages of 256
    int kb_total;                // 64-value K blocks (scale atoms per 128-row block)
    int n_m2, n_n2, tiles;       // 256 x 256 tiles
    int split;                   // 1, or 2: two K halves per tile on two clusters
    float alpha;
    float *part;                 // split 2: hand-off halves [tiles][2][2][4][32 x 128] f32
    unsigned int *counter;       // split 2: [tiles][2][2][4] flags, zero between launches
};

// ------------------------------------------------------------ pair helpers
__device__ __forceinline__ uint32_t c2_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of `local` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t c2_mapa(const void *local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
__device__ __forceinline__ void c2_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void c2_arrive_remote(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(cl_addr) : "memory");
}
// bounded wait with cluster-scope acquire (arrivals from the peer CTA)
__device__ __forceinline__ bool c2_wait(uint64_t *bar, uint32_t parity, unsigned site) {
    auto try1 = [&]() -> bool {
        uint32_t ok;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
        return ok != 0;
    };
    if (try1()) return true;
    const uint64_t t0 = fr_now_ns();
    for (uint32_t i = 0;; ++i) {
        if (try1()) return true;
        if ((i & 63) == 0 && fr_now_ns() - t0 > g_fr_wait_ns) {
            fr_flag(FR_ST_TIMEOUT | (site << FR_ST_SITE_SHIFT));
            return false;
        }
    }
}
__device__ __forceinline__ void c2_tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void c2_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// scale atom (32 rows x 128 bits, broadcast to the four lane quadrants) from
// each CTA's shared memory into its own TMEM
__device__ __forceinline__ void c2_cp_sf(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" :: "r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void c2_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}
// arrive on this CTA's `bar` once this thread's tcgen05 operations are done
__device__ __forceinline__ void c2_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}
// ... on `bar` at the same offset in both CTAs of the pair
__device__ __forceinline__ void c2_commit_pair(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(smem_u32(bar)), "h"(static_cast<uint16_t>(3)) : "memory");
}
// tensor load into this CTA's shared memory, completion counted on the
// pair's barrier at cluster address `bar_cl` (CTA 0's)
__device__ __forceinline__ void c2_load(void *dst, const CUtensorMap *map, int x, int y, uint32_t bar_cl) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cl) : "memory");
}
__device__ __forceinline__ void c2_store(const CUtensorMap *map, int x, int y, const void *src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(src)) : "memory");
}
__device__ __forceinline__ void c2_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void c2_store_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void c2_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One 32 x 32 box of this warp's rows (lane = row) through a staging
// buffer: when the buffer is reused, lane 0 first lets the previous box's
// store finish reading it; every lane writes its row (128-byte swizzle: 16-byte chunk i of row r at
// chunk i ^ (r & 7), conflict-free), then lane 0 issues the tensor store of
// the box at (column x, row y).
__device__ __forceinline__ void c2_box_store(const CUtensorMap *tmD, uint8_t *stg, int &nbox, const float *v, int x,
                                             int y, int lane, bool reuse) {
    uint8_t *sb = stg;
    if (reuse && lane == 0) c2_store_wait_read0();
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4 *>(sb + lane * 128 + ((i ^ (lane & 7)) << 4)) =
            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
        c2_store(tmD, x, y, sb);
        c2_store_commit();
    }
    ++nbox;
}

// Work unit u of a launch: tile u / split, K stages [kh nkt / split,
// (kh + 1) nkt / split) with kh = u % split
struct C2Unit {
    int mt, nt, kh, kt0, kt1;
};
__device__ __forceinline__ C2Unit c2_unit(const C2Args &g, int u) {
    C2Unit w;
    const int t = u / g.split;
    w.kh = u % g.split;
    w.mt = t % g.n_m2;
    w.nt = t / g.n_m2;
    w.kt0 = w.kh * g.nkt / g.split;
    w.kt1 = (w.kh + 1) * g.nkt / g.split;
    return w;
}

// Two-way K split (split = 2, one unit per cluster, both halves of a tile in
// flight together): the unit with K half kh finishes accumulator columns
// [128 kh, 128 kh + 128) of its rows and hands the other 128 columns to its
// partner through `part` ([tile][rank][column half][quadrant][32 rows x 128]
// f32, written as 512-byte lines); per (tile, rank, half, quadrant) a flag
// counts the hand-off and the receiving warp resets it.  a + b = b + a in
// fp32, so the result does not depend on which unit finishes first.
__device__ __forceinline__ float *c2_part(const C2Args &g, int t, int rank, int h, int q) {
    return g.part + ((((static_cast<int64_t>(t) * 2 + rank) * 2 + h) * 4 + q) * (32 * 128));
}

template <int EPI>
__global__ void __launch_bounds__(P_THREADS, 1) k_gemm_c2(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB,
                                                         const __grid_constant__ CUtensorMap tmSFA,
                                                         const __grid_constant__ CUtensorMap tmSFB,
                                                         const __grid_constant__ CUtensorMap tmD, const C2Args g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *stg_all = smem + C2_STAGES * C2_STAGE;
    uint64_t *full = reinterpret_cast<uint64_t *>(stg_all + P_EPI_WARPS * C2_STG);
    uint64_t *empty = full + C2_STAGES;
    uint64_t *sf_ready = empty + C2_STAGES;
    uint64_t *acc_full = sf_ready + C2_STAGES;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *epi_done = acc_empty + 1;
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(epi_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = c2_rank();
    const bool lead = rank == 0;
    const int cl = static_cast<int>(blockIdx.x >> 1), ncl = static_cast<int>(gridDim.x >> 1);
    const int units = g.tiles * g.split;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C2_STAGES; ++s) {
            mbar_init(&full[s], 1);                          // CTA 0's producer (armed with both CTAs' bytes)
            mbar_init(&empty[s], 1);                         // the MMA thread's commit
            mbar_init(&sf_ready[s], 2);                      // both copier threads
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * P_EPI_WARPS);               // the pair's epilogue warps
        mbar_init(epi_done, P_EPI_WARPS);
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmSFA);
        tma_prefetch_desc(&tmSFB);
        tma_prefetch_desc(&tmD);
    }
    if (warp == 1) c2_tmem_alloc(tmem_s, P_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    c2_cluster_sync();                                       // the peer's barriers exist before any signal
    tc_fence_after();
    const uint32_t tbase = *tmem_s;
    fr_pdl_wait();                                           // A comes from the previous kernel

    if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 40;" ::: "memory");
    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer (both CTAs)
            int64_t it = 0;
            bool ok = true;
            for (int u = cl; ok && u < units; u += ncl) {
                const C2Unit w = c2_unit(g, u);
                const int arow = w.mt * 256 + 128 * static_cast<int>(rank);
                const int brow = w.nt * 256 + 128 * static_cast<int>(rank);
                const int sfa_y = (2 * w.mt + static_cast<int>(rank)) * g.kb_total;
                const int sfb_y0 = (2 * w.nt) * g.kb_total, sfb_y1 = (2 * w.nt + 1) * g.kb_total;
                for (int kt = w.kt0; kt < w.kt1; ++kt, ++it) {
                    const int s = static_cast<int>(it % C2_STAGES);
                    if (it >= C2_STAGES &&
                        !mbar_wait(&empty[s], static_cast<uint32_t>((it / C2_STAGES) - 1) & 1u, 80)) {
                        ok = false;
                        break;
                    }
                    if (lead) mbar_expect_tx(&full[s], 2 * C2_STAGE);
                    const uint32_t bar = c2_mapa(&full[s], 0);
                    uint8_t *st = smem + s * C2_STAGE;
                    c2_load(st, &tmA, kt * 128, arow, bar);
                    c2_load(st + C2_A, &tmB, kt * 128, brow, bar);
                    c2_load(st + C2_A + C2_B, &tmSFA, 0, sfa_y + 4 * kt, bar);
                    c2_load(st + C2_A + C2_B + C2_SFA, &tmSFB, 0, sfb_y0 + 4 * kt, bar);
                    c2_load(st + C2_A + C2_B + C2_SFA + 2048, &tmSFB, 0, sfb_y1 + 4 * kt, bar);
                }
            }
            // CTA 0 sees every stage land (its MMA thread consumes them all);
            // the peer's loads complete on CTA 0's barriers before CTA 0's
            // MMA thread passes them, which the final cluster sync orders
            if (lead)
                for (int64_t j = it > C2_STAGES ? it - C2_STAGES : 0; j < it; ++j)
                    mbar_wait(&full[j % C2_STAGES], static_cast<uint32_t>(j / C2_STAGES) & 1u, 81);
        }
    } else if (warp == 1) {
        if (lane == 0 && lead) {
            // ---------------- MMA issuer (CTA 0)
            const uint32_t idesc = idesc_nvf4(256, 256);
            int64_t it = 0;
            int seg = 0;
            bool ok = true;
            for (int u = cl; u < units; u += ncl, ++seg) {
                const C2Unit w = c2_unit(g, u);
                if (seg > 0 && ok) {
                    ok = c2_wait(acc_empty, static_cast<uint32_t>(seg - 1) & 1u, 82);
                    tc_fence_after();
                }
                for (int kt = w.kt0; kt < w.kt1 && ok; ++kt, ++it) {
                    const int s = static_cast<int>(it % C2_STAGES);
                    if (!mbar_wait(&sf_ready[s], static_cast<uint32_t>(it / C2_STAGES) & 1u, 83)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint8_t *st = smem + s * C2_STAGE;
                    const uint32_t a_addr = smem_u32(st), b_addr = smem_u32(st + C2_A);
                    const uint32_t t_sfa = tbase + 256 + static_cast<uint32_t>(s) * 48, t_sfb = t_sfa + 16;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        c2_mma(tbase, sdesc_sw128(a_addr + 32 * j), sdesc_sw128(b_addr + 32 * j), idesc, t_sfa + 4 * j,
                               t_sfb + 8 * j, (kt > w.kt0 || j > 0) ? 1u : 0u);
                    c2_commit_pair(&empty[s]);
                }
                // always signal the unit, so no epilogue waits on an issuer
                // that gave up (the status word says so)
                c2_commit_pair(acc_full);
            }
        }
    } else if (warp == 2 || warp == 3) {
        if (lane == 0 && lead) {
            // ---------------- scale-factor copiers (CTA 0): copier 0 the
            // A atoms and B half 0's first two, copier 1 the other six
            const int cid = warp - 2;
            int64_t it = 0;
            bool ok = true;
            for (int u = cl; ok && u < units; u += ncl) {
                const C2Unit w = c2_unit(g, u);
                for (int kt = w.kt0; kt < w.kt1; ++kt, ++it) {
                    const int s = static_cast<int>(it % C2_STAGES);
                    if (!mbar_wait(&full[s], static_cast<uint32_t>(it / C2_STAGES) & 1u, 84)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sfa_addr = smem_u32(smem + s * C2_STAGE + C2_A + C2_B);
                    const uint32_t sfb_addr = sfa_addr + C2_SFA;
                    const uint32_t t_sfa = tbase + 256 + static_cast<uint32_t>(s) * 48, t_sfb = t_sfa + 16;
                    if (cid == 0) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) c2_cp_sf(t_sfa + 4 * j, sdesc_plain(sfa_addr + 512 * j, 128));
#pragma unroll
                        for (int j = 0; j < 2; ++j) c2_cp_sf(t_sfb + 8 * j, sdesc_plain(sfb_addr + 512 * j, 128));
                    } else {
#pragma unroll
                        for (int j = 2; j < 4; ++j) c2_cp_sf(t_sfb + 8 * j, sdesc_plain(sfb_addr + 512 * j, 128));
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            c2_cp_sf(t_sfb + 8 * j + 4, sdesc_plain(sfb_addr + 2048 + 512 * j, 128));
                    }
                    c2_commit(&sf_ready[s]);
                }
            }
        }
    } else {
        // ---------------- epilogue warps 4..11 (both CTAs)
        asm volatile("setmaxnreg.inc.sync.aligned.u32 232;" ::: "memory");
        const int q = warp & 3;                              // TMEM lane quadrant
        const int ch = (warp - 4) >> 2;                      // accumulator column half
        const uint32_t acc_empty_cl = c2_mapa(acc_empty, 0);
        int nbox = 0, seg = 0;
        for (int u = cl; u < units; u += ncl, ++seg) {
            const C2Unit w = c2_unit(g, u);
            const int t = u / g.split;
            // the last unit's boxes go through the operand ring, idle by then
            // (four boxes per warp, no wait between them); earlier ones
            // through the warp's own box buffer while the next unit streams
            const bool last = u + ncl >= units;
            uint8_t *stg = last ? smem + (warp - 4) * (4 * 4096) : stg_all + (warp - 4) * C2_STG;
            const bool ok = c2_wait(acc_full, static_cast<uint32_t>(seg) & 1u, 85);
            tc_fence_after();
            uint32_t r[P_CW];
            if (ok) {
                const uint32_t ta = tbase + (static_cast<uint32_t>(32 * q) << 16) + 128 * ch;
#pragma unroll
                for (int c = 0; c < P_CW / 32; ++c) tmem_ld32_async(ta + 32 * c, r + 32 * c);
#pragma unroll
                for (int c = 0; c < P_CW / 32; ++c) tmem_ld_wait_dep(r + 32 * c);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) c2_arrive_remote(acc_empty_cl);  // the accumulator may be overwritten
            if (!ok) break;
            float *v = reinterpret_cast<float *>(r);
            if (g.split == 2) {
                float4 *mine = reinterpret_cast<float4 *>(c2_part(g, t, static_cast<int>(rank), ch, q)) + lane;
                unsigned int *flag = g.counter + ((static_cast<int64_t>(t) * 2 + rank) * 2 + ch) * 4 + q;
                if (ch != w.kh) {
                    // hand these 128 columns to the partner unit
#pragma unroll
                    for (int i = 0; i < 32; ++i) mine[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    fence_acq_rel_gpu();
                    __syncwarp();
                    if (lane == 0) atomicAdd(flag, 1u);
                    continue;
                }
                // finish them: wait (bounded) for the partner's half, add
                int got = 0;
                if (lane == 0) {
                    const uint64_t t0 = fr_now_ns();
                    for (;;) {
                        unsigned int fv;
                        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(fv) : "l"(flag) : "memory");
                        if (fv != 0u) { got = 1; break; }
                        if (fr_now_ns() - t0 > g_fr_wait_ns) {
                            fr_flag(FR_ST_TIMEOUT | (87u << FR_ST_SITE_SHIFT));
                            break;
                        }
                    }
                    if (got) *flag = 0u;                     // nobody else touches it before the next launch
                }
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) break;
                fence_acq_rel_gpu();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float4 o = __ldcg(mine + i * 32);
                    v[4 * i] += o.x;
                    v[4 * i + 1] += o.y;
                    v[4 * i + 2] += o.z;
                    v[4 * i + 3] += o.w;
                }
            }
            const int row = w.mt * 256 + 128 * static_cast<int>(rank) + 32 * q;
            if (EPI == P_SWIGLU) {
                // (gate, up) column pairs -> silu(gate) * up, 64 outputs
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        float up = v[64 * c + 2 * i + 1] * g.alpha;
                        const float gate = v[64 * c + 2 * i] * g.alpha;
                        up *= silu_f(gate);
                        o[i] = up;
                    }
                    const int x = w.nt * 128 + 64 * ch + 32 * c;
                    if (row < g.M && x < g.N / 2)
                        c2_box_store(&tmD, last ? stg + c * 4096 : stg, nbox, o, x, row, lane, !last);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = v[32 * c + i] * g.alpha;
                    const int x = w.nt * 256 + 128 * ch + 32 * c;
                    if (row < g.M && x < g.N)
                        c2_box_store(&tmD, last ? stg + c * 4096 : stg, nbox, o, x, row, lane, !last);
                }
            }
        }
        if (lane == 0) c2_store_wait_all();                  // every box written before the CTA leaves
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_done);
    }
    __syncwarp();
    if (warp == 1) mbar_wait(epi_done, 0, 86);             // this CTA's TMEM reads are done
    tc_fence_before();
    __syncwarp();
    c2_cluster_sync();                                       // and the peer's; no operand still in flight
    fr_pdl_trigger();
    if (warp == 1) {
        tc_fence_after();
        c2_tmem_dealloc(tbase, P_TMEM_COLS);
    }
}

} // namespace frb
