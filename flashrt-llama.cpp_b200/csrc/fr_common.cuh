// fr_common.cuh -- shared device helpers for the B200 NVFP4 x q8_1 kernels.
//
// Formats (ggml's, read in place, never repacked on the GEMV path):
//   block_nvfp4: 36 B per 64 elements = d[4] (one UE4M3 per 16 elements,
//                ggml decode halves it) + qs[32] (sub-block s in qs[8s..8s+7],
//                byte j = elem j low nibble, elem j+8 high nibble), the values
//                being kvalues_mxfp4 = 2 * E2M1.
//                Reference: src/fr_repack.cu:4-10, include/fr_kernels.h:13-15.
//   block_q8_1 : 36 B per 32 elements = half2 ds (d, sum) + int8 qs[32].
//                Reference: src/fr_win_flint_batched.cuh:400-408.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <cfloat>

#include "../../include/fr_b200.h"

namespace frb {

constexpr int NV_BYTES = 36;   // block_nvfp4
constexpr int NV_ELEMS = 64;
constexpr int Q8_BYTES = 36;   // block_q8_1
constexpr int Q8_ELEMS = 32;

// ---------------------------------------------------------------- status
// Device-side status word: bounded waits that give up OR a code into it and
// return instead of hanging or trapping.  The host reads it with
// fr_device_status().  (The library is one translation unit, so the
// definition lives here.)
__device__ unsigned int g_fr_status = 0;

constexpr unsigned FR_ST_TIMEOUT   = 0x1u;      // a bounded wait ran out
constexpr unsigned FR_ST_BADINPUT  = 0x2u;      // an index/route outside its range was skipped
constexpr unsigned FR_ST_SITE_SHIFT = 8;        // site id of the first timeout

__device__ __forceinline__ void fr_flag(unsigned bits) { atomicOr(&g_fr_status, bits); }

// nanoseconds since an arbitrary epoch (%globaltimer)
__device__ __forceinline__ uint64_t fr_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every spin in these kernels gives up after g_fr_wait_ns nanoseconds
// (kernels run for microseconds; the bound only matters when something is
// broken).  2 s unless fr_set_wait_ns shortened it.
constexpr uint64_t FR_WAIT_NS_MAX = 2000000000ull;
__device__ unsigned long long g_fr_wait_ns = FR_WAIT_NS_MAX;

// ---------------------------------------------------------------- PDL
// GPU-scope acquire/release fence: with a relaxed atomic it forms the
// release (writer) and acquire (reader) halves of a message hand-off, which
// is all the stream-K partial sums need (lighter than a sequentially
// consistent fence).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fr_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void fr_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- smem / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or ~the hint elapses, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
// Bounded wait on phase `parity`: false (and the status word flagged with
// `site`) when the phase did not complete within g_fr_wait_ns.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned site) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = fr_now_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 63) == 0 && fr_now_ns() - t0 > g_fr_wait_ns) {
            fr_flag(FR_ST_TIMEOUT | (site << FR_ST_SITE_SHIFT));
            return false;
        }
    }
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast);
// completion counted in bytes on `bar`.  16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- number formats
// prmt in its generic mode: selector nibble bit 3 set -> sign-replicate the
// selected byte.  Used with an all-positive table so that a negative E2M1
// code (bit 3 set) selects 0.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// |kvalues_mxfp4| for codes 0..7: {0,1,2,3,4,6,8,12}
constexpr uint32_t KV_LO = 0x03020100u;
constexpr uint32_t KV_HI = 0x0C080604u;

// Decode one qs word (8 codes: bytes c0..c3, low and high nibbles) into four
// byte vectors for dp4a: for each 16-bit half h the output bytes are, in
// order, the codes of nibbles 0..3 of that half, i.e. elements
// (j, j+8, j+1, j+9) with j = 4i + 2h for qs word i of a sub-block.
//   pos[h] = |kv| where the code is non-negative, else 0
//   neg[h] = |kv| where the code is negative, else 0
// so that  sum kv*a = dp4a(pos, a) - dp4a(neg, a).
struct nv_word { uint32_t p0, p1, n0, n1; };
__device__ __forceinline__ nv_word nv_decode(uint32_t w) {
    const uint32_t x = w ^ 0x88888888u;
    nv_word r;
    r.p0 = prmt(KV_LO, KV_HI, w);
    r.p1 = prmt(KV_LO, KV_HI, w >> 16);
    r.n0 = prmt(KV_LO, KV_HI, x);
    r.n1 = prmt(KV_LO, KV_HI, x >> 16);
    return r;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// Four UE4M3 scale bytes -> floats with ggml's semantics up to a factor 2:
// standard e4m3 magnitude (sign bit ignored), codes 0x7F/0xFF -> 0.  The
// caller folds ggml's 1/2 into the activation scale (exact).
__device__ __forceinline__ void ue4m3x4(uint32_t d, float out[4]) {
    const uint32_t m = d & 0x7F7F7F7Fu;
    uint32_t h01, h23;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(static_cast<unsigned short>(m & 0xFFFFu)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(static_cast<unsigned short>(m >> 16)));
    const __half2 a = *reinterpret_cast<const __half2 *>(&h01);
    const __half2 b = *reinterpret_cast<const __half2 *>(&h23);
    // 0x7F decodes to NaN in e4m3; fmaxf(NaN, 0) = 0 matches ggml's zero.
    out[0] = fmaxf(__low2float(a), 0.0f);
    out[1] = fmaxf(__high2float(a), 0.0f);
    out[2] = fmaxf(__low2float(b), 0.0f);
    out[3] = fmaxf(__high2float(b), 0.0f);
}

// q8_1 of one 32-value chunk, lane = element: amax and the xor-butterfly
// sum, d = amax/127 and q = roundf(x/d) with IEEE division, ds = half2(d, sum)
// (reference frt_q8_1_chunk, src/fr_win_flint_sm120.cu:289-300).
struct q8_lane { int8_t q; float d; float sum; };
__device__ __forceinline__ q8_lane q8_1_chunk(float xi) {
    float amax = fabsf(xi);
    float sum = xi;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
    }
    const float d = __fdiv_rn(amax, 127.0f);
    q8_lane r;
    r.q = amax == 0.0f ? static_cast<int8_t>(0) : static_cast<int8_t>(roundf(__fdiv_rn(xi, d)));
    r.d = d;
    r.sum = sum;
    return r;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

} // namespace frb
