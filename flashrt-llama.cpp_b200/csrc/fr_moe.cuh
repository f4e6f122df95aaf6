// fr_moe.cuh -- MoE routing, token permute, expert-grouped matvec, combine.
//
//   k_route         : one launch for the router logits (f32), the softmax
//                     top-k per token (one warp per token, the reference's
//                     algorithm, src/fr_win_qwen36_sm120.cu:1826-1870) and the
//                     token permute eoff/slots/act (src/fr_win_flint_batched_
//                     moe.cuh:76-166), chained by last-arriver counters, plus
//                     the experts' activation input in extra CTAs.  Slots inside
//                     an expert are in slot order, so the grouping is
//                     deterministic (the reference's atomics leave it
//                     unspecified).
//   k_group_ids     : the same permute for ids given by the caller (mul_mat_id)
//   k_moe_gemv      : CTA = (active expert, row chunk).  The chunk's weight rows
//                     are bulk-copied into shared memory once and stay resident
//                     while the expert's tokens pass through in windows of TT,
//                     so every used expert's rows are read from HBM once per
//                     call, whatever the number of tokens routed to it.
//   k_moe_combine   : out[t] = sum_k part[t,k] * w[t,k] in slot order (+ resid)
//                     (src/fr_win_flint_batched_moe.cuh:342-379).
#pragma once

#include "fr_gemv.cuh"
#include "fr_fp4mv.cuh"

namespace frb {

constexpr int MOE_MAX_E = 256;
constexpr int MOE_MAX_USED = 32;
constexpr int MOE_MAX_SLOTS = 8192;   // T * n_used handled by the single-CTA permute

// ------------------------------------------------------------ router tile
// logits[t, e] for 4 experts x 4 tokens (e0, t0), fp32, by 256 threads
__device__ __forceinline__ void router_tile(const float *__restrict__ x, int64_t ldx, const float *__restrict__ wr,
                                            float *__restrict__ logits, int T, int K, int E, int e0, int t0) {
    __shared__ float red[8][16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float acc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[r][u] = 0.0f;
    for (int k = tid * 4; k < K; k += 256 * 4) {
        float4 wv[4], xv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            wv[r] = (e0 + r < E) ? *reinterpret_cast<const float4 *>(wr + static_cast<int64_t>(e0 + r) * K + k)
                                 : make_float4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            xv[u] = (t0 + u < T) ? *reinterpret_cast<const float4 *>(x + static_cast<int64_t>(t0 + u) * ldx + k)
                                 : make_float4(0, 0, 0, 0);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int u = 0; u < 4; ++u)
                acc[r][u] += wv[r].x * xv[u].x + wv[r].y * xv[u].y + wv[r].z * xv[u].z + wv[r].w * xv[u].w;
    }
    // warp sums of the tile's real tokens only (T = 1: 4 of the 16)
    const int nu = min(4, T - t0);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (u >= nu) continue;
            float v = acc[r][u];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) red[warp][r * 4 + u] = v;
        }
    __syncthreads();
    if (tid < 16 && (tid & 3) < nu) {
        const int r = tid >> 2, u = tid & 3;
        float v = red[0][tid];
#pragma unroll
        for (int w = 1; w < 8; ++w) v += red[w][tid];
        if (e0 + r < E && t0 + u < T) logits[static_cast<int64_t>(t0 + u) * E + e0 + r] = v;
    }
}

// ------------------------------------------------------------ top-k
// Softmax top-k of a token, the reference's algorithm
// (src/fr_win_qwen36_sm120.cu:1826-1870): softmax in fp32, n_used rounds of
// warp argmax (ties -> lower id), weights renormalised by max(sum, clamp).
// The rounds are restated as ranks: expert e is picked in round r when r
// probabilities beat it (higher, or equal with a lower id), so every thread
// of the CTA counts the rank of one (token, expert) pair at once instead of
// one warp running n_used dependent shuffle butterflies.  The float
// operations that fix the weights' bits keep the reference's order: the
// softmax as one warp per token, then each lane adds its own winners in
// round order and the warp sums those partials with the same butterfly.

// phase 1, one warp per token: probabilities into p[0, E) (NaN -> -FLT_MAX).
// Logits are read through L2 (other CTAs wrote them).
__device__ __forceinline__ void topk_softmax(const float *__restrict__ l, int E, float *__restrict__ p) {
    const int lane = threadIdx.x & 31;
    const int per = E / 32;
    float wt[MOE_MAX_E / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        wt[i] = (i < per) ? __ldcg(l + lane + 32 * i) : -INFINITY;
        mx = fmaxf(mx, wt[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        if (i < per) {
            wt[i] = expf(wt[i] - mx);
            sum += wt[i];
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        if (i < per) {
            float v = wt[i] * inv;
            if (isnan(v)) v = -FLT_MAX;
            p[lane + 32 * i] = v;
        }
    }
}

// phase 2, every thread of the block: rank[u][e] for the nu tokens whose
// probabilities are p[u][0, E) (rows MOE_MAX_E apart, E a multiple of 32)
__device__ __forceinline__ void topk_ranks(const float *__restrict__ p, int *__restrict__ rank, int nu, int E) {
    for (int u = 0; u < nu; ++u) {
        const float *pu = p + u * MOE_MAX_E;
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            const float v = pu[e];
            int r = 0;
            for (int j = 0; j < E; j += 4) {
                const float4 q = *reinterpret_cast<const float4 *>(pu + j);
                r += (q.x > v || (q.x == v && j < e)) ? 1 : 0;
                r += (q.y > v || (q.y == v && j + 1 < e)) ? 1 : 0;
                r += (q.z > v || (q.z == v && j + 2 < e)) ? 1 : 0;
                r += (q.w > v || (q.w == v && j + 3 < e)) ? 1 : 0;
            }
            rank[u * MOE_MAX_E + e] = r;
        }
    }
}

// phase 3, one warp per token: ids_row[r] / w_row[r] for the n_used winners
// (n_used <= 32).  Lane L's partial adds its experts L + 32 i that won, in
// round order, as the rounds' `wsum += bv` on the winner's lane does.
__device__ __forceinline__ void topk_finish(const float *__restrict__ p, const int *__restrict__ rank, int E,
                                            int n_used, float clamp_val, int32_t *__restrict__ ids_row,
                                            float *__restrict__ w_row) {
    const int lane = threadIdx.x & 31;
    const int per = E / 32;
    int rk[MOE_MAX_E / 32];
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) rk[i] = (i < per) ? rank[lane + 32 * i] : E;
    float wsum = 0.0f;
    for (int r = 0; r < n_used; ++r) {
#pragma unroll
        for (int i = 0; i < MOE_MAX_E / 32; ++i)
            if (rk[i] == r) wsum += p[lane + 32 * i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, off);
    wsum = fmaxf(wsum, clamp_val);
    const float invs = 1.0f / wsum;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        if (rk[i] < n_used) {
            ids_row[rk[i]] = lane + 32 * i;
            w_row[rk[i]] = p[lane + 32 * i] * invs;
        }
    }
}

// The rounds themselves, one warp per token: the form for chunks of 2..4
// tokens, whose four warps run their rounds side by side (there the CTA-wide
// rank counting measured slower: MoE layer at T=64 108.7 -> 117.7 us).
__device__ __forceinline__ void topk_token(const float *__restrict__ l, int E, int n_used, float clamp_val,
                                           int32_t *__restrict__ ids_row, float *__restrict__ w_row) {
    const int lane = threadIdx.x & 31;
    const int per = E / 32;
    float wt[MOE_MAX_E / 32];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        wt[i] = (i < per) ? __ldcg(l + lane + 32 * i) : -INFINITY;
        mx = fmaxf(mx, wt[i]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        if (i < per) {
            wt[i] = expf(wt[i] - mx);
            sum += wt[i];
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < MOE_MAX_E / 32; ++i) {
        if (i < per) {
            wt[i] *= inv;
            if (isnan(wt[i])) wt[i] = -FLT_MAX;
        } else {
            wt[i] = -INFINITY;
        }
    }
    float wsum = 0.0f, outw = 0.0f;
    for (int k = 0; k < n_used; ++k) {
        float bv = wt[0];
        int be = lane;
#pragma unroll
        for (int i = 1; i < MOE_MAX_E / 32; ++i) {
            if (wt[i] > bv) { bv = wt[i]; be = lane + 32 * i; }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, bv, off);
            const int e = __shfl_xor_sync(0xffffffffu, be, off);
            if (v > bv || (v == bv && e < be)) { bv = v; be = e; }
        }
        if ((be & 31) == lane) {
#pragma unroll
            for (int i = 0; i < MOE_MAX_E / 32; ++i)
                if (i == (be >> 5)) wt[i] = -INFINITY;
            wsum += bv;
        }
        if (k == lane) outw = bv;
        if (lane == 0) ids_row[k] = be;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, off);
    wsum = fmaxf(wsum, clamp_val);
    const float invs = 1.0f / wsum;
    if (lane < n_used) w_row[lane] = outw * invs;
}

// ------------------------------------------------------------ permute
// exclusive prefix sum over the block (any multiple of 32 threads); `scratch`
// holds 33 ints; returns the block total through *total
__device__ __forceinline__ int block_excl_scan(int v, int *scratch, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
    }
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? scratch[lane] : 0;
        int wi = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, wi, off);
            if (lane >= off) wi += o;
        }
        if (lane < nw) scratch[lane] = wi - w;
        if (lane == 31) scratch[32] = wi;
    }
    __syncthreads();
    const int r = scratch[warp] + inc - v;
    *total = scratch[32];
    __syncthreads();
    return r;
}

// Stable grouping of S slots by expert (get(s) = expert of slot s, or -1 for
// no expert) into eoff[E+1], slots[] (each expert's slots in slot order) and
// act[E+1] (active experts ascending, -1 padded, count at act[E]): the token
// permute of src/fr_win_flint_batched_moe.cuh:76-166, deterministic.  Each
// warp owns a contiguous run of slots and walks it 32 at a time; lanes of
// one expert find each other with __match_any_sync, so the cost is
// O(S / threads) per thread.  cnt holds (blockDim / 32) * E ints; scratch 33.
// E <= blockDim.  Every thread of the block calls it.
template <typename F>
__device__ __forceinline__ void group_slots_warp(F get, int S, int E, int32_t *__restrict__ eoff,
                                                 int32_t *__restrict__ slots, int32_t *__restrict__ act, int *cnt,
                                                 int *scratch) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int per = ((S + nw - 1) / nw + 31) & ~31;
    const int lo = warp * per, hi = min(S, lo + per);
    for (int i = tid; i < nw * E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int base = lo; base < hi; base += 32) {
        const int sl = base + lane;
        const int e = sl < hi ? get(sl) : -1;
        const unsigned m = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && lane == __ffs(m) - 1) cnt[warp * E + e] += __popc(m);
    }
    __syncthreads();
    // per expert: running offsets over the warps, then the block scan
    int tot = 0;
    if (tid < E) {
        for (int w = 0; w < nw; ++w) {
            const int c = cnt[w * E + tid];
            cnt[w * E + tid] = tot;
            tot += c;
        }
    }
    int n_slot = 0, n_act = 0;
    const int off = block_excl_scan(tot, scratch, &n_slot);
    const int rank = block_excl_scan(tot > 0 ? 1 : 0, scratch, &n_act);
    if (tid < E) {
        eoff[tid] = off;
        if (tot > 0) act[rank] = tid;
        for (int w = 0; w < nw; ++w) cnt[w * E + tid] += off;
    }
    if (tid == 0) {
        eoff[E] = n_slot;
        act[E] = n_act;
    }
    for (int i = n_act + tid; i < E; i += blockDim.x) act[i] = -1;
    __syncthreads();
    for (int base = lo; base < hi; base += 32) {
        const int sl = base + lane;
        const int e = sl < hi ? get(sl) : -1;
        const unsigned m = __match_any_sync(0xffffffffu, e);
        int pos = 0;
        if (e >= 0) pos = cnt[warp * E + e] + __popc(m & ((1u << lane) - 1u));
        __syncwarp();
        if (e >= 0) {
            slots[pos] = sl;
            if (lane == __ffs(m) - 1) cnt[warp * E + e] += __popc(m);
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------ fused routing
// One launch: router logits (4 experts x 4 tokens per CTA), softmax top-k of
// each 4-token chunk by the last of its CTAs to finish, the permute by the
// last chunk to finish (counters zero on entry, reset by the last arrivals,
// so graph replays need no reset), and -- in extra CTAs, independent of the
// routing -- the expert matvecs' activation input: q8_1 rows of x (aux 1) or
// its per-token FP4 digit images (aux 2).
struct RouteArgs {
    const float *x;
    int64_t ldx;
    const float *wr;
    int T, K, E, n_used;
    float clamp_val;
    float *logits;
    int32_t *ids;
    float *wts;
    int32_t *eoff, *slots, *act;
    unsigned int *cnt;           // [n_tc + 1]
    int n_rt;                    // router CTAs = (E / 4) * n_tc
    int aux;                     // 0 none, 1 q8_1, 2 FP4 images
    uint8_t *q8;                 // aux 1: [T][K / 32 blocks]
    int64_t ldq;
    uint8_t *img;                // aux 2: per token, t_stride bytes
    float *gtab;
    int64_t t_stride;
    int img_slices;
};

__global__ void __launch_bounds__(256) k_route(const RouteArgs a) {
    fr_pdl_wait();
    fr_pdl_trigger();
    extern __shared__ int sm_route[];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int b = blockIdx.x;
    if (b >= a.n_rt) {
        const int c = b - a.n_rt;
        if (a.aux == 1) {
            const int lane = tid & 31, nc = a.K / Q8_ELEMS;
            const int64_t blk_id = static_cast<int64_t>(c) * 8 + warp;
            if (blk_id >= static_cast<int64_t>(a.T) * nc) return;
            const int t = static_cast<int>(blk_id / nc), ch = static_cast<int>(blk_id % nc);
            const q8_lane r = q8_1_chunk(a.x[static_cast<int64_t>(t) * a.ldx + static_cast<int64_t>(ch) * Q8_ELEMS + lane]);
            uint8_t *blk = a.q8 + (t * a.ldq + ch) * Q8_BYTES;
            blk[4 + lane] = static_cast<uint8_t>(r.q);
            if (lane == 0) *reinterpret_cast<__half2 *>(blk) = __halves2half2(__float2half_rn(r.d), __float2half_rn(r.sum));
        } else if (a.aux == 2) {
            act_fp4_row(a.x, a.ldx, nullptr, 0, a.K, FM_DIGITS, a.img, nullptr, a.gtab, a.t_stride, c / a.img_slices,
                        c % a.img_slices, a.img_slices);
        }
        return;
    }
    const int n_ec = a.E / 4, n_tc = (a.T + 3) / 4;
    const int ec = b % n_ec, tc = b / n_ec;
    router_tile(a.x, a.ldx, a.wr, a.logits, a.T, a.K, a.E, ec * 4, tc * 4);
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.cnt[tc], 1u) == static_cast<unsigned>(n_ec - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // this chunk's tokens: warp u routes token 4 tc + u (probabilities and
    // ranks in the shared scratch the permute uses afterwards)
    const int t = tc * 4 + warp;
    const int nu = min(4, a.T - tc * 4);
    float *ps = reinterpret_cast<float *>(sm_route);                 // [4][MOE_MAX_E]
    int *rk = sm_route + 4 * MOE_MAX_E;                              // [4][MOE_MAX_E]
    if (nu == 1) {
        // one token (T = 1): its ranks counted by the whole CTA
        if (warp == 0) topk_softmax(a.logits + static_cast<int64_t>(t) * a.E, a.E, ps);
        __syncthreads();
        topk_ranks(ps, rk, 1, a.E);
        __syncthreads();
        if (warp == 0)
            topk_finish(ps, rk, a.E, a.n_used, a.clamp_val, a.ids + static_cast<int64_t>(t) * a.n_used,
                        a.wts + static_cast<int64_t>(t) * a.n_used);
    } else if (warp < nu) {
        topk_token(a.logits + static_cast<int64_t>(t) * a.E, a.E, a.n_used, a.clamp_val,
                   a.ids + static_cast<int64_t>(t) * a.n_used, a.wts + static_cast<int64_t>(t) * a.n_used);
    }
    __threadfence();
    __syncthreads();
    if (n_tc > 1) {
        // the permute needs every chunk's ids: the last chunk does it
        if (tid == 0) {
            a.cnt[tc] = 0;
            s_last = atomicAdd(&a.cnt[n_tc], 1u) == static_cast<unsigned>(n_tc - 1);
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
    } else if (tid == 0) {
        a.cnt[tc] = 0;
    }
    const int32_t *ids = a.ids;
    group_slots_warp([&](int s) { return __ldcg(ids + s); }, a.T * a.n_used, a.E, a.eoff, a.slots, a.act, sm_route,
                     sm_route + 8 * MOE_MAX_E);
    if (tid == 0 && n_tc > 1) a.cnt[n_tc] = 0;
}

// permute for caller-given ids [T, n_used] (row stride ids_ld); out-of-range
// ids are flagged in the status word and routed to no expert, except -1 when
// `skip_neg` is set (an empty slot of a fixed-capacity exchange).
__global__ void __launch_bounds__(1024) k_group_ids(const int32_t *__restrict__ ids, int64_t ids_ld, int T,
                                                    int n_used, int E, int32_t *__restrict__ eoff,
                                                    int32_t *__restrict__ slots, int32_t *__restrict__ act,
                                                    int skip_neg) {
    fr_pdl_wait();
    fr_pdl_trigger();
    extern __shared__ int sm_i[];
    auto get = [&](int s) {
        int e = ids[static_cast<int64_t>(s / n_used) * ids_ld + s % n_used];
        if (e < 0 || e >= E) e = -1;
        return e;
    };
    // flag bad ids once
    for (int s = threadIdx.x; s < T * n_used; s += blockDim.x) {
        const int e = ids[static_cast<int64_t>(s / n_used) * ids_ld + s % n_used];
        if ((e < 0 || e >= E) && !(skip_neg && e == -1)) fr_flag(FR_ST_BADINPUT);
    }
    group_slots_warp(get, T * n_used, E, eoff, slots, act, sm_i, sm_i + (blockDim.x >> 5) * E);
}

// ------------------------------------------------------------ grouped matvec
struct MoeParams {
    const uint8_t *w0, *w1;     // expert-major rows; w1 = up rows for the SwiGLU pair
    int64_t e_stride;           // bytes per expert
    int64_t w_ld;               // bytes per row
    int N, K;                   // rows per expert, row length
    const uint8_t *q8;          // q8_1 rows: token rows (bcast) or slot rows
    int64_t ldq;                // blocks per q8 row
    const float *xf;            // or f32 rows (same indexing), quantized to q8_1 while staged
    int64_t ldxf;
    int bcast, n_used, E;
    const int32_t *eoff, *slots, *act;
    const float *s0, *s1;       // per-expert scales [E] (nullable)
    float *out;                 // row of slot (t, k): out + t*ld_tok + k*ld_slot
    int64_t ld_tok, ld_slot;
    int rows_per_cta, chunks, rows_per_stage, slot_bytes, word_mode;
    // fused combine (plain form, slot rows packed [T][n_used][N]; c_out null
    // otherwise): the last CTA of a row chunk to finish, over the active
    // experts, writes c_out[t][rows] = sum_k out[t][k][rows] * c_wts[t][k]
    // (+ c_resid) -- k_moe_combine's arithmetic; c_cnt[chunk] zero on entry
    const float *c_wts, *c_resid;
    float *c_out;
    unsigned int *c_cnt;
    int c_T;
};

// out[t, r] of the slot-order combine (k ascending); shared by k_moe_combine
// and the fused form, so both round alike
__device__ __forceinline__ float moe_combine_value(const float *pt, const float *ws, int n_used, int64_t n_embd) {
    float sum = pt[0] * ws[0];
    for (int k = 1; k < n_used; ++k) sum += pt[static_cast<int64_t>(k) * n_embd] * ws[k];
    return sum;
}

template <int LG, int TT, bool DUAL>
__global__ void __launch_bounds__(GV_THREADS) k_moe_gemv(const MoeParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NB = p.K / NV_ELEMS;
    const int RS = p.rows_per_stage;
    __shared__ int tok_row[TT];       // q8 row per staged token
    __shared__ int out_off[TT];       // t*ld_tok + k*ld_slot
    bool bad = false;                 // a bounded wait of this warp gave up

    fr_pdl_wait();
    const int a = blockIdx.x / p.chunks, chunk = blockIdx.x % p.chunks;
    const int n_act = p.act[p.E];
    if (a >= n_act) return;
    const int e = p.act[a];
    const int s_begin = p.eoff[e], s_end = p.eoff[e + 1];
    const int r_begin = chunk * p.rows_per_cta;
    const int n_rows = min(p.N, r_begin + p.rows_per_cta) - r_begin;
    if (n_rows <= 0 || e < 0 || e >= p.E) return;
    const int n_st = (n_rows + RS - 1) / RS;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + 2048;
    int4 *act_q = reinterpret_cast<int4 *>(ring + static_cast<size_t>(n_st) * p.slot_bytes);
    float2 *act_d = reinterpret_cast<float2 *>(act_q + static_cast<size_t>(TT) * NB * 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < n_st; ++s) mbar_init(&full[s], p.word_mode ? 32 : 1);
        fence_mbar_init();
    }
    __syncthreads();
    const uint8_t *w0 = p.w0 + static_cast<int64_t>(e) * p.e_stride;
    const uint8_t *w1 = DUAL ? p.w1 + static_cast<int64_t>(e) * p.e_stride : nullptr;

    if (warp == GV_CWARPS) {
        // producer: every stage of this chunk into its own slot (no reuse)
        for (int i = 0; i < n_st; ++i) {
            const int rows = min(RS, n_rows - i * RS);
            const int64_t off = static_cast<int64_t>(r_begin + i * RS) * p.w_ld;
            uint8_t *dst = ring + static_cast<size_t>(i) * p.slot_bytes;
            if (p.word_mode) {
                const int wpr = static_cast<int>(p.w_ld / 4);
                uint32_t *d32 = reinterpret_cast<uint32_t *>(dst);
                const uint32_t *a0 = reinterpret_cast<const uint32_t *>(w0 + off);
                for (int k = lane; k < rows * wpr; k += 32) d32[k] = __ldg(a0 + k);
                if (DUAL) {
                    const uint32_t *a1 = reinterpret_cast<const uint32_t *>(w1 + off);
                    for (int k = lane; k < rows * wpr; k += 32) d32[RS * wpr + k] = __ldg(a1 + k);
                }
                mbar_arrive(&full[i]);
            } else if (lane == 0) {
                const uint32_t bytes = static_cast<uint32_t>(rows * p.w_ld);
                mbar_expect_tx(&full[i], DUAL ? 2 * bytes : bytes);
                bulk_g2s(dst, w0 + off, bytes, &full[i]);
                if (DUAL) bulk_g2s(dst + RS * p.w_ld, w1 + off, bytes, &full[i]);
            }
        }
        return;
    }

    const float sc0 = p.s0 ? p.s0[e] : 1.0f;
    const float sc1 = (DUAL && p.s1) ? p.s1[e] : 1.0f;
    const int g = lane / LG, j = lane % LG;
    const int nc = p.K / Q8_ELEMS;
    bool waited = false;

    for (int w0t = s_begin; w0t < s_end; w0t += TT) {
        const int nt = min(TT, s_end - w0t);
        if (threadIdx.x < nt) {
            const int sl = p.slots[w0t + threadIdx.x];
            const int t = sl / p.n_used, k = sl % p.n_used;
            tok_row[threadIdx.x] = p.bcast ? t : sl;
            out_off[threadIdx.x] = static_cast<int>(t * p.ld_tok + k * p.ld_slot);
        }
        named_bar(1, GV_CWARPS * 32);
        // stage the window's activations (gathered rows)
        {
            uint8_t *aq = reinterpret_cast<uint8_t *>(act_q);
            float *ad = reinterpret_cast<float *>(act_d);
            for (int c = warp; c < nt * nc; c += GV_CWARPS) {
                const int t = c / nc, ch = c % nc;
                int8_t q;
                float dh;                            // the f16-rounded q8_1 scale
                if (p.xf != nullptr) {
                    const q8_lane r = q8_1_chunk(
                        p.xf[static_cast<int64_t>(tok_row[t]) * p.ldxf + static_cast<int64_t>(ch) * Q8_ELEMS + lane]);
                    q = static_cast<int8_t>(r.q);
                    dh = __half2float(__float2half_rn(r.d));
                } else {
                    const uint8_t *blk = p.q8 + (static_cast<int64_t>(tok_row[t]) * p.ldq + ch) * Q8_BYTES;
                    q = static_cast<int8_t>(blk[4 + lane]);
                    dh = __low2float(*reinterpret_cast<const __half2 *>(blk));
                }
                const int b = ch >> 1;
                const int s = ((ch & 1) << 1) | (lane >> 4);
                const int sl = (t * NB + b) * 4 + (s ^ ((b >> 1) & 3));
                aq[sl * 16 + act_perm(lane & 15)] = static_cast<uint8_t>(q);
                if (lane == 0) ad[(t * NB + b) * 2 + (ch & 1)] = 0.5f * dh;
            }
        }
        named_bar(1, GV_CWARPS * 32);
        for (int i = warp; i < n_st; i += GV_CWARPS) {
            // after a copy that never arrived (status word flagged) the warp
            // computes nothing more, but stays for the named barriers
            if (bad) continue;
            if (!waited && !mbar_wait(&full[i], 0, 3)) {
                bad = true;
                continue;
            }
            const int rows = min(RS, n_rows - i * RS);
            const uint8_t *st = ring + static_cast<size_t>(i) * p.slot_bytes;
            float acc0[TT], acc1[TT];
#pragma unroll
            for (int t = 0; t < TT; ++t) { acc0[t] = 0.0f; acc1[t] = 0.0f; }
            if (g < rows) {
                const uint8_t *row0 = st + static_cast<size_t>(g) * p.w_ld;
                for (int b = j; b < NB; b += LG) {
                    gv_block<TT>(reinterpret_cast<const uint32_t *>(row0 + b * NV_BYTES), b, NB, nt, act_q, act_d, acc0);
                    if (DUAL)
                        gv_block<TT>(reinterpret_cast<const uint32_t *>(row0 + RS * p.w_ld + b * NV_BYTES), b, NB, nt,
                                     act_q, act_d, acc1);
                }
            }
#pragma unroll
            for (int t = 0; t < TT; ++t) {
#pragma unroll
                for (int off = LG / 2; off > 0; off >>= 1) {
                    acc0[t] += __shfl_xor_sync(0xffffffffu, acc0[t], off);
                    if (DUAL) acc1[t] += __shfl_xor_sync(0xffffffffu, acc1[t], off);
                }
            }
            if (j == 0 && g < rows) {
                const int row = r_begin + i * RS + g;
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    if (t < nt) {
                        float v;
                        if (DUAL) {
                            float result = acc1[t];
                            result *= sc1;
                            float gate = acc0[t];
                            gate *= sc0;
                            result *= silu_f(gate);
                            v = result;
                        } else {
                            v = acc0[t] * sc0;
                        }
                        p.out[static_cast<int64_t>(out_off[t]) + row] = v;
                    }
                }
            }
        }
        waited = true;
        named_bar(1, GV_CWARPS * 32);
    }
    fr_pdl_trigger();
    if (!DUAL && p.c_out != nullptr) {
        // this CTA's slot rows are written: count it for its chunk; the last
        // of the chunk's active experts combines the chunk's rows
        __shared__ int s_last;
        __shared__ float s_w[4 * MOE_MAX_USED];
        fence_acq_rel_gpu();
        named_bar(1, GV_CWARPS * 32);
        if (threadIdx.x == 0)
            s_last = atomicAdd(&p.c_cnt[chunk], 1u) == static_cast<unsigned>(n_act - 1);
        named_bar(1, GV_CWARPS * 32);
        if (!s_last) return;
        fence_acq_rel_gpu();
        for (int t0 = 0; t0 < p.c_T; t0 += 4) {
            const int tn = min(4, p.c_T - t0);
            for (int i = threadIdx.x; i < tn * p.n_used; i += GV_CWARPS * 32)
                s_w[i] = p.c_wts[static_cast<int64_t>(t0) * p.n_used + i];
            named_bar(1, GV_CWARPS * 32);
            for (int i = threadIdx.x; i < tn * n_rows; i += GV_CWARPS * 32) {
                const int tl = i / n_rows, r = r_begin + i % n_rows, t = t0 + tl;
                const float *pt = p.out + static_cast<int64_t>(t) * p.n_used * p.N + r;
                float sum = moe_combine_value(pt, s_w + tl * p.n_used, p.n_used, p.N);
                if (p.c_resid) sum = sum + p.c_resid[static_cast<int64_t>(t) * p.N + r];
                p.c_out[static_cast<int64_t>(t) * p.N + r] = sum;
            }
            named_bar(1, GV_CWARPS * 32);
        }
        if (threadIdx.x == 0) p.c_cnt[chunk] = 0;
    }
}

// ------------------------------------------------------------ combine
// out[t, r] = sum_k part[t*n_used + k, r] * w[t, k]  (k ascending) (+ resid)
__global__ void __launch_bounds__(256) k_moe_combine(const float *__restrict__ part, const float *__restrict__ wts,
                                                     const float *__restrict__ resid, float *__restrict__ out,
                                                     int n_used, int n_embd) {
    fr_pdl_wait();
    fr_pdl_trigger();
    __shared__ float ws[MOE_MAX_USED];
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (threadIdx.x < n_used) ws[threadIdx.x] = wts[static_cast<int64_t>(t) * n_used + threadIdx.x];
    __syncthreads();
    if (r >= n_embd) return;
    const float *pt = part + static_cast<int64_t>(t) * n_used * n_embd + r;
    float sum = moe_combine_value(pt, ws, n_used, n_embd);
    if (resid) sum = sum + resid[static_cast<int64_t>(t) * n_embd + r];
    out[static_cast<int64_t>(t) * n_embd + r] = sum;
}

// ------------------------------------------------------------ expert parallel
// Fixed-capacity exchange buffers, one per rank, mapped by every peer (CUDA
// IPC): [flags 64 u32 (32 dispatch, 32 return)][consumed counts of the two
// waits][recv_x P x cap x K f32][recv_eid P x cap i32][back cap x K f32],
// cap = T_max * n_used slots.  Slot s of token t is t * n_used + k.
constexpr int EP_CTAS = 64;

// Dispatch: every slot's activation row goes to the expert owner's recv_x at
// [this rank][slot], with the owner-local expert id; every other rank gets -1
// for that slot, and slots past S (this call's T * n_used) get -1 everywhere,
// so each call rewrites the whole [this rank] band of every peer.  Each CTA
// then counts itself into every rank's dispatch flag[rank].
__global__ void __launch_bounds__(256) k_ep_dispatch(const float *__restrict__ x, int64_t ldx,
                                                     const int32_t *__restrict__ ids, int S, int cap, int n_used,
                                                     int E_p, int K, uint8_t *const *peer_base, int npeers, int rank,
                                                     int64_t off_x, int64_t off_eid, int64_t flag_off) {
    fr_pdl_wait();
    const int per = (cap + gridDim.x - 1) / gridDim.x;
    const int s_lo = blockIdx.x * per, s_hi = min(cap, s_lo + per);
    for (int s = s_lo; s < s_hi; ++s) {
        const int e = s < S ? ids[s] : -1;
        const int dest = e >= 0 ? e / E_p : -1;
        if (threadIdx.x < npeers) {
            int32_t *eid = reinterpret_cast<int32_t *>(peer_base[threadIdx.x] + off_eid) +
                           static_cast<int64_t>(rank) * cap + s;
            *eid = static_cast<int>(threadIdx.x) == dest ? e - dest * E_p : -1;
        }
        if (dest >= 0) {
            const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<int64_t>(s / n_used) * ldx);
            float4 *dst = reinterpret_cast<float4 *>(peer_base[dest] + off_x) +
                          (static_cast<int64_t>(rank) * cap + s) * (K / 4);
            for (int i = threadIdx.x; i < K / 4; i += blockDim.x) dst[i] = src[i];
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

// Return: the expert outputs of the rows this rank received (y [P x cap, K])
// go back to the source rank's `back` at the slot they came from; then each
// CTA counts itself into every rank's return flag[rank].
__global__ void __launch_bounds__(256) k_ep_return(const float *__restrict__ y, const int32_t *__restrict__ recv_eid,
                                                   int cap, int K, uint8_t *const *peer_base, int npeers, int rank,
                                                   int64_t off_back, int64_t flag_off) {
    fr_pdl_wait();
    const int rows = npeers * cap;
    const int per = (rows + gridDim.x - 1) / gridDim.x;
    const int r_lo = blockIdx.x * per, r_hi = min(rows, r_lo + per);
    for (int r = r_lo; r < r_hi; ++r) {
        if (recv_eid[r] < 0) continue;
        const int src = r / cap, s = r % cap;
        const float4 *from = reinterpret_cast<const float4 *>(y + static_cast<int64_t>(r) * K);
        float4 *to = reinterpret_cast<float4 *>(peer_base[src] + off_back) + static_cast<int64_t>(s) * (K / 4);
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) to[i] = from[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < npeers; ++q)
            atomicAdd_system(reinterpret_cast<unsigned int *>(peer_base[q] + flag_off) + rank, 1u);
    }
    fr_pdl_trigger();
}

} // namespace frb
