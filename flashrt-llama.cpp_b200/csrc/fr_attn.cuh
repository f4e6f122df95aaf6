// fr_attn.cuh -- the decode-step kernels around the NVFP4 matmuls of the
// synthetic MoE decoder: RMSNorm, RoPE + f16 KV-cache
// append, GQA decode attention on the tcgen05 tensor cores, NVFP4 token
// embedding rows, greedy arg-max, and the step's position counter.
//
// Reference: the Flint windows' decode attention frt_fa_decode /
// frt_fa_combine and their split plan (src/fr_win_flint_sm120.cu:2411-2846,
// :2866-2930), the QK-norm / RoPE front (:478-884), the host restatements of
// RMSNorm and SiLU (src/fr_win_flint_batched.cuh:466-476), and the fused QKV
// post (include/fr_kernels.h qkv_post: RoPE + f16 store of K, f16 store of V).
//
// Layouts:
//   x, xn         [T, H] f32 (T = sequences of the batch, one token each)
//   qkv           [T, (nh + 2 nkv) * d] f32: q heads, then k heads, then v heads
//   q_r           [T, nh, d] f32, RoPE'd and pre-scaled by 1/sqrt(d)
//   K / V cache   per layer [T, nkv, ctx, d] f16 (a sequence's rows of one KV
//                 head contiguous, so a chunk of keys is one contiguous box)
//   attention out [T, nh * d] f32
#pragma once

#include "fr_tc.cuh"

namespace frb {

constexpr int AT_D = 128;          // head dimension
constexpr int AT_G = 8;            // query heads per KV head (32 / 4)
constexpr int AT_CH = 128;          // keys per chunk
constexpr int AT_THREADS = 256;    // two head groups of four per key

// ------------------------------------------------------------------ RMSNorm
// y = x / sqrt(mean(x^2) + eps) * w (w nullable = 1); one CTA per row.  Each
// thread loads all of its values (and weights) at once -- a decode step runs
// two of these per layer at T = 1, where latency is all there is.
constexpr int RN_MAXV = 8;           // float4 per thread: the vector path covers H <= 8192
__global__ void __launch_bounds__(256) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w,
                                                 float *__restrict__ y, int H, float eps) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const float *xr = x + static_cast<int64_t>(blockIdx.x) * H;
    float *yr = y + static_cast<int64_t>(blockIdx.x) * H;
    const bool vec = (H & 3) == 0 && H <= 4 * 256 * RN_MAXV && (reinterpret_cast<uintptr_t>(xr) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(yr) & 15) == 0 && (w == nullptr || (reinterpret_cast<uintptr_t>(w) & 15) == 0);
    const int H4 = H >> 2;
    float4 v[RN_MAXV], wv[RN_MAXV];
    float ss = 0.0f;
    if (vec) {
#pragma unroll
        for (int u = 0; u < RN_MAXV; ++u) {
            const int k = threadIdx.x + u * 256;
            v[u] = k < H4 ? reinterpret_cast<const float4 *>(xr)[k] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            wv[u] = (w != nullptr && k < H4) ? reinterpret_cast<const float4 *>(w)[k] : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        }
#pragma unroll
        for (int u = 0; u < RN_MAXV; ++u)
            ss = fmaf(v[u].w, v[u].w, fmaf(v[u].z, v[u].z, fmaf(v[u].y, v[u].y, fmaf(v[u].x, v[u].x, ss))));
    } else {
        for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    }
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float scale = rsqrtf(red[0] / static_cast<float>(H) + eps);
    if (vec) {
#pragma unroll
        for (int u = 0; u < RN_MAXV; ++u) {
            const int k = threadIdx.x + u * 256;
            if (k < H4)
                reinterpret_cast<float4 *>(yr)[k] = make_float4(v[u].x * scale * wv[u].x, v[u].y * scale * wv[u].y,
                                                                v[u].z * scale * wv[u].z, v[u].w * scale * wv[u].w);
        }
    } else {
        for (int i = threadIdx.x; i < H; i += blockDim.x) yr[i] = w ? xr[i] * scale * w[i] : xr[i] * scale;
    }
}

// ------------------------------------------------------------ RoPE + KV append
// NeoX rotation (dimension pairs i, i + d/2) at position *pos with
// theta_i = pos * theta_scale^i, theta_scale = base^(-2/d), cos / sin of
// theta in f32 -- the arithmetic of ggml's rope_neox as the reference's QKV
// post restates it (src/fr_qkv_post.cu:71-131, no YaRN correction, freq_scale
// and attn_factor 1); q rows scaled by qscale; K and V rows of the step stored
// as f16 at row *pos of the layer's cache.  grid (T, ceil((nh + nkv) / 4)),
// 256 threads: thread = one rotated pair of one of the CTA's four heads (its
// loads, power and cos / sin issued at once), plus a slice of the V row.
__global__ void __launch_bounds__(256) k_rope_kv(const float *__restrict__ qkv, const int32_t *__restrict__ pos_p,
                                                 float *__restrict__ q_r, __half *__restrict__ kc,
                                                 __half *__restrict__ vc, int nh, int nkv, int ctx, float base,
                                                 float qscale) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int t = blockIdx.x;
    const int pos = *pos_p;
    const int half = AT_D / 2;
    const int width = (nh + 2 * nkv) * AT_D;
    const float *row = qkv + static_cast<int64_t>(t) * width;
    const int hd = blockIdx.y * 4 + (threadIdx.x >> 6), j = threadIdx.x & 63;
    // this CTA's slice of the V row (loaded with the pair)
    const int nv = nkv * AT_D, per_v = (nv + gridDim.y - 1) / gridDim.y;
    const int vi = blockIdx.y * per_v + threadIdx.x;
    const bool has_v = threadIdx.x < per_v && vi < nv;
    const float vv = has_v ? row[(nh + nkv) * AT_D + vi] : 0.0f;
    if (hd < nh + nkv) {
        const float a = row[hd * AT_D + j], b = row[hd * AT_D + j + half];
        const float theta_scale = powf(base, -2.0f / static_cast<float>(AT_D));
        const float theta = static_cast<float>(pos) * powf(theta_scale, static_cast<float>(j));
        const float cs = cosf(theta), sn = sinf(theta);
        const float ra = a * cs - b * sn, rb = a * sn + b * cs;
        if (hd < nh) {
            float *qo = q_r + (static_cast<int64_t>(t) * nh + hd) * AT_D;
            qo[j] = ra * qscale;
            qo[j + half] = rb * qscale;
        } else {
            const int g = hd - nh;
            __half *ko = kc + ((static_cast<int64_t>(t) * nkv + g) * ctx + pos) * AT_D;
            ko[j] = __float2half_rn(ra);
            ko[j + half] = __float2half_rn(rb);
        }
    }
    if (has_v) {
        const int g = vi / AT_D, c = vi % AT_D;
        vc[((static_cast<int64_t>(t) * nkv + g) * ctx + pos) * AT_D + c] = __float2half_rn(vv);
    }
}

// ggml's kvalues_mxfp4 (twice the E2M1 value) of a 4-bit code
__device__ __forceinline__ float kvalue_nvfp4(int c) {
    const int m = c & 7;
    const int mag = m < 5 ? m : (m == 5 ? 6 : (m == 6 ? 8 : 12));
    return static_cast<float>((c & 8) ? -mag : mag);
}

// --------------------------------------------------------- NVFP4 embedding rows
// x[t, :] = dequant(table row tok[t]) with ggml's NVFP4 reading (value =
// E2M1(code) * UE4M3(scale), scale sign ignored, 0x7F -> 0); the token is
// prompt[t * prompt_ld + pos] while pos < prompt_len, else gen[t] (the last
// step's arg-max).  One CTA per token, one thread per 64-value block.
__global__ void __launch_bounds__(256) k_embed_nvfp4(const uint8_t *__restrict__ table, int64_t row_bytes,
                                                     const int32_t *__restrict__ prompt, int prompt_ld,
                                                     int prompt_len, const int32_t *__restrict__ gen,
                                                     const int32_t *__restrict__ pos_p, float *__restrict__ x, int H,
                                                     int vocab) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int t = blockIdx.x;
    const int pos = *pos_p;
    int tok = pos < prompt_len ? prompt[static_cast<int64_t>(t) * prompt_ld + pos] : gen[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) fr_flag(FR_ST_BADINPUT);
        tok = 0;
    }
    const uint8_t *r = table + static_cast<int64_t>(tok) * row_bytes;
    float *xo = x + static_cast<int64_t>(t) * H;
    for (int b = threadIdx.x; b < H / 64; b += blockDim.x) {
        const uint8_t *blk = r + static_cast<int64_t>(b) * NV_BYTES;
        float sc[4];
        ue4m3x4(*reinterpret_cast<const uint32_t *>(blk), sc);   // ggml's value: kvalue * ue4m3 / 2
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint8_t byte = blk[4 + 8 * s + j];
                xo[64 * b + 16 * s + j] = kvalue_nvfp4(byte & 15) * sc[s] * 0.5f;
                xo[64 * b + 16 * s + j + 8] = kvalue_nvfp4(byte >> 4) * sc[s] * 0.5f;
            }
        }
    }
}

// ------------------------------------------------------------------- arg-max
// tok[t] = argmax_v logits[t, v] (ties: the lowest index; NaN never wins).
// grid (AM_SLICES, T): each CTA scans a contiguous slice with its loads in
// flight together and leaves (max, index); the last CTA of the row (arrival
// counter) reduces the slices.  The (value, index) order with ties to the
// lower index is a total order, so the reduction order does not matter.
constexpr int AM_SLICES = 64;
__device__ __forceinline__ void am_take(float &best, int &bi, float ob, int oi) {
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
}
__global__ void __launch_bounds__(256) k_argmax(const float *__restrict__ logits, int V, int32_t *__restrict__ tok,
                                                float *__restrict__ part_v, int *__restrict__ part_i,
                                                unsigned int *__restrict__ cnt) {
    fr_pdl_wait();
    fr_pdl_trigger();
    const int t = blockIdx.y, sl = blockIdx.x, ns = gridDim.x;
    const float *r = logits + static_cast<int64_t>(t) * V;
    const int per = (V + ns - 1) / ns;
    const int v0 = sl * per, v1 = min(V, v0 + per);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int b = v0 + threadIdx.x; b < v1; b += 8 * 256) {
        float f[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) f[u] = (b + u * 256 < v1) ? r[b + u * 256] : -INFINITY;
#pragma unroll
        for (int u = 0; u < 8; ++u) am_take(best, bi, f[u], b + u * 256);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        am_take(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    __shared__ float sb[8];
    __shared__ int si[8];
    __shared__ int s_last;
    if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) am_take(sb[0], si[0], sb[w], si[w]);
        part_v[t * ns + sl] = sb[0];
        part_i[t * ns + sl] = si[0];
        __threadfence();
        s_last = atomicAdd(&cnt[t], 1u) == static_cast<unsigned>(ns - 1);
    }
    __syncthreads();
    if (!s_last) return;
    if (threadIdx.x < 32) {
        __threadfence();
        best = -INFINITY;
        bi = 0x7fffffff;
        for (int k = threadIdx.x; k < ns; k += 32) am_take(best, bi, __ldcg(part_v + t * ns + k), __ldcg(part_i + t * ns + k));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            am_take(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
        if (threadIdx.x == 0) {
            tok[t] = bi == 0x7fffffff ? 0 : bi;
            cnt[t] = 0u;
        }
    }
}

// the step's position advances once every kernel of the step has read it
__global__ void k_pos_advance(int32_t *pos_p) {
    fr_pdl_wait();
    fr_pdl_trigger();
    if (threadIdx.x == 0) *pos_p += 1;
}

// fr_copy_pinned: 16-byte copy, grid-stride, after the previous kernel of
// the stream (it may still read the destination), ahead of the next one
__global__ void __launch_bounds__(256) k_copy16(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int64_t n) {
    fr_pdl_wait();
    fr_pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * 256)
        dst[i] = src[i];
}

// ------------------------------------------------------ GQA decode attention
// CTA (s, g, t) of a grid (S, nkv, T) handles KV head g of sequence t over the
// key chunks s, s + S, s + 2S, ... of AT_CH keys below the step's length, both
// matmuls of a chunk on the tensor cores (tcgen05.mma kind::f16, f32 in TMEM):
//   S^T [128 keys x 16] = K_chunk [128 x 128] . Q^T   (Q: 8 heads, 8 zero rows)
//   softmax over the keys (thread = key = TMEM lane), P^T in f16
//   O^T [128 dims x 16] = V_chunk^T [128 x 128] . P^T (V read MN-major as the TMA wrote it)
// so K and V are read once per KV head for all 8 heads.  Across its chunks a
// CTA keeps the running max m, sum l and output o per head (online softmax,
// o in registers: thread = head dimension x 4 heads); the next chunk's K / V
// TMA is issued as soon as the current chunk's K and V have been consumed, so
// it overlaps the softmax and the P.V product (V has two buffers, so the
// next chunk's V lands while this chunk's P.V product still reads its own).  With S = 1 the CTA writes
// o / l directly; otherwise each CTA writes (m, l, o) and the last CTA of
// (t, g) to finish merges the splits in split order (deterministic).  The
// host picks S so that the grid fills the SMs (S = ctx / AT_CH at T = 1, one
// CTA per (t, g) at batch 64).  Rows past the step's keys are masked (the
// cache is zero-initialised, so they are finite).
struct AtArgs {
    const float *q;              // [T, nh, d], RoPE'd, pre-scaled
    const int32_t *pos;          // keys = *pos + 1
    int nh, nkv, ctx;
    float *part;                 // [T][nkv][splits][16 + 8 * 128]: m[8], l[8], o[8][128]
    unsigned int *counter;       // [T * nkv], zero on entry, reset by the merging CTA
    float *out;                  // [T, nh * d]
};

constexpr int AT_SLAB = 128 * 128;                 // 128 rows x 128 B
constexpr int AT_QSLAB = 16 * 128;                 // 16 rows x 128 B
constexpr int AT_PART = 16 + AT_G * AT_D;
constexpr size_t AT_SMEM = 1024 + 6 * AT_SLAB + 4 * AT_QSLAB + 512 + 64;   // K, 2 x V, Q, P, scratch

__device__ __forceinline__ void tc_mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__host__ __device__ constexpr uint32_t idesc_f16_f32acc(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__global__ void __launch_bounds__(AT_THREADS) k_attn_decode(const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmV,
                                                            const AtArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *Ks = smem;                        // 2 slabs: keys x dims [0, 64) and [64, 128)
    uint8_t *Vb = Ks + 2 * AT_SLAB;            // 2 buffers of V, each as K
    uint8_t *Qs = Vb + 4 * AT_SLAB;            // 2 slabs: 16 heads x dims
    uint8_t *Pt = Qs + 2 * AT_QSLAB;           // 2 slabs: 16 heads x keys
    float *red = reinterpret_cast<float *>(Pt + 2 * AT_QSLAB);     // [4][8] maxima, [4][8] sums, M, L, alpha
    uint64_t *bars = reinterpret_cast<uint64_t *>(red + 96);       // tma, mma
    uint32_t *tmem_s = reinterpret_cast<uint32_t *>(bars + 2);
    int *flag = reinterpret_cast<int *>(tmem_s + 1);
    float *M = red + 64, *L = red + 72, *AL = red + 80;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
    // thread = TMEM lane kd = wq * 32 + lane (a key of the chunk for the
    // scores, a head dimension for the output) x heads [4 hg, 4 hg + 4)
    const int wq = warp & 3, hg = warp >> 2;
    const int kd = wq * 32 + lane;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 0) tmem_alloc(tmem_s, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_s;
    fr_pdl_wait();                                     // q, the cache rows and pos come from earlier kernels
    const int n = *a.pos + 1;
    const int nch = (n + AT_CH - 1) / AT_CH;           // chunks holding the step's keys
    const int splits = gridDim.x;
    const int row_base = (t * a.nkv + g) * a.ctx;
    float *part = a.part + ((static_cast<int64_t>(t) * a.nkv + g) * splits + s) * AT_PART;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    bool ok = true, tma_pending = false;
    uint32_t ph0 = 0, ph1 = 0;
    if (s < nch) {
        if (tid == 0) {
            mbar_expect_tx(&bars[0], 4 * AT_SLAB);
            tma_load_2d(Ks, &tmK, 0, row_base + s * AT_CH, &bars[0]);
            tma_load_2d(Ks + AT_SLAB, &tmK, 64, row_base + s * AT_CH, &bars[0]);
            tma_load_2d(Vb, &tmV, 0, row_base + s * AT_CH, &bars[0]);
            tma_load_2d(Vb + AT_SLAB, &tmV, 64, row_base + s * AT_CH, &bars[0]);
        }
        tma_pending = true;
        // Q tile (f16, 128-byte swizzled K-major): 16 rows x 16 chunks of 8 dims; rows 8..15 zero
        for (int i = tid; i < 16 * 16; i += AT_THREADS) {
            const int h = i >> 4, c = i & 15;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (h < AT_G) {
                const float4 *qp = reinterpret_cast<const float4 *>(
                    a.q + (static_cast<int64_t>(t) * a.nh + g * AT_G + h) * AT_D + 8 * c);
                const float4 f0 = qp[0], f1 = qp[1];
                const __half2 h0 = __floats2half2_rn(f0.x, f0.y), h1 = __floats2half2_rn(f0.z, f0.w);
                const __half2 h2 = __floats2half2_rn(f1.x, f1.y), h3 = __floats2half2_rn(f1.z, f1.w);
                v = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                               *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            }
            *reinterpret_cast<uint4 *>(Qs + (c >> 3) * AT_QSLAB + h * 128 + (((c & 7) ^ (h & 7)) << 4)) = v;
        }
        // P^T rows 8..15 stay zero
        for (int i = tid; i < 8 * 16; i += AT_THREADS) {
            const int h = 8 + (i >> 4), c = i & 15;
            *reinterpret_cast<uint4 *>(Pt + (c >> 3) * AT_QSLAB + h * 128 + (((c & 7) ^ (h & 7)) << 4)) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        if (tid < AT_G) {
            M[tid] = -INFINITY;
            L[tid] = 0.0f;
        }
        fence_proxy_async();
        __syncthreads();
        int it = 0;
#pragma unroll 1
        for (int c = s; c < nch && ok; c += splits, ++it) {
            const int nk = min(AT_CH, n - c * AT_CH);
            uint8_t *Vs = Vb + (it & 1) * 2 * AT_SLAB;
            ok = mbar_wait(&bars[0], ph0, 50);
            if (ok) {
                ph0 ^= 1u;
                tma_pending = false;
            }
            if (tid == 0 && ok) {
                tc_fence_after();
                const uint32_t idesc = idesc_f16_f32acc(128, 16);
                for (int j = 0; j < 8; ++j) {
                    const int sl = j >> 2, ko = (j & 3) * 32;
                    tc_mma_f16_ss(tm, sdesc_sw128(smem_u32(Ks + sl * AT_SLAB) + ko),
                                  sdesc_sw128(smem_u32(Qs + sl * AT_QSLAB) + ko), idesc, j > 0 ? 1u : 0u);
                }
                tc_commit(&bars[1]);
            }
            if (ok) {
                ok = mbar_wait(&bars[1], ph1, 51);
            }
            ph1 ^= 1u;
            tc_fence_after();
            float sv[4];
            {
                uint32_t r[16];
                tmem_ld16(tm + (static_cast<uint32_t>(wq * 32) << 16), r);
#pragma unroll
                for (int h4 = 0; h4 < 4; ++h4)
                    sv[h4] = (ok && kd < nk) ? __uint_as_float(r[4 * hg + h4]) : -INFINITY;
            }
#pragma unroll
            for (int h4 = 0; h4 < 4; ++h4) {
                float m = sv[h4];
#pragma unroll
                for (int sh = 16; sh > 0; sh >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, sh));
                if (lane == 0) red[wq * 8 + 4 * hg + h4] = m;
            }
            tc_fence_before();
            ok = __syncthreads_and(ok) != 0;
            // K of this chunk is consumed and the other V buffer's last P.V
            // product is done: the next chunk's copies go out now
            if (ok && c + splits < nch) {
                if (tid == 0) {
                    const int row = row_base + (c + splits) * AT_CH;
                    uint8_t *Vn = Vb + ((it + 1) & 1) * 2 * AT_SLAB;
                    mbar_expect_tx(&bars[0], 4 * AT_SLAB);
                    tma_load_2d(Ks, &tmK, 0, row, &bars[0]);
                    tma_load_2d(Ks + AT_SLAB, &tmK, 64, row, &bars[0]);
                    tma_load_2d(Vn, &tmV, 0, row, &bars[0]);
                    tma_load_2d(Vn + AT_SLAB, &tmV, 64, row, &bars[0]);
                }
                tma_pending = true;
            }
            if (tid < AT_G) {
                const float mc = fmaxf(fmaxf(red[tid], red[8 + tid]), fmaxf(red[16 + tid], red[24 + tid]));
                const float mo = M[tid], mn = fmaxf(mo, mc);
                AL[tid] = mo > -INFINITY ? expf(mo - mn) : 0.0f;     // rescale of what came before
                M[tid] = mn;
            }
            __syncthreads();
#pragma unroll
            for (int h4 = 0; h4 < 4; ++h4) {
                const int h = 4 * hg + h4;
                const float mh = M[h];
                const __half p16 = __float2half_rn(kd < nk && mh > -INFINITY ? expf(sv[h4] - mh) : 0.0f);
                float l = __half2float(p16);           // the sum of the probabilities the MMA multiplies
#pragma unroll
                for (int sh = 16; sh > 0; sh >>= 1) l += __shfl_xor_sync(0xffffffffu, l, sh);
                if (lane == 0) red[32 + wq * 8 + h] = l;
                const int kk = kd & 63;
                *reinterpret_cast<__half *>(Pt + (kd >> 6) * AT_QSLAB + h * 128 + (((kk >> 3) ^ (h & 7)) << 4) +
                                            (kk & 7) * 2) = p16;
            }
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            if (tid < AT_G)
                L[tid] = fmaf(L[tid], AL[tid], (red[32 + tid] + red[40 + tid]) + (red[48 + tid] + red[56 + tid]));
            if (tid == 0 && ok) {
                tc_fence_after();
                // keys [16 j, 16 j + 16) are rows 16 j.. of both V slabs; A (V^T) MN-major
                const uint32_t idesc_pv = idesc_f16_f32acc(128, 16) | (1u << 15);
                for (int j = 0; j < 8; ++j) {
                    const int sl = j >> 2, ko = (j & 3) * 32;
                    tc_mma_f16_ss(tm + 16, sdesc_sw128_mn(smem_u32(Vs) + j * 16 * 128, AT_SLAB, 1024),
                                  sdesc_sw128(smem_u32(Pt + sl * AT_QSLAB) + ko), idesc_pv, j > 0 ? 1u : 0u);
                }
                tc_commit(&bars[1]);
            }
            if (ok) ok = mbar_wait(&bars[1], ph1, 52);
            ph1 ^= 1u;
            tc_fence_after();
            {
                uint32_t r[16];
                tmem_ld16(tm + (static_cast<uint32_t>(wq * 32) << 16) + 16, r);
#pragma unroll
                for (int h4 = 0; h4 < 4; ++h4)
                    o[h4] = fmaf(o[h4], AL[4 * hg + h4], ok ? __uint_as_float(r[4 * hg + h4]) : 0.0f);
            }
            tc_fence_before();
            ok = __syncthreads_and(ok) != 0;
        }
        // a copy still in flight after a timed-out wait lands before the CTA leaves
        if (tma_pending && tid == 0) mbar_wait(&bars[0], ph0, 53);
        __syncthreads();
        if (splits == 1) {
#pragma unroll
            for (int h4 = 0; h4 < 4; ++h4) {
                const int h = 4 * hg + h4;
                a.out[(static_cast<int64_t>(t) * a.nh + g * AT_G + h) * AT_D + kd] = ok ? o[h4] / L[h] : 0.0f;
            }
        } else {
#pragma unroll
            for (int h4 = 0; h4 < 4; ++h4) part[16 + (4 * hg + h4) * AT_D + kd] = ok ? o[h4] : 0.0f;
            if (tid < AT_G) {
                part[tid] = M[tid];
                part[8 + tid] = L[tid];
            }
        }
    }
    if (splits > 1) {
        // the last CTA of (t, g) merges the splits
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            unsigned int *cnt = a.counter + t * a.nkv + g;
            const unsigned prev = atomicAdd(cnt, 1u);
            *flag = prev == static_cast<unsigned>(splits - 1);
            if (*flag) *cnt = 0u;
        }
        __syncthreads();
        if (*flag) {
            // merge: every split's (m, l) into shared memory with all loads in
            // flight, the per-head weights exp(m_s - max) once, then each thread
            // (= head dimension) its outputs with its split loads issued together
            __threadfence();
            const int ns = min(splits, nch);
            const float *base = a.part + (static_cast<int64_t>(t) * a.nkv + g) * splits * AT_PART;
            float *ml = reinterpret_cast<float *>(Ks);        // [split][16]: m[8], l[8]; then w [split][8]
            float *wts = ml + 16 * ns;
            for (int i = tid; i < 16 * ns; i += AT_THREADS) ml[i] = __ldcg(base + (i >> 4) * AT_PART + (i & 15));
            __syncthreads();
            if (tid < AT_G) {
                float mx = -INFINITY;
                for (int s2 = 0; s2 < ns; ++s2) mx = fmaxf(mx, ml[s2 * 16 + tid]);
                float lsum = 0.0f;
                for (int s2 = 0; s2 < ns; ++s2) {
                    const float w = expf(ml[s2 * 16 + tid] - mx);
                    wts[s2 * 8 + tid] = w;
                    lsum = fmaf(w, ml[s2 * 16 + 8 + tid], lsum);
                }
                red[tid] = lsum;                           // (the softmax's scratch is free by now)
            }
            __syncthreads();
            // thread = head dimension of one of the two head groups
            const int d = tid & (AT_D - 1);
            constexpr int MS = 16, MH = 4;                 // splits x heads whose loads go out together
#pragma unroll 1
            for (int h0 = (tid >> 7) * MH; h0 < AT_G; h0 += 2 * MH) {
                float acc[MH];
#pragma unroll
                for (int hh = 0; hh < MH; ++hh) acc[hh] = 0.0f;
                for (int s0 = 0; s0 < ns; s0 += MS) {
                    float v[MH][MS];
#pragma unroll
                    for (int hh = 0; hh < MH; ++hh)
#pragma unroll
                        for (int u = 0; u < MS; ++u)
                            v[hh][u] = s0 + u < ns ? __ldcg(base + (s0 + u) * AT_PART + 16 + (h0 + hh) * AT_D + d)
                                                   : 0.0f;
#pragma unroll
                    for (int hh = 0; hh < MH; ++hh)
#pragma unroll
                        for (int u = 0; u < MS; ++u)
                            if (s0 + u < ns) acc[hh] = fmaf(wts[(s0 + u) * 8 + h0 + hh], v[hh][u], acc[hh]);
                }
#pragma unroll
                for (int hh = 0; hh < MH; ++hh)
                    a.out[(static_cast<int64_t>(t) * a.nh + g * AT_G + h0 + hh) * AT_D + d] = acc[hh] / red[h0 + hh];
            }
        }
    }
    fr_pdl_trigger();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, 32);
    }
}

} // namespace frb
