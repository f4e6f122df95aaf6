/*
 * fr_b200.h -- C-ABI of the B200 (sm_100a) NVFP4-weight x q8_1-activation
 * matmul hot path, a drop-in for FlashRT-llama.cpp's NVFP4 mul_mat /
 * mul_mat_id path.
 *
 * Conventions (the reference's, include/fr_kernels.h:1-6 and
 * docs/development.md:11-25):
 *   - raw device pointers, the caller's cudaStream_t, no framework types;
 *   - every entry returns an int: 0 on success, -1 on a shape / alignment /
 *     null-pointer precondition, -3 on a layout overflow, -cudaError_t on a
 *     CUDA launch error (the reference's codes), and the FR_E* codes below
 *     for conditions the reference has no code for;
 *   - nothing aborts; nothing allocates while the stream is being captured
 *     (an entry that would have to grow a workspace then returns
 *     FR_ECAPTURE).
 *
 * Formats: ggml's block_nvfp4 (36 B per 64 values: 4 UE4M3 sub-block scales
 * + 32 bytes of E2M1 codes, sub-block s in qs[8s..8s+7], byte j = value j in
 * the low nibble and value j+8 in the high nibble) and block_q8_1 (36 B per
 * 32 values: half d, half sum, int8 qs[32]).  Weights [N rows, K] are rows of
 * K/64 blocks, `w_ld` bytes apart; activations / outputs are row-major f32.
 */
#ifndef FR_B200_H
#define FR_B200_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ codes */
#define FR_OK          0
#define FR_EINVAL     (-1)    /* shape / alignment / null pointer (reference -1) */
#define FR_ELAYOUT    (-3)    /* scale layout larger than the buffer (reference -3) */
#define FR_ECAPTURE   (-901)  /* a workspace would have to grow during stream capture */
#define FR_EINJECTED  (-902)  /* host-side fault injection fired (fr_fault_inject) */
#define FR_ENODEVICE  (-903)  /* no sm_100 device current */

int         fr_version(void);
const char *fr_strerror(int rc);

/* Device-side status word: bounded waits inside the kernels that give up set
 * bit 0 (and a site id in bits 8..15) and return instead of hanging;
 * out-of-range routing ids set bit 1.  Reads (and optionally clears) the
 * word of the current device.  Synchronises the device. */
int fr_device_status(uint32_t *status, int clear);

/* Limit of every bounded device-side wait, in nanoseconds (default and
 * maximum 2 s, minimum 1 us).  A wait that runs out sets status bit 0 with its
 * site and lets its kernel return.  Applies to the current device, from the
 * next launch on.  Returns the previous limit, or a negative code. */
int64_t fr_set_wait_ns(int64_t ns);

/* Host-side fault injection (test aid): the next call of the entry point
 * whose name equals `site` returns FR_EINJECTED before launching anything.
 * NULL clears.  Also read once from the environment variable FR_FAULT. */
int fr_fault_inject(const char *site);

/* Number of kernels this library has launched in this process. */
uint64_t fr_kernel_launches(void);

/* Matvec kernel selection (config knob, like the reference's FRT_* switches):
 * 0 = by shape (tensor-core kernel when K % 256 == 0 and rows are 16-byte
 * aligned, else the dp4a kernel), 1 = dp4a kernel, 2 = tensor-core kernel
 * where the shape allows.  Initialised once from FR_MATVEC=auto|dp4a|tc.
 * Returns the previous setting, or -1 for an invalid argument. */
int fr_set_matvec_path(int path);

/* ------------------------------------------------------------------ sizes */
int64_t fr_nvfp4_row_bytes(int64_t K);   /* K/64 * 36 */
int64_t fr_q8_1_row_bytes(int64_t K);    /* K/32 * 36 */

/* --------------------------------------------------- (a1) quantize_q8_1
 * x [T, ldx] f32 -> q8 [T, ldq blocks] block_q8_1.  K % 32 == 0.
 * Bit-exact: d = amax/127, q = roundf(x/d) (IEEE division), ds = half2(d, sum
 * in xor-butterfly order).  Replaces frt_q8_1_chunk / frt_b_q8
 * (src/fr_win_flint_sm120.cu:289-300, src/fr_win_flint_batched.cuh:178-190)
 * and ggml-cuda's quantize_q8_1 in front of mmvq. */
int fr_quantize_q8_1(const float *x, int64_t ldx, void *q8, int64_t ldq,
                     int T, int K, cudaStream_t stream);

/* ------------------------------------------- (a3/a4) NVFP4 x q8_1 matvec
 * y[t, n] = scale * dot(W[n], q8[t]) (+ resid[t, n]) for t < T, n < N.
 * scale / resid nullable (1.0 / none).  K % 64 == 0, 1 <= T <= 128.
 * Replaces the mmvq NVFP4 x q8_1 decode GEMV and the Flint row dots
 * (src/fr_win_flint_sm120.cu:320-414, windows :889-920, :1201-1232) and the
 * batched frt_m_gemv / frt_b_gemv (src/fr_win_flint_bmma.cuh:193-310,
 * src/fr_win_flint_batched.cuh:215-289). */
int fr_gemv_nvfp4_q8_1(const void *w, int64_t w_ld, const void *q8, int64_t ldq,
                       const float *scale, const float *resid, int64_t ldr,
                       float *y, int64_t ldy, int N, int K, int T, cudaStream_t stream);

/* Same, with the q8_1 quantization of f32 x [T, ldx] fused into the kernel. */
int fr_gemv_nvfp4_f32(const void *w, int64_t w_ld, const float *x, int64_t ldx,
                      const float *scale, const float *resid, int64_t ldr,
                      float *y, int64_t ldy, int N, int K, int T, cudaStream_t stream);

/* Gate/up pair with the fused mmvq SwiGLU epilogue
 * y = (su * dot(Wu[n], q8)) * silu(sg * dot(Wg[n], q8))
 * (src/fr_win_flint_sm120.cu:1944-1952, frt_dense_gu :1024-1101). */
int fr_gemv_nvfp4_q8_1_swiglu(const void *wg, const void *wu, int64_t w_ld,
                              const void *q8, int64_t ldq, const float *sg, const float *su,
                              float *y, int64_t ldy, int N, int K, int T, cudaStream_t stream);

/* ggml_mul_mat(src0 = NVFP4 [N, K], src1 = f32 [T, K]) -> dst f32 [T, N] with
 * ggml's q8_1 activation semantics: the f32 rows are quantized to q8_1 and
 * multiplied by the NVFP4 rows.  The op surface of ggml_cuda_mul_mat for an
 * NVFP4 src0 (hosts/llama.cpp/patches/0001-...:109-121, the Thor predicate
 * src/fr_dispatch.cu:267-289).  T >= 1 (no upper bound). */
int fr_mul_mat_nvfp4(const void *src0, int64_t nb01, const float *src1, int64_t ld1,
                     float *dst, int64_t ldd, int N, int K, int T, cudaStream_t stream);

/* Dense SwiGLU FFN (the Flint DENSEFFN window, src/fr_win_flint_sm120.cu:
 * 1024-1101): out[t] = sd * Wd . q8( swiglu(Wg, Wu; q8(x[t])) ) (+ resid[t]).
 * x / resid / out are [T, n_embd]; Wg, Wu [n_ff, n_embd]; Wd [n_embd, n_ff].
 * The optional check buffers (nullable) receive the intermediates the
 * reference's check mode inspects: glu [T, n_ff] f32, glu_q8 [T, n_ff/32]
 * blocks. */
int fr_ffn_nvfp4(const float *x, const void *wg, const void *wu, const void *wd,
                 const float *sg, const float *su, const float *sd, const float *resid,
                 float *out, int T, int n_embd, int n_ff,
                 float *chk_glu, void *chk_glu_q8, cudaStream_t stream);

/* The same dense FFN for callers that cannot allocate device memory.
 * No counterpart in the reference.
 *
 * fr_ffn_nvfp4 grows a private workspace with cudaMalloc the first time it
 * sees a larger shape.  Some callers cannot allow that: code running while a
 * stream is being captured into a CUDA graph (cudaMalloc is not permitted
 * there), hosts such as ggml whose allocator plans every buffer of a graph up
 * front and expects operators not to allocate behind its back, and serving
 * processes with a fixed device-memory budget.  This entry point allocates
 * nothing: its intermediates (q8_1 of x, the GLU, q8_1 of the GLU) live in a
 * static device array of FR_FFN_NOALLOC_SCRATCH_BYTES that every GPU which
 * loads the library holds until the process exits.
 *   - Required scratch: T * (n_embd/32*36 + n_ff*4 + n_ff/32*36) bytes; a
 *     call that needs more returns FR_ETOOBIG and launches nothing.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls share the one array and it keeps the last call's contents.
 *     Every intermediate is fully rewritten by each call, so nothing needs
 *     clearing, but calls that overlap on the GPU (different streams without
 *     ordering between them) race on the array: order them on one stream or
 *     with events.
 *   - It always runs the dp4a matvec (the kernel that needs no workspace),
 *     whatever fr_set_matvec_path says, so its results can differ from
 *     fr_ffn_nvfp4's within the matvec tolerance, and at larger T it is
 *     slower than the tensor-core path fr_ffn_nvfp4 would pick. */
#define FR_FFN_NOALLOC_SCRATCH_BYTES (8u << 20)
#define FR_ETOOBIG    (-904)  /* request larger than the static scratch */
int fr_ffn_nvfp4_noalloc(const float *x, const void *wg, const void *wu, const void *wd,
                         const float *sg, const float *su, const float *sd, const float *resid,
                         float *out, int T, int n_embd, int n_ff, cudaStream_t stream);

/* -------------------------------------------------------------- (a7/a8) MoE routing
 * logits[t, e] = x[t] . W_r[e] (f32), softmax over E, n_used rounds of
 * arg-max (lower expert id wins ties), w = p / max(sum p_sel, clamp)
 * (frt_router_fused, src/fr_win_qwen36_sm120.cu:1785-1870), then the token
 * permute (src/fr_win_flint_batched_moe.cuh:76-166): eoff [E+1] (first
 * grouped slot of each expert), slots [T*n_used] (slot ids t*n_used + k grouped
 * by expert, in slot order inside an expert), act [E+1] (active experts
 * ascending, count at act[E]).  E % 32 == 0, E <= 256, n_used <= 32, K % 4 == 0. */
int fr_moe_route(const float *x, int64_t ldx, const float *w_r, int T, int K, int E,
                 int n_used, float clamp_val, float *logits, int32_t *ids, float *wts,
                 int32_t *eoff, int32_t *slots, int32_t *act, cudaStream_t stream);

/* ------------------------------------------------------- (a9) mul_mat_id
 * ggml_mul_mat_id: dst[t, k, :] = W[ids[t, k]] . q8(x[t, k or 0]) for t < T,
 * k < n_used.  W is E experts of [N, K] NVFP4 rows (nb01 bytes per row, nb02
 * bytes per expert).  x rows: x + t*x_ld_tok + k*x_ld_slot floats
 * (x_ld_slot = 0 broadcasts one row per token, the gate/up case).
 * dst rows: dst + t*dst_ld_tok + k*dst_ld_slot.  Rows are grouped by expert
 * so every used expert's weights are read once per call.  The hook
 * ggml_cuda_frt_moe_mul_mat_id (src/fr_win_qwen36_sm120.cu:2502-2618)
 * with the q8_1 arithmetic of ggml's MMVQ/MMQ mul_mat_id. */
int fr_mul_mat_id_nvfp4(const void *w, int64_t nb01, int64_t nb02, int E,
                        const float *x, int64_t x_ld_slot, int64_t x_ld_tok,
                        const int32_t *ids, int64_t ids_ld,
                        float *dst, int64_t dst_ld_slot, int64_t dst_ld_tok,
                        int T, int n_used, int N, int K, cudaStream_t stream);

/* --------------------------------------------- (a7-a10) fused MoE FFN layer
 * route -> grouped gate/up (SwiGLU) -> q8_1 of the GLU -> grouped down ->
 * weighted slot-order combine: out[t] = sum_k w[t,k] * sd[e] * Wd[e] . q8(glu)
 * (+ resid[t]).  Experts: Wg/Wu [E][n_ff, n_embd], Wd [E][n_embd, n_ff];
 * per-expert scales sg/su/sd [E] (nullable -> 1).  W_r [E, n_embd] f32.
 * Check buffers (nullable): ids/wts [T, n_used], glu [T, n_used, n_ff] f32,
 * part [T, n_used, n_embd] f32 (unweighted per-slot down outputs). */
int fr_moe_ffn_nvfp4(const float *x, const float *w_r, const void *wg, const void *wu,
                     const void *wd, const float *sg, const float *su, const float *sd,
                     const float *resid, float *out, int T, int n_embd, int n_ff, int E,
                     int n_used, float clamp_val,
                     int32_t *chk_ids, float *chk_wts, float *chk_glu, float *chk_part,
                     cudaStream_t stream);

/* Expert FFN over pre-routed rows (the expert-parallel building block): row s
 * of x [S, ldx] goes through expert eid[s] (0 <= eid < E): SwiGLU of the
 * grouped gate/up matvecs, q8_1 of the GLU, grouped down matvec, scaled by
 * sd[e]: out[s] = sd[e] * Wd[e] . q8(swiglu(...)).  Every expert that appears
 * is read once.  Rows with an out-of-range id are flagged (status bit 1) and
 * left untouched.  The routed/shared MOEFFN window's expert part,
 * src/fr_win_flint_sm120.cu:1890-2094. */
int fr_moe_experts_nvfp4(const float *x, int64_t ldx, const int32_t *eid, int S,
                         const void *wg, const void *wu, const void *wd,
                         const float *sg, const float *su, const float *sd,
                         float *out, int64_t ldo, int n_embd, int n_ff, int E, cudaStream_t stream);

/* Weighted slot-order combine: out[t] = sum_k w[t,k] * part[t*n_used + k]
 * (k ascending) (+ resid[t]); part rows n_embd floats, out / resid [T, n_embd]
 * (src/fr_win_flint_batched_moe.cuh:342-379). */
int fr_moe_combine(const float *part, const float *wts, const float *resid, float *out,
                   int T, int n_used, int n_embd, cudaStream_t stream);

/* ------------------------------------------------ (a2-a4) tile-major weights
 * A one-time repack of a ggml block_nvfp4 matrix [N, K] (rows w_ld bytes
 * apart) into tiles of 128 rows x 256 values, each one contiguous 18 KB block
 * (16 KB of E2M1 codes in the 128-byte-swizzled K-major order the tcgen05
 * block-scaled MMA reads, 2 KB of UE4M3 sub-block scale atoms), tiles of a
 * row block consecutive along K.  Same bytes as the ggml tensor when
 * N % 128 == 0 and K % 256 == 0 (rows / blocks past the end are zero).  The
 * reference repacks NVFP4 weights once at load for its tensor-core GEMM in
 * the same way (include/fr_kernels.h:45-51, src/fr_repack.cu:1-13); here the
 * tiled layout feeds the decode matvec on the FP4 tensor cores, which streams
 * each CTA's tiles as one contiguous byte range.
 *   fr_nvfp4_tiled_bytes : size of the tiled copy (-1 on bad shape)
 *   fr_nvfp4_tile        : repack (K % 64 == 0)
 *   fr_gemv_tiled        : y[t] = scale * W . x_q[t] (+ resid[t]); exactly one
 *                          of x (f32 rows, quantized to q8_1 on the fly) or q8
 *                          (q8_1 rows, ldq blocks apart) is non-null
 *   fr_gemv_tiled_swiglu : y[t] = silu(sg * Wg . x_q[t]) * (su * Wu . x_q[t])
 *   fr_ffn_tiled         : fr_ffn_nvfp4 on tiled weights
 * K % 256 == 0 for the matvecs. */
int64_t fr_nvfp4_tiled_bytes(int N, int K);
int fr_nvfp4_tile(const void *w, int64_t w_ld, int N, int K, void *dst, cudaStream_t stream);
int fr_gemv_tiled(const void *wt, int N, int K, const float *x, int64_t ldx, const void *q8, int64_t ldq,
                  const float *scale, const float *resid, int64_t ldr, float *y, int64_t ldy, int T,
                  cudaStream_t stream);
int fr_gemv_tiled_swiglu(const void *wg_t, const void *wu_t, int N, int K, const float *x, int64_t ldx,
                         const void *q8, int64_t ldq, const float *sg, const float *su, float *y, int64_t ldy, int T,
                         cudaStream_t stream);
int fr_ffn_tiled(const float *x, const void *wg_t, const void *wu_t, const void *wd_t, const float *sg,
                 const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                 float *chk_glu, cudaStream_t stream);

/* ------------------------------------ (a7-a10) MoE on tiled expert weights
 * The expert matrices repacked by fr_nvfp4_tile as one stacked [E * N, K]
 * matrix (N % 128 == 0, so expert e's tiles start at e * N/128 * K/256 *
 * 18432 bytes -- the ggml tensor's own expert stride).  The per-expert
 * matvecs then run on the FP4 tensor cores: each active expert's slots are
 * cut into windows of up to 16 tokens, and every row block of every used
 * expert is streamed once per window (once per call unless more than 16
 * tokens chose the expert), with the window count taken on the device from
 * the routing (no host sync, graph-capturable).
 *   fr_mul_mat_id_tiled : fr_mul_mat_id_nvfp4 on tiled experts [E][N, K]
 *                         (N % 128 == 0, K % 256 == 0; a per-slot input must
 *                         have x_ld_tok == n_used * x_ld_slot).  Replaces the
 *                         hook ggml_cuda_frt_moe_mul_mat_id
 *                         (src/fr_win_qwen36_sm120.cu:2502-2618) for
 *                         repacked expert tensors.
 *   fr_moe_ffn_tiled    : fr_moe_ffn_nvfp4 on tiled experts (n_embd and n_ff
 *                         multiples of 256); same routing, grouping, check
 *                         buffers and slot-order combine. */
int fr_mul_mat_id_tiled(const void *w_t, int E, int N, int K, const float *x, int64_t x_ld_slot,
                        int64_t x_ld_tok, const int32_t *ids, int64_t ids_ld, float *dst, int64_t dst_ld_slot,
                        int64_t dst_ld_tok, int T, int n_used, cudaStream_t stream);
int fr_moe_ffn_tiled(const float *x, const float *w_r, const void *wg_t, const void *wu_t, const void *wd_t,
                     const float *sg, const float *su, const float *sd, const float *resid, float *out, int T,
                     int n_embd, int n_ff, int E, int n_used, float clamp_val, int32_t *chk_ids, float *chk_wts,
                     float *chk_glu, float *chk_part, cudaStream_t stream);

/* ------------------------------------------------------ (e) tensor parallel
 * One rank's step of the dense FFN sharded over n_ff (P = nranks ranks, shard
 * F_p = n_ff / P): rank r holds gate/up rows [r*F_p, (r+1)*F_p) and, of every
 * down row, the NVFP4 blocks of columns [r*F_p, (r+1)*F_p) (wd_shard is
 * [n_embd rows][F_p/64 blocks], rows F_p/64*36 bytes apart).  Each rank
 * computes its GLU columns and its partial down output locally; the down
 * matvec's epilogue stores the partial rows into this rank's slot of every
 * rank's partial array over NVLink and counts its CTAs into every rank's
 * flags; a bounded wait then sums the P partials in rank order (the same
 * order on every rank), adds `resid` and writes `out` [T, n_embd] on every
 * rank.  n_ff % (64 * P) == 0, so no q8_1 or NVFP4 block straddles a shard.
 * peer_base is a device array of the P ranks' base addresses of one shared
 * buffer of fr_tp_buffer_bytes(T, n_embd, n_ff, P) bytes, zeroed once before
 * first use; local_base is this rank's own base.  All ranks call with the
 * same T.  The reference is single-device; no counterpart. */
int64_t fr_tp_buffer_bytes(int T, int n_embd, int n_ff, int nranks);
/* The partial outputs are double-buffered by step parity inside the buffer (a
 * device-side step count picks the half), so a rank that runs a step ahead
 * never overwrites partials a slower rank is still summing; consecutive steps
 * need no host synchronisation.  The buffer's size fixes its token capacity
 * (the T given to fr_tp_buffer_bytes): every call on it passes the same
 * buffer_bytes and T up to that capacity.
 * fr_tp_wait: the step's completion wait alone (nothing summed): returns once
 * each of the nranks flag counters of this rank's buffer grew by `expect`
 * publications since the last wait, or when the wait limit runs out (status
 * bit 0, site 30).  For failure handling and tests; a step already waits. */
int fr_tp_wait(void *local_base, int64_t buffer_bytes, int n_embd, int nranks, unsigned expect,
               cudaStream_t stream);
/* fr_tp_ffn_nvfp4 on tile-major shards (fr_nvfp4_tile of the gate/up row
 * shards [F_p, n_embd] and of the down K-shard [n_embd, F_p]);
 * n_ff % (256 * nranks) == 0 and n_embd % 256 == 0. */
int fr_tp_ffn_tiled(const float *x, const void *wg_t, const void *wu_t, const void *wd_t, const float *sg,
                    const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                    int nranks, int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes,
                    cudaStream_t stream);
int fr_tp_ffn_nvfp4(const float *x, const void *wg_shard, const void *wu_shard, const void *wd_shard,
                    const float *sg, const float *su, const float *sd, const float *resid, float *out,
                    int T, int n_embd, int n_ff, int nranks, int rank,
                    void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream);

/* The dense FFN row-sharded over P ranks -- the partitioning BASELINE's
 * north star names: rank r holds gate/up rows [r F_p, (r+1) F_p) (F_p = n_ff
 * / P) and down rows [r E_p, (r+1) E_p) (E_p = n_embd / P, each row over the
 * whole n_ff).  q8_1(x) is computed on every rank; each rank's GLU columns
 * are quantized to q8_1 and stored into every rank's copy of the full q8_1
 * GLU over NVLink (the all-gather of the GLU, 3.6x smaller than f32 and
 * exact: q8_1 blocks never straddle a shard); a bounded wait; each rank's
 * output rows go into column block r of every rank's output (the output
 * all-gather); a second bounded wait adds the residual.  Every output value
 * is one row's dot product on one GPU, so the result equals one GPU's dp4a
 * FFN bit for bit.  The exchange buffers are double-buffered by step parity
 * as for fr_tp_ffn_nvfp4; a buffer of fr_tp_rows_buffer_bytes(T_max, ...)
 * bytes per rank, zeroed once; all ranks call with the same T <= T_max.
 * n_ff % (64 P) == 0, n_embd % 64 == 0, n_embd % P == 0. */
int64_t fr_tp_rows_buffer_bytes(int T, int n_embd, int n_ff, int nranks);
int fr_tp_ffn_rows(const float *x, const void *wg_shard, const void *wu_shard, const void *wd_shard,
                   const float *sg, const float *su, const float *sd, const float *resid, float *out,
                   int T, int n_embd, int n_ff, int nranks, int rank,
                   void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream);

/* ------------------------------------------------------ (e) expert parallel
 * One rank's step of the MoE layer with E/P experts per rank (rank r owns
 * experts [r*E/P, (r+1)*E/P); wg/wu/wd_local hold their rows) and its own T
 * tokens.  The router runs replicated; every routed slot's activation row is
 * stored into the expert owner's exchange buffer over NVLink (fixed capacity
 * T_max * n_used slots per source rank, empty slots marked), a bounded wait
 * sees every rank's rows in, the owner runs its experts, the outputs go back
 * to the source slots the same way, and the token owner combines them in slot
 * order -- the arithmetic and order of fr_moe_ffn_nvfp4 on one GPU, so the
 * result is identical.  No host synchronisation; CUDA-graph capturable.
 * peer_base / local_base: a buffer of fr_ep_buffer_bytes(T_max, n_embd,
 * n_used, P) bytes per rank as for fr_tp_ffn_nvfp4.  All ranks call with the
 * same T.  The reference is single-device; no counterpart. */
int64_t fr_ep_buffer_bytes(int T_max, int n_embd, int n_used, int nranks);
int fr_ep_moe_nvfp4(const float *x, const float *w_r, const void *wg_local, const void *wu_local,
                    const void *wd_local, const float *sg, const float *su, const float *sd, const float *resid,
                    float *out, int T, int T_max, int n_embd, int n_ff, int E, int n_used, float clamp_val, int nranks,
                    int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream);
/* The same layer with this rank's experts repacked tile-major
 * (fr_nvfp4_tile on its stacked [E/P * N, K] expert tensors): the received
 * rows run on the FP4 tensor cores (windows of up to 8 rows per expert);
 * results equal fr_moe_ffn_tiled's to the f32 rounding of the split-K
 * partial sums.  n_embd, n_ff multiples of 256. */
int fr_ep_moe_tiled(const float *x, const float *w_r, const void *wg_t, const void *wu_t, const void *wd_t,
                    const float *sg, const float *su, const float *sd, const float *resid, float *out, int T,
                    int T_max, int n_embd, int n_ff, int E, int n_used, float clamp_val, int nranks, int rank,
                    void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream);

/* Peer buffers for fr_tp_ffn_nvfp4 without any library-side multicast
 * object: fr_ipc_alloc returns a zeroed device buffer and its 64-byte CUDA
 * IPC handle (exchanged between the ranks by the host), fr_ipc_open maps a
 * peer's handle into this process, fr_ipc_close / fr_ipc_free release them. */
int fr_ipc_alloc(int64_t bytes, void **dev_ptr, void *handle64);
int fr_ipc_open(const void *handle64, void **dev_ptr);
int fr_ipc_close(void *dev_ptr);
int fr_ipc_free(void *dev_ptr);

/* ------------------------------------------------- (a5/a6) W4A4 tcgen05 path
 * The reference's Thor launch interface (include/fr_kernels.h:21-57), same
 * arguments, same meaning, same return codes; C++ callers also get the
 * namespace ggml_cuda_flashrt forwarders at the end of this header. */
int64_t fr_sf_bytes(int64_t rows, int64_t K);        /* include/fr_kernels.h:25-29 */
int64_t fr_packed_bytes(int64_t rows, int64_t K);    /* include/fr_kernels.h:31-33 */
/* include/fr_kernels.h:49-50 */
int fr_quantize_act_f32(const float *src, void *dst_packed, void *dst_sfa,
                        int M, int K, cudaStream_t stream);
/* include/fr_kernels.h:56-57 */
int fr_repack_weight(const void *ggml_blocks, void *dst_packed, void *dst_sf,
                     int N, int K, cudaStream_t stream);
/* D [M, N] = alpha * A [M, K] . B [N, K]^T, NVFP4 x NVFP4 block-scaled on
 * tcgen05 (kind::mxf4nvf4), f32 out: a persistent kernel, one CTA per SM,
 * 128 x 256 tiles whose K stages are divided evenly over the CTAs (partial
 * tiles added in a fixed order: deterministic).  K % 64 == 0, N % 16 == 0.
 * include/fr_kernels.h:41-44 */
int fr_gemm_f32out(const void *A_packed, const void *SFA, const void *B_packed, const void *SFB,
                   float *D, int M, int N, int K, float alpha, bool widen, cudaStream_t stream);
/* include/fr_kernels.h:59-65: repack a gate and an up matrix (ggml
 * block_nvfp4, each [n_ff, K]) into one B operand of 2 * n_ff rows, row 2j =
 * gate row j, row 2j+1 = up row j (packed [2 n_ff, K/2], dst_sf of
 * fr_sf_bytes(2 n_ff, K)), byte for byte the reference's
 * repack_weight_pair_interleaved (src/fr_repack.cu:66-136). */
int fr_repack_weight_pair_interleaved(const void *gate_blocks, const void *up_blocks, void *dst_packed,
                                      void *dst_sf, int n_ff, int K, cudaStream_t stream);
/* The prefill FFN's gate/up GEMM with the SwiGLU fused into its epilogue:
 * D [M, n_ff] f32 = silu(alpha * A . G^T) * (alpha * A . U^T), B_pair from
 * fr_repack_weight_pair_interleaved, so the [M, 2 n_ff] gate/up product is
 * never written.  The reference fuses GeGLU the same way
 * (vendor/csrc/gemm/fp4/cutlass_fp4_gemm_geglu_il_sm100.cuh:1-25); this is
 * its SiLU form.  K % 64 == 0, n_ff % 8 == 0. */
int fr_gemm_swiglu_f32out(const void *A_packed, const void *SFA, const void *B_pair, const void *SFB_pair,
                          float *D, int M, int n_ff, int K, float alpha, cudaStream_t stream);

/* ------------------------------------- (f1/f2) decode step of the MoE decoder
 * The kernels around the NVFP4 matmuls of a decode step of the synthetic
 * 48-layer MoE decoder (llama.cpp runs these ops as
 * ggml graph nodes, and the reference replaces the attention part with its
 * Flint windows frt_fa_decode / frt_fa_combine, src/fr_win_flint_sm120.cu:
 * 2411-2846, and the QKV post, include/fr_kernels.h qkv_post).  T sequences
 * decode one token each per step; `pos` is a device int32 holding the step's
 * position (the same for every sequence); it is read after the previous
 * kernel completes, so a whole step can be captured once as a CUDA graph and
 * replayed.
 *   fr_rmsnorm_f32     y = x / sqrt(mean(x^2) + eps) * w  (w nullable = 1), [T, H]
 *   fr_rope_kv_f16     qkv [T, (nh + 2 nkv) * d] (q heads, k heads, v heads):
 *                      NeoX RoPE (pairs i, i + d/2, theta_i = pos *
 *                      base^(-2i/d)) of q (scaled by 1/sqrt(d), into q_r
 *                      [T, nh, d] f32) and k, which with v is appended as f16
 *                      at row pos of the caches [T, nkv, ctx, d]
 *   fr_attn_decode_f16 GQA decode attention over keys 0..pos: out [T, nh * d]
 *                      = softmax(q k^T) v per head, KV head of head h = h /
 *                      (nh / nkv); tcgen05 tensor cores (f16 operands, f32
 *                      accumulation, probabilities rounded to f16 for the PV
 *                      product); d == 128, nh == 8 nkv, ctx % 128 == 0; the
 *                      caches zero-initialised before first use.  Each
 *                      (sequence, KV head) walks its 128-key chunks over S
 *                      CTAs, S = min(ctx / 128, 2 x SMs / (T x nkv)) (the
 *                      FR_ATTN_SPLITS environment variable, read once, sets S
 *                      for tuning); with S > 1 the last CTA merges the splits
 *                      in split order, so results are deterministic for a
 *                      given S
 *   fr_embed_nvfp4     x[t] = NVFP4 row of token prompt[t * prompt_ld + pos]
 *                      while pos < prompt_len, else of gen[t]
 *   fr_argmax_f32      tok[t] = argmax logits[t, :] (ties: lowest index)
 *   fr_pos_advance     *pos += 1 (the step's last kernel)
 *   fr_synth_nvfp4_device  NVFP4 rows with the synthetic weight distribution
 *                      (codes uniform over 0..15, scales e4m3(|N(0,1)| *
 *                      sigma)), generated on the device for multi-GB models */
int fr_rmsnorm_f32(const float *x, const float *w, float *y, int T, int H, float eps, cudaStream_t stream);
int fr_rope_kv_f16(const float *qkv, const int32_t *pos, float *q_r, void *kcache, void *vcache, int T, int nh,
                   int nkv, int head_dim, int ctx, float rope_base, cudaStream_t stream);
int fr_attn_decode_f16(const float *q_r, const void *kcache, const void *vcache, const int32_t *pos, float *out,
                       int T, int nh, int nkv, int head_dim, int ctx, cudaStream_t stream);
int fr_embed_nvfp4(const void *table, int vocab, int H, const int32_t *prompt, int prompt_ld, int prompt_len,
                   const int32_t *gen, const int32_t *pos, float *x, int T, cudaStream_t stream);
int fr_argmax_f32(const float *logits, int T, int V, int32_t *tok, cudaStream_t stream);
int fr_pos_advance(int32_t *pos, cudaStream_t stream);
int fr_synth_nvfp4_device(uint64_t seed, int64_t rows, int64_t K, double scale_sigma, void *out,
                          cudaStream_t stream);

/* ------------------------------------------------------ host transfers
 * fr_copy_pinned: copies `bytes` between device memory and page-locked host
 * memory (either side may be host; cudaHostAlloc / pin_memory buffers) with
 * SM loads and stores over PCIe inside the stream's PDL chain, instead of a
 * copy-engine memcpy, whose fixed latency dominates the few KB a decode step
 * moves and which breaks the chain of programmatic launches around it.  It
 * waits for the previous kernel of the stream to finish before it writes.
 * Host pointers must be mapped (cudaHostGetDevicePointer succeeds: true of
 * every page-locked allocation on a unified-address system); both addresses
 * and `bytes` 16-byte aligned.  FR_EINVAL otherwise.  Not a reference
 * interface: the ggml backend's tensor_set/get do the same transfers with
 * cudaMemcpyAsync. */
int fr_copy_pinned(void *dst, const void *src, int64_t bytes, cudaStream_t stream);

/* ------------------------------------------------------ synthetic inputs
 * Host-side, deterministic (splitmix64 + Box-Muller in double) generator of
 * the benchmark inputs: NVFP4 rows with E2M1 codes uniform over 0..15 and
 * sub-block scales e4m3(|N(0,1)| * scale_sigma) (RNE), and N(mean, std) f32. */
void fr_synth_nvfp4(uint64_t seed, int64_t rows, int64_t K, double scale_sigma, void *out_blocks);
void fr_synth_normal(uint64_t seed, int64_t n, double mean, double stddev, float *out);

#ifdef __cplusplus
} /* extern "C" */

/* Drop-in C++ spellings of the reference launch interface. */
namespace ggml_cuda_flashrt {
static inline int64_t round_up_i64(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
static inline int64_t sf_bytes(int64_t rows, int64_t K) { return fr_sf_bytes(rows, K); }
static inline int64_t packed_bytes(int64_t rows, int64_t K) { return fr_packed_bytes(rows, K); }
static inline int gemm_f32out(const void *A_packed, const void *SFA, const void *B_packed,
                              const void *SFB, float *D, int M, int N, int K, float alpha,
                              bool widen, cudaStream_t stream) {
    return fr_gemm_f32out(A_packed, SFA, B_packed, SFB, D, M, N, K, alpha, widen, stream);
}
static inline int quantize_act_f32(const float *src, void *dst_packed, void *dst_sfa, int M, int K,
                                   cudaStream_t stream) {
    return fr_quantize_act_f32(src, dst_packed, dst_sfa, M, K, stream);
}
static inline int repack_weight(const void *ggml_blocks, void *dst_packed, void *dst_sf, int N, int K,
                                cudaStream_t stream) {
    return fr_repack_weight(ggml_blocks, dst_packed, dst_sf, N, K, stream);
}
} /* namespace ggml_cuda_flashrt */
#endif

#endif /* FR_B200_H */
