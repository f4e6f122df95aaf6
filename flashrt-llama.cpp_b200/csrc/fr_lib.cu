// fr_lib.cu -- the library's single CUDA translation unit: kernels from the
// fr_*.cuh headers plus the C-ABI entry points of include/fr_b200.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "fr_common.cuh"
#include "fr_runtime.cuh"
#include "fr_gemv.cuh"
#include "fr_moe.cuh"
#include "fr_w4a4.cuh"
#include "fr_gemm.cuh"
#include "fr_gemm2.cuh"
#include "fr_attn.cuh"
#include "fr_tcgemv.cuh"
#include "fr_fp4mv.cuh"
#include "fr_fp4tile.cuh"
#include "fr_fp4moe.cuh"

#include <cudaTypedefs.h>

namespace frb {

std::atomic<uint64_t> g_launches{0};

static bool tc_shape_ok(const void *w0, const void *w1, int64_t w_ld, int K);
static int tc_matvec(const uint8_t *w0, const uint8_t *w1, int64_t w_ld, int N, int K, const float *x, int64_t ldx,
                     const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                     int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream);
static int fp4_matvec(const uint8_t *w0, const uint8_t *w1, int64_t w_ld, int N, int K, const float *x, int64_t ldx,
                      const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                      int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream);
// tensor-parallel output of the plain form (see FtArgs); ctas_out receives
// the number of CTAs launched, which each count into the flags
struct TpOut {
    uint8_t *const *peer_base;
    int npeers, rank;
    int64_t peer_off, flag_off;
    const unsigned int *epoch;   // step parity of the receiving slots
    int64_t par_bytes;
    unsigned *ctas_out;
};
static int fp4t_matvec(const uint8_t *w0, const uint8_t *w1, int N, int K, const float *x, int64_t ldx,
                       const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                       int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream,
                       float *amax_out = nullptr, const float *amax_in = nullptr, const TpOut *tp = nullptr);
constexpr int FP4_MAX_T = 16;                      // tokens per launch of the FP4 tensor-core matvecs
// Which matvec runs on weights in ggml's layout: the dp4a kernel for up to two
// tokens and for shapes the TMA paths cannot take, the f16 tensor-core kernel
// for batches; the FP4 tensor-core kernel on ggml's layout (TMA boxes of row
// segments, slower than the tiled layout's contiguous stream) when forced.
// The path can be forced (FR_MATVEC / fr_set_matvec_path).
enum MvKind : int { MV_DP4A = 0, MV_TC16 = 1, MV_FP4 = 2 };
static MvKind mv_kind(const void *w0, const void *w1, int64_t w_ld, int K, int T) {
    const int path = matvec_path();
    if (path == 1 || !tc_shape_ok(w0, w1, w_ld, K)) return MV_DP4A;
    if (path == 2) return MV_TC16;
    if (path == 3) return MV_FP4;
    return T <= 2 ? MV_DP4A : MV_TC16;
}
static bool use_tc(const void *w0, const void *w1, int64_t w_ld, int K, int T) {
    return mv_kind(w0, w1, w_ld, K, T) != MV_DP4A;
}
// tensor-core matvec of either kind (the caller checked use_tc)
static int tcx_matvec(const uint8_t *w0, const uint8_t *w1, int64_t w_ld, int N, int K, const float *x, int64_t ldx,
                      const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                      int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream) {
    if (mv_kind(w0, w1, w_ld, K, T) == MV_FP4)
        return fp4_matvec(w0, w1, w_ld, N, K, x, ldx, q8, ldq, T, s0, s1, resid, ldr, y, ldy, dual, stream);
    return tc_matvec(w0, w1, w_ld, N, K, x, ldx, q8, ldq, T, s0, s1, resid, ldr, y, ldy, dual, stream);
}

// ------------------------------------------------------------- device info
const DevInfo &dev_info() {
    static DevInfo infos[64];
    static bool have[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    std::lock_guard<std::mutex> lk(mu);
    if (!have[dev]) {
        DevInfo d;
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        infos[dev] = d;
        have[dev] = true;
    }
    return infos[dev];
}

// ------------------------------------------------------------- fault injection
static std::mutex g_fault_mu;
static std::string g_fault_site;
static bool g_fault_env_read = false;

bool fault_hit(const char *site) {
    std::lock_guard<std::mutex> lk(g_fault_mu);
    if (!g_fault_env_read) {
        g_fault_env_read = true;
        const char *e = getenv("FR_FAULT");
        if (e && *e) g_fault_site = e;
    }
    if (!g_fault_site.empty() && g_fault_site == site) {
        g_fault_site.clear();
        return true;
    }
    return false;
}

// ------------------------------------------------------------- workspaces
int workspace_get(int purpose, size_t bytes, cudaStream_t stream, void **out) {
    static Workspace ws[64][WS_COUNT];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || purpose < 0 || purpose >= WS_COUNT) return FR_EINVAL;
    std::lock_guard<std::mutex> lk(mu);
    Workspace &w = ws[dev][purpose];
    if (w.cap < bytes) {
        if (stream_capturing(stream)) return FR_ECAPTURE;
        if (w.ptr) {
            cudaError_t e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return cuda_rc(e);
            cudaFree(w.ptr);
            w.ptr = nullptr;
            w.cap = 0;
        }
        size_t cap = std::max<size_t>(bytes, 1 << 20);
        cudaError_t e = cudaMalloc(&w.ptr, cap);
        if (e != cudaSuccess) { w.ptr = nullptr; return cuda_rc(e); }
        w.cap = cap;
    }
    *out = w.ptr;
    return FR_OK;
}

int workspace_get_zeroed(int purpose, size_t bytes, cudaStream_t stream, void **out) {
    // its own grow-only buffers, cleared on every (re)allocation
    static Workspace ws[64][WS_COUNT];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || purpose < 0 || purpose >= WS_COUNT) return FR_EINVAL;
    std::lock_guard<std::mutex> lk(mu);
    Workspace &w = ws[dev][purpose];
    if (w.cap < bytes) {
        if (stream_capturing(stream)) return FR_ECAPTURE;
        if (w.ptr) {
            cudaError_t e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return cuda_rc(e);
            cudaFree(w.ptr);
            w.ptr = nullptr;
            w.cap = 0;
        }
        const size_t cap = std::max<size_t>(bytes, 1 << 20);
        cudaError_t e = cudaMalloc(&w.ptr, cap);
        if (e != cudaSuccess) { w.ptr = nullptr; return cuda_rc(e); }
        e = cudaMemsetAsync(w.ptr, 0, cap, stream);
        if (e != cudaSuccess) return cuda_rc(e);
        w.cap = cap;
    }
    *out = w.ptr;
    return FR_OK;
}

static std::atomic<int> g_matvec_path{-1};
int matvec_path() {
    int v = g_matvec_path.load();
    if (v < 0) {
        const char *e = getenv("FR_MATVEC");
        v = 0;
        if (e && std::string(e) == "dp4a") v = 1;
        if (e && std::string(e) == "tc") v = 2;
        if (e && std::string(e) == "fp4") v = 3;
        g_matvec_path.store(v);
    }
    return v;
}

// ------------------------------------------------------------- matvec launcher
struct GvPlan {
    int LG, TT, R2, SR, rows_per_cta, grid, n_slots, slot_bytes;
    size_t smem;
};

static int pick_lg(int NB) {
    int best = 32;
    double best_u = -1.0;
    for (int lg = 32; lg >= 4; lg >>= 1) {
        const int it = (NB + lg - 1) / lg;
        const double u = static_cast<double>(NB) / (lg * it);
        if (u > best_u + 1e-9) { best_u = u; best = lg; }
    }
    return best;
}

static int pow2_tokens(int nt) { return nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8; }

static size_t gv_act_bytes(int nt, int K) { return static_cast<size_t>(nt) * (K / 64) * (64 + 8); }

// One CTA per SM; a stage is 8 warps x (32/LG) lane groups x R2 rows, sized
// to 16-80 KB so each operand moves in one large bulk copy; the ring holds as
// many stages as shared memory allows (2..8).
static GvPlan gv_plan(int N, int K, int64_t w_ld, int T, bool dual) {
    const DevInfo &di = dev_info();
    GvPlan pl{};
    const int NB = K / 64;
    pl.LG = pick_lg(NB);
    const int gpw = 32 / pl.LG;
    constexpr int CW = GV_MAIN_CW;
    const int smem_cap = (di.smem_optin > 0 ? di.smem_optin : 227 * 1024) - 1024;
    const long row_bytes = w_ld * (dual ? 2 : 1);
    int nt = std::min(T, 8);
    while (nt > 1 && gv_act_bytes(nt, K) + 2048 + 2 * static_cast<size_t>(CW * gpw) * row_bytes >
                         static_cast<size_t>(smem_cap))
        nt = nt / 2;
    pl.TT = pow2_tokens(nt);
    const size_t act = gv_act_bytes(nt, K);
    const int sms = std::max(1, di.sms);
    pl.rows_per_cta = (N + sms - 1) / sms;
    pl.grid = (N + pl.rows_per_cta - 1) / pl.rows_per_cta;
    // the largest stage (<= 80 KB, two fit) that still gives the CTA at least
    // two stages, so its first rows are decoded while the rest arrive
    pl.R2 = 1;
    if (pl.TT <= 2) {
        for (int r2 : {4, 2}) {
            const long st = static_cast<long>(CW) * gpw * r2 * row_bytes;
            if (st <= 80 * 1024 && 2 * st + 2048 + static_cast<long>(act) <= smem_cap &&
                pl.rows_per_cta >= 2 * CW * gpw * r2) {
                pl.R2 = r2;
                break;
            }
        }
    }
    pl.SR = CW * gpw * pl.R2;
    pl.slot_bytes = static_cast<int>((pl.SR * row_bytes + 15) / 16 * 16);
    const long budget = smem_cap - 2048 - static_cast<long>(act);
    // no more ring slots than the CTA has stages: a small matvec then leaves
    // shared memory for the next launch's CTAs to start streaming early
    const long n_st = (pl.rows_per_cta + pl.SR - 1) / pl.SR;
    pl.n_slots = static_cast<int>(std::max(1L, std::min(std::min(8L, n_st), budget / pl.slot_bytes)));
    pl.smem = 2048 + static_cast<size_t>(pl.n_slots) * pl.slot_bytes + act;
    return pl;
}

template <int LG, int TT, int EPI, int R2>
static int gv_launch_inst(const GvParams &p, const GvPlan &pl, cudaStream_t stream) {
    auto kern = k_gemv<LG, TT, EPI, R2, GV_MAIN_CW>;
    static bool attr_done[64] = {};
    const int arc = allow_max_smem(kern, attr_done);
    if (arc != FR_OK) return arc;
    return launch_pdl(kern, dim3(pl.grid), dim3((GV_MAIN_CW + 1) * 32), pl.smem, stream, p);
}

template <int LG, int EPI>
static int gv_launch_tt(const GvParams &p, const GvPlan &pl, cudaStream_t stream) {
    if (pl.TT == 1) {
        if (pl.R2 == 4) return gv_launch_inst<LG, 1, EPI, 4>(p, pl, stream);
        if (pl.R2 == 2) return gv_launch_inst<LG, 1, EPI, 2>(p, pl, stream);
        return gv_launch_inst<LG, 1, EPI, 1>(p, pl, stream);
    }
    if (pl.TT == 2) {
        if (pl.R2 == 4) return gv_launch_inst<LG, 2, EPI, 4>(p, pl, stream);
        if (pl.R2 == 2) return gv_launch_inst<LG, 2, EPI, 2>(p, pl, stream);
        return gv_launch_inst<LG, 2, EPI, 1>(p, pl, stream);
    }
    if (pl.TT == 4) return gv_launch_inst<LG, 4, EPI, 1>(p, pl, stream);
    return gv_launch_inst<LG, 8, EPI, 1>(p, pl, stream);
}

template <int EPI>
static int gv_launch_lg(const GvParams &p, const GvPlan &pl, cudaStream_t stream) {
    switch (pl.LG) {
    case 32: return gv_launch_tt<32, EPI>(p, pl, stream);
    case 16: return gv_launch_tt<16, EPI>(p, pl, stream);
    case 8: return gv_launch_tt<8, EPI>(p, pl, stream);
    default: return gv_launch_tt<4, EPI>(p, pl, stream);
    }
}

// Runs the matvec over all T tokens (token windows of at most TT per launch).
static int gemv_run(GvParams p, int T, bool dual, cudaStream_t stream) {
    const GvPlan pl = gv_plan(p.N, p.K, p.w_ld, T, dual);
    p.rows_per_cta = pl.rows_per_cta;
    p.rows_per_stage = pl.SR;
    p.n_slots = pl.n_slots;
    p.slot_bytes = pl.slot_bytes;
    p.word_mode = (p.w_ld % 16 != 0 || (reinterpret_cast<uintptr_t>(p.w0) & 15) ||
                   (p.w1 && (reinterpret_cast<uintptr_t>(p.w1) & 15))) ? 1 : 0;
    for (int t0 = 0; t0 < T; t0 += pl.TT) {
        p.t0 = t0;
        p.nt = std::min(pl.TT, T - t0);
        const int rc = dual ? gv_launch_lg<GV_SWIGLU>(p, pl, stream) : gv_launch_lg<GV_PLAIN>(p, pl, stream);
        if (rc != FR_OK) return rc;
    }
    return FR_OK;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int check_gemv_shape(const void *w, int64_t w_ld, int N, int K, int T) {
    if (!w || N <= 0 || K <= 0 || T <= 0) return FR_EINVAL;
    if (K % 64 != 0) return FR_EINVAL;
    if (w_ld < static_cast<int64_t>(K / 64) * NV_BYTES || w_ld % 4 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) & 3) != 0) return FR_EINVAL;
    return FR_OK;
}

static int quantize_launch2(const float *x, int64_t ldx, int n_in, int64_t ldx_in, void *q8, int64_t ldq, int rows,
                            int K, cudaStream_t stream) {
    const int64_t chunks = static_cast<int64_t>(rows) * (K / 32);
    const int grid = static_cast<int>((chunks + 7) / 8);
    return launch_pdl(k_quantize_q8_1, dim3(grid), dim3(256), 0, stream, x, ldx, n_in, ldx_in,
                      static_cast<uint8_t *>(q8), ldq, rows, K);
}

static int quantize_launch(const float *x, int64_t ldx, void *q8, int64_t ldq, int T, int K, cudaStream_t stream) {
    return quantize_launch2(x, ldx, 1, 0, q8, ldq, T, K, stream);
}

} // namespace frb

using namespace frb;

// ======================================================================
// C-ABI
// ======================================================================
extern "C" {

int fr_version(void) { return 1; }

const char *fr_strerror(int rc) {
    switch (rc) {
    case FR_OK: return "ok";
    case FR_EINVAL: return "invalid shape, alignment or pointer";
    case FR_ELAYOUT: return "scale layout larger than the buffer";
    case FR_ECAPTURE: return "workspace growth refused during stream capture";
    case FR_EINJECTED: return "injected fault";
    case FR_ENODEVICE: return "no suitable CUDA device";
    case FR_ETOOBIG: return "request larger than the static scratch";
    default: break;
    }
    if (rc < 0 && rc > -1000) return cudaGetErrorString(static_cast<cudaError_t>(-rc));
    return "unknown error";
}

int fr_device_status(uint32_t *status, int clear) {
    if (!status) return FR_EINVAL;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_rc(e);
    unsigned v = 0;
    e = cudaMemcpyFromSymbol(&v, g_fr_status, sizeof(v));
    if (e != cudaSuccess) return cuda_rc(e);
    *status = v;
    if (clear) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(g_fr_status, &z, sizeof(z));
        if (e != cudaSuccess) return cuda_rc(e);
    }
    return FR_OK;
}

int64_t fr_set_wait_ns(int64_t ns) {
    if (ns < 1000 || ns > static_cast<int64_t>(FR_WAIT_NS_MAX)) return FR_EINVAL;
    unsigned long long prev = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&prev, g_fr_wait_ns, sizeof(prev));
    if (e != cudaSuccess) return cuda_rc(e);
    const unsigned long long v = static_cast<unsigned long long>(ns);
    e = cudaMemcpyToSymbol(g_fr_wait_ns, &v, sizeof(v));
    if (e != cudaSuccess) return cuda_rc(e);
    return static_cast<int64_t>(prev);
}

int fr_fault_inject(const char *site) {
    std::lock_guard<std::mutex> lk(g_fault_mu);
    g_fault_env_read = true;
    g_fault_site = site ? site : "";
    return FR_OK;
}

uint64_t fr_kernel_launches(void) { return g_launches.load(); }

int fr_set_matvec_path(int path) {
    if (path < 0 || path > 3) return FR_EINVAL;
    const int prev = matvec_path();
    g_matvec_path.store(path);
    return prev;
}

int64_t fr_nvfp4_row_bytes(int64_t K) { return K / 64 * NV_BYTES; }
int64_t fr_q8_1_row_bytes(int64_t K) { return K / 32 * Q8_BYTES; }

int fr_quantize_q8_1(const float *x, int64_t ldx, void *q8, int64_t ldq, int T, int K, cudaStream_t stream) {
    if (fault_hit("fr_quantize_q8_1")) return FR_EINJECTED;
    if (!x || !q8 || T <= 0 || K <= 0 || K % 32 != 0 || ldx < K || ldq < K / 32) return FR_EINVAL;
    return quantize_launch(x, ldx, q8, ldq, T, K, stream);
}

int fr_gemv_nvfp4_q8_1(const void *w, int64_t w_ld, const void *q8, int64_t ldq, const float *scale,
                       const float *resid, int64_t ldr, float *y, int64_t ldy, int N, int K, int T,
                       cudaStream_t stream) {
    if (fault_hit("fr_gemv_nvfp4_q8_1")) return FR_EINJECTED;
    int rc = check_gemv_shape(w, w_ld, N, K, T);
    if (rc != FR_OK) return rc;
    if (!q8 || !y || ldq < K / 32 || ldy < N || (resid && ldr < N)) return FR_EINVAL;
    if (use_tc(w, nullptr, w_ld, K, T))
        return tcx_matvec(static_cast<const uint8_t *>(w), nullptr, w_ld, N, K, nullptr, 0,
                         static_cast<const uint8_t *>(q8), ldq, T, scale, nullptr, resid, ldr, y, ldy, false, stream);
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(w);
    p.w_ld = w_ld;
    p.q8 = static_cast<const uint8_t *>(q8);
    p.ldq = ldq;
    p.s0 = scale;
    p.resid = resid;
    p.ldr = ldr;
    p.y = y;
    p.ldy = ldy;
    p.N = N;
    p.K = K;
    return gemv_run(p, T, false, stream);
}

int fr_gemv_nvfp4_f32(const void *w, int64_t w_ld, const float *x, int64_t ldx, const float *scale,
                      const float *resid, int64_t ldr, float *y, int64_t ldy, int N, int K, int T,
                      cudaStream_t stream) {
    if (fault_hit("fr_gemv_nvfp4_f32")) return FR_EINJECTED;
    int rc = check_gemv_shape(w, w_ld, N, K, T);
    if (rc != FR_OK) return rc;
    if (!x || !y || ldx < K || ldy < N || (resid && ldr < N)) return FR_EINVAL;
    if (use_tc(w, nullptr, w_ld, K, T))
        return tcx_matvec(static_cast<const uint8_t *>(w), nullptr, w_ld, N, K, x, ldx, nullptr, 0, T, scale, nullptr,
                         resid, ldr, y, ldy, false, stream);
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(w);
    p.w_ld = w_ld;
    p.x = x;
    p.ldx = ldx;
    p.s0 = scale;
    p.resid = resid;
    p.ldr = ldr;
    p.y = y;
    p.ldy = ldy;
    p.N = N;
    p.K = K;
    return gemv_run(p, T, false, stream);
}

int fr_gemv_nvfp4_q8_1_swiglu(const void *wg, const void *wu, int64_t w_ld, const void *q8, int64_t ldq,
                              const float *sg, const float *su, float *y, int64_t ldy, int N, int K, int T,
                              cudaStream_t stream) {
    if (fault_hit("fr_gemv_nvfp4_q8_1_swiglu")) return FR_EINJECTED;
    int rc = check_gemv_shape(wg, w_ld, N, K, T);
    if (rc != FR_OK) return rc;
    if (!wu || (reinterpret_cast<uintptr_t>(wu) & 3) || !q8 || !y || ldq < K / 32 || ldy < N) return FR_EINVAL;
    if (use_tc(wg, wu, w_ld, K, T))
        return tcx_matvec(static_cast<const uint8_t *>(wg), static_cast<const uint8_t *>(wu), w_ld, N, K, nullptr, 0,
                         static_cast<const uint8_t *>(q8), ldq, T, sg, su, nullptr, 0, y, ldy, true, stream);
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(wg);
    p.w1 = static_cast<const uint8_t *>(wu);
    p.w_ld = w_ld;
    p.q8 = static_cast<const uint8_t *>(q8);
    p.ldq = ldq;
    p.s0 = sg;
    p.s1 = su;
    p.y = y;
    p.ldy = ldy;
    p.N = N;
    p.K = K;
    return gemv_run(p, T, true, stream);
}

int fr_mul_mat_nvfp4(const void *src0, int64_t nb01, const float *src1, int64_t ld1, float *dst, int64_t ldd,
                     int N, int K, int T, cudaStream_t stream) {
    if (fault_hit("fr_mul_mat_nvfp4")) return FR_EINJECTED;
    int rc = check_gemv_shape(src0, nb01, N, K, T);
    if (rc != FR_OK) return rc;
    if (!src1 || !dst || ld1 < K || ldd < N) return FR_EINVAL;
    if (use_tc(src0, nullptr, nb01, K, T))
        return tcx_matvec(static_cast<const uint8_t *>(src0), nullptr, nb01, N, K, src1, ld1, nullptr, 0, T, nullptr,
                         nullptr, nullptr, 0, dst, ldd, false, stream);
    if (T <= 2) return fr_gemv_nvfp4_f32(src0, nb01, src1, ld1, nullptr, nullptr, 0, dst, ldd, N, K, T, stream);
    void *q8 = nullptr;
    rc = workspace_get(WS_Q8, static_cast<size_t>(T) * (K / 32) * Q8_BYTES, stream, &q8);
    if (rc != FR_OK) return rc;
    rc = quantize_launch(src1, ld1, q8, K / 32, T, K, stream);
    if (rc != FR_OK) return rc;
    return fr_gemv_nvfp4_q8_1(src0, nb01, q8, K / 32, nullptr, nullptr, 0, dst, ldd, N, K, T, stream);
}

int fr_ffn_nvfp4(const float *x, const void *wg, const void *wu, const void *wd, const float *sg,
                 const float *su, const float *sd, const float *resid, float *out, int T, int n_embd,
                 int n_ff, float *chk_glu, void *chk_glu_q8, cudaStream_t stream) {
    if (fault_hit("fr_ffn_nvfp4")) return FR_EINJECTED;
    if (!x || !wg || !wu || !wd || !out || T <= 0 || n_embd % 256 != 0 || n_ff % 256 != 0) return FR_EINVAL;
    if (!aligned16(wg) || !aligned16(wu) || !aligned16(wd)) return FR_EINVAL;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(n_ff) / 64 * NV_BYTES;
    int rc;
    float *glu = chk_glu;
    if (!glu) {
        void *p = nullptr;
        rc = workspace_get(WS_GLU, static_cast<size_t>(T) * n_ff * sizeof(float), stream, &p);
        if (rc != FR_OK) return rc;
        glu = static_cast<float *>(p);
    }
    if (use_tc(wg, wu, ld_gu, n_embd, T) && use_tc(wd, nullptr, ld_d, n_ff, T)) {
        // tensor-core path: the hi/lo activation kernels quantize x and the GLU
        // to q8_1 on the way (no q8_1 blocks needed)
        rc = tcx_matvec(static_cast<const uint8_t *>(wg), static_cast<const uint8_t *>(wu), ld_gu, n_ff, n_embd, x,
                       n_embd, nullptr, 0, T, sg, su, nullptr, 0, glu, n_ff, true, stream);
        if (rc != FR_OK) return rc;
        if (chk_glu_q8) {
            rc = quantize_launch(glu, n_ff, chk_glu_q8, n_ff / 32, T, n_ff, stream);
            if (rc != FR_OK) return rc;
        }
        return tcx_matvec(static_cast<const uint8_t *>(wd), nullptr, ld_d, n_embd, n_ff, glu, n_ff, nullptr, 0, T, sd,
                         nullptr, resid, n_embd, out, n_embd, false, stream);
    }
    // q8_1(x) in its own small kernel: under PDL it overlaps the start of the
    // gate/up weight stream, which a quantizing prologue would delay
    void *q8x = nullptr;
    rc = workspace_get(WS_Q8, static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES, stream, &q8x);
    if (rc != FR_OK) return rc;
    rc = quantize_launch(x, n_embd, q8x, n_embd / 32, T, n_embd, stream);
    if (rc != FR_OK) return rc;
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(wg);
    p.w1 = static_cast<const uint8_t *>(wu);
    p.w_ld = ld_gu;
    p.q8 = static_cast<const uint8_t *>(q8x);
    p.ldq = n_embd / 32;
    p.s0 = sg;
    p.s1 = su;
    p.y = glu;
    p.ldy = n_ff;
    p.N = n_ff;
    p.K = n_embd;
    rc = gemv_run(p, T, true, stream);
    if (rc != FR_OK) return rc;
    // q8_1 of the GLU, likewise a separate kernel overlapped by PDL
    void *gq8 = chk_glu_q8;
    if (!gq8) {
        rc = workspace_get(WS_GLUQ8, static_cast<size_t>(T) * (n_ff / 32) * Q8_BYTES, stream, &gq8);
        if (rc != FR_OK) return rc;
    }
    rc = quantize_launch(glu, n_ff, gq8, n_ff / 32, T, n_ff, stream);
    if (rc != FR_OK) return rc;
    GvParams q{};
    q.w0 = static_cast<const uint8_t *>(wd);
    q.w_ld = ld_d;
    q.q8 = static_cast<const uint8_t *>(gq8);
    q.ldq = n_ff / 32;
    q.s0 = sd;
    q.resid = resid;
    q.ldr = n_embd;
    q.y = out;
    q.ldy = n_embd;
    q.N = n_embd;
    q.K = n_ff;
    return gemv_run(q, T, false, stream);
}

} // extern "C"

// ======================================================================
// Dense FFN without device allocation (static scratch).  For callers that
// cannot call cudaMalloc: graph capture, hosts whose allocator plans every
// buffer up front, fixed device-memory budgets.
// ======================================================================
namespace frb {

static __device__ __align__(256) unsigned char g_ffn_noalloc_scratch[FR_FFN_NOALLOC_SCRATCH_BYTES];

// Device address of g_ffn_noalloc_scratch for the current device.  In host
// code the array's name is only a host-side stand-in, so the address is looked
// up once per device with that device current and cached.
static int ffn_noalloc_scratch(unsigned char **out) {
    static unsigned char *addr[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_rc(e);
    if (dev < 0 || dev >= 64) return FR_ENODEVICE;
    std::lock_guard<std::mutex> lk(mu);
    if (addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_ffn_noalloc_scratch);
        if (e != cudaSuccess) return cuda_rc(e);
        addr[dev] = static_cast<unsigned char *>(p);
    }
    *out = addr[dev];
    return FR_OK;
}

} // namespace frb

extern "C" int fr_ffn_nvfp4_noalloc(const float *x, const void *wg, const void *wu, const void *wd,
                                    const float *sg, const float *su, const float *sd, const float *resid,
                                    float *out, int T, int n_embd, int n_ff, cudaStream_t stream) {
    if (fault_hit("fr_ffn_nvfp4_noalloc")) return FR_EINJECTED;
    if (!x || !wg || !wu || !wd || !out || T <= 0 || n_embd % 256 != 0 || n_ff % 256 != 0) return FR_EINVAL;
    if (!aligned16(wg) || !aligned16(wu) || !aligned16(wd)) return FR_EINVAL;
    const size_t q8x_bytes = static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES;
    const size_t glu_bytes = static_cast<size_t>(T) * n_ff * sizeof(float);
    const size_t gq8_bytes = static_cast<size_t>(T) * (n_ff / 32) * Q8_BYTES;
    // each piece starts on a 256-byte boundary
    const size_t o_glu = (q8x_bytes + 255) / 256 * 256;
    const size_t o_gq8 = o_glu + (glu_bytes + 255) / 256 * 256;
    if (o_gq8 + gq8_bytes > FR_FFN_NOALLOC_SCRATCH_BYTES) return FR_ETOOBIG;
    unsigned char *scratch = nullptr;
    int rc = ffn_noalloc_scratch(&scratch);
    if (rc != FR_OK) return rc;
    void *q8x = scratch;
    float *glu = reinterpret_cast<float *>(scratch + o_glu);
    void *gq8 = scratch + o_gq8;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(n_ff) / 64 * NV_BYTES;
    rc = quantize_launch(x, n_embd, q8x, n_embd / 32, T, n_embd, stream);
    if (rc != FR_OK) return rc;
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(wg);
    p.w1 = static_cast<const uint8_t *>(wu);
    p.w_ld = ld_gu;
    p.q8 = static_cast<const uint8_t *>(q8x);
    p.ldq = n_embd / 32;
    p.s0 = sg;
    p.s1 = su;
    p.y = glu;
    p.ldy = n_ff;
    p.N = n_ff;
    p.K = n_embd;
    rc = gemv_run(p, T, true, stream);
    if (rc != FR_OK) return rc;
    rc = quantize_launch(glu, n_ff, gq8, n_ff / 32, T, n_ff, stream);
    if (rc != FR_OK) return rc;
    GvParams q{};
    q.w0 = static_cast<const uint8_t *>(wd);
    q.w_ld = ld_d;
    q.q8 = static_cast<const uint8_t *>(gq8);
    q.ldq = n_ff / 32;
    q.s0 = sd;
    q.resid = resid;
    q.ldr = n_embd;
    q.y = out;
    q.ldy = n_embd;
    q.N = n_embd;
    q.K = n_ff;
    return gemv_run(q, T, false, stream);
}

// ======================================================================
// MoE: routing, mul_mat_id, fused MoE FFN
// ======================================================================
namespace frb {

struct MoePlan {
    int LG, TT, RS, rows_per_cta, chunks, grid, slot_bytes;
    size_t smem;
};

static MoePlan moe_plan(int N, int K, int64_t w_ld, bool dual, int max_active, int max_tok) {
    const DevInfo &di = dev_info();
    MoePlan pl{};
    const int NB = K / 64;
    pl.LG = pick_lg(NB);
    pl.RS = 32 / pl.LG;
    pl.slot_bytes = static_cast<int>((pl.RS * w_ld * (dual ? 2 : 1) + 15) / 16 * 16);
    pl.TT = pow2_tokens(std::max(1, std::min(8, max_tok)));
    const size_t act = static_cast<size_t>(pl.TT) * NB * 72;
    const int smem_cap = di.smem_optin > 0 ? di.smem_optin : 227 * 1024;
    const long half = (smem_cap - 2048) / 2 - 2048 - 1024 - static_cast<long>(act);
    const long full = smem_cap - 4096 - 1024 - static_cast<long>(act);
    long budget = half >= pl.slot_bytes * 4 ? half : full;
    int max_st = static_cast<int>(std::min<long>(256, budget / pl.slot_bytes));
    max_st = std::max(1, max_st);
    const int target = std::max(1, 2 * di.sms);
    const long rows_total = static_cast<long>(N) * std::max(1, max_active);
    int rpc = static_cast<int>((rows_total + target - 1) / target);
    rpc = (rpc + pl.RS - 1) / pl.RS * pl.RS;
    rpc = std::max(pl.RS, std::min(rpc, max_st * pl.RS));
    pl.rows_per_cta = rpc;
    pl.chunks = (N + rpc - 1) / rpc;
    pl.grid = std::max(1, max_active) * pl.chunks;
    const int n_st = (rpc + pl.RS - 1) / pl.RS;
    pl.smem = 2048 + static_cast<size_t>(n_st) * pl.slot_bytes + act;
    return pl;
}

template <int LG, int TT, bool DUAL>
static int moe_launch_inst(const MoeParams &p, const MoePlan &pl, cudaStream_t stream) {
    auto kern = k_moe_gemv<LG, TT, DUAL>;
    static bool attr_done[64] = {};
    const int arc = allow_max_smem(kern, attr_done);
    if (arc != FR_OK) return arc;
    return launch_pdl(kern, dim3(pl.grid), dim3(GV_THREADS), pl.smem, stream, p);
}

template <int LG, bool DUAL>
static int moe_launch_tt(const MoeParams &p, const MoePlan &pl, cudaStream_t stream) {
    switch (pl.TT) {
    case 1: return moe_launch_inst<LG, 1, DUAL>(p, pl, stream);
    case 2: return moe_launch_inst<LG, 2, DUAL>(p, pl, stream);
    case 4: return moe_launch_inst<LG, 4, DUAL>(p, pl, stream);
    default: return moe_launch_inst<LG, 8, DUAL>(p, pl, stream);
    }
}

// fused_combine (plain form; nullable): if the combine is light enough to
// ride on the last CTA of each row chunk (p.c_* set by the caller), it is
// fused and *fused_combine is set; otherwise p.c_out is cleared.
template <bool DUAL>
static int moe_launch(MoeParams p, int max_active, int max_tok, cudaStream_t stream, bool *fused_combine = nullptr) {
    const MoePlan pl = moe_plan(p.N, p.K, p.w_ld, DUAL, max_active, max_tok);
    if (fused_combine) *fused_combine = false;
    if (!DUAL && p.c_out != nullptr) {
        bool ok = static_cast<long>(p.c_T) * pl.rows_per_cta <= 4096 && p.n_used <= MOE_MAX_USED;
        if (ok) {
            void *cnt = nullptr;
            ok = workspace_get_zeroed(WS_MOECNT, static_cast<size_t>(pl.chunks) * sizeof(unsigned), stream, &cnt) ==
                 FR_OK;
            p.c_cnt = static_cast<unsigned int *>(cnt);
        }
        if (ok) {
            if (fused_combine) *fused_combine = true;
        } else {
            p.c_out = nullptr;
        }
    }
    p.rows_per_cta = pl.rows_per_cta;
    p.chunks = pl.chunks;
    p.rows_per_stage = pl.RS;
    p.slot_bytes = pl.slot_bytes;
    p.word_mode = (p.w_ld % 16 != 0 || p.e_stride % 16 != 0 || (reinterpret_cast<uintptr_t>(p.w0) & 15) ||
                   (p.w1 && (reinterpret_cast<uintptr_t>(p.w1) & 15))) ? 1 : 0;
    switch (pl.LG) {
    case 32: return moe_launch_tt<32, DUAL>(p, pl, stream);
    case 16: return moe_launch_tt<16, DUAL>(p, pl, stream);
    case 8: return moe_launch_tt<8, DUAL>(p, pl, stream);
    default: return moe_launch_tt<4, DUAL>(p, pl, stream);
    }
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// k_group_ids: per-warp expert counts of its 32 warps plus the scan scratch
static int group_smem(int, int) { return static_cast<int>((32 * MOE_MAX_E + 33) * sizeof(int32_t)); }

// Routing (k_route).  aux: 0 = nothing else; 1 = q8_1 rows of x into q8
// (ldq blocks per row); 2 = per-token FP4 digit images of x into img/gtab
// (t_stride bytes per token) -- both computed by extra CTAs of the launch.
static int route_launch(const float *x, int64_t ldx, const float *w_r, int T, int K, int E, int n_used,
                        float clamp_val, float *logits, int32_t *ids, float *wts, int32_t *eoff, int32_t *slots,
                        int32_t *act, cudaStream_t stream, int aux = 0, uint8_t *q8 = nullptr, int64_t ldq = 0,
                        uint8_t *img = nullptr, float *gtab = nullptr, int64_t t_stride = 0) {
    const int n_tc = (T + 3) / 4;
    void *cnt = nullptr;
    int rc = workspace_get_zeroed(WS_ROUTE, static_cast<size_t>(n_tc + 1) * sizeof(unsigned), stream, &cnt);
    if (rc != FR_OK) return rc;
    RouteArgs a{};
    a.x = x;
    a.ldx = ldx;
    a.wr = w_r;
    a.T = T;
    a.K = K;
    a.E = E;
    a.n_used = n_used;
    a.clamp_val = clamp_val;
    a.logits = logits;
    a.ids = ids;
    a.wts = wts;
    a.eoff = eoff;
    a.slots = slots;
    a.act = act;
    a.cnt = static_cast<unsigned int *>(cnt);
    a.n_rt = (E / 4) * n_tc;
    a.aux = aux;
    int n_aux = 0;
    if (aux == 1) {
        a.q8 = q8;
        a.ldq = ldq;
        n_aux = static_cast<int>((static_cast<int64_t>(T) * (K / Q8_ELEMS) + 7) / 8);
    } else if (aux == 2) {
        const int nq = K / Q8_ELEMS;
        a.img = img;
        a.gtab = gtab;
        a.t_stride = t_stride;
        a.img_slices = std::max(1, std::min((nq + 7) / 8, std::max(1, 256 / T)));
        n_aux = T * a.img_slices;
    }
    const size_t smem = (8 * MOE_MAX_E + 33) * sizeof(int);
    return launch_pdl(k_route, dim3(a.n_rt + n_aux), dim3(256), smem, stream, a);
}

static int check_route_shape(int T, int K, int E, int n_used) {
    if (T <= 0 || K <= 0 || K % 4 != 0 || E <= 0 || E % 32 != 0 || E > MOE_MAX_E) return FR_EINVAL;
    if (n_used <= 0 || n_used > MOE_MAX_USED || n_used > E) return FR_EINVAL;
    if (static_cast<long>(T) * n_used > MOE_MAX_SLOTS) return FR_EINVAL;
    return FR_OK;
}

} // namespace frb

extern "C" {

int fr_moe_route(const float *x, int64_t ldx, const float *w_r, int T, int K, int E, int n_used, float clamp_val,
                 float *logits, int32_t *ids, float *wts, int32_t *eoff, int32_t *slots, int32_t *act,
                 cudaStream_t stream) {
    if (fault_hit("fr_moe_route")) return FR_EINJECTED;
    int rc = check_route_shape(T, K, E, n_used);
    if (rc != FR_OK) return rc;
    if (!x || !w_r || !logits || !ids || !wts || !eoff || !slots || !act || ldx < K) return FR_EINVAL;
    if (!aligned16(x) || !aligned16(w_r) || ldx % 4 != 0) return FR_EINVAL;
    return route_launch(x, ldx, w_r, T, K, E, n_used, clamp_val, logits, ids, wts, eoff, slots, act, stream);
}

int fr_mul_mat_id_nvfp4(const void *w, int64_t nb01, int64_t nb02, int E, const float *x, int64_t x_ld_slot,
                        int64_t x_ld_tok, const int32_t *ids, int64_t ids_ld, float *dst, int64_t dst_ld_slot,
                        int64_t dst_ld_tok, int T, int n_used, int N, int K, cudaStream_t stream) {
    if (fault_hit("fr_mul_mat_id_nvfp4")) return FR_EINJECTED;
    if (!w || !x || !ids || !dst || T <= 0 || n_used <= 0 || N <= 0 || K <= 0 || K % 64 != 0) return FR_EINVAL;
    if (E <= 0 || E > MOE_MAX_E || n_used > 64 || static_cast<long>(T) * n_used > MOE_MAX_SLOTS) return FR_EINVAL;
    if (nb01 < static_cast<int64_t>(K / 64) * NV_BYTES || nb01 % 4 != 0 || nb02 < nb01 * N || nb02 % 4 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) & 3) || ids_ld < n_used || x_ld_tok < K) return FR_EINVAL;
    const bool bcast = x_ld_slot == 0;
    const int qrows = bcast ? T : T * n_used;
    const size_t q8_bytes = align256(static_cast<size_t>(qrows) * (K / 32) * Q8_BYTES);
    const size_t grp_bytes = align256(static_cast<size_t>(2 * (E + 1) + T * n_used) * sizeof(int32_t));
    void *wsp = nullptr;
    int rc = workspace_get(WS_MOE, q8_bytes + grp_bytes, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *q8 = static_cast<uint8_t *>(wsp);
    int32_t *eoff = reinterpret_cast<int32_t *>(q8 + q8_bytes);
    int32_t *act = eoff + (E + 1);
    int32_t *slots = act + (E + 1);
    static bool attr_done[64] = {};
    rc = allow_max_smem(k_group_ids, attr_done);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_group_ids, dim3(1), dim3(1024), group_smem(T, n_used), stream, ids, ids_ld, T, n_used, E, eoff,
                    slots, act, 0);
    if (rc != FR_OK) return rc;
    rc = bcast ? quantize_launch2(x, x_ld_tok, 1, 0, q8, K / 32, T, K, stream)
               : quantize_launch2(x, x_ld_tok, n_used, x_ld_slot, q8, K / 32, T * n_used, K, stream);
    if (rc != FR_OK) return rc;
    MoeParams p{};
    p.w0 = static_cast<const uint8_t *>(w);
    p.e_stride = nb02;
    p.w_ld = nb01;
    p.N = N;
    p.K = K;
    p.q8 = q8;
    p.ldq = K / 32;
    p.bcast = bcast ? 1 : 0;
    p.n_used = n_used;
    p.E = E;
    p.eoff = eoff;
    p.slots = slots;
    p.act = act;
    p.out = dst;
    p.ld_tok = dst_ld_tok;
    p.ld_slot = dst_ld_slot;
    return moe_launch<false>(p, std::min(E, T * n_used), T, stream);
}

int fr_moe_ffn_nvfp4(const float *x, const float *w_r, const void *wg, const void *wu, const void *wd, const float *sg,
                     const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                     int E, int n_used, float clamp_val, int32_t *chk_ids, float *chk_wts, float *chk_glu,
                     float *chk_part, cudaStream_t stream) {
    if (fault_hit("fr_moe_ffn_nvfp4")) return FR_EINJECTED;
    int rc = check_route_shape(T, n_embd, E, n_used);
    if (rc != FR_OK) return rc;
    if (!x || !w_r || !wg || !wu || !wd || !out || n_embd % 64 != 0 || n_ff % 64 != 0) return FR_EINVAL;
    if (!aligned16(x) || !aligned16(w_r)) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(wg) & 3) || (reinterpret_cast<uintptr_t>(wu) & 3) ||
        (reinterpret_cast<uintptr_t>(wd) & 3))
        return FR_EINVAL;
    const int S = T * n_used;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(n_ff) / 64 * NV_BYTES;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_logits = take(static_cast<size_t>(T) * E * 4);
    const size_t o_ids = take(static_cast<size_t>(S) * 4);
    const size_t o_wts = take(static_cast<size_t>(S) * 4);
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_q8x = take(static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES);
    const size_t o_glu = take(static_cast<size_t>(S) * n_ff * 4);
    const size_t o_part = take(static_cast<size_t>(S) * n_embd * 4);
    void *wsp = nullptr;
    rc = workspace_get(WS_MOE, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *base = static_cast<uint8_t *>(wsp);
    float *logits = reinterpret_cast<float *>(base + o_logits);
    int32_t *ids = chk_ids ? chk_ids : reinterpret_cast<int32_t *>(base + o_ids);
    float *wts = chk_wts ? chk_wts : reinterpret_cast<float *>(base + o_wts);
    int32_t *eoff = reinterpret_cast<int32_t *>(base + o_eoff);
    int32_t *act = reinterpret_cast<int32_t *>(base + o_act);
    int32_t *slots = reinterpret_cast<int32_t *>(base + o_slots);
    uint8_t *q8x = base + o_q8x;
    float *glu = chk_glu ? chk_glu : reinterpret_cast<float *>(base + o_glu);
    float *part = chk_part ? chk_part : reinterpret_cast<float *>(base + o_part);

    rc = route_launch(x, n_embd, w_r, T, n_embd, E, n_used, clamp_val, logits, ids, wts, eoff, slots, act, stream,
                      1, q8x, n_embd / 32);
    if (rc != FR_OK) return rc;
    MoeParams p{};
    p.w0 = static_cast<const uint8_t *>(wg);
    p.w1 = static_cast<const uint8_t *>(wu);
    p.e_stride = ld_gu * n_ff;
    p.w_ld = ld_gu;
    p.N = n_ff;
    p.K = n_embd;
    p.q8 = q8x;
    p.ldq = n_embd / 32;
    p.bcast = 1;
    p.n_used = n_used;
    p.E = E;
    p.eoff = eoff;
    p.slots = slots;
    p.act = act;
    p.s0 = sg;
    p.s1 = su;
    p.out = glu;
    p.ld_tok = static_cast<int64_t>(n_used) * n_ff;
    p.ld_slot = n_ff;
    const int max_active = std::min(E, S);
    rc = moe_launch<true>(p, max_active, T, stream);
    if (rc != FR_OK) return rc;
    // the down matvec quantizes the GLU rows to q8_1 as it stages them, and
    // (for few tokens) its last CTA per row chunk does the combine
    MoeParams q{};
    q.w0 = static_cast<const uint8_t *>(wd);
    q.e_stride = ld_d * n_embd;
    q.w_ld = ld_d;
    q.N = n_embd;
    q.K = n_ff;
    q.xf = glu;
    q.ldxf = n_ff;
    q.bcast = 0;
    q.n_used = n_used;
    q.E = E;
    q.eoff = eoff;
    q.slots = slots;
    q.act = act;
    q.s0 = sd;
    q.out = part;
    q.ld_tok = static_cast<int64_t>(n_used) * n_embd;
    q.ld_slot = n_embd;
    q.c_wts = wts;
    q.c_resid = resid;
    q.c_out = out;
    q.c_T = T;
    bool fused = false;
    rc = moe_launch<false>(q, max_active, T, stream, &fused);
    if (rc != FR_OK) return rc;
    if (fused) return FR_OK;
    return launch_pdl(k_moe_combine, dim3((n_embd + 255) / 256, T), dim3(256), 0, stream,
                      static_cast<const float *>(part), static_cast<const float *>(wts), resid, out, n_used, n_embd);
}

} // extern "C"

// ======================================================================
// W4A4: quantize_act_f32, repack_weight, gemm_f32out (include/fr_kernels.h)
// ======================================================================
namespace frb {

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [rows, row_bytes] uint8 matrix, box `box_rows` rows x 128 bytes, 128-byte swizzle
static int make_map_sw128(CUtensorMap *map, const void *base, int64_t rows, int64_t row_bytes,
                          uint32_t box_rows = 128) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

// Scale atoms of 128-row blocks ([rows / 128][K / 64] atoms of 512 B) as a
// 2D u32 tensor, one box = four consecutive atoms (one K stage of a block)
static int make_map_sf(CUtensorMap *map, const void *base, int64_t row_blocks, int64_t kb_total) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(row_blocks * kb_total)};
    cuuint64_t strides[1] = {512};
    cuuint32_t box[2] = {128, 4};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

// f32 output [rows, cols] (row stride ld floats), 32 x 32 boxes, 128-byte swizzle
static int make_map_out(CUtensorMap *map, float *base, int64_t rows, int64_t cols, int64_t ld) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

// The SM-pair GEMM (fr_gemm2.cuh): 256 x 256 tiles, one cluster of two CTAs
// per SM pair, static round-robin over the tiles.
static int gemm_c2_run(int epi, const void *A_packed, const void *SFA, const void *B_packed, const void *SFB, float *D,
                       int M, int N, int K, float alpha, int split, cudaStream_t stream) {
    const DevInfo &di = dev_info();
    C2Args g{};
    g.split = split;
    g.M = M;
    g.N = N;
    g.K = K;
    g.nkt = K / 256;
    g.kb_total = K / 64;
    g.n_m2 = (M + 255) / 256;
    g.n_n2 = (N + 255) / 256;
    g.tiles = g.n_m2 * g.n_n2;
    g.alpha = alpha;
    CUtensorMap ma, mb, msa, msb, md;
    int rc = make_map_sw128(&ma, A_packed, M, K / 2, 128);
    if (rc == FR_OK) rc = make_map_sw128(&mb, B_packed, N, K / 2, 128);
    if (rc == FR_OK) rc = make_map_sf(&msa, SFA, (M + 127) / 128, g.kb_total);
    if (rc == FR_OK) rc = make_map_sf(&msb, SFB, (N + 127) / 128, g.kb_total);
    const int nout = epi == P_SWIGLU ? N / 2 : N;
    if (rc == FR_OK) rc = make_map_out(&md, D, M, nout, nout);
    if (rc != FR_OK) return rc;
    if (split == 2) {
        // hand-off halves and their flags (zero between launches)
        void *part = nullptr, *cnt = nullptr;
        rc = workspace_get(WS_GPART, static_cast<size_t>(g.tiles) * 16 * 32 * 128 * sizeof(float), stream, &part);
        if (rc != FR_OK) return rc;
        rc = workspace_get_zeroed(WS_GCNT, static_cast<size_t>(g.tiles) * 16 * sizeof(unsigned int), stream, &cnt);
        if (rc != FR_OK) return rc;
        g.part = static_cast<float *>(part);
        g.counter = static_cast<unsigned int *>(cnt);
    }
    // split 2: one unit per cluster, so the two halves of a tile run together
    const int ncl = std::max(1, std::min(g.tiles * split, di.sms / 2));
    auto kern = epi == P_SWIGLU ? k_gemm_c2<P_SWIGLU> : k_gemm_c2<P_PLAIN>;
    static bool done[2][64] = {};
    rc = allow_max_smem(kern, done[epi == P_SWIGLU ? 1 : 0]);
    if (rc != FR_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * ncl);
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = C2_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, msa, msb, md, g);
    if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
    return cuda_rc(e);
}

// The persistent W4A4 GEMM (fr_gemm.cuh): whole 128x256 tiles on one CTA per
// SM when the tiles fill the SMs, else every tile split into S equal K ranges
// (grid = tiles x S), partial slots [grid][128 x 256] f32 and per-tile arrival
// counters in grow-only workspaces.
static int gemm_p_run(int epi, const void *A_packed, const void *SFA, const void *B_packed, const void *SFB, float *D,
                      int M, int N, int K, float alpha, cudaStream_t stream) {
    if (!A_packed || !SFA || !B_packed || !SFB || !D || M <= 0 || N <= 0 || K <= 0) return FR_EINVAL;
    if (K % 64 != 0 || N % 16 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(D) & 15) || (reinterpret_cast<uintptr_t>(A_packed) & 15) ||
        (reinterpret_cast<uintptr_t>(B_packed) & 15) || (reinterpret_cast<uintptr_t>(SFA) & 15) ||
        (reinterpret_cast<uintptr_t>(SFB) & 15))
        return FR_EINVAL;
    const DevInfo &di = dev_info();
    if (di.cc_major != 10) return FR_ENODEVICE;
    // SM pairs (FR_GEMM_PAIR=0 keeps the one-SM kernel; whole K stages,
    // output rows 16-byte aligned): whole tiles when the 256 x 256 tiles
    // nearly fill the pairs, two K halves per tile when half as many tiles
    // do (both halves of every tile then run at once)
    {
        static const char *pv = getenv("FR_GEMM_PAIR");
        const bool pair_ok = !(pv && *pv == '0');
        const int64_t tiles2 = static_cast<int64_t>((M + 255) / 256) * ((N + 255) / 256);
        const int nout = epi == P_SWIGLU ? N / 2 : N;
        const int pairs = di.sms / 2;
        if (pair_ok && M >= 256 && K % 256 == 0 && nout % 4 == 0 && tiles2 < (1 << 24)) {
            if (tiles2 >= pairs * 7 / 8)
                return gemm_c2_run(epi, A_packed, SFA, B_packed, SFB, D, M, N, K, alpha, 1, stream);
            if (2 * tiles2 <= pairs && 2 * tiles2 >= pairs * 5 / 8 && K >= 512)
                return gemm_c2_run(epi, A_packed, SFA, B_packed, SFB, D, M, N, K, alpha, 2, stream);
        }
    }
    PGemmArgs g{};
    g.sfa = static_cast<const uint8_t *>(SFA);
    g.sfb = static_cast<const uint8_t *>(SFB);
    g.D = D;
    g.ldd = epi == P_SWIGLU ? N / 2 : N;
    g.M = M;
    g.N = N;
    g.K = K;
    g.nkt = (K + P_BK - 1) / P_BK;
    g.n_m = (M + P_BM - 1) / P_BM;
    g.n_n = (N + P_BN - 1) / P_BN;
    const int64_t tiles = static_cast<int64_t>(g.n_m) * g.n_n;
    if (tiles > (1 << 24)) return FR_EINVAL;
    g.tiles = static_cast<int>(tiles);
    g.alpha = alpha;
    // whole tiles when they fill the SMs, else an even K split of every tile
    int grid;
    if (tiles >= di.sms) {
        g.split = 0;
        grid = di.sms;
    } else {
        g.split = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(di.sms / tiles, g.nkt)));
        grid = static_cast<int>(tiles * g.split);
    }
    void *part = nullptr, *cnt = nullptr;
    int rc = FR_OK;
    if (g.split > 1) {
        rc = workspace_get(WS_GPART, static_cast<size_t>(grid) * P_SLOT_FLOATS * sizeof(float), stream, &part);
        if (rc != FR_OK) return rc;
    }
    rc = workspace_get_zeroed(WS_GCNT, static_cast<size_t>(2 * tiles) * sizeof(unsigned int), stream, &cnt);
    if (rc != FR_OK) return rc;
    g.part = static_cast<float *>(part);
    g.counter = static_cast<unsigned int *>(cnt);
    CUtensorMap ma, mb;
    rc = make_map_sw128(&ma, A_packed, M, K / 2, P_BM);
    if (rc != FR_OK) return rc;
    rc = make_map_sw128(&mb, B_packed, N, K / 2, P_BN);
    if (rc != FR_OK) return rc;
    if (epi == P_SWIGLU) {
        static bool done[64] = {};
        rc = allow_max_smem(k_gemm_p<P_SWIGLU>, done);
        if (rc != FR_OK) return rc;
        return launch_pdl(k_gemm_p<P_SWIGLU>, dim3(grid), dim3(P_THREADS), P_SMEM, stream, ma, mb, g);
    }
    static bool done[64] = {};
    rc = allow_max_smem(k_gemm_p<P_PLAIN>, done);
    if (rc != FR_OK) return rc;
    return launch_pdl(k_gemm_p<P_PLAIN>, dim3(grid), dim3(P_THREADS), P_SMEM, stream, ma, mb, g);
}

} // namespace frb

extern "C" {

int64_t fr_sf_bytes(int64_t rows, int64_t K) { return (rows + 127) / 128 * 128 * (((K / 16) + 3) / 4 * 4); }
int64_t fr_packed_bytes(int64_t rows, int64_t K) { return rows * (K / 2); }

int fr_quantize_act_f32(const float *src, void *dst_packed, void *dst_sfa, int M, int K, cudaStream_t stream) {
    if (fault_hit("fr_quantize_act_f32")) return FR_EINJECTED;
    if (!src || !dst_packed || !dst_sfa || M <= 0 || K <= 0 || K % 16 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst_packed) & 7)) return FR_EINVAL;
    const int nb = K / 16;
    return launch_pdl(k_quantize_act, dim3((nb + 127) / 128, M), dim3(128), 0, stream,
                      reinterpret_cast<const float4 *>(src), static_cast<uint2 *>(dst_packed),
                      static_cast<uint8_t *>(dst_sfa), M, K);
}

int fr_repack_weight(const void *ggml_blocks, void *dst_packed, void *dst_sf, int N, int K, cudaStream_t stream) {
    if (fault_hit("fr_repack_weight")) return FR_EINJECTED;
    if (!ggml_blocks || !dst_packed || !dst_sf || N <= 0 || K <= 0 || K % 64 != 0) return FR_EINVAL;
    if (reinterpret_cast<uintptr_t>(dst_packed) & 7) return FR_EINVAL;
    // the layout's largest offset must fit the caller's sf_bytes(N, K) buffer
    if (sf_offset(N - 1, K - 16, K) + 1 > fr_sf_bytes(N, K)) return FR_ELAYOUT;
    const int K16 = K / 16;
    return launch_pdl(k_repack, dim3((K16 + 127) / 128, N), dim3(128), 0, stream,
                      static_cast<const uint8_t *>(ggml_blocks), static_cast<uint2 *>(dst_packed),
                      static_cast<uint8_t *>(dst_sf), N, K, 1, 0);
}

int fr_gemm_f32out(const void *A_packed, const void *SFA, const void *B_packed, const void *SFB, float *D, int M,
                   int N, int K, float alpha, bool widen, cudaStream_t stream) {
    (void) widen;   // the reference ignores it too (src/fr_gemm_f32out.cu:196-197)
    if (fault_hit("fr_gemm_f32out")) return FR_EINJECTED;
    return gemm_p_run(P_PLAIN, A_packed, SFA, B_packed, SFB, D, M, N, K, alpha, stream);
}

int fr_gemm_swiglu_f32out(const void *A_packed, const void *SFA, const void *B_pair, const void *SFB_pair, float *D,
                          int M, int n_ff, int K, float alpha, cudaStream_t stream) {
    if (fault_hit("fr_gemm_swiglu_f32out")) return FR_EINJECTED;
    if (n_ff <= 0 || n_ff % 8 != 0) return FR_EINVAL;
    return gemm_p_run(P_SWIGLU, A_packed, SFA, B_pair, SFB_pair, D, M, 2 * n_ff, K, alpha, stream);
}

int fr_repack_weight_pair_interleaved(const void *gate_blocks, const void *up_blocks, void *dst_packed, void *dst_sf,
                                      int n_ff, int K, cudaStream_t stream) {
    if (fault_hit("fr_repack_weight_pair_interleaved")) return FR_EINJECTED;
    if (!gate_blocks || !up_blocks || !dst_packed || !dst_sf || n_ff <= 0 || K <= 0 || K % 64 != 0) return FR_EINVAL;
    if (reinterpret_cast<uintptr_t>(dst_packed) & 7) return FR_EINVAL;
    const int N2 = 2 * n_ff;
    if (sf_offset(N2 - 1, K - 16, K) + 1 > fr_sf_bytes(N2, K)) return FR_ELAYOUT;
    const int K16 = K / 16;
    int rc = launch_pdl(k_repack, dim3((K16 + 127) / 128, n_ff), dim3(128), 0, stream,
                        static_cast<const uint8_t *>(gate_blocks), static_cast<uint2 *>(dst_packed),
                        static_cast<uint8_t *>(dst_sf), n_ff, K, 2, 0);
    if (rc != FR_OK) return rc;
    return launch_pdl(k_repack, dim3((K16 + 127) / 128, n_ff), dim3(128), 0, stream,
                      static_cast<const uint8_t *>(up_blocks), static_cast<uint2 *>(dst_packed),
                      static_cast<uint8_t *>(dst_sf), n_ff, K, 2, 1);
}

} // extern "C"

// ======================================================================
// Tensor-core matvec (k_tcgemv) host side, and the dispatch between it and
// the dp4a kernel
// ======================================================================
namespace frb {

// TMA map of block_nvfp4 rows: [N rows, K/64*36 bytes], box 144 B x R rows
static int make_map_wrows(CUtensorMap *map, const void *base, int N, int K, int64_t w_ld, int R) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 64 * NV_BYTES), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(w_ld)};
    cuuint32_t box[2] = {TG_WBOX, static_cast<cuuint32_t>(R)};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

// TMA map of the hi/lo activation: f16 [NP rows, Kp], box 64 x NP, 128 B swizzle
static int make_map_act(CUtensorMap *map, const void *base, int NP, int Kp) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(Kp), static_cast<cuuint64_t>(NP)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(Kp) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(NP)};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

static bool tc_shape_ok(const void *w0, const void *w1, int64_t w_ld, int K) {
    if (K % 256 != 0 || w_ld % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(w0) & 15) return false;
    if (w1 && (reinterpret_cast<uintptr_t>(w1) & 15)) return false;
    const DevInfo &di = dev_info();
    return di.cc_major == 10;
}

template <int NP, int EPI>
static int tc_launch(const CUtensorMap &m0, const CUtensorMap &m1, const CUtensorMap &mb, TgArgs a, int grid,
                     cudaStream_t stream) {
    constexpr int NM = EPI == TG_SWIGLU ? 2 : 1;
    constexpr int STAGE = NM * TG_WBYTES + 4 * NP * 128;
    auto kern = k_tcgemv<NP, EPI>;
    static bool attr_done[64] = {};
    int rc = allow_max_smem(kern, attr_done);
    if (rc != FR_OK) return rc;
    const int cap = dev_info().smem_optin - 2048;
    a.n_stages = std::max(1, std::min(4, cap / STAGE));
    const size_t smem = 1024 + static_cast<size_t>(a.n_stages) * STAGE + 256;
    return launch_pdl(kern, dim3(grid), dim3(TG_THREADS), smem, stream, m0, m1, mb, a);
}

// y[t] = W . x_q[t] (PLAIN) or SwiGLU(Wg . x_q[t], Wu . x_q[t]) for T tokens,
// activations given as f32 rows (x) or q8_1 blocks (q8).
static int tc_matvec(const uint8_t *w0, const uint8_t *w1, int64_t w_ld, int N, int K, const float *x, int64_t ldx,
                     const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                     int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream) {
    const DevInfo &di = dev_info();
    const int G = std::max(1, di.sms);
    const int NP = T <= 8 ? 16 : T <= 16 ? 32 : T <= 32 ? 64 : 128;
    const int TW = NP / 2;
    const int Kp = (K + 255) / 256 * 256;
    const int n_kt = Kp / 256;
    // K split so that tiles of (up to) 128 rows fill the SMs: every CTA
    // re-reads the activation of its K range (2 x T f16 columns, 4 x the
    // bytes of the NVFP4 weights it decodes at T = 64), so fewer, fuller row
    // tiles keep that L2 traffic down; the split partials are added by the
    // last CTA of each (row tile, quadrant, column range)
    int ksplit = std::max(1, std::min(n_kt, G / ((N + 127) / 128)));
    // tuning cap (FR_TC_KSPLIT_MAX)
    static const char *kv = getenv("FR_TC_KSPLIT_MAX");
    if (kv && *kv) ksplit = std::max(1, std::min(ksplit, atoi(kv)));
    const int kt_per = (n_kt + ksplit - 1) / ksplit;
    ksplit = (n_kt + kt_per - 1) / kt_per;
    // rows per tile: the row tiles of one K split take G / ksplit CTAs
    const int R = std::min(128, std::max(1, (N + G / ksplit - 1) / (G / ksplit)));
    const int n_rt = (N + R - 1) / R;

    void *actp = nullptr;
    int rc = workspace_get(WS_ACT, static_cast<size_t>(NP) * Kp * 2, stream, &actp);
    if (rc != FR_OK) return rc;
    // counters live at a fixed place (the first TG_MAX_COUNTERS words, zero
    // after allocation and reset by every last split), partials after them
    constexpr size_t TG_MAX_COUNTERS = 1 << 16;
    if (ksplit > 1 && static_cast<size_t>(n_rt) * 16 > TG_MAX_COUNTERS) return FR_EINVAL;
    const size_t part_floats = static_cast<size_t>(n_rt) * ksplit * 2 * TW * 128;
    const size_t part_off = TG_MAX_COUNTERS * 4;
    void *wsp = nullptr;
    rc = workspace_get_zeroed(WS_TGPART, part_off + part_floats * 4, stream, &wsp);
    if (rc != FR_OK) return rc;
    void *partp = static_cast<uint8_t *>(wsp) + part_off;

    CUtensorMap m0, m1, mb;
    rc = make_map_wrows(&m0, w0, N, K, w_ld, R);
    if (rc != FR_OK) return rc;
    rc = make_map_wrows(&m1, dual ? w1 : w0, N, K, w_ld, R);
    if (rc != FR_OK) return rc;
    rc = make_map_act(&mb, actp, NP, Kp);
    if (rc != FR_OK) return rc;

    TgArgs a{};
    a.N = N;
    a.K = K;
    a.R = R;
    a.n_kt = n_kt;
    a.ksplit = ksplit;
    a.kt_per_split = kt_per;
    a.s0 = s0;
    a.s1 = s1;
    a.resid = resid;
    a.ldr = ldr;
    a.y = y;
    a.ldy = ldy;
    a.part = static_cast<float *>(partp);
    a.counter = static_cast<unsigned int *>(wsp);
    for (int t0 = 0; t0 < T; t0 += TW) {
        const int tw = std::min(TW, T - t0);
        const int64_t chunks = static_cast<int64_t>(TW) * (Kp / 32);
        rc = launch_pdl(k_act_hilo, dim3(static_cast<unsigned>((chunks + 7) / 8)), dim3(256), 0, stream,
                        x ? x + t0 * ldx : static_cast<const float *>(nullptr), ldx,
                        q8 ? q8 + t0 * ldq * Q8_BYTES : static_cast<const uint8_t *>(nullptr), ldq, tw, K, Kp, NP,
                        static_cast<__half *>(actp));
        if (rc != FR_OK) return rc;
        a.T = tw;
        a.t0 = t0;
        const int grid = n_rt * ksplit;
        switch (NP) {
        case 16: rc = dual ? tc_launch<16, TG_SWIGLU>(m0, m1, mb, a, grid, stream) : tc_launch<16, TG_PLAIN>(m0, m1, mb, a, grid, stream); break;
        case 32: rc = dual ? tc_launch<32, TG_SWIGLU>(m0, m1, mb, a, grid, stream) : tc_launch<32, TG_PLAIN>(m0, m1, mb, a, grid, stream); break;
        case 64: rc = dual ? tc_launch<64, TG_SWIGLU>(m0, m1, mb, a, grid, stream) : tc_launch<64, TG_PLAIN>(m0, m1, mb, a, grid, stream); break;
        default: rc = dual ? tc_launch<128, TG_SWIGLU>(m0, m1, mb, a, grid, stream) : tc_launch<128, TG_PLAIN>(m0, m1, mb, a, grid, stream); break;
        }
        if (rc != FR_OK) return rc;
    }
    return FR_OK;
}

template <int NCOL, int EPI>
static int fp4_launch(const CUtensorMap &m0, const CUtensorMap &m1, FmArgs a, int grid, cudaStream_t stream) {
    using S = FmShape<NCOL, EPI>;
    auto kern = k_fp4mv<NCOL, EPI>;
    static bool attr_done[64] = {};
    int rc = allow_max_smem(kern, attr_done);
    if (rc != FR_OK) return rc;
    // ring depths: two or three MMA-ready stages, up to four activation
    // stages, the rest of shared memory for raw weight stages (the HBM
    // prefetch depth)
    const int bar_bytes = 512;
    const int cap = dev_info().smem_optin - 1024 - bar_bytes;
    int nc = 3, nb = 4;
    if (nb * S::BST > 40 * 1024) nb = 2;
    int nr = (cap - nc * S::CAN - nb * S::BST) / S::RAW;
    if (nr < 4) {
        nc = 2;
        nr = (cap - nc * S::CAN - nb * S::BST) / S::RAW;
    }
    // tuning overrides (FR_FP4_RINGS="raw,mma,act"), clamped to shared memory
    static const char *ov = getenv("FR_FP4_RINGS");
    if (ov && *ov) {
        int r = 0, c = 0, b = 0;
        if (sscanf(ov, "%d,%d,%d", &r, &c, &b) == 3 && r >= 2 && c >= 1 && b >= 1 &&
            r * S::RAW + c * S::CAN + b * S::BST <= cap) {
            nr = r;
            nc = c;
            nb = b;
        }
    }
    if (nr < 2) return FR_EINVAL;
    a.n_can = nc;
    a.n_b = nb;
    a.n_raw = std::min(nr, 8);
    const size_t smem = 1024 + static_cast<size_t>(a.n_can) * S::CAN + static_cast<size_t>(a.n_b) * S::BST +
                        static_cast<size_t>(a.n_raw) * S::RAW + bar_bytes;
    return launch_pdl(kern, dim3(grid), dim3(S::THREADS), smem, stream, m0, m1, a);
}

template <int NCOL, int EPI, int NT>
static int fp4t_launch(FtArgs a, int grid, cudaStream_t stream) {
    using S = FtShape<NCOL, EPI, NT>;
    auto kern = k_fp4t<NCOL, EPI, NT>;
    static bool attr_done[64] = {};
    int rc = allow_max_smem(kern, attr_done);
    if (rc != FR_OK) return rc;
    // about 110 KB of weights in flight per SM (measured best for one pass
    // over a matrix: more only lengthens the memory queues); each ring stage
    // also holds its activation columns; TMEM's 256 scale columns bound the
    // ring, whose depth is a multiple of the issue groups
    const int extra = 2048;                                  // scale atom, factors, barriers
    const int cap = dev_info().smem_optin - 1024 - extra;
    const int per = S::WST + S::BST;
    const int nw_tmem = (256 - 4 * S::NISS) / (16 * S::NI);
    // the down projection (one matrix) follows the activation kernel of the
    // GLU: a deeper ring prefetches more of its weights meanwhile
    int nw = std::max(2, std::min(((EPI == FM_PLAIN ? 184 : 110) * 1024 + S::WST - 1) / S::WST, 8));
    nw = std::min(nw, nw_tmem);
    // tuning override (FR_FP4T_RINGS="stages"), within the limits
    static const char *ov = getenv("FR_FP4T_RINGS");
    if (ov && *ov) {
        const int w = atoi(ov);
        if (w >= 2 && w <= nw_tmem && w * per <= cap) nw = w;
    }
    while (nw > 2 && nw * per > cap) --nw;
    nw -= nw % S::P;
    if (nw < 2 || nw * per > cap) return FR_EINVAL;
    a.n_w = nw;
    a.n_b = nw;
    const size_t smem = 1024 + static_cast<size_t>(nw) * per + extra;
    return launch_pdl(kern, dim3(grid), dim3(S::THREADS), smem, stream, a);
}

template <int NCOL>
static int fp4t_launch2(const FtArgs &a, int grid, bool dual, int nt, cudaStream_t stream) {
    if (dual) return fp4t_launch<NCOL, FM_SWIGLU, 1>(a, grid, stream);
    return nt == 2 ? fp4t_launch<NCOL, FM_PLAIN, 2>(a, grid, stream) : fp4t_launch<NCOL, FM_PLAIN, 1>(a, grid, stream);
}

// FP4 tensor-core matvec on tile-major weights (k_tile_nvfp4's layout):
// k_act_fp4 builds the activation columns of a window of FP4_MAX_T tokens,
// k_fp4t streams the weights once per window.
// amax_out (nullable): per token, the largest |y| of every 32-row group
// ([T][ceil(N / 128) * 4]); amax_in (nullable, with f32 x): the same maxima
// of x's row, so the activation kernel needs no scan of it ([T][K / 32]).
static int fp4t_matvec(const uint8_t *w0, const uint8_t *w1, int N, int K, const float *x, int64_t ldx,
                       const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                       int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream, float *amax_out,
                       const float *amax_in, const TpOut *tp) {
    if (!w0 || (dual && !w1) || N <= 0 || K <= 0 || K % 256 != 0 || T <= 0 || !y) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w0) & 15) || (w1 && (reinterpret_cast<uintptr_t>(w1) & 15))) return FR_EINVAL;
    const DevInfo &di = dev_info();
    if (di.cc_major != 10) return FR_ENODEVICE;
    const int n_kq = K / 256, n_rb = (N + 127) / 128;
    const int nt = (!dual && n_kq % 2 == 0) ? 2 : 1;         // K stages per pipeline step
    const int nsr = n_kq / nt;
    const int U = n_rb * nsr;
    const int G = std::max(1, std::min(di.sms, U));
    const int per_min = std::max(1, U / G);
    const int maxp = std::min(G, (nsr + per_min - 1) / per_min + 1);
    const int TW = std::min(T, FP4_MAX_T);
    const int NCOL = FM_DIGITS * TW <= 16 ? 16 : FM_DIGITS * TW <= 32 ? 32 : FM_DIGITS * TW <= 64 ? 64 : 128;
    const int TMAX = NCOL / FM_DIGITS;

    constexpr size_t MAX_COUNTERS = 1 << 16;
    if (static_cast<size_t>(n_rb) * 4 > MAX_COUNTERS) return FR_EINVAL;
    const size_t part_floats = static_cast<size_t>(n_rb) * maxp * 2 * TMAX * 128;
    const size_t part_off = MAX_COUNTERS * 4;
    void *wsp = nullptr;
    int rc = workspace_get_zeroed(WS_TGPART, part_off + part_floats * 4, stream, &wsp);
    if (rc != FR_OK) return rc;
    const size_t b_bytes = static_cast<size_t>(n_kq) * NCOL * 128;
    const size_t sf_bytes = static_cast<size_t>(n_kq) * 4 * 512;
    void *actp = nullptr;
    rc = workspace_get(WS_FP4, b_bytes + sf_bytes + static_cast<size_t>(TMAX) * FM_GSTRIDE * 4, stream, &actp);
    if (rc != FR_OK) return rc;
    uint8_t *bimg = static_cast<uint8_t *>(actp);
    uint8_t *sfb = bimg + b_bytes;
    float *gtab = reinterpret_cast<float *>(sfb + sf_bytes);

    FtArgs a{};
    a.N = N;
    a.K = K;
    a.n_kq = n_kq;
    a.n_units = U;
    a.maxp = maxp;
    a.w0 = w0;
    a.w1 = dual ? w1 : w0;
    a.bimg = bimg;
    a.gtab = gtab;
    a.s0 = s0;
    a.s1 = s1;
    a.resid = resid;
    a.ldr = ldr;
    a.y = y;
    a.ldy = ldy;
    a.part = reinterpret_cast<float *>(static_cast<uint8_t *>(wsp) + part_off);
    a.counter = static_cast<unsigned int *>(wsp);
    a.amax_out = amax_out;
    a.amax_ld = n_rb * 4;
    if (tp != nullptr) {
        if (dual) return FR_EINVAL;
        a.peer_base = tp->peer_base;
        a.npeers = tp->npeers;
        a.rank = tp->rank;
        a.peer_off = tp->peer_off;
        a.flag_off = tp->flag_off;
        a.epoch = tp->epoch;
        a.par_bytes = tp->par_bytes;
        if (tp->ctas_out) *tp->ctas_out = static_cast<unsigned>(G) * static_cast<unsigned>((T + TW - 1) / TW);
    }
    const int nq = K / Q8_ELEMS;
    for (int t0 = 0; t0 < T; t0 += TW) {
        const int tw = std::min(TW, T - t0);
        a.T = tw;
        a.t0 = t0;
        const int slices = std::max(1, std::min((nq + 7) / 8, std::max(1, 256 / tw)));
        rc = launch_pdl(k_act_fp4, dim3(slices, tw), dim3(256), 0, stream,
                        x ? x + t0 * ldx : static_cast<const float *>(nullptr), ldx,
                        q8 ? q8 + t0 * ldq * Q8_BYTES : static_cast<const uint8_t *>(nullptr), ldq, K, NCOL, bimg, sfb,
                        gtab, static_cast<int64_t>(0),
                        (x && amax_in) ? amax_in + static_cast<int64_t>(t0) * nq : static_cast<const float *>(nullptr),
                        nq);
        if (rc != FR_OK) return rc;
        switch (NCOL) {
        case 16: rc = fp4t_launch2<16>(a, G, dual, nt, stream); break;
        case 32: rc = fp4t_launch2<32>(a, G, dual, nt, stream); break;
        case 64: rc = fp4t_launch2<64>(a, G, dual, nt, stream); break;
        default: rc = fp4t_launch2<128>(a, G, dual, nt, stream); break;
        }
        if (rc != FR_OK) return rc;
    }
    return FR_OK;
}

// FP4 tensor-core matvec: k_act_fp4 writes the activation columns of up to
// FP4_MAX_T tokens, k_fp4mv streams the weights once per such window.
static int fp4_matvec(const uint8_t *w0, const uint8_t *w1, int64_t w_ld, int N, int K, const float *x, int64_t ldx,
                      const uint8_t *q8, int64_t ldq, int T, const float *s0, const float *s1, const float *resid,
                      int64_t ldr, float *y, int64_t ldy, bool dual, cudaStream_t stream) {
    const DevInfo &di = dev_info();
    const int G = std::max(1, di.sms);
    const int TW = std::min(T, FP4_MAX_T);
    const int NCOL = FM_DIGITS * TW <= 16 ? 16 : FM_DIGITS * TW <= 32 ? 32 : FM_DIGITS * TW <= 64 ? 64 : 128;
    const int TMAX = NCOL / FM_DIGITS;
    const int n_kt = K / FM_KS;
    int ksplit = std::max(1, std::min(n_kt, (128 * G) / std::max(1, N)));
    const int kt_per = (n_kt + ksplit - 1) / ksplit;
    ksplit = (n_kt + kt_per - 1) / kt_per;
    const int R = std::min(128, std::max(1, static_cast<int>((static_cast<int64_t>(N) * ksplit + G - 1) / G)));
    const int n_rt = (N + R - 1) / R;

    // activation columns, their scale atoms, the column factors
    const size_t b_bytes = static_cast<size_t>(n_kt) * NCOL * 128;
    const size_t sf_bytes = static_cast<size_t>(n_kt) * 4 * 512;
    const size_t g_bytes = static_cast<size_t>(TMAX) * FM_GSTRIDE * 4;
    void *actp = nullptr;
    int rc = workspace_get(WS_FP4, b_bytes + sf_bytes + g_bytes, stream, &actp);
    if (rc != FR_OK) return rc;
    uint8_t *bimg = static_cast<uint8_t *>(actp);
    uint8_t *sfb = bimg + b_bytes;
    float *gtab = reinterpret_cast<float *>(sfb + sf_bytes);

    constexpr size_t MAX_COUNTERS = 1 << 16;
    if (static_cast<size_t>(n_rt) * 4 > MAX_COUNTERS) return FR_EINVAL;
    const size_t part_floats = static_cast<size_t>(n_rt) * ksplit * 2 * TMAX * 128;
    const size_t part_off = MAX_COUNTERS * 4;
    void *wsp = nullptr;
    rc = workspace_get_zeroed(WS_TGPART, part_off + part_floats * 4, stream, &wsp);
    if (rc != FR_OK) return rc;

    CUtensorMap m0, m1;
    rc = make_map_wrows(&m0, w0, N, K, w_ld, R);
    if (rc != FR_OK) return rc;
    rc = make_map_wrows(&m1, dual ? w1 : w0, N, K, w_ld, R);
    if (rc != FR_OK) return rc;

    FmArgs a{};
    a.N = N;
    a.K = K;
    a.R = R;
    a.n_kt = n_kt;
    a.ksplit = ksplit;
    a.kt_per_split = kt_per;
    a.bimg = bimg;
    a.sfb = sfb;
    a.gtab = gtab;
    a.s0 = s0;
    a.s1 = s1;
    a.resid = resid;
    a.ldr = ldr;
    a.y = y;
    a.ldy = ldy;
    a.part = static_cast<float *>(static_cast<void *>(static_cast<uint8_t *>(wsp) + part_off));
    a.counter = static_cast<unsigned int *>(wsp);
    const int nq = K / Q8_ELEMS;
    for (int t0 = 0; t0 < T; t0 += TW) {
        const int tw = std::min(TW, T - t0);
        const int slices = std::max(1, std::min((nq + 7) / 8, std::max(1, 256 / tw)));
        rc = launch_pdl(k_act_fp4, dim3(slices, tw), dim3(256), 0, stream,
                        x ? x + t0 * ldx : static_cast<const float *>(nullptr), ldx,
                        q8 ? q8 + t0 * ldq * Q8_BYTES : static_cast<const uint8_t *>(nullptr), ldq, K, NCOL, bimg,
                        sfb, gtab, static_cast<int64_t>(0), static_cast<const float *>(nullptr), 0);
        if (rc != FR_OK) return rc;
        a.T = tw;
        a.t0 = t0;
        const int grid = n_rt * ksplit;
        switch (NCOL) {
        case 16: rc = dual ? fp4_launch<16, FM_SWIGLU>(m0, m1, a, grid, stream) : fp4_launch<16, FM_PLAIN>(m0, m1, a, grid, stream); break;
        case 32: rc = dual ? fp4_launch<32, FM_SWIGLU>(m0, m1, a, grid, stream) : fp4_launch<32, FM_PLAIN>(m0, m1, a, grid, stream); break;
        case 64: rc = dual ? fp4_launch<64, FM_SWIGLU>(m0, m1, a, grid, stream) : fp4_launch<64, FM_PLAIN>(m0, m1, a, grid, stream); break;
        default: rc = dual ? fp4_launch<128, FM_SWIGLU>(m0, m1, a, grid, stream) : fp4_launch<128, FM_PLAIN>(m0, m1, a, grid, stream); break;
        }
        if (rc != FR_OK) return rc;
    }
    return FR_OK;
}

} // namespace frb

// ======================================================================
// Expert-parallel building blocks: expert FFN over pre-routed rows, combine
// ======================================================================
extern "C" {

} // extern "C"

namespace frb {
// Expert FFN over pre-routed rows; skip_neg: rows with expert id -1 are empty
// slots of a fixed-capacity exchange and are left out (their output rows are
// not written).
static int moe_experts_impl(const float *x, int64_t ldx, const int32_t *eid, int S, const void *wg, const void *wu,
                            const void *wd, const float *sg, const float *su, const float *sd, float *out, int64_t ldo,
                            int n_embd, int n_ff, int E, int skip_neg, cudaStream_t stream) {
    if (S < 0 || E <= 0 || E > MOE_MAX_E || n_embd <= 0 || n_ff <= 0) return FR_EINVAL;
    if (S == 0) return FR_OK;
    if (!x || !eid || !wg || !wu || !wd || !out || n_embd % 64 != 0 || n_ff % 64 != 0) return FR_EINVAL;
    if (ldx < n_embd || ldo < n_embd || S > MOE_MAX_SLOTS) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(wg) & 3) || (reinterpret_cast<uintptr_t>(wu) & 3) ||
        (reinterpret_cast<uintptr_t>(wd) & 3))
        return FR_EINVAL;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(n_ff) / 64 * NV_BYTES;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_glu = take(static_cast<size_t>(S) * n_ff * 4);
    void *wsp = nullptr;
    int rc = workspace_get(WS_MOE, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *base = static_cast<uint8_t *>(wsp);
    int32_t *eoff = reinterpret_cast<int32_t *>(base + o_eoff);
    int32_t *act = reinterpret_cast<int32_t *>(base + o_act);
    int32_t *slots = reinterpret_cast<int32_t *>(base + o_slots);
    float *glu = reinterpret_cast<float *>(base + o_glu);
    static bool attr_done[64] = {};
    rc = allow_max_smem(k_group_ids, attr_done);
    if (rc != FR_OK) return rc;
    // each row is one "token" with one slot
    rc = launch_pdl(k_group_ids, dim3(1), dim3(1024), group_smem(S, 1), stream, eid, static_cast<int64_t>(1), S, 1, E,
                    eoff, slots, act, skip_neg);
    if (rc != FR_OK) return rc;
    // both matvecs quantize their f32 input rows to q8_1 as they stage them
    MoeParams p{};
    p.w0 = static_cast<const uint8_t *>(wg);
    p.w1 = static_cast<const uint8_t *>(wu);
    p.e_stride = ld_gu * n_ff;
    p.w_ld = ld_gu;
    p.N = n_ff;
    p.K = n_embd;
    p.xf = x;
    p.ldxf = ldx;
    p.bcast = 1;
    p.n_used = 1;
    p.E = E;
    p.eoff = eoff;
    p.slots = slots;
    p.act = act;
    p.s0 = sg;
    p.s1 = su;
    p.out = glu;
    p.ld_tok = n_ff;
    p.ld_slot = 0;
    const int max_active = std::min(E, S);
    rc = moe_launch<true>(p, max_active, S, stream);
    if (rc != FR_OK) return rc;
    MoeParams q{};
    q.w0 = static_cast<const uint8_t *>(wd);
    q.e_stride = ld_d * n_embd;
    q.w_ld = ld_d;
    q.N = n_embd;
    q.K = n_ff;
    q.xf = glu;
    q.ldxf = n_ff;
    q.bcast = 1;
    q.n_used = 1;
    q.E = E;
    q.eoff = eoff;
    q.slots = slots;
    q.act = act;
    q.s0 = sd;
    q.out = out;
    q.ld_tok = ldo;
    q.ld_slot = 0;
    return moe_launch<false>(q, max_active, S, stream);
}
} // namespace frb

extern "C" {

int fr_moe_experts_nvfp4(const float *x, int64_t ldx, const int32_t *eid, int S, const void *wg, const void *wu,
                         const void *wd, const float *sg, const float *su, const float *sd, float *out, int64_t ldo,
                         int n_embd, int n_ff, int E, cudaStream_t stream) {
    if (fault_hit("fr_moe_experts_nvfp4")) return FR_EINJECTED;
    return moe_experts_impl(x, ldx, eid, S, wg, wu, wd, sg, su, sd, out, ldo, n_embd, n_ff, E, 0, stream);
}

int fr_moe_combine(const float *part, const float *wts, const float *resid, float *out, int T, int n_used, int n_embd,
                   cudaStream_t stream) {
    if (fault_hit("fr_moe_combine")) return FR_EINJECTED;
    if (T < 0 || n_used <= 0 || n_used > MOE_MAX_USED || n_embd <= 0) return FR_EINVAL;
    if (T == 0) return FR_OK;
    if (!part || !wts || !out) return FR_EINVAL;
    return launch_pdl(k_moe_combine, dim3((n_embd + 255) / 256, T), dim3(256), 0, stream, part, wts, resid, out, n_used,
                      n_embd);
}

} // extern "C"

// ======================================================================
// Tensor-parallel FFN over NVLink peer stores
// ======================================================================
namespace frb {

// shared buffer layout: [flags 32] u32, the reduce kernel's per-CTA consumed
// counts [TP_WAIT_CTAS][32] u32 and step counts [TP_WAIT_CTAS] u32, then
// (256-byte aligned) two parity halves of the ranks' partial outputs, each
// [P][T][n_embd] f32 with slot r written by rank r, then this rank's local
// staging rows [T][n_embd] f32 (the push path's matvec output).  The halves'
// size follows from the buffer's size -- T_cap tokens, the T the buffer was
// sized for -- so every call on one buffer agrees on where they lie whatever
// its own T.
constexpr int TP_WAIT_CTAS = 32;
struct TpLayout {
    int64_t flags, seen, epoch, part, half, stage, total;
    int64_t t_cap;
};
static int64_t tp_part_off() { return (4LL * 32 + 4LL * 32 * TP_WAIT_CTAS + 4LL * TP_WAIT_CTAS + 255) / 256 * 256; }
static TpLayout tp_layout_cap(int64_t t_cap, int n_embd, int P) {
    TpLayout l{};
    l.flags = 0;
    l.seen = 4LL * 32;
    l.epoch = l.seen + 4LL * 32 * TP_WAIT_CTAS;
    l.part = tp_part_off();
    l.t_cap = t_cap;
    l.half = static_cast<int64_t>(P) * t_cap * n_embd * 4;
    l.stage = l.part + 2 * l.half;
    l.total = l.stage + t_cap * n_embd * 4;
    return l;
}
// the layout of a buffer of `bytes` bytes (t_cap = 0 when it holds no token)
static TpLayout tp_layout_buf(int64_t bytes, int n_embd, int P) {
    const int64_t per_tok = (2LL * P + 1) * n_embd * 4;
    const int64_t t_cap = bytes > tp_part_off() ? (bytes - tp_part_off()) / per_tok : 0;
    return tp_layout_cap(t_cap, n_embd, P);
}

// CTAs the matvec launches for (N, K, T) -- what each rank counts into the flags
static unsigned gemv_ctas(int N, int K, int64_t w_ld, int T, bool dual) {
    const GvPlan pl = gv_plan(N, K, w_ld, T, dual);
    const int windows = (T + pl.TT - 1) / pl.TT;
    return static_cast<unsigned>(pl.grid * windows);
}

} // namespace frb

extern "C" {

int64_t fr_nvfp4_tiled_bytes(int N, int K) {
    if (N <= 0 || K <= 0 || K % 64 != 0) return -1;
    return static_cast<int64_t>((N + 127) / 128) * ((K + 255) / 256) * FT_TILE;
}

int fr_nvfp4_tile(const void *w, int64_t w_ld, int N, int K, void *dst, cudaStream_t stream) {
    if (fault_hit("fr_nvfp4_tile")) return FR_EINJECTED;
    if (!w || !dst || N <= 0 || K <= 0 || K % 64 != 0) return FR_EINVAL;
    if (w_ld < static_cast<int64_t>(K / 64) * NV_BYTES || w_ld % 4 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) & 3) || (reinterpret_cast<uintptr_t>(dst) & 15)) return FR_EINVAL;
    const int n_kq = (K + 255) / 256;
    const int64_t total = static_cast<int64_t>((N + 127) / 128) * 128 * n_kq * 4;
    return launch_pdl(k_tile_nvfp4, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, stream,
                      static_cast<const uint8_t *>(w), w_ld, N, K, n_kq, static_cast<uint8_t *>(dst), total);
}

int fr_gemv_tiled(const void *wt, int N, int K, const float *x, int64_t ldx, const void *q8, int64_t ldq,
                  const float *scale, const float *resid, int64_t ldr, float *y, int64_t ldy, int T,
                  cudaStream_t stream) {
    if (fault_hit("fr_gemv_tiled")) return FR_EINJECTED;
    if ((x == nullptr) == (q8 == nullptr)) return FR_EINVAL;
    return fp4t_matvec(static_cast<const uint8_t *>(wt), nullptr, N, K, x, ldx, static_cast<const uint8_t *>(q8),
                       ldq, T, scale, nullptr, resid, ldr, y, ldy, false, stream);
}

int fr_gemv_tiled_swiglu(const void *wg_t, const void *wu_t, int N, int K, const float *x, int64_t ldx,
                         const void *q8, int64_t ldq, const float *sg, const float *su, float *y, int64_t ldy, int T,
                         cudaStream_t stream) {
    if (fault_hit("fr_gemv_tiled_swiglu")) return FR_EINJECTED;
    if ((x == nullptr) == (q8 == nullptr)) return FR_EINVAL;
    return fp4t_matvec(static_cast<const uint8_t *>(wg_t), static_cast<const uint8_t *>(wu_t), N, K, x, ldx,
                       static_cast<const uint8_t *>(q8), ldq, T, sg, su, nullptr, 0, y, ldy, true, stream);
}

int fr_ffn_tiled(const float *x, const void *wg_t, const void *wu_t, const void *wd_t, const float *sg,
                 const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                 float *chk_glu, cudaStream_t stream) {
    if (fault_hit("fr_ffn_tiled")) return FR_EINJECTED;
    if (!x || !wg_t || !wu_t || !wd_t || !out || T <= 0 || n_embd % 256 != 0 || n_ff % 256 != 0) return FR_EINVAL;
    float *glu = chk_glu;
    if (!glu) {
        void *p = nullptr;
        const int rc = workspace_get(WS_GLU, static_cast<size_t>(T) * n_ff * sizeof(float), stream, &p);
        if (rc != FR_OK) return rc;
        glu = static_cast<float *>(p);
    }
    // the gate/up epilogue leaves the GLU's row-group maxima for the down's
    // activation kernel
    void *am = nullptr;
    int rc = workspace_get(WS_AMAX, static_cast<size_t>(T) * (n_ff / 32) * sizeof(float), stream, &am);
    if (rc != FR_OK) return rc;
    rc = fp4t_matvec(static_cast<const uint8_t *>(wg_t), static_cast<const uint8_t *>(wu_t), n_ff, n_embd, x,
                     n_embd, nullptr, 0, T, sg, su, nullptr, 0, glu, n_ff, true, stream, static_cast<float *>(am));
    if (rc != FR_OK) return rc;
    return fp4t_matvec(static_cast<const uint8_t *>(wd_t), nullptr, n_embd, n_ff, glu, n_ff, nullptr, 0, T, sd,
                       nullptr, resid, n_embd, out, n_embd, false, stream, nullptr, static_cast<const float *>(am));
}

} // extern "C"

// ======================================================================
// MoE experts on the FP4 tensor cores (tile-major expert weights)
// ======================================================================
namespace frb {

template <int NCOL, int EPI>
static int fp4e_launch(FeArgs a, int grid, cudaStream_t stream) {
    using S = FtShape<NCOL, EPI, 1>;
    using H = FeShape<NCOL, EPI>;
    auto kern = k_fp4e<NCOL, EPI>;
    static bool attr_done[64] = {};
    int rc = allow_max_smem(kern, attr_done);
    if (rc != FR_OK) return rc;
    const int extra = fe_extra_bytes() + 64;
    const int cap = dev_info().smem_optin - 1024 - extra;
    // TMEM: accumulators in columns [0, 256), then 16 scale columns per
    // weight tile of the ring and 4 per issuer for the activation atom; each
    // ring stage holds a weight stage and its activation atoms
    const int nw_tmem = (256 - 4 * H::NISS) / (16 * H::NM);
    const int per = S::WST + S::BST;
    int nw = std::max(2, std::min(((EPI == FM_PLAIN ? 184 : 146) * 1024 + S::WST - 1) / S::WST, 8));
    nw = std::min(nw, nw_tmem);
    static const char *ov = getenv("FR_FP4E_RINGS");
    if (ov && *ov) {
        const int w = atoi(ov);
        if (w >= 2 && w <= nw_tmem && w * per <= cap) nw = w;
    }
    while (nw > 2 && nw * per > cap) --nw;
    // each issue group owns the ring slots s with s % P == its index
    nw -= nw % H::P;
    if (nw < 2 || nw * per > cap) return FR_EINVAL;
    a.n_w = nw;
    a.n_b = nw;
    const size_t smem = 1024 + static_cast<size_t>(nw) * per + extra;
    return launch_pdl(kern, dim3(grid), dim3(H::THREADS), smem, stream, a);
}

// MMA columns of the window: 8 per token.  Windows of 8 tokens let two issue
// groups (and, for one matrix, two accumulator sets) fit in TMEM; the plain
// projection takes 16-token windows when more than 64 tokens make re-reads
// of an expert's rows likely.
static int fe_ncol(int max_tok, bool dual) {
    const int tw = std::min(std::max(1, max_tok), (dual || max_tok <= 64) ? 8 : FP4_MAX_T);
    return FM_DIGITS * tw <= 16 ? 16 : FM_DIGITS * tw <= 32 ? 32 : FM_DIGITS * tw <= 64 ? 64 : 128;
}

// Per-source-row activation images of `rows` f32 rows (k_act_fp4), then the
// expert matvec of one projection.  `a` carries the routing, weights and
// output; max_tok bounds the tokens any expert receives (picks the window).
static int fp4e_run(FeArgs a, bool dual, const float *x, int64_t ldx, int rows, int max_tok, int max_active,
                    uint8_t *img, float *gtab, cudaStream_t stream) {
    const DevInfo &di = dev_info();
    if (di.cc_major != 10) return FR_ENODEVICE;
    const int n_kq = a.K / 256;
    const int nq = a.K / Q8_ELEMS;
    const int slices = std::max(1, std::min((nq + 7) / 8, std::max(1, 256 / std::max(1, rows))));
    int rc = FR_OK;
    if (x != nullptr) {                                      // else the images are already built
        rc = launch_pdl(k_act_fp4, dim3(slices, rows), dim3(256), 0, stream, x, ldx,
                        static_cast<const uint8_t *>(nullptr), static_cast<int64_t>(0), a.K, FM_DIGITS, img,
                        static_cast<uint8_t *>(nullptr), gtab, static_cast<int64_t>(n_kq) * 1024,
                        static_cast<const float *>(nullptr), 0);
        if (rc != FR_OK) return rc;
    }
    const int NCOL = fe_ncol(max_tok, dual);
    const int TMAX = NCOL / FM_DIGITS;
    const int G = std::max(1, di.sms);
    const long max_windows = std::min<long>(a.E, max_active) + (static_cast<long>(rows) * (a.bcast ? a.n_used : 1)) / TMAX + 1;
    const size_t cnt_bytes = align256(static_cast<size_t>(max_windows) * a.n_rb * 4 * sizeof(unsigned));
    const size_t part_bytes = static_cast<size_t>(G) * 2 * 2 * TMAX * 128 * sizeof(float);
    // counters (kept at zero between calls; grow-only, cleared when they
    // grow) and partials live in separate buffers, so a call that needs more
    // counters never finds another call's partials over them
    void *cnt = nullptr, *prt = nullptr;
    rc = workspace_get_zeroed(WS_FE, cnt_bytes, stream, &cnt);
    if (rc != FR_OK) return rc;
    rc = workspace_get(WS_FE, part_bytes, stream, &prt);
    if (rc != FR_OK) return rc;
    a.counter = static_cast<unsigned int *>(cnt);
    a.part = static_cast<float *>(prt);
    a.max_rbg = static_cast<int>(max_windows * a.n_rb);
    a.img = img;
    a.gtab = gtab;
    a.n_kq = n_kq;
    if (dual) {
        switch (NCOL) {
        case 16: return fp4e_launch<16, FM_SWIGLU>(a, G, stream);
        case 32: return fp4e_launch<32, FM_SWIGLU>(a, G, stream);
        case 64: return fp4e_launch<64, FM_SWIGLU>(a, G, stream);
        default: return fp4e_launch<64, FM_SWIGLU>(a, G, stream);
        }
    }
    switch (NCOL) {
    case 16: return fp4e_launch<16, FM_PLAIN>(a, G, stream);
    case 32: return fp4e_launch<32, FM_PLAIN>(a, G, stream);
    case 64: return fp4e_launch<64, FM_PLAIN>(a, G, stream);
    default: return fp4e_launch<128, FM_PLAIN>(a, G, stream);
    }
}

static bool fe_shape_ok(int N, int K) { return N > 0 && K > 0 && N % 128 == 0 && K % 256 == 0; }

// Expert FFN over pre-routed rows (row s to expert eid[s]; -1 skipped when
// skip_neg) on tile-major experts: grouping, then the gate/up pair and the
// down projection on the FP4 tensor cores.
static int moe_experts_tiled_impl(const float *x, int64_t ldx, const int32_t *eid, int S, const void *wg_t,
                                  const void *wu_t, const void *wd_t, const float *sg, const float *su,
                                  const float *sd, float *out, int64_t ldo, int n_embd, int n_ff, int E, int skip_neg,
                                  cudaStream_t stream) {
    if (S < 0 || E <= 0 || E > FE_MAX_E || !fe_shape_ok(n_ff, n_embd) || !fe_shape_ok(n_embd, n_ff)) return FR_EINVAL;
    if (S == 0) return FR_OK;
    if (!x || !eid || !wg_t || !wu_t || !wd_t || !out || ldx < n_embd || ldo < n_embd || S > MOE_MAX_SLOTS)
        return FR_EINVAL;
    if (!aligned16(wg_t) || !aligned16(wu_t) || !aligned16(wd_t)) return FR_EINVAL;
    const int kq_gu = n_embd / 256, kq_d = n_ff / 256;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_gx = take(static_cast<size_t>(S) * FM_GSTRIDE * 4);
    const size_t o_ix = take(static_cast<size_t>(S) * kq_gu * 1024);
    const size_t o_glu = take(static_cast<size_t>(S) * n_ff * 4);
    const size_t o_gg = take(static_cast<size_t>(S) * FM_GSTRIDE * 4);
    const size_t o_ig = take(static_cast<size_t>(S) * kq_d * 1024);
    void *wsp = nullptr;
    int rc = workspace_get(WS_MOE, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *base = static_cast<uint8_t *>(wsp);
    int32_t *eoff = reinterpret_cast<int32_t *>(base + o_eoff);
    int32_t *act = reinterpret_cast<int32_t *>(base + o_act);
    int32_t *slots = reinterpret_cast<int32_t *>(base + o_slots);
    float *glu = reinterpret_cast<float *>(base + o_glu);
    static bool attr_done[64] = {};
    rc = allow_max_smem(k_group_ids, attr_done);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_group_ids, dim3(1), dim3(1024), group_smem(S, 1), stream, eid, static_cast<int64_t>(1), S, 1, E,
                    eoff, slots, act, skip_neg);
    if (rc != FR_OK) return rc;
    const int max_active = std::min(E, S);
    FeArgs a{};
    a.N = n_ff;
    a.K = n_embd;
    a.n_rb = n_ff / 128;
    a.E = E;
    a.n_used = 1;
    a.bcast = 0;
    a.eoff = eoff;
    a.slots = slots;
    a.act = act;
    a.w0 = static_cast<const uint8_t *>(wg_t);
    a.w1 = static_cast<const uint8_t *>(wu_t);
    a.e_stride = static_cast<int64_t>(n_ff / 128) * kq_gu * FT_TILE;
    a.s0 = sg;
    a.s1 = su;
    a.y = glu;
    a.ld_tok = n_ff;
    a.ld_slot = 0;
    rc = fp4e_run(a, true, x, ldx, S, S, max_active, base + o_ix, reinterpret_cast<float *>(base + o_gx), stream);
    if (rc != FR_OK) return rc;
    FeArgs d{};
    d.N = n_embd;
    d.K = n_ff;
    d.n_rb = n_embd / 128;
    d.E = E;
    d.n_used = 1;
    d.bcast = 0;
    d.eoff = eoff;
    d.slots = slots;
    d.act = act;
    d.w0 = static_cast<const uint8_t *>(wd_t);
    d.w1 = d.w0;
    d.e_stride = static_cast<int64_t>(n_embd / 128) * kq_d * FT_TILE;
    d.s0 = sd;
    d.y = out;
    d.ld_tok = ldo;
    d.ld_slot = 0;
    return fp4e_run(d, false, glu, n_ff, S, S, max_active, base + o_ig, reinterpret_cast<float *>(base + o_gg),
                    stream);
}

} // namespace frb

extern "C" {

int fr_moe_ffn_tiled(const float *x, const float *w_r, const void *wg_t, const void *wu_t, const void *wd_t,
                     const float *sg, const float *su, const float *sd, const float *resid, float *out, int T,
                     int n_embd, int n_ff, int E, int n_used, float clamp_val, int32_t *chk_ids, float *chk_wts,
                     float *chk_glu, float *chk_part, cudaStream_t stream) {
    if (fault_hit("fr_moe_ffn_tiled")) return FR_EINJECTED;
    int rc = check_route_shape(T, n_embd, E, n_used);
    if (rc != FR_OK) return rc;
    if (!x || !w_r || !wg_t || !wu_t || !wd_t || !out) return FR_EINVAL;
    if (!fe_shape_ok(n_ff, n_embd) || !fe_shape_ok(n_embd, n_ff) || E > FE_MAX_E) return FR_EINVAL;
    if (!aligned16(x) || !aligned16(w_r) || !aligned16(wg_t) || !aligned16(wu_t) || !aligned16(wd_t)) return FR_EINVAL;
    const int S = T * n_used;
    const int kq_gu = n_embd / 256, kq_d = n_ff / 256;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_logits = take(static_cast<size_t>(T) * E * 4);
    const size_t o_ids = take(static_cast<size_t>(S) * 4);
    const size_t o_wts = take(static_cast<size_t>(S) * 4);
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_gx = take(static_cast<size_t>(T) * FM_GSTRIDE * 4);
    const size_t o_ix = take(static_cast<size_t>(T) * kq_gu * 1024);
    const size_t o_glu = take(static_cast<size_t>(S) * n_ff * 4);
    const size_t o_gg = take(static_cast<size_t>(S) * FM_GSTRIDE * 4);
    const size_t o_ig = take(static_cast<size_t>(S) * kq_d * 1024);
    const size_t o_part = take(static_cast<size_t>(S) * n_embd * 4);
    void *wsp = nullptr;
    rc = workspace_get(WS_MOE, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *base = static_cast<uint8_t *>(wsp);
    float *logits = reinterpret_cast<float *>(base + o_logits);
    int32_t *ids = chk_ids ? chk_ids : reinterpret_cast<int32_t *>(base + o_ids);
    float *wts = chk_wts ? chk_wts : reinterpret_cast<float *>(base + o_wts);
    int32_t *eoff = reinterpret_cast<int32_t *>(base + o_eoff);
    int32_t *act = reinterpret_cast<int32_t *>(base + o_act);
    int32_t *slots = reinterpret_cast<int32_t *>(base + o_slots);
    float *glu = chk_glu ? chk_glu : reinterpret_cast<float *>(base + o_glu);
    float *part = chk_part ? chk_part : reinterpret_cast<float *>(base + o_part);

    rc = route_launch(x, n_embd, w_r, T, n_embd, E, n_used, clamp_val, logits, ids, wts, eoff, slots, act, stream,
                      2, nullptr, 0, base + o_ix, reinterpret_cast<float *>(base + o_gx),
                      static_cast<int64_t>(kq_gu) * 1024);
    if (rc != FR_OK) return rc;
    const int max_active = std::min(E, S);
    FeArgs a{};
    a.N = n_ff;
    a.K = n_embd;
    a.n_rb = n_ff / 128;
    a.E = E;
    a.n_used = n_used;
    a.bcast = 1;
    a.eoff = eoff;
    a.slots = slots;
    a.act = act;
    a.w0 = static_cast<const uint8_t *>(wg_t);
    a.w1 = static_cast<const uint8_t *>(wu_t);
    a.e_stride = static_cast<int64_t>(n_ff / 128) * kq_gu * FT_TILE;
    a.s0 = sg;
    a.s1 = su;
    a.y = glu;
    a.ld_tok = static_cast<int64_t>(n_used) * n_ff;
    a.ld_slot = n_ff;
    rc = fp4e_run(a, true, nullptr, 0, T, T, max_active, base + o_ix, reinterpret_cast<float *>(base + o_gx),
                  stream);
    if (rc != FR_OK) return rc;
    FeArgs d{};
    d.N = n_embd;
    d.K = n_ff;
    d.n_rb = n_embd / 128;
    d.E = E;
    d.n_used = n_used;
    d.bcast = 0;
    d.eoff = eoff;
    d.slots = slots;
    d.act = act;
    d.w0 = static_cast<const uint8_t *>(wd_t);
    d.w1 = d.w0;
    d.e_stride = static_cast<int64_t>(n_embd / 128) * kq_d * FT_TILE;
    d.s0 = sd;
    d.y = part;
    d.ld_tok = static_cast<int64_t>(n_used) * n_embd;
    d.ld_slot = n_embd;
    rc = fp4e_run(d, false, glu, n_ff, S, T, max_active, base + o_ig, reinterpret_cast<float *>(base + o_gg), stream);
    if (rc != FR_OK) return rc;
    return launch_pdl(k_moe_combine, dim3((n_embd + 255) / 256, T), dim3(256), 0, stream,
                      static_cast<const float *>(part), static_cast<const float *>(wts), resid, out, n_used, n_embd);
}

int fr_mul_mat_id_tiled(const void *w_t, int E, int N, int K, const float *x, int64_t x_ld_slot, int64_t x_ld_tok,
                        const int32_t *ids, int64_t ids_ld, float *dst, int64_t dst_ld_slot, int64_t dst_ld_tok,
                        int T, int n_used, cudaStream_t stream) {
    if (fault_hit("fr_mul_mat_id_tiled")) return FR_EINJECTED;
    if (!w_t || !x || !ids || !dst || T <= 0 || n_used <= 0 || n_used > MOE_MAX_USED) return FR_EINVAL;
    if (!fe_shape_ok(N, K) || E <= 0 || E > FE_MAX_E || static_cast<long>(T) * n_used > MOE_MAX_SLOTS) return FR_EINVAL;
    if (!aligned16(w_t) || ids_ld < n_used || x_ld_tok < K) return FR_EINVAL;
    const bool bcast = x_ld_slot == 0;
    // the slot rows of a per-slot input must be evenly spaced (one row stride)
    if (!bcast && (x_ld_slot < K || x_ld_tok != static_cast<int64_t>(n_used) * x_ld_slot)) return FR_EINVAL;
    const int rows = bcast ? T : T * n_used;
    const int64_t ldx = bcast ? x_ld_tok : x_ld_slot;
    const int S = T * n_used;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_g = take(static_cast<size_t>(rows) * FM_GSTRIDE * 4);
    const size_t o_img = take(static_cast<size_t>(rows) * (K / 256) * 1024);
    void *wsp = nullptr;
    int rc = workspace_get(WS_MOE, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *base = static_cast<uint8_t *>(wsp);
    int32_t *eoff = reinterpret_cast<int32_t *>(base + o_eoff);
    int32_t *act = reinterpret_cast<int32_t *>(base + o_act);
    int32_t *slots = reinterpret_cast<int32_t *>(base + o_slots);
    static bool attr_done[64] = {};
    rc = allow_max_smem(k_group_ids, attr_done);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_group_ids, dim3(1), dim3(1024), group_smem(T, n_used), stream, ids, ids_ld, T, n_used, E, eoff,
                    slots, act, 0);
    if (rc != FR_OK) return rc;
    FeArgs a{};
    a.N = N;
    a.K = K;
    a.n_rb = N / 128;
    a.E = E;
    a.n_used = n_used;
    a.bcast = bcast ? 1 : 0;
    a.eoff = eoff;
    a.slots = slots;
    a.act = act;
    a.w0 = static_cast<const uint8_t *>(w_t);
    a.w1 = a.w0;
    a.e_stride = static_cast<int64_t>(N / 128) * (K / 256) * FT_TILE;
    a.y = dst;
    a.ld_tok = dst_ld_tok;
    a.ld_slot = dst_ld_slot;
    return fp4e_run(a, false, x, ldx, rows, T, std::min(E, S), base + o_img, reinterpret_cast<float *>(base + o_g),
                    stream);
}

} // extern "C"

namespace frb {
// expert-parallel exchange buffer (see k_ep_dispatch)
struct EpLayout {
    int64_t flags_d, flags_r, seen_d, seen_r, recv_x, recv_eid, back, total;
};
static EpLayout ep_layout(int T, int n_embd, int n_used, int P) {
    const int64_t cap = static_cast<int64_t>(T) * n_used;
    EpLayout l{};
    l.flags_d = 0;
    l.flags_r = 128;
    l.seen_d = 256;
    l.seen_r = 384;
    l.recv_x = 512;
    l.recv_eid = l.recv_x + (P * cap * n_embd * 4 + 255) / 256 * 256;
    l.back = l.recv_eid + (P * cap * 4 + 255) / 256 * 256;
    l.total = l.back + (cap * n_embd * 4 + 255) / 256 * 256;
    return l;
}
} // namespace frb

extern "C" {

int64_t fr_ep_buffer_bytes(int T_max, int n_embd, int n_used, int nranks) {
    if (T_max <= 0 || n_embd <= 0 || n_used <= 0 || nranks <= 0) return -1;
    return ep_layout(T_max, n_embd, n_used, nranks).total;
}

} // extern "C"

namespace frb {
static int ep_moe_impl(const float *x, const float *w_r, const void *wg_local, const void *wu_local,
                       const void *wd_local, const float *sg, const float *su, const float *sd, const float *resid,
                       float *out, int T, int T_max, int n_embd, int n_ff, int E, int n_used, float clamp_val,
                       int nranks, int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes,
                       bool tiled, cudaStream_t stream) {
    int rc = check_route_shape(T, n_embd, E, n_used);
    if (rc != FR_OK) return rc;
    if (!x || !w_r || !wg_local || !wu_local || !wd_local || !out || !peer_base || !local_base) return FR_EINVAL;
    if (nranks <= 0 || nranks > 32 || rank < 0 || rank >= nranks || E % nranks != 0 || T > T_max) return FR_EINVAL;
    if (n_embd % 64 != 0 || n_ff % 64 != 0 || !aligned16(x) || !aligned16(w_r)) return FR_EINVAL;
    const int cap = T_max * n_used;
    if (static_cast<int64_t>(nranks) * cap > MOE_MAX_SLOTS) return FR_EINVAL;
    const EpLayout L = ep_layout(T_max, n_embd, n_used, nranks);
    if (buffer_bytes < L.total) return FR_EINVAL;
    uint8_t *base = static_cast<uint8_t *>(local_base);
    uint8_t *const *pb = reinterpret_cast<uint8_t *const *>(peer_base);
    const int E_p = E / nranks;
    const int S = T * n_used;
    // routing (replicated router) and this rank's expert outputs live in a
    // workspace of their own: the expert FFN uses the MoE workspace
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_logits = take(static_cast<size_t>(T) * E * 4);
    const size_t o_ids = take(static_cast<size_t>(S) * 4);
    const size_t o_wts = take(static_cast<size_t>(S) * 4);
    const size_t o_eoff = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_act = take(static_cast<size_t>(E + 1) * 4);
    const size_t o_slots = take(static_cast<size_t>(S) * 4);
    const size_t o_y = take(static_cast<size_t>(nranks) * cap * n_embd * 4);
    void *wsp = nullptr;
    rc = workspace_get(WS_ACT2, off, stream, &wsp);
    if (rc != FR_OK) return rc;
    uint8_t *w = static_cast<uint8_t *>(wsp);
    int32_t *ids = reinterpret_cast<int32_t *>(w + o_ids);
    float *wts = reinterpret_cast<float *>(w + o_wts);
    float *y = reinterpret_cast<float *>(w + o_y);
    rc = route_launch(x, n_embd, w_r, T, n_embd, E, n_used, clamp_val, reinterpret_cast<float *>(w + o_logits), ids,
                      wts, reinterpret_cast<int32_t *>(w + o_eoff), reinterpret_cast<int32_t *>(w + o_slots),
                      reinterpret_cast<int32_t *>(w + o_act), stream);
    if (rc != FR_OK) return rc;
    // rows to the expert owners
    rc = launch_pdl(k_ep_dispatch, dim3(EP_CTAS), dim3(256), 0, stream, x, static_cast<int64_t>(n_embd),
                    static_cast<const int32_t *>(ids), S, cap, n_used, E_p, n_embd, pb, nranks, rank, L.recv_x,
                    L.recv_eid, L.flags_d);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_tp_reduce, dim3(1), dim3(256), 0, stream, reinterpret_cast<const unsigned int *>(base + L.flags_d),
                    reinterpret_cast<unsigned int *>(base + L.seen_d), nranks, static_cast<unsigned>(EP_CTAS),
                    static_cast<const float *>(nullptr), static_cast<int64_t>(0), static_cast<const float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<int64_t>(1), static_cast<float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<unsigned int *>(nullptr), static_cast<int64_t>(0), 1);
    if (rc != FR_OK) return rc;
    // this rank's experts over everything it received (empty slots skipped)
    if (tiled)
        rc = moe_experts_tiled_impl(reinterpret_cast<const float *>(base + L.recv_x), n_embd,
                                    reinterpret_cast<const int32_t *>(base + L.recv_eid), nranks * cap, wg_local,
                                    wu_local, wd_local, sg, su, sd, y, n_embd, n_embd, n_ff, E_p, 1, stream);
    else
        rc = moe_experts_impl(reinterpret_cast<const float *>(base + L.recv_x), n_embd,
                              reinterpret_cast<const int32_t *>(base + L.recv_eid), nranks * cap, wg_local, wu_local,
                              wd_local, sg, su, sd, y, n_embd, n_embd, n_ff, E_p, 1, stream);
    if (rc != FR_OK) return rc;
    // outputs back to the slots they came from
    rc = launch_pdl(k_ep_return, dim3(EP_CTAS), dim3(256), 0, stream, static_cast<const float *>(y),
                    reinterpret_cast<const int32_t *>(base + L.recv_eid), cap, n_embd, pb, nranks, rank, L.back,
                    L.flags_r);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_tp_reduce, dim3(1), dim3(256), 0, stream, reinterpret_cast<const unsigned int *>(base + L.flags_r),
                    reinterpret_cast<unsigned int *>(base + L.seen_r), nranks, static_cast<unsigned>(EP_CTAS),
                    static_cast<const float *>(nullptr), static_cast<int64_t>(0), static_cast<const float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<int64_t>(1), static_cast<float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<unsigned int *>(nullptr), static_cast<int64_t>(0), 1);
    if (rc != FR_OK) return rc;
    return launch_pdl(k_moe_combine, dim3((n_embd + 255) / 256, T), dim3(256), 0, stream,
                      reinterpret_cast<const float *>(base + L.back), static_cast<const float *>(wts), resid, out,
                      n_used, n_embd);
}
} // namespace frb

extern "C" {

int fr_ep_moe_nvfp4(const float *x, const float *w_r, const void *wg_local, const void *wu_local,
                    const void *wd_local, const float *sg, const float *su, const float *sd, const float *resid,
                    float *out, int T, int T_max, int n_embd, int n_ff, int E, int n_used, float clamp_val, int nranks,
                    int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream) {
    if (fault_hit("fr_ep_moe_nvfp4")) return FR_EINJECTED;
    return ep_moe_impl(x, w_r, wg_local, wu_local, wd_local, sg, su, sd, resid, out, T, T_max, n_embd, n_ff, E,
                       n_used, clamp_val, nranks, rank, peer_base, local_base, buffer_bytes, false, stream);
}

int fr_ep_moe_tiled(const float *x, const float *w_r, const void *wg_t, const void *wu_t, const void *wd_t,
                    const float *sg, const float *su, const float *sd, const float *resid, float *out, int T,
                    int T_max, int n_embd, int n_ff, int E, int n_used, float clamp_val, int nranks, int rank,
                    void *const *peer_base, void *local_base, int64_t buffer_bytes, cudaStream_t stream) {
    if (fault_hit("fr_ep_moe_tiled")) return FR_EINJECTED;
    return ep_moe_impl(x, w_r, wg_t, wu_t, wd_t, sg, su, sd, resid, out, T, T_max, n_embd, n_ff, E, n_used,
                       clamp_val, nranks, rank, peer_base, local_base, buffer_bytes, true, stream);
}

int fr_ipc_alloc(int64_t bytes, void **dev_ptr, void *handle64) {
    if (bytes <= 0 || !dev_ptr || !handle64) return FR_EINVAL;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    void *p = nullptr;
    int rc = cuda_rc(cudaMalloc(&p, static_cast<size_t>(bytes)));
    if (rc != FR_OK) return rc;
    rc = cuda_rc(cudaMemset(p, 0, static_cast<size_t>(bytes)));
    cudaIpcMemHandle_t h;
    if (rc == FR_OK) rc = cuda_rc(cudaIpcGetMemHandle(&h, p));
    if (rc != FR_OK) {
        cudaFree(p);
        return rc;
    }
    std::memcpy(handle64, &h, sizeof(h));
    *dev_ptr = p;
    return FR_OK;
}

int fr_ipc_open(const void *handle64, void **dev_ptr) {
    if (!handle64 || !dev_ptr) return FR_EINVAL;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, sizeof(h));
    return cuda_rc(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int fr_ipc_close(void *dev_ptr) { return dev_ptr ? cuda_rc(cudaIpcCloseMemHandle(dev_ptr)) : FR_EINVAL; }

int fr_ipc_free(void *dev_ptr) { return dev_ptr ? cuda_rc(cudaFree(dev_ptr)) : FR_EINVAL; }

int64_t fr_tp_buffer_bytes(int T, int n_embd, int n_ff, int nranks) {
    if (T <= 0 || n_embd <= 0 || n_ff <= 0 || nranks <= 0) return -1;
    return tp_layout_cap(T, n_embd, nranks).total;
}

} // extern "C"

namespace frb {
// One rank's tensor-parallel FFN step; `tiled`: the shards are in the
// tile-major layout (FP4 tensor-core matvecs), else ggml's layout.
static int tp_ffn_impl(const float *x, const void *wg_shard, const void *wu_shard, const void *wd_shard,
                       const float *sg, const float *su, const float *sd, const float *resid, float *out, int T,
                       int n_embd, int n_ff, int nranks, int rank, void *const *peer_base, void *local_base,
                       int64_t buffer_bytes, bool tiled, cudaStream_t stream) {
    if (!x || !wg_shard || !wu_shard || !wd_shard || !out || !peer_base || !local_base) return FR_EINVAL;
    if (T <= 0 || nranks <= 0 || nranks > 32 || rank < 0 || rank >= nranks) return FR_EINVAL;
    // the n_ff shard boundary falls on NVFP4 block (64) boundaries, so the
    // GLU's q8_1 blocks and the down rows' NVFP4 blocks never straddle it
    if (n_embd % 64 != 0 || n_ff % (64 * nranks) != 0) return FR_EINVAL;
    const TpLayout L = tp_layout_buf(buffer_bytes, n_embd, nranks);
    if (T > L.t_cap) return FR_EINVAL;
    uint8_t *base = static_cast<uint8_t *>(local_base);
    uint8_t *const *pb = reinterpret_cast<uint8_t *const *>(peer_base);
    const int F_p = n_ff / nranks;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(F_p) / 64 * NV_BYTES;
    const int64_t slot_off = L.part + static_cast<int64_t>(rank) * T * n_embd * 4;
    const unsigned int *flags = reinterpret_cast<const unsigned int *>(base + L.flags);
    unsigned int *seen = reinterpret_cast<unsigned int *>(base + L.seen);
    unsigned int *epoch = reinterpret_cast<unsigned int *>(base + L.epoch);
    const float *parts = reinterpret_cast<const float *>(base + L.part);
    const int64_t n_out = static_cast<int64_t>(T) * n_embd;
    void *glu_p = nullptr;
    int rc = workspace_get(WS_GLU, static_cast<size_t>(T) * F_p * sizeof(float), stream, &glu_p);
    if (rc != FR_OK) return rc;
    float *glu = static_cast<float *>(glu_p);

    unsigned expect;
    if (tiled || (use_tc(wg_shard, wu_shard, ld_gu, n_embd, T) && use_tc(wd_shard, nullptr, ld_d, F_p, T))) {
        // tensor-core matvecs: on tile-major shards the down matvec's
        // epilogue stores the partial output into every rank's slot itself;
        // on ggml's layout it goes into this rank's own slot and a push
        // kernel stores it into every peer's slot
        constexpr int PUSH_CTAS = 64;
        if (tiled) {
            // the down matvec's epilogue stores its rows into every rank's
            // slot and counts each CTA into the flags: no push kernel
            void *am = nullptr;
            rc = workspace_get(WS_AMAX, static_cast<size_t>(T) * (F_p / 32) * sizeof(float), stream, &am);
            if (rc != FR_OK) return rc;
            rc = fp4t_matvec(static_cast<const uint8_t *>(wg_shard), static_cast<const uint8_t *>(wu_shard), F_p,
                             n_embd, x, n_embd, nullptr, 0, T, sg, su, nullptr, 0, glu, F_p, true, stream,
                             static_cast<float *>(am));
            if (rc != FR_OK) return rc;
            unsigned ctas = 0;
            const TpOut to{pb, nranks, rank, slot_off, L.flags, epoch, L.half, &ctas};
            rc = fp4t_matvec(static_cast<const uint8_t *>(wd_shard), nullptr, n_embd, F_p, glu, F_p, nullptr, 0, T,
                             sd, nullptr, nullptr, 0, reinterpret_cast<float *>(base + L.stage), n_embd, false,
                             stream, nullptr,
                             static_cast<const float *>(am), &to);
            if (rc != FR_OK) return rc;
            expect = ctas;
        } else {
            rc = tcx_matvec(static_cast<const uint8_t *>(wg_shard), static_cast<const uint8_t *>(wu_shard), ld_gu,
                            F_p, n_embd, x, n_embd, nullptr, 0, T, sg, su, nullptr, 0, glu, F_p, true, stream);
            if (rc != FR_OK) return rc;
            // the down matvec writes this rank's partial rows into its local
            // staging area; the push kernel stores them into this rank's slot
            // of every rank (the step's parity half)
            rc = tcx_matvec(static_cast<const uint8_t *>(wd_shard), nullptr, ld_d, n_embd, F_p, glu, F_p, nullptr, 0,
                            T, sd, nullptr, nullptr, 0, reinterpret_cast<float *>(base + L.stage), n_embd, false,
                            stream);
            if (rc != FR_OK) return rc;
            rc = launch_pdl(k_tp_push, dim3(PUSH_CTAS), dim3(256), 0, stream, pb, nranks, rank, L.stage, slot_off,
                            L.half, static_cast<const unsigned int *>(epoch), static_cast<int64_t>(n_embd), T, n_embd,
                            L.flags);
            expect = PUSH_CTAS;
        }
        if (rc != FR_OK) return rc;
    } else {
        void *q8x = nullptr, *q8g = nullptr;
        rc = workspace_get(WS_Q8, static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES, stream, &q8x);
        if (rc != FR_OK) return rc;
        rc = workspace_get(WS_GLUQ8, static_cast<size_t>(T) * (F_p / 32) * Q8_BYTES, stream, &q8g);
        if (rc != FR_OK) return rc;
        rc = quantize_launch(x, n_embd, q8x, n_embd / 32, T, n_embd, stream);
        if (rc != FR_OK) return rc;
        // gate/up: this rank's GLU columns, locally
        GvParams p{};
        p.w0 = static_cast<const uint8_t *>(wg_shard);
        p.w1 = static_cast<const uint8_t *>(wu_shard);
        p.w_ld = ld_gu;
        p.q8 = static_cast<const uint8_t *>(q8x);
        p.ldq = n_embd / 32;
        p.s0 = sg;
        p.s1 = su;
        p.y = glu;
        p.ldy = F_p;
        p.N = F_p;
        p.K = n_embd;
        rc = gemv_run(p, T, true, stream);
        if (rc != FR_OK) return rc;
        rc = quantize_launch(glu, F_p, q8g, F_p / 32, T, F_p, stream);
        if (rc != FR_OK) return rc;
        // down over this rank's K range: the partial output of every row goes
        // into this rank's slot on every rank, then the flags are raised
        GvParams q{};
        q.w0 = static_cast<const uint8_t *>(wd_shard);
        q.w_ld = ld_d;
        q.q8 = static_cast<const uint8_t *>(q8g);
        q.ldq = F_p / 32;
        q.s0 = sd;
        q.y = nullptr;
        q.ldy = n_embd;
        q.N = n_embd;
        q.K = F_p;
        q.peer_base = pb;
        q.npeers = nranks;
        q.rank = rank;
        q.peer_off = slot_off;
        q.flag_off = L.flags;
        q.col_off = 0;
        q.epoch = epoch;
        q.par_bytes = L.half;
        rc = gemv_run(q, T, false, stream);
        if (rc != FR_OK) return rc;
        expect = gemv_ctas(n_embd, F_p, ld_d, T, false);
    }
    // wait for every rank's partial, sum them in rank order, add the residual.
    // Always TP_WAIT_CTAS CTAs: each keeps its own consumed count.
    return launch_pdl(k_tp_reduce, dim3(TP_WAIT_CTAS), dim3(256), 0, stream, flags, seen, nranks, expect, parts,
                      n_out, resid, static_cast<int64_t>(n_embd), static_cast<int64_t>(n_embd), out,
                      static_cast<int64_t>(n_embd), epoch, L.half / 4, nranks);
}

} // namespace frb

extern "C" {

int fr_tp_wait(void *local_base, int64_t buffer_bytes, int n_embd, int nranks, unsigned expect,
               cudaStream_t stream) {
    if (fault_hit("fr_tp_wait")) return FR_EINJECTED;
    if (!local_base || n_embd <= 0 || nranks <= 0 || nranks > 32) return FR_EINVAL;
    const TpLayout L = tp_layout_buf(buffer_bytes, n_embd, nranks);
    if (L.t_cap <= 0) return FR_EINVAL;
    uint8_t *base = static_cast<uint8_t *>(local_base);
    // every consumed-count row advances, as in a step's reduce; nothing is summed
    return launch_pdl(k_tp_reduce, dim3(TP_WAIT_CTAS), dim3(256), 0, stream,
                      reinterpret_cast<const unsigned int *>(base + L.flags),
                      reinterpret_cast<unsigned int *>(base + L.seen), nranks, expect,
                      static_cast<const float *>(nullptr), static_cast<int64_t>(0),
                      static_cast<const float *>(nullptr), static_cast<int64_t>(0), static_cast<int64_t>(1),
                      static_cast<float *>(nullptr), static_cast<int64_t>(0), static_cast<unsigned int *>(nullptr),
                      static_cast<int64_t>(0), 1);
}

int fr_tp_ffn_nvfp4(const float *x, const void *wg_shard, const void *wu_shard, const void *wd_shard, const float *sg,
                    const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                    int nranks, int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes,
                    cudaStream_t stream) {
    if (fault_hit("fr_tp_ffn_nvfp4")) return FR_EINJECTED;
    return tp_ffn_impl(x, wg_shard, wu_shard, wd_shard, sg, su, sd, resid, out, T, n_embd, n_ff, nranks, rank,
                       peer_base, local_base, buffer_bytes, false, stream);
}

} // extern "C"

namespace frb {
// Row-sharded tensor-parallel FFN buffer: [flags of the GLU exchange 32]
// [flags of the output exchange 32] u32, per-CTA consumed counts of both
// [TP_WAIT_CTAS][32] and step counts [TP_WAIT_CTAS], then two parity halves,
// each [T_cap][n_ff / 32] q8_1 blocks of the GLU followed (256-aligned) by
// [T_cap][n_embd] f32 of the output; capacity from the buffer's size.
struct TpRowsLayout {
    int64_t flags_g, flags_o, seen_g, seen_o, epoch, part, q8, out, half, total, t_cap;
};
static int64_t tpr_hdr() {
    return (4LL * 64 + 2 * 4LL * 32 * TP_WAIT_CTAS + 4LL * TP_WAIT_CTAS + 255) / 256 * 256;
}
static int64_t tpr_half(int64_t t_cap, int n_embd, int n_ff) {
    const int64_t q8 = (t_cap * (n_ff / 32) * Q8_BYTES + 255) / 256 * 256;
    return q8 + t_cap * n_embd * 4;
}
static TpRowsLayout tpr_layout_cap(int64_t t_cap, int n_embd, int n_ff) {
    TpRowsLayout l{};
    l.flags_g = 0;
    l.flags_o = 4LL * 32;
    l.seen_g = 4LL * 64;
    l.seen_o = l.seen_g + 4LL * 32 * TP_WAIT_CTAS;
    l.epoch = l.seen_o + 4LL * 32 * TP_WAIT_CTAS;
    l.part = tpr_hdr();
    l.t_cap = t_cap;
    l.half = tpr_half(t_cap, n_embd, n_ff);
    l.q8 = 0;
    l.out = (t_cap * (n_ff / 32) * Q8_BYTES + 255) / 256 * 256;
    l.total = l.part + 2 * l.half;
    return l;
}
static TpRowsLayout tpr_layout_buf(int64_t bytes, int n_embd, int n_ff) {
    int64_t t = 0;
    while (t < (1 << 16) && tpr_layout_cap(t + 1, n_embd, n_ff).total <= bytes) ++t;
    return tpr_layout_cap(t, n_embd, n_ff);
}
} // namespace frb

extern "C" {

int64_t fr_tp_rows_buffer_bytes(int T, int n_embd, int n_ff, int nranks) {
    if (T <= 0 || n_embd <= 0 || n_ff <= 0 || nranks <= 0) return -1;
    return tpr_layout_cap(T, n_embd, n_ff).total;
}

int fr_tp_ffn_rows(const float *x, const void *wg_shard, const void *wu_shard, const void *wd_shard, const float *sg,
                   const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                   int nranks, int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes,
                   cudaStream_t stream) {
    if (fault_hit("fr_tp_ffn_rows")) return FR_EINJECTED;
    if (!x || !wg_shard || !wu_shard || !wd_shard || !out || !peer_base || !local_base) return FR_EINVAL;
    if (T <= 0 || nranks <= 0 || nranks > 32 || rank < 0 || rank >= nranks) return FR_EINVAL;
    if (n_embd % 64 != 0 || n_ff % 64 != 0 || n_ff % (64 * nranks) != 0 || n_embd % nranks != 0) return FR_EINVAL;
    const TpRowsLayout L = tpr_layout_buf(buffer_bytes, n_embd, n_ff);
    if (T > L.t_cap) return FR_EINVAL;
    uint8_t *base = static_cast<uint8_t *>(local_base);
    uint8_t *const *pb = reinterpret_cast<uint8_t *const *>(peer_base);
    unsigned int *epoch = reinterpret_cast<unsigned int *>(base + L.epoch);
    const int F_p = n_ff / nranks, E_p = n_embd / nranks;
    const int64_t ld_gu = static_cast<int64_t>(n_embd) / 64 * NV_BYTES;
    const int64_t ld_d = static_cast<int64_t>(n_ff) / 64 * NV_BYTES;
    void *q8x = nullptr, *glu_p = nullptr;
    int rc = workspace_get(WS_Q8, static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES, stream, &q8x);
    if (rc != FR_OK) return rc;
    rc = workspace_get(WS_GLU, static_cast<size_t>(T) * F_p * sizeof(float), stream, &glu_p);
    if (rc != FR_OK) return rc;
    float *glu = static_cast<float *>(glu_p);
    // q8_1(x) on every rank (identical bits), then this rank's GLU columns
    rc = quantize_launch(x, n_embd, q8x, n_embd / 32, T, n_embd, stream);
    if (rc != FR_OK) return rc;
    GvParams p{};
    p.w0 = static_cast<const uint8_t *>(wg_shard);
    p.w1 = static_cast<const uint8_t *>(wu_shard);
    p.w_ld = ld_gu;
    p.q8 = static_cast<const uint8_t *>(q8x);
    p.ldq = n_embd / 32;
    p.s0 = sg;
    p.s1 = su;
    p.y = glu;
    p.ldy = F_p;
    p.N = F_p;
    p.K = n_embd;
    rc = gemv_run(p, T, true, stream);
    if (rc != FR_OK) return rc;
    // all-gather of the GLU as q8_1 blocks: every rank's blocks into every rank
    constexpr int PUSH_CTAS = 64;
    rc = launch_pdl(k_q8_push, dim3(PUSH_CTAS), dim3(256), 0, stream, static_cast<const float *>(glu),
                    static_cast<int64_t>(F_p), T, F_p, rank * F_p, pb, nranks, rank, L.part + L.q8, L.half,
                    static_cast<const unsigned int *>(epoch), static_cast<int64_t>(n_ff / 32), L.flags_g);
    if (rc != FR_OK) return rc;
    rc = launch_pdl(k_tp_reduce, dim3(TP_WAIT_CTAS), dim3(256), 0, stream,
                    reinterpret_cast<const unsigned int *>(base + L.flags_g),
                    reinterpret_cast<unsigned int *>(base + L.seen_g), nranks, static_cast<unsigned>(PUSH_CTAS),
                    static_cast<const float *>(nullptr), static_cast<int64_t>(0), static_cast<const float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<int64_t>(1), static_cast<float *>(nullptr),
                    static_cast<int64_t>(0), static_cast<unsigned int *>(nullptr), static_cast<int64_t>(0), 1);
    if (rc != FR_OK) return rc;
    // this rank's output rows over the whole GLU, stored into column block
    // rank * E_p of every rank's output (the output all-gather)
    GvParams q{};
    q.w0 = static_cast<const uint8_t *>(wd_shard);
    q.w_ld = ld_d;
    q.q8 = base + L.part + L.q8;
    q.q8_epoch = epoch;
    q.q8_par = L.half;
    q.ldq = n_ff / 32;
    q.s0 = sd;
    q.y = nullptr;
    q.ldy = n_embd;
    q.N = E_p;
    q.K = n_ff;
    q.peer_base = pb;
    q.npeers = nranks;
    q.rank = rank;
    q.peer_off = L.part + L.out;
    q.flag_off = L.flags_o;
    q.col_off = static_cast<int64_t>(rank) * E_p;
    q.epoch = epoch;
    q.par_bytes = L.half;
    rc = gemv_run(q, T, false, stream);
    if (rc != FR_OK) return rc;
    const unsigned expect = gemv_ctas(E_p, n_ff, ld_d, T, false);
    // wait for every rank's column block, add the residual, advance the parity
    return launch_pdl(k_tp_reduce, dim3(TP_WAIT_CTAS), dim3(256), 0, stream,
                      reinterpret_cast<const unsigned int *>(base + L.flags_o),
                      reinterpret_cast<unsigned int *>(base + L.seen_o), nranks, expect,
                      reinterpret_cast<const float *>(base + L.part + L.out), static_cast<int64_t>(T) * n_embd,
                      resid, static_cast<int64_t>(n_embd), static_cast<int64_t>(n_embd), out,
                      static_cast<int64_t>(n_embd), epoch, L.half / 4, 1);
}

int fr_tp_ffn_tiled(const float *x, const void *wg_t, const void *wu_t, const void *wd_t, const float *sg,
                    const float *su, const float *sd, const float *resid, float *out, int T, int n_embd, int n_ff,
                    int nranks, int rank, void *const *peer_base, void *local_base, int64_t buffer_bytes,
                    cudaStream_t stream) {
    if (fault_hit("fr_tp_ffn_tiled")) return FR_EINJECTED;
    if (nranks <= 0 || n_embd % 256 != 0 || n_ff % (256 * nranks) != 0) return FR_EINVAL;
    return tp_ffn_impl(x, wg_t, wu_t, wd_t, sg, su, sd, resid, out, T, n_embd, n_ff, nranks, rank, peer_base,
                       local_base, buffer_bytes, true, stream);
}

} // extern "C"

// ======================================================================
// Decode-step kernels of the synthetic MoE decoder
// ======================================================================
namespace frb {

// [rows, 128] f16 rows (256 B), box 64 halves x 128 rows, 128-byte swizzle
static int make_map_kv(CUtensorMap *map, const void *base, int64_t rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return FR_ENODEVICE;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(AT_D), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(AT_D * 2)};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FR_OK : FR_EINVAL;
}

// splitmix64
__device__ __forceinline__ uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// NVFP4 blocks with BASELINE's distribution, generated on the device (for
// multi-GB synthetic models): codes uniform over 0..15, sub-block scales
// e4m3(|N(0,1)| * sigma) RNE (Box-Muller on two hashed uniforms).
__global__ void k_synth_nvfp4(uint64_t seed, int64_t nblocks, float sigma, uint8_t *out) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint8_t *blk = out + b * NV_BYTES;
    uint64_t h = sm64(seed ^ (static_cast<uint64_t>(b) * 0xD1B54A32D192ED03ull));
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
        const uint64_t r = sm64(h + s);
        const double u1 = (static_cast<double>(r >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        const double u2 = static_cast<double>(sm64(r) >> 11) * (1.0 / 9007199254740992.0);
        const double rad = sqrt(-2.0 * log(u1));
        const float n0 = static_cast<float>(fabs(rad * cos(6.283185307179586 * u2))) * sigma;
        const float n1 = static_cast<float>(fabs(rad * sin(6.283185307179586 * u2))) * sigma;
        blk[s] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(n0, __NV_SATFINITE, __NV_E4M3));
        blk[s + 1] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(n1, __NV_SATFINITE, __NV_E4M3));
    }
    // 32 bytes of codes (uniform over all 16 values); blocks are 36 bytes
    // apart, so 4-byte stores
    uint32_t *codes = reinterpret_cast<uint32_t *>(blk + 4);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint64_t r = sm64(h ^ (0xA5A5A5A5ull + w));
        codes[2 * w] = static_cast<uint32_t>(r);
        codes[2 * w + 1] = static_cast<uint32_t>(r >> 32);
    }
}

} // namespace frb

extern "C" {

int fr_synth_nvfp4_device(uint64_t seed, int64_t rows, int64_t K, double scale_sigma, void *out,
                          cudaStream_t stream) {
    if (!out || rows <= 0 || K <= 0 || K % 64 != 0) return FR_EINVAL;
    const int64_t nb = rows * (K / 64);
    const unsigned grid = static_cast<unsigned>((nb + 255) / 256);
    k_synth_nvfp4<<<grid, 256, 0, stream>>>(seed, nb, static_cast<float>(scale_sigma), static_cast<uint8_t *>(out));
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
    return cuda_rc(e);
}

int fr_rmsnorm_f32(const float *x, const float *w, float *y, int T, int H, float eps, cudaStream_t stream) {
    if (fault_hit("fr_rmsnorm_f32")) return FR_EINJECTED;
    if (!x || !y || T <= 0 || H <= 0) return FR_EINVAL;
    return launch_pdl(k_rmsnorm, dim3(T), dim3(256), 0, stream, x, w, y, H, eps);
}

int fr_rope_kv_f16(const float *qkv, const int32_t *pos, float *q_r, void *kcache, void *vcache, int T, int nh,
                   int nkv, int head_dim, int ctx, float rope_base, cudaStream_t stream) {
    if (fault_hit("fr_rope_kv_f16")) return FR_EINJECTED;
    if (!qkv || !pos || !q_r || !kcache || !vcache || T <= 0 || nh <= 0 || nkv <= 0 || ctx <= 0) return FR_EINVAL;
    if (head_dim != AT_D) return FR_EINVAL;
    return launch_pdl(k_rope_kv, dim3(T, (nh + nkv + 3) / 4), dim3(256), 0, stream, qkv, pos, q_r,
                      static_cast<__half *>(kcache),
                      static_cast<__half *>(vcache), nh, nkv, ctx, rope_base, 1.0f / sqrtf(static_cast<float>(AT_D)));
}

int fr_attn_decode_f16(const float *q_r, const void *kcache, const void *vcache, const int32_t *pos, float *out,
                       int T, int nh, int nkv, int head_dim, int ctx, cudaStream_t stream) {
    if (fault_hit("fr_attn_decode_f16")) return FR_EINJECTED;
    if (!q_r || !kcache || !vcache || !pos || !out || T <= 0 || nkv <= 0) return FR_EINVAL;
    if (head_dim != AT_D || nh != AT_G * nkv || ctx <= 0 || ctx % AT_CH != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(kcache) & 15) || (reinterpret_cast<uintptr_t>(vcache) & 15) ||
        (reinterpret_cast<uintptr_t>(q_r) & 15))
        return FR_EINVAL;
    const DevInfo &di = dev_info();
    if (di.cc_major != 10) return FR_ENODEVICE;
    // a sequence's chunks split S ways so that the grid fills the SMs (two
    // CTAs resident on each); at batch 64 one CTA walks all of its chunks
    int splits = std::min(ctx / AT_CH, std::max(1, 2 * di.sms / (T * nkv)));
    static const char *sv = getenv("FR_ATTN_SPLITS");
    if (sv && *sv) splits = std::max(1, std::min(ctx / AT_CH, atoi(sv)));
    void *part = nullptr, *cnt = nullptr;
    int rc = workspace_get(WS_ATPART, static_cast<size_t>(T) * nkv * splits * AT_PART * sizeof(float), stream, &part);
    if (rc != FR_OK) return rc;
    rc = workspace_get_zeroed(WS_ATCNT, static_cast<size_t>(T) * nkv * sizeof(unsigned int), stream, &cnt);
    if (rc != FR_OK) return rc;
    CUtensorMap mk, mv;
    const int64_t rows = static_cast<int64_t>(T) * nkv * ctx;
    rc = make_map_kv(&mk, kcache, rows);
    if (rc != FR_OK) return rc;
    rc = make_map_kv(&mv, vcache, rows);
    if (rc != FR_OK) return rc;
    static bool done[64] = {};
    rc = allow_max_smem(k_attn_decode, done);
    if (rc != FR_OK) return rc;
    AtArgs a{q_r, pos, nh, nkv, ctx, static_cast<float *>(part), static_cast<unsigned int *>(cnt), out};
    return launch_pdl(k_attn_decode, dim3(splits, nkv, T), dim3(AT_THREADS), AT_SMEM, stream, mk, mv, a);
}

int fr_embed_nvfp4(const void *table, int vocab, int H, const int32_t *prompt, int prompt_ld, int prompt_len,
                   const int32_t *gen, const int32_t *pos, float *x, int T, cudaStream_t stream) {
    if (fault_hit("fr_embed_nvfp4")) return FR_EINJECTED;
    if (!table || !pos || !x || !gen || T <= 0 || vocab <= 0 || H <= 0 || H % 64 != 0) return FR_EINVAL;
    if (prompt_len > 0 && !prompt) return FR_EINVAL;
    return launch_pdl(k_embed_nvfp4, dim3(T), dim3(256), 0, stream, static_cast<const uint8_t *>(table),
                      static_cast<int64_t>(H / 64 * NV_BYTES), prompt, prompt_ld, prompt_len, gen, pos, x, H, vocab);
}

int fr_argmax_f32(const float *logits, int T, int V, int32_t *tok, cudaStream_t stream) {
    if (fault_hit("fr_argmax_f32")) return FR_EINJECTED;
    if (!logits || !tok || T <= 0 || V <= 0 || T > 65535) return FR_EINVAL;
    // per-slice maxima and the rows' arrival counters (zero between calls)
    void *part = nullptr, *cnt = nullptr;
    int rc = workspace_get(WS_ARGMAX, static_cast<size_t>(T) * AM_SLICES * 8, stream, &part);
    if (rc != FR_OK) return rc;
    rc = workspace_get_zeroed(WS_AMCNT, static_cast<size_t>(T) * sizeof(unsigned int), stream, &cnt);
    if (rc != FR_OK) return rc;
    float *pv = static_cast<float *>(part);
    int *pi = reinterpret_cast<int *>(pv + static_cast<size_t>(T) * AM_SLICES);
    return launch_pdl(k_argmax, dim3(AM_SLICES, T), dim3(256), 0, stream, logits, V, tok, pv, pi,
                      static_cast<unsigned int *>(cnt));
}

int fr_pos_advance(int32_t *pos, cudaStream_t stream) {
    if (!pos) return FR_EINVAL;
    return launch_pdl(k_pos_advance, dim3(1), dim3(32), 0, stream, pos);
}

int fr_copy_pinned(void *dst, const void *src, int64_t bytes, cudaStream_t stream) {
    if (fault_hit("fr_copy_pinned")) return FR_EINJECTED;
    if (!dst || !src || bytes < 0 || bytes % 16 != 0) return FR_EINVAL;
    if ((reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15)) return FR_EINVAL;
    if (bytes == 0) return FR_OK;
    // the device-side address of each side (host memory must be mapped)
    auto dev_addr = [](const void *p, void **out) -> bool {
        cudaPointerAttributes a{};
        if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
            *out = const_cast<void *>(p);
            return true;
        }
        if (a.type == cudaMemoryTypeHost && a.devicePointer != nullptr) {
            *out = a.devicePointer;
            return true;
        }
        return false;
    };
    void *d = nullptr, *sp = nullptr;
    if (!dev_addr(dst, &d) || !dev_addr(src, &sp)) return FR_EINVAL;
    const int64_t n16 = bytes / 16;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((n16 + threads - 1) / threads, 4LL * dev_info().sms);
    return launch_pdl(k_copy16, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, stream,
                      static_cast<const uint4 *>(sp), static_cast<uint4 *>(d), n16);
}

} // extern "C"
