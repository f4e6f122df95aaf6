// fr_lib.cu -- the library's single CUDA translation unit: kernels from the
// fr_*.cuh headers plus the C-ABI entry points of include/fr_b200.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "fr_common.cuh"
#include "fr_runtime.cuh"
#include "fr_gemv.cuh"

namespace frb {

std::atomic<uint64_t> g_launches{0};

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

// ------------------------------------------------------------- matvec launcher
struct GvPlan {
    int LG, TT, rows_per_stage, rows_per_cta, grid, n_slots, slot_bytes;
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

static GvPlan gv_plan(int N, int K, int64_t w_ld, int T, bool dual) {
    const DevInfo &di = dev_info();
    GvPlan pl{};
    const int NB = K / 64;
    pl.LG = pick_lg(NB);
    pl.rows_per_stage = 32 / pl.LG;
    pl.slot_bytes = static_cast<int>((pl.rows_per_stage * w_ld * (dual ? 2 : 1) + 15) / 16 * 16);
    const int smem_cap = di.smem_optin > 0 ? di.smem_optin : 227 * 1024;
    // tokens per launch: as many as fit next to a minimal ring
    int nt = std::min(T, 8);
    while (nt > 1 && gv_act_bytes(nt, K) + 2048 + static_cast<size_t>(GV_CWARPS) * pl.slot_bytes > static_cast<size_t>(smem_cap) - 4096)
        nt = nt / 2;
    pl.TT = pow2_tokens(nt);
    if (pl.TT > nt) pl.TT = pow2_tokens(nt);
    const size_t act = gv_act_bytes(nt, K);
    // two CTAs per SM when the ring fits in half the shared memory, else one
    const int per_sm_budget = (smem_cap - 2048) / 2 - 1024;
    int ctas_per_sm = 2;
    long ring_budget = per_sm_budget - 2048 - static_cast<long>(act);
    if (ring_budget < static_cast<long>(GV_CWARPS) * pl.slot_bytes * 2) {
        ctas_per_sm = 1;
        ring_budget = smem_cap - 4096 - static_cast<long>(act);
    }
    int depth = static_cast<int>(ring_budget / (static_cast<long>(GV_CWARPS) * pl.slot_bytes));
    depth = std::max(1, std::min(depth, 6));
    pl.n_slots = GV_CWARPS * depth;
    const int stages = (N + pl.rows_per_stage - 1) / pl.rows_per_stage;
    const int max_grid = std::max(1, di.sms * ctas_per_sm);
    const int st_per_cta = (stages + max_grid - 1) / max_grid;
    pl.rows_per_cta = st_per_cta * pl.rows_per_stage;
    pl.grid = (N + pl.rows_per_cta - 1) / pl.rows_per_cta;
    pl.smem = 2048 + static_cast<size_t>(pl.n_slots) * pl.slot_bytes + act;
    return pl;
}

template <int LG, int TT, int EPI>
static int gv_launch_inst(const GvParams &p, const GvPlan &pl, cudaStream_t stream) {
    auto kern = k_gemv<LG, TT, EPI>;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        const DevInfo &di = dev_info();
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin);
        if (e != cudaSuccess) return cuda_rc(e);
        attr_done[dev & 63] = true;
    }
    return launch_pdl(kern, dim3(pl.grid), dim3(GV_THREADS), pl.smem, stream, p);
}

template <int LG, int EPI>
static int gv_launch_tt(const GvParams &p, const GvPlan &pl, cudaStream_t stream) {
    switch (pl.TT) {
    case 1: return gv_launch_inst<LG, 1, EPI>(p, pl, stream);
    case 2: return gv_launch_inst<LG, 2, EPI>(p, pl, stream);
    case 4: return gv_launch_inst<LG, 4, EPI>(p, pl, stream);
    default: return gv_launch_inst<LG, 8, EPI>(p, pl, stream);
    }
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
    p.rows_per_stage = pl.rows_per_stage;
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

static int quantize_launch(const float *x, int64_t ldx, void *q8, int64_t ldq, int T, int K, cudaStream_t stream) {
    const int64_t chunks = static_cast<int64_t>(T) * (K / 32);
    const int grid = static_cast<int>((chunks + 7) / 8);
    return launch_pdl(k_quantize_q8_1, dim3(grid), dim3(256), 0, stream, x, ldx,
                      static_cast<uint8_t *>(q8), ldq, T, K);
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

int fr_fault_inject(const char *site) {
    std::lock_guard<std::mutex> lk(g_fault_mu);
    g_fault_env_read = true;
    g_fault_site = site ? site : "";
    return FR_OK;
}

uint64_t fr_kernel_launches(void) { return g_launches.load(); }

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
    void *q8x = nullptr;
    float *glu = chk_glu;
    void *gq8 = chk_glu_q8;
    rc = workspace_get(WS_Q8, static_cast<size_t>(T) * (n_embd / 32) * Q8_BYTES, stream, &q8x);
    if (rc != FR_OK) return rc;
    if (!glu) {
        void *p = nullptr;
        rc = workspace_get(WS_GLU, static_cast<size_t>(T) * n_ff * sizeof(float), stream, &p);
        if (rc != FR_OK) return rc;
        glu = static_cast<float *>(p);
    }
    if (!gq8) {
        rc = workspace_get(WS_GLUQ8, static_cast<size_t>(T) * (n_ff / 32) * Q8_BYTES, stream, &gq8);
        if (rc != FR_OK) return rc;
    }
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
