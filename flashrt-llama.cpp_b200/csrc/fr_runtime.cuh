// fr_runtime.cuh -- host-side plumbing shared by the entry points: device
// properties, launch helper (PDL attribute), error mapping, fault injection,
// launch counting, grow-only per-device workspaces.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/fr_b200.h"

namespace frb {

extern std::atomic<uint64_t> g_launches;

struct DevInfo {
    int sms = 0;
    int smem_optin = 0;
    int cc_major = 0, cc_minor = 0;
};
const DevInfo &dev_info();

// -cudaError_t, the reference's convention (src/fr_quant_act.cu:106-108)
inline int cuda_rc(cudaError_t e) { return e == cudaSuccess ? FR_OK : -static_cast<int>(e); }

// host-side fault injection: true (and consumed) when `site` is armed
bool fault_hit(const char *site);

inline bool stream_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) return false;
    return st != cudaStreamCaptureStatusNone;
}

// Launch `kern` with the programmatic-stream-serialization attribute so it
// joins the caller's PDL chain (griddepcontrol in the kernels).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    if (e == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
    return cuda_rc(e);
}

// Allow `kern` the largest dynamic shared memory the device offers next to
// its static shared memory (once per device and kernel).
template <typename K>
int allow_max_smem(K kern, bool *done_per_dev) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (done_per_dev[dev & 63]) return FR_OK;
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return cuda_rc(e);
    const DevInfo &di = dev_info();
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             di.smem_optin - static_cast<int>(fa.sharedSizeBytes));
    if (e != cudaSuccess) return cuda_rc(e);
    done_per_dev[dev & 63] = true;
    return FR_OK;
}

// Grow-only device workspace, one per (device, purpose).  Never shrinks and
// never moves while large enough, so captured graphs stay valid; refuses to
// grow while the stream is capturing (the reference's rule,
// src/fr_dispatch.cu:135-160).
struct Workspace {
    void *ptr = nullptr;
    size_t cap = 0;
};
int workspace_get(int purpose, size_t bytes, cudaStream_t stream, void **out);

enum WsPurpose : int { WS_Q8 = 0, WS_GLU = 1, WS_GLUQ8 = 2, WS_MOE = 3, WS_ACT = 4, WS_TGPART = 5, WS_ACT2 = 6,
                       WS_FP4 = 7, WS_FE = 8, WS_ROUTE = 9, WS_AMAX = 10,
                       WS_MOECNT = 11, WS_GPART = 12, WS_GCNT = 13, WS_ATPART = 14, WS_ATCNT = 15, WS_ARGMAX = 16, WS_AMCNT = 17,
                       WS_COUNT = 18 };

// Same, but the buffer is zero-filled whenever it is (re)allocated (for
// counters that kernels keep at zero between calls).
int workspace_get_zeroed(int purpose, size_t bytes, cudaStream_t stream, void **out);

// Matvec implementation choice: 0 = by shape, 1 = dp4a kernel, 2 = tensor-core
// kernel.  Read once from FR_MATVEC (auto | dp4a | tc); fr_set_matvec_path
// overrides it.
int matvec_path();

} // namespace frb
