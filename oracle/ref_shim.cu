// ref_shim.cu -- C linkage for the reference's own Thor W4A4 launch interface
// (include/fr_kernels.h:25-57 of the reference, namespace ggml_cuda_flashrt),
// so that the tests and the benchmark's comparison leg can call the
// reference's compiled kernels through ctypes.  TEST INFRASTRUCTURE ONLY: it is
// built into oracle/_ref/libfrref.so together with the reference's unmodified
// src/fr_quant_act.cu, src/fr_repack.cu and src/fr_gemm_f32out.cu (compiled
// where they lie) by oracle/ref.mk, and nothing in the product links it.
#include "fr_kernels.h"

extern "C" {

int frref_quantize_act_f32(const float *src, void *dst_packed, void *dst_sfa, int M, int K, cudaStream_t s) {
    return ggml_cuda_flashrt::quantize_act_f32(src, dst_packed, dst_sfa, M, K, s);
}

int frref_repack_weight(const void *blocks, void *dst_packed, void *dst_sf, int N, int K, cudaStream_t s) {
    return ggml_cuda_flashrt::repack_weight(blocks, dst_packed, dst_sf, N, K, s);
}

int frref_gemm_f32out(const void *A, const void *SFA, const void *B, const void *SFB, float *D, int M, int N, int K,
                      float alpha, int widen, cudaStream_t s) {
    return ggml_cuda_flashrt::gemm_f32out(A, SFA, B, SFB, D, M, N, K, alpha, widen != 0, s);
}

int frref_repack_weight_pair_interleaved(const void *gate, const void *up, void *dst_packed, void *dst_sf, int n_ff,
                                         int K, cudaStream_t s) {
    return ggml_cuda_flashrt::repack_weight_pair_interleaved(gate, up, dst_packed, dst_sf, n_ff, K, s);
}

long long frref_sf_bytes(long long rows, long long K) { return ggml_cuda_flashrt::sf_bytes(rows, K); }

} // extern "C"
