"""ctypes binding of libfrb200.so (the C-ABI in include/fr_b200.h).

PyTorch is used only for device memory and streams: every compute call goes
through the C entry points, and there is no fallback -- if the library is
missing or a call fails, a FrError is raised.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libfrb200.so")
INCLUDE = os.path.join(os.path.dirname(_PKG), "include", "fr_b200.h")

_lib = None


class FrError(RuntimeError):
    def __init__(self, fn: str, rc: int):
        msg = f"{fn} returned {rc}"
        try:
            msg += f" ({lib().fr_strerror(rc).decode()})"
        except Exception:  # noqa: BLE001 - best effort message
            pass
        super().__init__(msg)
        self.rc = rc


def build(jobs: int = 2) -> str:
    """Compile libfrb200.so in place (nvcc for sm_100a)."""
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", _PKG], check=True)
    return LIB_PATH


_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_f32 = C.c_float

SIGNATURES = {
    "fr_version": (_i32, []),
    "fr_strerror": (C.c_char_p, [_i32]),
    "fr_device_status": (_i32, [C.POINTER(C.c_uint32), _i32]),
    "fr_fault_inject": (_i32, [C.c_char_p]),
    "fr_set_wait_ns": (_i64, [_i64]),
    "fr_kernel_launches": (C.c_uint64, []),
    "fr_set_matvec_path": (_i32, [_i32]),
    "fr_nvfp4_row_bytes": (_i64, [_i64]),
    "fr_q8_1_row_bytes": (_i64, [_i64]),
    "fr_quantize_q8_1": (_i32, [_vp, _i64, _vp, _i64, _i32, _i32, _vp]),
    "fr_gemv_nvfp4_q8_1": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp]),
    "fr_gemv_nvfp4_f32": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp]),
    "fr_gemv_nvfp4_q8_1_swiglu": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp]),
    "fr_mul_mat_nvfp4": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp]),
    "fr_ffn_nvfp4": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "fr_ffn_nvfp4_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "fr_nvfp4_tiled_bytes": (_i64, [_i32, _i32]),
    "fr_nvfp4_tile": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp]),
    "fr_gemv_tiled": (_i32, [_vp, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i32, _vp]),
    "fr_gemv_tiled_swiglu": (_i32, [_vp, _vp, _i32, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i32, _vp]),
    "fr_ffn_tiled": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp]),
    "fr_mul_mat_id_tiled": (_i32, [_vp, _i32, _i32, _i32, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i32, _i32,
                                   _vp]),
    "fr_moe_ffn_tiled": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                C.c_float, _vp, _vp, _vp, _vp, _vp]),
    "fr_tp_buffer_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "fr_tp_wait": (_i32, [_vp, _i64, _i32, _i32, C.c_uint32, _vp]),
    "fr_tp_rows_buffer_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "fr_tp_ffn_rows": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                              _i64, _vp]),
    "fr_tp_ffn_nvfp4": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                               _i64, _vp]),
    "fr_tp_ffn_tiled": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                               _i64, _vp]),
    "fr_ep_buffer_bytes": (_i64, [_i32, _i32, _i32, _i32]),
    "fr_ep_moe_nvfp4": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                               _f32, _i32, _i32, _vp, _vp, _i64, _vp]),
    "fr_ep_moe_tiled": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                               _f32, _i32, _i32, _vp, _vp, _i64, _vp]),
    "fr_ipc_alloc": (_i32, [_i64, C.POINTER(C.c_void_p), _vp]),
    "fr_ipc_open": (_i32, [_vp, C.POINTER(C.c_void_p)]),
    "fr_ipc_close": (_i32, [_vp]),
    "fr_ipc_free": (_i32, [_vp]),
    "fr_moe_route": (_i32, [_vp, _i64, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "fr_mul_mat_id_nvfp4": (_i32, [_vp, _i64, _i64, _i32, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64,
                                   _i32, _i32, _i32, _i32, _vp]),
    "fr_moe_ffn_nvfp4": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                _i32, _f32, _vp, _vp, _vp, _vp, _vp]),
    "fr_moe_experts_nvfp4": (_i32, [_vp, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32,
                                    _i32, _vp]),
    "fr_moe_combine": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "fr_sf_bytes": (_i64, [_i64, _i64]),
    "fr_packed_bytes": (_i64, [_i64, _i64]),
    "fr_quantize_act_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "fr_repack_weight": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "fr_gemm_f32out": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _f32, C.c_bool, _vp]),
    "fr_gemm_swiglu_f32out": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _f32, _vp]),
    "fr_repack_weight_pair_interleaved": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _vp]),
    "fr_rmsnorm_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "fr_rope_kv_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp]),
    "fr_attn_decode_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    "fr_embed_nvfp4": (_i32, [_vp, _i32, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _vp]),
    "fr_argmax_f32": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "fr_pos_advance": (_i32, [_vp, _vp]),
    "fr_copy_pinned": (_i32, [_vp, _vp, _i64, _vp]),
    "fr_synth_nvfp4_device": (_i32, [C.c_uint64, _i64, _i64, C.c_double, _vp, _vp]),
    "fr_synth_nvfp4": (None, [C.c_uint64, _i64, _i64, C.c_double, _vp]),
    "fr_synth_normal": (None, [C.c_uint64, _i64, C.c_double, C.c_double, _vp]),
}


def lib():
    """Load libfrb200.so (building it first if it is absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name, None)
            if fn is None:      # reported by tests/test_abi.py
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def call(name: str, *args) -> int:
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise FrError(name, rc)
    return rc


# ------------------------------------------------------------ torch helpers

def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def row_bytes(K: int) -> int:
    return K // 64 * 36


def q8_row_bytes(K: int) -> int:
    return K // 32 * 36


def synth_nvfp4(seed: int, rows: int, K: int, scale_sigma: float = 0.05):
    """numpy uint8 [rows, K/64*36] of NVFP4 blocks (host)."""
    import numpy as np
    out = np.empty((rows, row_bytes(K)), np.uint8)
    lib().fr_synth_nvfp4(seed, rows, K, scale_sigma, out.ctypes.data)
    return out


def synth_normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0):
    import numpy as np
    out = np.empty(n, np.float32)
    lib().fr_synth_normal(seed, n, mean, std, out.ctypes.data)
    return out


def set_matvec_path(path: int) -> int:
    """0 = by shape, 1 = dp4a kernel, 2 = tensor-core kernel; returns the previous."""
    return int(lib().fr_set_matvec_path(path))


def device_status(clear: bool = True) -> int:
    v = C.c_uint32(0)
    call("fr_device_status", C.byref(v), 1 if clear else 0)
    return int(v.value)


def quantize_q8_1(x, out=None, stream=None):
    import torch
    T, K = x.shape
    if out is None:
        out = torch.empty((T, q8_row_bytes(K)), dtype=torch.uint8, device=x.device)
    call("fr_quantize_q8_1", _ptr(x), x.stride(0), _ptr(out), out.stride(0) // 36, T, K, _stream(stream))
    return out


def gemv_q8_1(w, q8, N, K, T, scale=None, resid=None, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=q8.device)
    ldr = resid.stride(0) if resid is not None else 0
    call("fr_gemv_nvfp4_q8_1", _ptr(w), w.stride(0), _ptr(q8), q8.stride(0) // 36, _ptr(scale), _ptr(resid),
         ldr, _ptr(out), out.stride(0), N, K, T, _stream(stream))
    return out


def gemv_f32(w, x, N, K, scale=None, resid=None, out=None, stream=None):
    import torch
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=x.device)
    ldr = resid.stride(0) if resid is not None else 0
    call("fr_gemv_nvfp4_f32", _ptr(w), w.stride(0), _ptr(x), x.stride(0), _ptr(scale), _ptr(resid), ldr,
         _ptr(out), out.stride(0), N, K, T, _stream(stream))
    return out


def gemv_swiglu(wg, wu, q8, N, K, T, sg=None, su=None, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=q8.device)
    call("fr_gemv_nvfp4_q8_1_swiglu", _ptr(wg), _ptr(wu), wg.stride(0), _ptr(q8), q8.stride(0) // 36, _ptr(sg),
         _ptr(su), _ptr(out), out.stride(0), N, K, T, _stream(stream))
    return out


def mul_mat(w, x, N, K, out=None, stream=None):
    import torch
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=x.device)
    call("fr_mul_mat_nvfp4", _ptr(w), w.stride(0), _ptr(x), x.stride(0), _ptr(out), out.stride(0), N, K, T,
         _stream(stream))
    return out


def ffn(x, wg, wu, wd, n_embd, n_ff, sg=None, su=None, sd=None, resid=None, out=None, chk_glu=None,
        chk_glu_q8=None, stream=None):
    import torch
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, n_embd), dtype=torch.float32, device=x.device)
    call("fr_ffn_nvfp4", _ptr(x), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su), _ptr(sd), _ptr(resid),
         _ptr(out), T, n_embd, n_ff, _ptr(chk_glu), _ptr(chk_glu_q8), _stream(stream))
    return out


def moe_route(x, w_r, n_used, clamp=6.103515625e-5, stream=None):
    import torch
    T, K = x.shape
    E = w_r.shape[0]
    dev = x.device
    logits = torch.empty((T, E), dtype=torch.float32, device=dev)
    ids = torch.empty((T, n_used), dtype=torch.int32, device=dev)
    wts = torch.empty((T, n_used), dtype=torch.float32, device=dev)
    eoff = torch.empty(E + 1, dtype=torch.int32, device=dev)
    slots = torch.empty(T * n_used, dtype=torch.int32, device=dev)
    act = torch.empty(E + 1, dtype=torch.int32, device=dev)
    call("fr_moe_route", _ptr(x), x.stride(0), _ptr(w_r), T, K, E, n_used, clamp, _ptr(logits), _ptr(ids),
         _ptr(wts), _ptr(eoff), _ptr(slots), _ptr(act), _stream(stream))
    return logits, ids, wts, eoff, slots, act


def mul_mat_id(w, E, N, K, x, ids, broadcast: bool, out=None, stream=None):
    """w: uint8 [E, N, K/64*36]; x: [T, K] (broadcast) or [T, n_used, K]; ids [T, n_used]."""
    import torch
    T, n_used = ids.shape
    if out is None:
        out = torch.empty((T, n_used, N), dtype=torch.float32, device=x.device)
    if broadcast:
        x_ld_slot, x_ld_tok = 0, x.stride(0)
    else:
        x_ld_slot, x_ld_tok = x.stride(1), x.stride(0)
    call("fr_mul_mat_id_nvfp4", _ptr(w), w.stride(1), w.stride(0), E, _ptr(x), x_ld_slot, x_ld_tok, _ptr(ids),
         ids.stride(0), _ptr(out), out.stride(1), out.stride(0), T, n_used, N, K, _stream(stream))
    return out


def tile_nvfp4(w, N, K, out=None, stream=None):
    """Repack a ggml block_nvfp4 matrix [N, K] (uint8 CUDA tensor, rows
    w.stride(0) bytes apart) into the tile-major layout (uint8 tensor)."""
    import torch
    nb = int(lib().fr_nvfp4_tiled_bytes(N, K))
    if nb < 0:
        raise ValueError(f"bad shape N={N} K={K}")
    if out is None:
        out = torch.empty(nb, dtype=torch.uint8, device=w.device)
    call("fr_nvfp4_tile", _ptr(w), w.stride(0), N, K, _ptr(out), _stream(stream))
    return out


def gemv_tiled(wt, N, K, x=None, q8=None, T=None, scale=None, resid=None, out=None, stream=None):
    """y = scale * W . x_q (+ resid) on tiled weights; x f32 [T, K] or q8 [T, K/32*36]."""
    import torch
    a = x if x is not None else q8
    T = a.shape[0] if T is None else T
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=a.device)
    call("fr_gemv_tiled", _ptr(wt), N, K, _ptr(x), x.stride(0) if x is not None else 0, _ptr(q8),
         q8.stride(0) // 36 if q8 is not None else 0, _ptr(scale), _ptr(resid),
         resid.stride(0) if resid is not None else 0, _ptr(out), out.stride(0), T, _stream(stream))
    return out


def gemv_tiled_swiglu(wg_t, wu_t, N, K, x=None, q8=None, T=None, sg=None, su=None, out=None, stream=None):
    import torch
    a = x if x is not None else q8
    T = a.shape[0] if T is None else T
    if out is None:
        out = torch.empty((T, N), dtype=torch.float32, device=a.device)
    call("fr_gemv_tiled_swiglu", _ptr(wg_t), _ptr(wu_t), N, K, _ptr(x), x.stride(0) if x is not None else 0,
         _ptr(q8), q8.stride(0) // 36 if q8 is not None else 0, _ptr(sg), _ptr(su), _ptr(out), out.stride(0), T,
         _stream(stream))
    return out


def ffn_tiled(x, wg_t, wu_t, wd_t, n_embd, n_ff, sg=None, su=None, sd=None, resid=None, out=None, chk_glu=None,
              stream=None):
    import torch
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, n_embd), dtype=torch.float32, device=x.device)
    call("fr_ffn_tiled", _ptr(x), _ptr(wg_t), _ptr(wu_t), _ptr(wd_t), _ptr(sg), _ptr(su), _ptr(sd), _ptr(resid),
         _ptr(out), T, n_embd, n_ff, _ptr(chk_glu), _stream(stream))
    return out


def moe_ffn(x, w_r, wg, wu, wd, n_embd, n_ff, E, n_used, sg=None, su=None, sd=None, resid=None, out=None,
            clamp=6.103515625e-5, check=False, stream=None):
    import torch
    T = x.shape[0]
    dev = x.device
    if out is None:
        out = torch.empty((T, n_embd), dtype=torch.float32, device=dev)
    chk = {}
    if check:
        chk["ids"] = torch.empty((T, n_used), dtype=torch.int32, device=dev)
        chk["wts"] = torch.empty((T, n_used), dtype=torch.float32, device=dev)
        chk["glu"] = torch.empty((T, n_used, n_ff), dtype=torch.float32, device=dev)
        chk["part"] = torch.empty((T, n_used, n_embd), dtype=torch.float32, device=dev)
    call("fr_moe_ffn_nvfp4", _ptr(x), _ptr(w_r), _ptr(wg), _ptr(wu), _ptr(wd), _ptr(sg), _ptr(su), _ptr(sd),
         _ptr(resid), _ptr(out), T, n_embd, n_ff, E, n_used, clamp, _ptr(chk.get("ids")), _ptr(chk.get("wts")),
         _ptr(chk.get("glu")), _ptr(chk.get("part")), _stream(stream))
    return (out, chk) if check else out


def tile_experts(w, E, N, K, out=None, stream=None):
    """Repack E stacked ggml block_nvfp4 experts [E, N, K] (uint8, experts
    N * w.stride(1) bytes apart, N % 128 == 0) into the tile-major layout."""
    rows = w.reshape(E * N, -1) if w.dim() == 3 else w
    return tile_nvfp4(rows, E * N, K, out=out, stream=stream)


def mul_mat_id_tiled(w_t, E, N, K, x, ids, broadcast: bool, out=None, stream=None):
    """mul_mat_id on tile_experts weights; x: [T, K] (broadcast) or [T, n_used, K]."""
    import torch
    T, n_used = ids.shape
    if out is None:
        out = torch.empty((T, n_used, N), dtype=torch.float32, device=x.device)
    if broadcast:
        x_ld_slot, x_ld_tok = 0, x.stride(0)
    else:
        x_ld_slot, x_ld_tok = x.stride(1), x.stride(0)
    call("fr_mul_mat_id_tiled", _ptr(w_t), E, N, K, _ptr(x), x_ld_slot, x_ld_tok, _ptr(ids), ids.stride(0),
         _ptr(out), out.stride(1), out.stride(0), T, n_used, _stream(stream))
    return out


def moe_ffn_tiled(x, w_r, wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used, sg=None, su=None, sd=None, resid=None,
                  out=None, clamp=6.103515625e-5, check=False, stream=None):
    """moe_ffn on tile_experts weights (FP4 tensor-core expert matvecs)."""
    import torch
    T = x.shape[0]
    dev = x.device
    if out is None:
        out = torch.empty((T, n_embd), dtype=torch.float32, device=dev)
    chk = {}
    if check:
        chk["ids"] = torch.empty((T, n_used), dtype=torch.int32, device=dev)
        chk["wts"] = torch.empty((T, n_used), dtype=torch.float32, device=dev)
        chk["glu"] = torch.empty((T, n_used, n_ff), dtype=torch.float32, device=dev)
        chk["part"] = torch.empty((T, n_used, n_embd), dtype=torch.float32, device=dev)
    call("fr_moe_ffn_tiled", _ptr(x), _ptr(w_r), _ptr(wg_t), _ptr(wu_t), _ptr(wd_t), _ptr(sg), _ptr(su), _ptr(sd),
         _ptr(resid), _ptr(out), T, n_embd, n_ff, E, n_used, clamp, _ptr(chk.get("ids")), _ptr(chk.get("wts")),
         _ptr(chk.get("glu")), _ptr(chk.get("part")), _stream(stream))
    return (out, chk) if check else out


def moe_experts(x, eid, wg, wu, wd, n_embd, n_ff, E, sg=None, su=None, sd=None, out=None, stream=None):
    """Expert FFN over pre-routed rows: x [S, n_embd] f32, eid [S] int32."""
    import torch
    S = x.shape[0]
    if out is None:
        out = torch.empty((S, n_embd), dtype=torch.float32, device=x.device)
    call("fr_moe_experts_nvfp4", _ptr(x), x.stride(0) if S else n_embd, _ptr(eid), S, _ptr(wg), _ptr(wu), _ptr(wd),
         _ptr(sg), _ptr(su), _ptr(sd), _ptr(out), out.stride(0) if S else n_embd, n_embd, n_ff, E, _stream(stream))
    return out


def moe_combine(part, wts, n_embd, resid=None, out=None, stream=None):
    """part [T*n_used, n_embd], wts [T, n_used] -> out [T, n_embd]."""
    import torch
    T, n_used = wts.shape
    if out is None:
        out = torch.empty((T, n_embd), dtype=torch.float32, device=part.device)
    call("fr_moe_combine", _ptr(part), _ptr(wts), _ptr(resid), _ptr(out), T, n_used, n_embd, _stream(stream))
    return out


def copy_pinned(dst, src, stream=None):
    """dst <- src (same byte size; device memory and/or page-locked host
    memory) by SM loads and stores inside the stream's PDL chain."""
    n = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() != n:
        raise ValueError("copy_pinned: sizes differ")
    call("fr_copy_pinned", _ptr(dst), _ptr(src), n, _stream(stream))
    return dst


def sf_bytes(rows: int, K: int) -> int:
    return int(lib().fr_sf_bytes(rows, K))


def quantize_act_f32(x, stream=None):
    import torch
    M, K = x.shape
    packed = torch.empty((M, K // 2), dtype=torch.uint8, device=x.device)
    sf = torch.zeros(sf_bytes(M, K), dtype=torch.uint8, device=x.device)
    call("fr_quantize_act_f32", _ptr(x), _ptr(packed), _ptr(sf), M, K, _stream(stream))
    return packed, sf


def repack_weight(blocks, N, K, stream=None):
    import torch
    packed = torch.empty((N, K // 2), dtype=torch.uint8, device=blocks.device)
    sf = torch.zeros(sf_bytes(N, K), dtype=torch.uint8, device=blocks.device)
    call("fr_repack_weight", _ptr(blocks), _ptr(packed), _ptr(sf), N, K, _stream(stream))
    return packed, sf


def gemm_f32out(A, SFA, B, SFB, M, N, K, alpha=1.0, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    call("fr_gemm_f32out", _ptr(A), _ptr(SFA), _ptr(B), _ptr(SFB), _ptr(out), M, N, K, alpha, False,
         _stream(stream))
    return out


def repack_weight_pair_interleaved(gate_blocks, up_blocks, n_ff, K, stream=None):
    import torch
    packed = torch.empty((2 * n_ff, K // 2), dtype=torch.uint8, device=gate_blocks.device)
    sf = torch.zeros(sf_bytes(2 * n_ff, K), dtype=torch.uint8, device=gate_blocks.device)
    call("fr_repack_weight_pair_interleaved", _ptr(gate_blocks), _ptr(up_blocks), _ptr(packed), _ptr(sf), n_ff, K,
         _stream(stream))
    return packed, sf


def gemm_swiglu_f32out(A, SFA, B_pair, SFB_pair, M, n_ff, K, alpha=1.0, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty((M, n_ff), dtype=torch.float32, device=A.device)
    call("fr_gemm_swiglu_f32out", _ptr(A), _ptr(SFA), _ptr(B_pair), _ptr(SFB_pair), _ptr(out), M, n_ff, K, alpha,
         _stream(stream))
    return out
