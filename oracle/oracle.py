"""ctypes view of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py as the checker.  The product never imports it.
Every function here forwards to oracle/fr_oracle.c, which cites the reference
lines it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile liboracle.so in place (make), return its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "or_f32_to_f16": (C.c_uint16, [C.c_float]),
            "or_f16_to_f32": (C.c_float, [C.c_uint16]),
            "or_ue4m3_half": (C.c_float, [C.c_uint8]),
            "or_e4m3_to_f32": (C.c_float, [C.c_uint8]),
            "or_f32_to_e4m3_satfinite": (C.c_uint8, [C.c_float]),
            "or_f32_to_e2m1_act": (C.c_uint8, [C.c_float]),
            "or_nvfp4_dequant": (None, [_u8p, C.c_int64, _f32p]),
            "or_quantize_q8_1": (None, [_f32p, C.c_int64, C.c_int, C.c_int, _u8p]),
            "or_quantize_q8_ggml_cpu": (None, [_f32p, C.c_int64, _i8p, _u16p]),
            "or_gemv_q8_1": (None, [_u8p, C.c_int64, _u8p, C.c_int64, C.c_float, C.c_int, C.c_int,
                                    C.c_int, _f64p, C.c_int64, C.c_int]),
            "or_gemv_q8_1_f32": (None, [_u8p, C.c_int64, _u8p, C.c_int64, C.c_float, C.c_int, C.c_int,
                                        C.c_int, _f32p, C.c_int64, C.c_int]),
            "or_silu": (C.c_float, [C.c_float]),
            "or_topk_softmax": (None, [_f32p, C.c_int, C.c_int, C.c_int, C.c_float, _i32p, _f32p]),
            "or_router_logits": (None, [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f64p]),
            "or_group_by_expert": (None, [_i32p, C.c_int, C.c_int, C.c_int, _i32p, _i32p, _i32p]),
            "or_sf_offset": (C.c_int64, [C.c_int64, C.c_int64, C.c_int64]),
            "or_sf_bytes": (C.c_int64, [C.c_int64, C.c_int64]),
            "or_quantize_act_f32": (None, [_f32p, C.c_int, C.c_int, _u8p, _u8p]),
            "or_repack_weight": (None, [_u8p, C.c_int, C.c_int, _u8p, _u8p]),
            "or_gemm_f32out": (None, [_u8p, _u8p, _u8p, _u8p, _f64p, C.c_int, C.c_int, C.c_int,
                                      C.c_float, C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


# ---------------------------------------------------------------- helpers

def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def nvfp4_dequant(blocks: np.ndarray) -> np.ndarray:
    b = _c(blocks, np.uint8).reshape(-1)
    nb = b.size // 36
    out = np.empty(nb * 64, np.float32)
    lib().or_nvfp4_dequant(b, nb, out)
    return out


def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """x [T, K] f32 -> uint8 [T, K/32*36] q8_1 blocks."""
    x = _c(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    T, K = x.shape
    out = np.empty((T, K // 32 * 36), np.uint8)
    lib().or_quantize_q8_1(x, K, T, K, out)
    return out


def quantize_q8_ggml_cpu(x: np.ndarray):
    x = _c(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 32, np.uint16)
    lib().or_quantize_q8_ggml_cpu(x, x.size, q, d)
    return q, d


def gemv_q8_1(w: np.ndarray, q8: np.ndarray, N: int, K: int, scale: float = 1.0,
              nthreads: int = 0) -> np.ndarray:
    """w uint8 [N, K/64*36], q8 uint8 [T, K/32*36] -> y f64 [T, N]."""
    w = _c(w, np.uint8)
    q8 = _c(q8, np.uint8)
    if q8.ndim == 1:
        q8 = q8[None]
    T = q8.shape[0]
    y = np.empty((T, N), np.float64)
    lib().or_gemv_q8_1(w.reshape(-1), K // 64 * 36, q8.reshape(-1), K // 32, scale, N, K, T,
                       y, N, nthreads)
    return y


def gemv_q8_1_f32(w, q8, N, K, scale=1.0, nthreads=0):
    w = _c(w, np.uint8)
    q8 = _c(q8, np.uint8)
    if q8.ndim == 1:
        q8 = q8[None]
    T = q8.shape[0]
    y = np.empty((T, N), np.float32)
    lib().or_gemv_q8_1_f32(w.reshape(-1), K // 64 * 36, q8.reshape(-1), K // 32, scale, N, K, T,
                           y, N, nthreads)
    return y


def silu(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    return np.array([lib().or_silu(float(v)) for v in x.reshape(-1)], np.float32).reshape(x.shape)


def silu_np(x: np.ndarray) -> np.ndarray:
    """Vectorised x / (1 + exp(-x)) in float32 (the same formula as or_silu)."""
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def router_logits(x, wr):
    x = _c(x, np.float32)
    wr = _c(wr, np.float32)
    T, K = x.shape
    E = wr.shape[0]
    out = np.empty((T, E), np.float64)
    lib().or_router_logits(x, wr, T, K, E, out)
    return out


def topk_softmax(logits, n_used, clamp=6.103515625e-5):
    logits = _c(logits, np.float32)
    T, E = logits.shape
    ids = np.empty((T, n_used), np.int32)
    w = np.empty((T, n_used), np.float32)
    lib().or_topk_softmax(logits, T, E, n_used, clamp, ids, w)
    return ids, w


def group_by_expert(ids, E):
    ids = _c(ids, np.int32)
    T, n_used = ids.shape
    eoff = np.empty(E + 1, np.int32)
    slots = np.empty(T * n_used, np.int32)
    act = np.empty(E + 1, np.int32)
    lib().or_group_by_expert(ids, T, n_used, E, eoff, slots, act)
    return eoff, slots, act


def sf_bytes(rows, K):
    return int(lib().or_sf_bytes(rows, K))


def sf_offset(row, k, K):
    return int(lib().or_sf_offset(row, k, K))


def quantize_act_f32(x):
    x = _c(x, np.float32)
    M, K = x.shape
    packed = np.zeros((M, K // 2), np.uint8)
    sf = np.zeros(sf_bytes(M, K), np.uint8)
    lib().or_quantize_act_f32(x, M, K, packed, sf)
    return packed, sf


def repack_weight(blocks, N, K):
    b = _c(blocks, np.uint8).reshape(-1)
    packed = np.zeros((N, K // 2), np.uint8)
    sf = np.zeros(sf_bytes(N, K), np.uint8)
    lib().or_repack_weight(b, N, K, packed, sf)
    return packed, sf


def gemm_f32out(A, SFA, B, SFB, M, N, K, alpha=1.0, nthreads=0):
    D = np.empty((M, N), np.float64)
    lib().or_gemm_f32out(_c(A, np.uint8).reshape(-1), _c(SFA, np.uint8), _c(B, np.uint8).reshape(-1),
                         _c(SFB, np.uint8), D, M, N, K, alpha, nthreads)
    return D


# ------------------------------------------------------------ comparisons

def tile_nvfp4(blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    """Tile-major NVFP4 layout (the library's fr_nvfp4_tile, test
    restatement): tiles of 128 rows x 256 values, tile (rb, kq) at
    (rb * n_kq + kq) * 18432; 16 KB of code bytes with row r's 16-byte unit c
    (block c >> 1, half c & 1 of its 32 code bytes, ggml byte order) at
    r * 128 + ((c ^ (r & 7)) << 4); then per block j a 512-byte scale atom with
    row r's sub-block scales at (r & 31) * 16 + (r >> 5) * 4, sign bit
    dropped and 0x7F read as 0 (ggml's ue4m3 reading, ggml-common.h).
    Padding rows / blocks are zero."""
    n_kq, n_rb = (K + 255) // 256, (N + 127) // 128
    b = np.zeros((n_rb * 128, n_kq * 4, 36), np.uint8)
    b[:N, :K // 64] = np.asarray(blocks, np.uint8).reshape(N, K // 64, 36)
    sc = b[:, :, :4] & 0x7F
    sc[sc == 0x7F] = 0
    codes = b[:, :, 4:].reshape(n_rb, 128, n_kq, 8, 16)           # rb, r, kq, c, 16
    out = np.zeros((n_rb, n_kq, 18432), np.uint8)
    r = np.arange(128)
    tiles_codes = np.zeros((n_rb, n_kq, 128, 8, 16), np.uint8)
    for c in range(8):
        phys = c ^ (r & 7)
        tiles_codes[:, :, r, phys, :] = codes[:, :, :, c, :].transpose(0, 2, 1, 3)[:, :, r, :]
    out[:, :, :16384] = tiles_codes.reshape(n_rb, n_kq, 16384)
    scs = sc.reshape(n_rb, 128, n_kq, 4, 4)                         # rb, r, kq, j, sb
    atoms = np.zeros((n_rb, n_kq, 4, 32, 4, 4), np.uint8)            # rb, kq, j, r & 31, r >> 5, sb
    atoms[:, :, :, r & 31, r >> 5, :] = scs.transpose(0, 2, 3, 1, 4)[:, :, :, r, :]
    out[:, :, 16384:] = atoms.reshape(n_rb, n_kq, 2048)
    return out.reshape(-1)


def rel_err(mine: np.ndarray, ref: np.ndarray, floor_frac: float = 1e-2) -> float:
    """max |mine - ref| / max(|ref|, floor_frac * rms(ref)): the relative error,
    with outputs smaller than 1% of the rms judged against 1% of the rms (a
    relative error of a value near zero measures cancellation, not the kernel)."""
    mine = np.asarray(mine, np.float64)
    ref = np.asarray(ref, np.float64)
    if not np.all(np.isfinite(mine)):
        return float("inf")
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    den = np.maximum(np.abs(ref), floor_frac * rms + 1e-30)
    return float(np.max(np.abs(mine - ref) / den)) if ref.size else 0.0


def norm_err(mine, ref) -> float:
    """||mine - ref||_2 / ||ref||_2."""
    mine = np.asarray(mine, np.float64)
    ref = np.asarray(ref, np.float64)
    den = float(np.linalg.norm(ref))
    return float(np.linalg.norm(mine - ref)) / den if den > 0 else float(np.linalg.norm(mine))


def ref_gate_bad(mine, ref, atol=1e-4, rtol=2e-3) -> int:
    """The reference's conjunctive gate (src/fr_win_flint_batched.cuh:478-489):
    bad iff abs > atol and rel > rtol, and any non-finite value is bad.  The
    reference applies it to unit-scale activations; outputs whose rms exceeds
    1 are judged in units of their rms (atol scaled by it), since a float32
    sum of outputs of magnitude ~1e3 cannot resolve 1e-4 absolutely."""
    mine = np.asarray(mine, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size:
        atol = atol * max(1.0, float(np.sqrt(np.mean(ref * ref))))
    d = np.abs(mine - ref)
    rel = d / (np.abs(ref) + 1e-6)
    bad = (d > atol) & (rel > rtol)
    bad |= ~np.isfinite(mine)
    return int(bad.sum())


# ---------------------------------------------------------------- the reference's own W4A4 build

_REF_PATH = os.path.join(_HERE, "_ref", "libfrref.so")
_ref = None


def ref_lib():
    """The reference's Thor W4A4 launch interface (src/fr_quant_act.cu,
    src/fr_repack.cu, src/fr_gemm_f32out.cu compiled unmodified for sm_100a by
    oracle/ref.mk, C linkage from oracle/ref_shim.cu), or None when that build
    is absent (it needs the reference sources, which only the build machine
    has).  GPU code: the pins in tests/ and bench.py's comparison leg call it
    on device pointers."""
    global _ref
    if _ref is None and os.path.exists(_REF_PATH):
        L = C.CDLL(_REF_PATH)
        vp = C.c_void_p
        L.frref_quantize_act_f32.restype = C.c_int
        L.frref_quantize_act_f32.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp]
        L.frref_repack_weight.restype = C.c_int
        L.frref_repack_weight.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp]
        L.frref_gemm_f32out.restype = C.c_int
        L.frref_gemm_f32out.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, vp]
        L.frref_sf_bytes.restype = C.c_longlong
        L.frref_sf_bytes.argtypes = [C.c_longlong, C.c_longlong]
        _ref = L
    return _ref


# ---------------------------------------------------------------- decode-step restatements (numpy, fp64)

def rmsnorm(x, w=None, eps=1e-6):
    """RMSNorm as the reference's host check states it (src/fr_win_flint_batched.cuh:468-474):
    sum of squares in double, scale = 1/sqrt(mean + eps)."""
    x = np.asarray(x, np.float64)
    scale = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    y = x * scale
    return y if w is None else y * np.asarray(w, np.float64)


def rope_neox(x, pos, base=1e6):
    """NeoX RoPE of heads x [..., d] at position pos: pairs (i, i + d/2),
    theta_i = pos * base^(-2i/d) (src/fr_qkv_post.cu:71-131), in fp64."""
    x = np.asarray(x, np.float64)
    d = x.shape[-1]
    i = np.arange(d // 2, dtype=np.float64)
    th = pos * base ** (-2.0 * i / d)
    c, s = np.cos(th), np.sin(th)
    a, b = x[..., : d // 2], x[..., d // 2:]
    return np.concatenate([a * c - b * s, a * s + b * c], -1)


def attention_decode(q, k, v):
    """Softmax attention of one token's query heads q [nh, d] (already scaled)
    over keys k, v [nkv, n, d] (GQA: head h reads KV head h // (nh / nkv)),
    fp64: the decode attention the reference's frt_fa_decode / frt_fa_combine
    compute (src/fr_win_flint_sm120.cu:2411-2846)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    nh, nkv = q.shape[0], k.shape[0]
    out = np.empty_like(q)
    for h in range(nh):
        g = h // (nh // nkv)
        s = k[g] @ q[h]
        p = np.exp(s - s.max())
        out[h] = (p @ v[g]) / p.sum()
    return out


def nvfp4_rows(blocks, rows):
    """Dequantized rows of an NVFP4 matrix (ggml values), f32 [len(rows), K]."""
    b = np.asarray(blocks, np.uint8)
    return np.stack([nvfp4_dequant(b[r]) for r in rows])
