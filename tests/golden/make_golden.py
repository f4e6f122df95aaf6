"""Generate the golden fixtures that pin the CPU oracle.

Run once in a container that has gguf-py (0.19.0, ggml's Python restatement
of its reference CPU quantizers) and torch:

    python tests/golden/make_golden.py

Outputs (committed, small):
  nvfp4_decode.npz  random block_nvfp4 bytes and gguf's NVFP4.dequantize_blocks
                    output, plus gguf's ue4m3 decode of every byte.
  q8_0_ggml.npz     f32 rows and gguf's Q8_0.quantize_blocks (ggml-quants.c's
                    quantize_row_q8_0_ref: d = amax/127, q = roundf(x * 1/d)),
                    the CPU form the reference's q8 checks compare against.
  e4m3_encode.npz   f32 values and torch.float8_e4m3fn's RNE encoding (values
                    inside the finite range, where it matches satfinite).
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    import gguf.quants as gq
    import torch

    rng = np.random.default_rng(0x5EED0001)

    # ---- NVFP4 decode: 256 blocks of random bytes; scale bytes avoid 0xFF,
    # the one code where gguf-py (decodes it as 240) and the reference
    # (src/fr_win_flint_batched.cuh:442-447: 0xFF -> 0) differ.
    blocks = rng.integers(0, 256, size=(256, 36), dtype=np.uint8)
    sc = blocks[:, :4]
    sc[sc == 0xFF] = 0x7F
    deq = gq.NVFP4.dequantize_blocks(blocks.copy())
    codes = np.arange(256, dtype=np.uint8)
    ue4m3 = gq.NVFP4.ue4m3_to_fp32(codes).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "nvfp4_decode.npz"), blocks=blocks,
                        deq=deq.astype(np.float32), ue4m3_half=ue4m3)

    # ---- q8_0 CPU quantizer (int8 values and the f16 scale)
    x = rng.standard_normal((64, 32)).astype(np.float32)
    x[3] = 0.0                                     # all-zero chunk
    x[5] *= 1e-30                                  # tiny values
    x[7, :] = np.linspace(-2.5, 2.5, 32, dtype=np.float32)
    q = gq.Q8_0.quantize_blocks(x.copy())
    d = q[:, :2].copy().view(np.float16).reshape(-1)
    qs = q[:, 2:].copy().view(np.int8)
    np.savez_compressed(os.path.join(HERE, "q8_0_ggml.npz"), x=x, d=d, qs=qs)

    # ---- e4m3 RNE encoder
    v = np.concatenate([
        rng.standard_normal(4096).astype(np.float32) * 0.05,
        rng.standard_normal(4096).astype(np.float32) * 30.0,
        np.array([0.0, -0.0, 2.0 ** -9, 2.0 ** -10, 1.5 * 2.0 ** -10, 448.0, -448.0, 440.0,
                  0.0068359375, 0.001953125, 240.0, 0.0625 * 1.0625], np.float32),
    ])
    v = v[np.abs(v) <= 448.0]
    enc = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.savez_compressed(os.path.join(HERE, "e4m3_encode.npz"), x=v, code=enc)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
