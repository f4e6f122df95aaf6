"""The tile-major NVFP4 layout's CPU restatement (oracle.tile_nvfp4) against
an element-by-element reading of its definition, and the C-ABI's size rule."""
import numpy as np
import pytest


@pytest.mark.parametrize("N,K", [(130, 512), (64, 320), (1, 64)])
def test_tile_oracle_matches_definition(O, fr, N, K):
    w = fr.synth_nvfp4(5 + N, N, K)
    w.reshape(N, K // 64, 36)[0, 0, 0] = 0x7F         # ggml reads 0x7F as zero
    w.reshape(N, K // 64, 36)[N - 1, 0, 1] |= 0x80    # and ignores the sign bit
    t = O.tile_nvfp4(w, N, K)
    n_kq, n_rb = (K + 255) // 256, (N + 127) // 128
    assert t.size == n_rb * n_kq * 18432
    seen = np.zeros(t.size, bool)
    for row in range(n_rb * 128):
        for kb in range(n_kq * 4):
            blk = w[row, kb * 36:(kb + 1) * 36] if row < N and kb < K // 64 else np.zeros(36, np.uint8)
            rb, r, kq, j = row >> 7, row & 127, kb >> 2, kb & 3
            base = (rb * n_kq + kq) * 18432
            for h in range(2):
                c = 2 * j + h
                o = base + r * 128 + ((c ^ (r & 7)) << 4)
                np.testing.assert_array_equal(t[o:o + 16], blk[4 + 16 * h:20 + 16 * h])
                seen[o:o + 16] = True
            for sb in range(4):
                v = int(blk[sb]) & 0x7F
                o = base + 16384 + j * 512 + (r & 31) * 16 + (r >> 5) * 4 + sb
                assert t[o] == (0 if v == 0x7F else v)
                seen[o] = True
    assert seen.all()


def test_tiled_bytes_rule(fr):
    L = fr.lib()
    assert L.fr_nvfp4_tiled_bytes(14336, 4096) == 14336 * 4096 // 64 * 36
    assert L.fr_nvfp4_tiled_bytes(130, 320) == 2 * 2 * 18432
    assert L.fr_nvfp4_tiled_bytes(1, 100) == -1
