// fr_synth.cpp -- deterministic synthetic inputs for tests and benchmarks
// (host side, no CUDA).  The benchmark configurations specify:
//   weights: E2M1 codes uniform over all 16 values, one e4m3 scale per 16
//            values drawn as |N(0,1)| * 0.05 and rounded to e4m3 (RNE);
//   activations / router weights: N(mean, std) f32.
// RNG: splitmix64, Box-Muller in double.  Rows (weights) and 64 Ki-element
// chunks (normals) get independent streams, so the output does not depend on
// the thread count.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/fr_b200.h"

namespace {

inline uint64_t splitmix64(uint64_t &s) {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// two N(0,1) draws
inline void box_muller(uint64_t &s, double &z0, double &z1) {
    const double u1 = (static_cast<double>(splitmix64(s) >> 11) + 1.0) * 0x1.0p-53;   // (0, 1]
    const double u2 = static_cast<double>(splitmix64(s) >> 11) * 0x1.0p-53;           // [0, 1)
    const double r = std::sqrt(-2.0 * std::log(u1));
    z0 = r * std::cos(6.283185307179586 * u2);
    z1 = r * std::sin(6.283185307179586 * u2);
}

// non-negative float -> e4m3 code, round to nearest even, saturating at 448
uint8_t e4m3_rne_pos(float f) {
    if (!(f > 0.0f)) return 0;
    if (f >= 448.0f) return 0x7E;
    uint32_t a;
    std::memcpy(&a, &f, 4);
    const uint32_t e = a >> 23;
    if (e < 121) {
        if (e < 117) return 0;
        const uint32_t m = (a & 0x7fffffu) | 0x800000u, sh = 141 - e;
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return static_cast<uint8_t>(q);
    }
    const uint32_t m = a & 0x7fffffu;
    uint32_t q = ((e - 120) << 3) | (m >> 20);
    const uint32_t rem = m & 0xfffffu;
    if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) q++;
    return static_cast<uint8_t>(q > 0x7E ? 0x7E : q);
}

template <typename F>
void parallel_for(int64_t n, F &&f) {
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 32) nt = 32;
    if (n < 64 || nt == 1) {
        for (int64_t i = 0; i < n; ++i) f(i);
        return;
    }
    std::vector<std::thread> th;
    for (unsigned k = 0; k < nt; ++k)
        th.emplace_back([&, k]() {
            for (int64_t i = k; i < n; i += nt) f(i);
        });
    for (auto &t : th) t.join();
}

} // namespace

extern "C" {

void fr_synth_nvfp4(uint64_t seed, int64_t rows, int64_t K, double scale_sigma, void *out_blocks) {
    uint8_t *out = static_cast<uint8_t *>(out_blocks);
    const int64_t nb = K / 64;
    parallel_for(rows, [&](int64_t r) {
        uint64_t s = seed * 0x100000001B3ull + static_cast<uint64_t>(r) * 0xD1B54A32D192ED03ull;
        uint8_t *row = out + r * nb * 36;
        for (int64_t b = 0; b < nb; ++b) {
            uint8_t *blk = row + b * 36;
            double z[4];
            box_muller(s, z[0], z[1]);
            box_muller(s, z[2], z[3]);
            for (int i = 0; i < 4; ++i) blk[i] = e4m3_rne_pos(static_cast<float>(std::fabs(z[i]) * scale_sigma));
            for (int w = 0; w < 4; ++w) {
                const uint64_t v = splitmix64(s);
                std::memcpy(blk + 4 + 8 * w, &v, 8);
            }
        }
    });
}

void fr_synth_normal(uint64_t seed, int64_t n, double mean, double stddev, float *out) {
    const int64_t CH = 1 << 16;
    const int64_t nch = (n + CH - 1) / CH;
    parallel_for(nch, [&](int64_t c) {
        uint64_t s = seed * 0x100000001B3ull + static_cast<uint64_t>(c) * 0xD1B54A32D192ED03ull + 0x5EEDull;
        const int64_t lo = c * CH, hi = std::min<int64_t>(n, lo + CH);
        for (int64_t i = lo; i < hi; i += 2) {
            double z0, z1;
            box_muller(s, z0, z1);
            out[i] = static_cast<float>(mean + stddev * z0);
            if (i + 1 < hi) out[i + 1] = static_cast<float>(mean + stddev * z1);
        }
    });
}

} // extern "C"
