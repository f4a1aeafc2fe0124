// qrc_gen.cuh -- seeded, counter-based synthetic inputs, identical on host and
// device.
//
// Element i of a stream is a pure function of (seed, i): splitmix64 (Steele,
// Lea & Flood, OOPSLA 2014) of a per-seed key plus a Weyl step of the counter.
// Only integer arithmetic, one IEEE int->float round-to-nearest conversion and
// exact power-of-two scales are used, so host and device produce the same bits
// and shards of one stream can be generated on different GPUs independently.
//   uniform[-1,1):  x = (m - 2^23) * 2^-23, m the top 24 bits of the hash.
//   normal(0,1):    Irwin-Hall sum of twelve 24-bit uniforms, centred,
//                   converted once to float, scaled by 2^-24 (variance 1).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define QRC_HD __host__ __device__ __forceinline__
#else
#define QRC_HD inline
#endif

namespace qrc_gen {

QRC_HD uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

QRC_HD uint64_t key_of(uint64_t seed) { return mix64(seed + 0x9E3779B97F4A7C15ull); }

// Draw k (0..15) of element i.
QRC_HD uint64_t draw(uint64_t key, uint64_t i, unsigned k) {
    return mix64(key + (i * 16u + k + 1u) * 0x9E3779B97F4A7C15ull);
}

QRC_HD float i64_to_f32_rn(int64_t v) {
#if defined(__CUDA_ARCH__)
    return __ll2float_rn((long long)v);
#else
    return (float)v;   // x86-64 cvtsi2ss: round to nearest even
#endif
}

QRC_HD float uniform_pm1(uint64_t key, uint64_t i) {
    const int32_t m = (int32_t)(draw(key, i, 0) >> 40);
    return (float)(m - (1 << 23)) * (1.0f / 8388608.0f);
}

QRC_HD float normal01(uint64_t key, uint64_t i) {
    int64_t s = 0;
    for (unsigned k = 0; k < 12; k++) s += (int64_t)(draw(key, i, k) >> 40);
    s -= (int64_t)6 << 24;
    return i64_to_f32_rn(s) * (1.0f / 16777216.0f);
}

// IEEE binary32 -> bfloat16, round to nearest even (NaN -> quiet NaN).
QRC_HD uint16_t f32_to_bf16_rn(float x) {
    uint32_t b;
#if defined(__CUDA_ARCH__)
    b = __float_as_uint(x);
#else
    __builtin_memcpy(&b, &x, 4);
#endif
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((b >> 16) & 0x8000u) | 0x7FC0u);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

// Seeded outlier position and sign for the synthetic workloads.
QRC_HD uint64_t outlier_index(uint64_t seed, uint64_t n) {
    return n ? draw(key_of(seed ^ 0x0D7C0FFEEull), 0, 0) % n : 0;
}
QRC_HD int outlier_sign(uint64_t seed) {
    return (draw(key_of(seed ^ 0x0D7C0FFEEull), 0, 1) >> 63) ? -1 : 1;
}

}  // namespace qrc_gen
