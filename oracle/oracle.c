/*
 * oracle.c -- CPU oracle for the side-aware FP32 absmax path and the fused
 * amax -> FP8 e4m3 quantize.
 *
 * THIS IS TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only the test suite, the
 * smoke check and the CPU-baseline leg of the benchmark load this library,
 * and only as the checker (or as the timed CPU baseline).  The product path
 * (the CUDA kernels behind include/qrc_b200.h) never calls into it.
 *
 * What it restates, and where the reference defines it:
 *   - absmax:  the reduction operator of QuickRunCUDA tests/side_aware.cu:216-219
 *              (`reduction_oob = 0.0f`, `fmaxf(a, fabsf(b))`), applied over every
 *              element of A exactly once (side_aware.cu:294-361), with the NaN
 *              behaviour of CUDA's fmaxf: any NaN input (quiet or signalling)
 *              never wins; -0.0 becomes +0.0; an empty or all-NaN input gives
 *              +0.0; denormals are kept (the oracle does not flush).
 *   - the chunk-side selection of side_aware.cu:299-318 (parity of the masked
 *     address bits XOR the per-2MiB-page bit picks which 4 KiB half of each
 *     8 KiB pair a side reads), restated in oracle_pair_half() so host tests can
 *     check that any side map still covers every byte exactly once.
 *   - the reference harness' `-r` fill (QuickRunCUDA.cpp:432-457) is a C++
 *     std::mt19937_64 stream and lives in oracle_mt.cpp next to this file.
 *   - e4m3: no reference code exists (the quantize is new); the encoder follows
 *     the OCP 8-bit floating point specification (OFP8, E4M3: bias 7, no
 *     infinities, S.1111.111 is NaN, max finite 448) with round-to-nearest-even
 *     and saturation to +-448, i.e. the semantics of `cvt.rn.satfinite.e4m3x2`.
 *
 * Synthetic data generators (seeded, counter based, bit-identical on host and
 * device because they use only integer arithmetic and one IEEE int->float
 * conversion): splitmix64 (Steele, Lea & Flood, "Fast splittable pseudorandom
 * number generators", OOPSLA 2014) keyed by (seed, element index).
 *   uniform[-1,1):  24 high bits m of the hash, x = (m - 2^23) * 2^-23.
 *   normal(0,1):    Irwin-Hall sum of twelve 24-bit uniforms, centred, then
 *                   one int64 -> float round-to-nearest conversion and an exact
 *                   power-of-two scale (variance 1).
 * The product has its own implementation of the same published algorithms;
 * the tests check the two agree bit for bit.
 *
 * Built with -O2 -fopenmp -ffp-contract=off and WITHOUT -ffast-math so that
 * fmaxf/fabsf, float multiply/divide and int->float conversion are IEEE.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <omp.h>

#define ORACLE_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* splitmix64 and the counter-based streams                                  */
/* ------------------------------------------------------------------------- */

static inline uint64_t sm64_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Stream key for a seed: one splitmix64 step of the seed. */
static inline uint64_t stream_key(uint64_t seed) {
    return sm64_mix(seed + 0x9E3779B97F4A7C15ull);
}

/* Draw `k` (0..15) of element `i` of the stream keyed by `key`. */
static inline uint64_t draw(uint64_t key, uint64_t i, unsigned k) {
    return sm64_mix(key + (i * 16u + k + 1u) * 0x9E3779B97F4A7C15ull);
}

ORACLE_API uint64_t oracle_splitmix64(uint64_t seed, uint64_t i, unsigned k) {
    return draw(stream_key(seed), i, k);
}

static inline float uniform_pm1(uint64_t key, uint64_t i) {
    int32_t m = (int32_t)(draw(key, i, 0) >> 40);            /* 0 .. 2^24-1 */
    return (float)(m - (1 << 23)) * (1.0f / 8388608.0f);    /* exact */
}

static inline float normal_ih(uint64_t key, uint64_t i) {
    int64_t s = 0;
    for (unsigned k = 0; k < 12; k++) s += (int64_t)(draw(key, i, k) >> 40);
    s -= (int64_t)6 << 24;
    return (float)s * (1.0f / 16777216.0f);                 /* RN convert, exact scale */
}

/* Fill out[j] = element (offset + j) of the uniform[-1,1) stream of `seed`. */
ORACLE_API void oracle_fill_uniform(uint64_t seed, uint64_t offset, size_t n, float* out) {
    const uint64_t key = stream_key(seed);
    #pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n; j++) out[j] = uniform_pm1(key, offset + j);
}

/* Fill out[j] = sigma * element (offset + j) of the normal stream of `seed`.
 * sigma must be a power of two for the result to be bit-reproducible. */
ORACLE_API void oracle_fill_normal(uint64_t seed, uint64_t offset, size_t n, float sigma, float* out) {
    const uint64_t key = stream_key(seed);
    #pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n; j++) out[j] = normal_ih(key, offset + j) * sigma;
}

/* IEEE binary32 -> bfloat16, round to nearest even; NaN -> 0x7FC0 | sign. */
ORACLE_API uint16_t oracle_f32_to_bf16(float x) {
    uint32_t b; memcpy(&b, &x, 4);
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((b >> 16) & 0x8000u) | 0x7FC0u);
    b += 0x7FFFu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

ORACLE_API float oracle_bf16_to_f32(uint16_t h) {
    uint32_t b = (uint32_t)h << 16; float x; memcpy(&x, &b, 4); return x;
}

/* bf16 normal(0, sigma) tensor: f32 Irwin-Hall sample * sigma, then RNE to bf16. */
ORACLE_API void oracle_fill_normal_bf16(uint64_t seed, uint64_t offset, size_t n, float sigma, uint16_t* out) {
    const uint64_t key = stream_key(seed);
    #pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n; j++) out[j] = oracle_f32_to_bf16(normal_ih(key, offset + j) * sigma);
}

/* Seeded outlier position in [0, n) and its sign (+1 / -1). */
ORACLE_API uint64_t oracle_outlier_index(uint64_t seed, uint64_t n) {
    return n ? draw(stream_key(seed ^ 0x0D7C0FFEEull), 0, 0) % n : 0;
}
ORACLE_API int oracle_outlier_sign(uint64_t seed) {
    return (draw(stream_key(seed ^ 0x0D7C0FFEEull), 0, 1) >> 63) ? -1 : 1;
}

/* ------------------------------------------------------------------------- */
/* absmax -- side_aware.cu:216-219 applied over the whole input              */
/* ------------------------------------------------------------------------- */

/* One step of the reference operator, fmaxf(acc, fabsf(x)) as CUDA evaluates
 * it (side_aware.cu:217-219 compiles to a GPU max that returns the non-NaN
 * operand for quiet AND signalling NaNs).  The C library's fmaxf differs: for a
 * signalling NaN it returns a quiet NaN (IEEE 754-2008 maxNum), which would
 * reset the running maximum.  So the step is written out: a NaN |x| compares
 * false and is skipped, acc itself is never NaN. */
static inline float absmax_step(float acc, float x) {
    const float v = fabsf(x);
    return v > acc ? v : acc;
}

/* Scalar loop, one thread: the literal restatement. */
ORACLE_API float oracle_absmax_f32_serial(const float* x, size_t n) {
    float m = 0.0f;                                   /* reduction_oob */
    for (size_t i = 0; i < n; i++) m = absmax_step(m, x[i]);
    return m;
}

/* OpenMP version (max is associative and commutative, so the grouping does not
 * change the bits).  nthreads <= 0 uses all available threads.  Returns the
 * number of threads actually used through *used (may be NULL). */
ORACLE_API float oracle_absmax_f32(const float* x, size_t n, int nthreads, int* used) {
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    float m = 0.0f;
    int got = 1;
    #pragma omp parallel num_threads(nthreads)
    {
        float t = 0.0f;
        #pragma omp for schedule(static) nowait
        for (size_t i = 0; i < n; i++) t = absmax_step(t, x[i]);
        #pragma omp critical
        { m = absmax_step(m, t); got = omp_get_num_threads(); }
    }
    if (used) *used = got;
    return m;
}

/* bf16 absmax (values widened exactly to f32, same operator). */
ORACLE_API float oracle_absmax_bf16(const uint16_t* x, size_t n) {
    float m = 0.0f;
    #pragma omp parallel
    {
        float t = 0.0f;
        #pragma omp for schedule(static) nowait
        for (size_t i = 0; i < n; i++) t = absmax_step(t, oracle_bf16_to_f32(x[i]));
        #pragma omp critical
        m = absmax_step(m, t);
    }
    return m;
}

/* ------------------------------------------------------------------------- */
/* The other reduction operators                                             */
/* ------------------------------------------------------------------------- */

/* The reference's operator is a swappable function (side_aware.cu:215-219,
 * and the note at :11); the product offers max, min, sum and sum of squares
 * besides absmax.  Their semantics, restated here:
 *   max / min: NaN elements are skipped (maxNum / minNum); -0 orders below
 *              +0; an empty or all-NaN input gives -inf (max) / +inf (min).
 *   sum / sum of squares: every element once, in double; NaN and infinities
 *              propagate as in IEEE addition.  The oracle sums with
 *              Neumaier's compensated algorithm (Neumaier 1974), so its result
 *              is within about one double rounding of the exact sum; it also
 *              returns sum |term| so that tests can bound any summation order's
 *              error by n * 2^-53 * sum |term|. */
static inline uint32_t f32_key(float f) {
    uint32_t b; memcpy(&b, &f, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

ORACLE_API float oracle_max_f32(const float* x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (!isnan(x[i]) && f32_key(x[i]) > f32_key(m)) m = x[i];
    return m;
}

ORACLE_API float oracle_min_f32(const float* x, size_t n) {
    float m = INFINITY;
    for (size_t i = 0; i < n; i++)
        if (!isnan(x[i]) && f32_key(x[i]) < f32_key(m)) m = x[i];
    return m;
}

static double neumaier(const float* x, size_t n, int square, double* abs_sum) {
    double s = 0.0, c = 0.0, a = 0.0, plain = 0.0;
    for (size_t i = 0; i < n; i++) {
        const double v = square ? (double)x[i] * (double)x[i] : (double)x[i];   /* a float's square is exact in double */
        const double t = s + v;
        if (fabs(s) >= fabs(v)) c += (s - t) + v; else c += (v - t) + s;
        s = t;
        a += fabs(v);
        plain += v;
    }
    if (abs_sum) *abs_sum = a;
    /* Floats cannot overflow a double sum, so a non-finite plain sum means an
     * infinity or NaN input: return IEEE addition's answer (inf, -inf or NaN). */
    return isfinite(plain) ? s + c : plain;
}

ORACLE_API double oracle_sum_f32(const float* x, size_t n, double* abs_sum) { return neumaier(x, n, 0, abs_sum); }
ORACLE_API double oracle_sumsq_f32(const float* x, size_t n, double* abs_sum) { return neumaier(x, n, 1, abs_sum); }

/* ------------------------------------------------------------------------- */
/* e4m3 (OCP OFP8) encode, RNE + satfinite                                   */
/* ------------------------------------------------------------------------- */

ORACLE_API uint8_t oracle_f32_to_e4m3(float x) {
    uint32_t b; memcpy(&b, &x, 4);
    const uint8_t sign = (uint8_t)((b >> 24) & 0x80u);
    const uint32_t a = b & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7F;                 /* NaN -> canonical NaN */
    if (a >= 0x7F800000u) return sign | 0x7E;         /* +-inf saturates to +-448 */
    const int e = (int)(a >> 23) - 127;               /* unbiased f32 exponent */
    if (e < -6) {
        /* e4m3 subnormal range: quantum 2^-9, codes 0..7; 8 is the first
         * normal (2^-6), and the code sequence is contiguous across. */
        float mag; memcpy(&mag, &a, 4);
        float q = nearbyintf(mag * 512.0f);           /* exact scale, RNE to integer */
        return sign | (uint8_t)q;
    }
    uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;       /* 24-bit significand */
    uint32_t r = mant >> 20;                           /* keep 1 + 3 bits: 8..15 */
    const uint32_t rem = mant & 0xFFFFFu, half = 0x80000u;
    int ee = e;
    if (rem > half || (rem == half && (r & 1u))) {
        r += 1;
        if (r == 16) { r = 8; ee += 1; }
    }
    if (ee > 8 || (ee == 8 && (r & 7u) == 7u)) return sign | 0x7E;   /* > 448 saturates */
    return sign | (uint8_t)(((uint32_t)(ee + 7) << 3) | (r & 7u));
}

ORACLE_API float oracle_e4m3_to_f32(uint8_t c) {
    const int s = c >> 7, e = (c >> 3) & 15, m = c & 7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), e - 10);
    return s ? -v : v;
}

/* Bulk encode (used by the exhaustive conversion test). */
ORACLE_API void oracle_f32_bits_to_e4m3(uint32_t first_bits, size_t n, uint8_t* out) {
    #pragma omp parallel for schedule(static)
    for (size_t j = 0; j < n; j++) {
        uint32_t b = first_bits + (uint32_t)j; float x; memcpy(&x, &b, 4);
        out[j] = oracle_f32_to_e4m3(x);
    }
}

/* scale = 448 / amax (IEEE round-to-nearest division); amax == 0 or inf -> 1. */
ORACLE_API float oracle_e4m3_scale(float amax) {
    if (!(amax > 0.0f) || isinf(amax)) return 1.0f;
    return 448.0f / amax;
}

/* Fused per-tensor quantize: amax over bf16 input, scale = 448/amax, then
 * q[i] = e4m3_rn_satfinite(f32(x[i]) * scale) with an IEEE f32 multiply. */
ORACLE_API float oracle_amax_quant_e4m3(const uint16_t* x, size_t n, uint8_t* q) {
    const float scale = oracle_e4m3_scale(oracle_absmax_bf16(x, n));
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        volatile float y = oracle_bf16_to_f32(x[i]) * scale;   /* no contraction */
        q[i] = oracle_f32_to_e4m3(y);
    }
    return scale;
}

/* ------------------------------------------------------------------------- */
/* Chunk-side selection -- side_aware.cu:299-318                             */
/* ------------------------------------------------------------------------- */

/* For the 2*chunk-byte pair that starts at absolute address `pair_addr`,
 * return which half (0 = first chunk, 1 = second) side `side` reads, given the
 * in-page hash mask and the page's side bit.  The first chunk is homed on side
 * parity(pair_addr & mask) ^ page_bit; a side reads the chunk homed on it. */
ORACLE_API int oracle_pair_half(uint64_t pair_addr, uint32_t mask, int page_bit, int side) {
    int first_side = (__builtin_popcountll(pair_addr & (uint64_t)mask) & 1) ^ (page_bit & 1);
    return first_side == side ? 0 : 1;
}
