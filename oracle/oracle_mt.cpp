// oracle_mt.cpp -- CPU oracle helper (TEST INFRASTRUCTURE, not product code).
//
// Reproduces the reference harness' `-r` fill of array A, QuickRunCUDA.cpp:432-457:
// the array is cut into chunks of 1 Mi dwords; chunk c draws its dwords from
// std::mt19937_64 seeded with (randomSeed + c) through
// std::uniform_int_distribution<uint>, each value ANDed with --randomMask.
// It uses the same C++ standard library engine and distribution as the
// reference harness, so golden outputs produced by running the reference
// kernel on `-r` data can be checked against the oracle's absmax on a
// bit-identical copy of that data.
#include <cstddef>
#include <cstdint>
#include <random>
#include <algorithm>

extern "C" __attribute__((visibility("default")))
void oracle_fill_ref_random(unsigned seed, unsigned mask, size_t n, uint32_t* out) {
    const size_t chunk_size = 1024 * 1024;
    const size_t num_chunks = (n + chunk_size - 1) / chunk_size;
    #pragma omp parallel for schedule(static)
    for (size_t chunk = 0; chunk < num_chunks; chunk++) {
        std::mt19937_64 rng(seed + chunk);
        std::uniform_int_distribution<unsigned> dist;
        const size_t end = std::min((chunk + 1) * chunk_size, n);
        for (size_t i = chunk * chunk_size; i < end; ++i) out[i] = dist(rng) & mask;
    }
}
