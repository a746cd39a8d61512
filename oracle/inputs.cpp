// Seeded input generation for the parity tests.  TEST INFRASTRUCTURE ONLY.
//
// The reference draws its inputs from one std::mt19937 engine and one
// std::normal_distribution<float> (or uniform_real_distribution<float>) object,
// filling A, then B, then C in order (tests/test_gemm_correctness.cu:23-30,
// tests/test_mxfp8_quantize.cu:12-16, :48-52).  The exact stream depends on the
// C++ standard library, so this file is built with g++/libstdc++, the same
// library the reference's tests are built with, and keeps one engine and one
// distribution object across all arrays of a call.
#include <cstdint>
#include <random>

extern "C" {

// Fill n_arrays arrays in order from one mt19937(seed) + normal(mean, std).
void orc_fill_normal(uint32_t seed, float mean, float stddev, int n_arrays,
                     float** arrays, const int64_t* sizes)
{
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (int a = 0; a < n_arrays; ++a)
        for (int64_t i = 0; i < sizes[a]; ++i) arrays[a][i] = dist(rng);
}

// Fill n_arrays arrays in order from one mt19937(seed) + uniform_real(lo, hi).
void orc_fill_uniform(uint32_t seed, float lo, float hi, int n_arrays,
                      float** arrays, const int64_t* sizes)
{
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (int a = 0; a < n_arrays; ++a)
        for (int64_t i = 0; i < sizes[a]; ++i) arrays[a][i] = dist(rng);
}

}  // extern "C"
