// common/random.hpp -- seeded initialisation of host containers.
//
// Same generator and distributions as the reference's driver
// (include/common/random.hpp:40-69 in gpu_algos): std::mt19937_64 seeded
// with `seed`; floating-point elements draw from
// uniform_real_distribution(0, 1) in their own type (float for half),
// integer elements from uniform_int_distribution(0, 100).  With the same
// C++ standard library the driver therefore produces the same inputs as the
// reference for the same --seed.
#pragma once

#include <random>
#include <type_traits>

#include <cuda_fp16.h>

template <typename Container>
void randomize_container(Container& data, long seed) {
    using T = std::remove_reference_t<decltype(*data.begin())>;
    std::mt19937_64 generator(static_cast<std::mt19937_64::result_type>(seed));
    if constexpr (std::is_integral_v<T>) {
        std::uniform_int_distribution<T> distribution(T(0), T(100));
        for (auto& v : data) v = distribution(generator);
    } else {
        using U = std::conditional_t<std::is_floating_point_v<T>, T, float>;
        std::uniform_real_distribution<U> distribution(U(0), U(1));
        for (auto& v : data) v = T(distribution(generator));
    }
}
