// common/benchmark_options.hpp -- options shared by every GLM executable
// (the reference's src/common/benchmark_options.cpp:23-33: same names,
// defaults and meanings).
#pragma once

#include <string>

#include "cxxopts.hpp"

constexpr int DEFAULT_GPU_MEM = 16;  // GPU memory size in GB
constexpr int DEFAULT_SEED = 42;
constexpr int DEFAULT_TOL_BITS = 4;

inline void add_benchmark_options(cxxopts::Options& options) {
    options.add_options()
        ("i,init-method", "How to generate data: random, increasing, decreasing",
         cxxopts::value<std::string>()->default_value("random"))
        ("gpumem", "GPU memory size", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_GPU_MEM)))
        ("seed", "Random seed", cxxopts::value<long>()->default_value(std::to_string(DEFAULT_SEED)))
        ("tol-bits", "Number of bits of precision lost due to arithmetic rounding",
         cxxopts::value<int>()->default_value(std::to_string(DEFAULT_TOL_BITS)))
        ("errors", "Display errors", cxxopts::value<bool>()->default_value("false"))
        ("verbose", "Verbose output", cxxopts::value<bool>()->default_value("false"))
        ("force,f", "Allow verbose output even if the input matrix is large",
         cxxopts::value<bool>()->default_value("false"))
        ("h,help", "Print usage");
}
