// glm_main.cuh -- shared main() body of the GLM executables: parse the
// options, build the spec, dispatch on --type to the eleven element types of
// the reference mains (src/cuda/benchmarks/glm/*.cu in gpu_algos) and run
// the driver.  Option errors print the help text and return 1.
#pragma once

#include <cstdint>
#include <iostream>

#include "common/benchmark_options.hpp"
#include "cuda/benchmark/benchmark_tensor3d.cuh"
#include "cxxopts.hpp"

template <typename Spec, template <typename> class Benchmark, template <CUDA_scalar> class Kernel>
int glm_main(const char* name, const char* description, int argc, char** argv) {
    cxxopts::Options options(name, description);
    add_benchmark_options(options);
    Spec::add_kernel_spec_options(options);
    try {
        const cxxopts::ParseResult parsed = options.parse(argc, argv);
        if (parsed.count("help")) {
            std::cout << options.help() << std::endl;
            return 0;
        }
        const Spec spec = Spec::make(parsed);
        const std::string& t = spec.type_;
        if (t == "half") return Benchmark<Kernel<__half>>(spec, options, parsed).run();
        if (t == "single" || t == "float") return Benchmark<Kernel<float>>(spec, options, parsed).run();
        if (t == "double") return Benchmark<Kernel<double>>(spec, options, parsed).run();
        if (t == "int8") return Benchmark<Kernel<std::int8_t>>(spec, options, parsed).run();
        if (t == "int16") return Benchmark<Kernel<std::int16_t>>(spec, options, parsed).run();
        if (t == "int32") return Benchmark<Kernel<std::int32_t>>(spec, options, parsed).run();
        if (t == "int64") return Benchmark<Kernel<std::int64_t>>(spec, options, parsed).run();
        if (t == "uint8") return Benchmark<Kernel<std::uint8_t>>(spec, options, parsed).run();
        if (t == "uint16") return Benchmark<Kernel<std::uint16_t>>(spec, options, parsed).run();
        if (t == "uint32") return Benchmark<Kernel<std::uint32_t>>(spec, options, parsed).run();
        if (t == "uint64") return Benchmark<Kernel<std::uint64_t>>(spec, options, parsed).run();
        throw cxxopts::exceptions::exception("Invalid type: " + t);
    } catch (const cxxopts::exceptions::exception& e) {
        std::cerr << "Error parsing options: " << e.what() << std::endl;
        std::cout << options.help() << std::endl;
        return 1;
    }
}
