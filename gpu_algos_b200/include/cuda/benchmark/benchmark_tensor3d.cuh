// benchmark_tensor3d.cuh -- the randomized-input driver of the GLM executables.
//
// Benchmark_Tensor3D_3In_1Out<Kernel> and Benchmark_Tensor3D_2In_1Out<Kernel>
// do what the reference's drivers do
// (include/cuda/benchmark/benchmark_tensor3d_{3in,2in}_1out.cuh in gpu_algos):
// build host tensors from the spec's extents, fill them (--init-method
// random / increasing / decreasing, seeds seed, seed+1, seed+2), allocate
// device memory on one stream, copy in, call kernel.run_device_kernel, copy
// the output (and temp) back, free, then recompute with kernel.run_host_kernel
// and compare element by element.  The summary lines keep the text the
// reference's sweep harness parses (test/gpu_algo_test/gpu_algo_test.py:569-600):
//   "Compute kernel: <ms> ms", "Max error     : ...", "Max error rel : ...",
//   "DONE: <ms> ms total", "[SUCCESS]" / "[FAILURE]".
// The verdict is E_max == 0 or E_max_rel <= 2^-(precision_bits - tol_bits).
#pragma once

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <iomanip>
#include <iostream>
#include <string>
#include <tuple>
#include <type_traits>

#include <cuda_runtime.h>

#include "common/types/tensor3d.hpp"
#include "cuda/check_errors.cuh"
#include "cuda/kernel_api/tensor3d_2in_1out.cuh"
#include "cuda/kernel_api/tensor3d_3in_1out.cuh"
#include "cuda/kernel_detect_types.cuh"
#include "cxxopts.hpp"

namespace bench_detail {

using Clock = std::chrono::high_resolution_clock;

inline double ms_since(Clock::time_point t0, Clock::time_point t1) {
    return std::chrono::duration<double, std::milli>(t1 - t0).count();
}

struct Common {
    long seed = 42;
    long gpu_mem = 16;
    bool verbose = false, errors = false, force = false;
    std::string init_method = "random";
    int tol_bits = 4;
};

template <typename Tolerance>
Common read_common(const cxxopts::Options& options, const cxxopts::ParseResult& parsed) {
    if (parsed.count("help")) {
        std::cout << options.help() << std::endl;
        std::exit(0);
    }
    Common c;
    c.seed = parsed["seed"].as<long>();
    c.gpu_mem = parsed["gpumem"].as<long>();
    c.verbose = parsed["verbose"].as<bool>();
    c.errors = parsed["errors"].as<bool>();
    c.force = parsed["force"].as<bool>();
    c.init_method = parsed["init-method"].as<std::string>();
    constexpr bool exact = std::is_integral_v<typename Tolerance::type>;
    if (exact && parsed.count("tol-bits")) {
        std::cout << "[ERROR] You may not use --tol-bits with integral types, which have no tolerance" << std::endl;
        std::cout << options.help() << std::endl;
        std::exit(1);
    }
    c.tol_bits = exact ? 0 : parsed["tol-bits"].as<int>();
    if (c.init_method != "random" && c.init_method != "increasing" && c.init_method != "decreasing") {
        std::cerr << "[ERROR] Invalid initialization method" << std::endl;
        std::exit(1);
    }
    return c;
}

template <typename T>
T from_index(size_t i) {
    if constexpr (std::is_same_v<T, __half>) return __half(static_cast<float>(i));
    else return static_cast<T>(i);
}

template <typename T>
double to_double(T v) {
    if constexpr (std::is_same_v<T, __half>) return double(__half2float(v));
    else return static_cast<double>(v);
}

template <typename T>
void init_tensor(Tensor3D<T>& t, const std::string& method, long seed) {
    const size_t n = t.vector_.size();
    if (method == "random") {
        t.randomize(seed);
    } else if (method == "increasing") {
        for (size_t i = 0; i < n; ++i) t.vector_[i] = from_index<T>(i);
    } else {
        for (size_t i = 0; i < n; ++i) t.vector_[i] = from_index<T>(n - i);
    }
}

template <typename T>
size_t bytes_of(const Tensor3D<T>& t) {
    return t.vector_.size() * sizeof(T);
}

template <typename T>
void print_dims(const char* label, const Tensor3D<T>& t) {
    std::cout << label << t.rows() << "x" << t.cols() << "x" << t.sheets() << "\n";
}

struct Errors {
    double e_max = 0, e_max_rel = 0;
    long e_col = 0, e_row = 0, e_sheet = 0, r_col = 0, r_row = 0, r_sheet = 0;
};

// Absolute and relative error of every element; NaN==NaN and same-signed
// infinities count as equal, a zero reference gives relative error 0.
template <typename T>
Errors compare(const Tensor3D<T>& gpu, const Tensor3D<T>& cpu, bool list) {
    Errors e;
    bool any = false;
    if (list) std::cout << "Non-zero error elements:\n";
    for (long s = 0; s < cpu.sheets(); ++s)
        for (long r = 0; r < cpu.rows(); ++r)
            for (long c = 0; c < cpu.cols(); ++c) {
                const double g = to_double(gpu(c, r, s)), h = to_double(cpu(c, r, s));
                const double delta = g - h;
                const bool same = (std::isnan(g) && std::isnan(h)) || (std::isinf(g) && std::isinf(h) && std::isnan(delta));
                const double ea = same ? 0.0 : std::fabs(delta);
                const double er = std::fabs(h) > 0 ? ea / std::fabs(h) : 0.0;
                if (ea > e.e_max) std::tie(e.e_max, e.e_col, e.e_row, e.e_sheet) = std::make_tuple(ea, c, r, s);
                if (er > e.e_max_rel) std::tie(e.e_max_rel, e.r_col, e.r_row, e.r_sheet) = std::make_tuple(er, c, r, s);
                if (list && ea != 0.0) {
                    any = true;
                    std::cout << "(" << c << ", " << r << ", " << s << "): result gpu =" << g << ", result cpu =" << h
                              << ", E          =" << ea << "\n";
                }
            }
    if (list && !any) std::cout << "No non-zero error elements found\n";
    return e;
}

// Times of the device steps, measured with events on the one stream.
struct DeviceSteps {
    float ms[5] = {0, 0, 0, 0, 0};
    static constexpr const char* names[5] = {"Allocate device memory", "Copy data to device", "Compute kernel",
                                             "Copy result back to host", "Free device memory"};
    void print() const {
        float total = 0;
        for (int i = 0; i < 5; ++i) {
            total += ms[i];
            std::cout << (i + 1) << " - " << std::setw(26) << names[i] << ": " << ms[i] << " ms (" << total
                      << " ms total)" << std::endl;
        }
    }
    float total() const { return ms[0] + ms[1] + ms[2] + ms[3] + ms[4]; }
};

template <typename Tolerance>
void print_summary(double total_ms, const Errors& e, int tol_bits, double cpu_ms, const DeviceSteps& steps) {
    const float tolerance = Tolerance::tolerance(tol_bits);
    std::cout << "DONE: " << total_ms << " ms total" << std::endl;
    std::cout << "Max error     : " << e.e_max << " at (" << e.e_row << ", " << e.e_col << ", " << e.e_sheet << ")" << std::endl;
    std::cout << "Max error rel : " << e.e_max_rel << " at (" << e.r_row << ", " << e.r_col << ", " << e.r_sheet << ")" << std::endl;
    std::cout << "Precision rel : " << Tolerance::precision << " (" << Tolerance::name() << " with "
              << Tolerance::precision_bits << " bits of precision)" << std::endl;
    std::cout << "Tolerance rel : " << tolerance << " assuming a loss of " << tol_bits << " bits of precision" << std::endl;
    std::cout << "Gross speedup : " << (steps.ms[2] > 0 ? cpu_ms / steps.ms[2] : 0.0) << std::endl;
    std::cout << "Net speedup   : " << (steps.total() > 0 ? cpu_ms / steps.total() : 0.0) << std::endl;
    if (e.e_max == 0 || e.e_max_rel <= tolerance) {
        std::cout << "[SUCCESS]     : Max error pct is within tolerance" << std::endl;
    } else {
        std::cout << "[FAILURE]     : Max error pct exceeds tolerance" << std::endl;
    }
}

// Runs the device side: allocation, copies in, `launch(device pointers)`,
// copies out, free -- each step timed with events on one stream.
template <typename Launch>
DeviceSteps run_device(const std::vector<std::pair<const void*, size_t>>& inputs,
                       const std::vector<std::pair<void*, size_t>>& outputs, Launch&& launch) {
    DeviceSteps steps;
    cudaStream_t stream;
    cuda_check_error(cudaStreamCreate(&stream), "cudaStreamCreate");
    cudaEvent_t ev[6];
    for (auto& e : ev) cuda_check_error(cudaEventCreate(&e), "cudaEventCreate");
    std::vector<void*> d_in(inputs.size(), nullptr), d_out(outputs.size(), nullptr);
    cuda_check_error(cudaEventRecord(ev[0], stream), "cudaEventRecord");
    for (size_t i = 0; i < inputs.size(); ++i)
        if (inputs[i].second) cuda_check_error(cudaMallocAsync(&d_in[i], inputs[i].second, stream), "cudaMallocAsync");
    for (size_t i = 0; i < outputs.size(); ++i)
        if (outputs[i].second) cuda_check_error(cudaMallocAsync(&d_out[i], outputs[i].second, stream), "cudaMallocAsync");
    cuda_check_error(cudaEventRecord(ev[1], stream), "cudaEventRecord");
    for (size_t i = 0; i < inputs.size(); ++i)
        if (inputs[i].second)
            cuda_check_error(cudaMemcpyAsync(d_in[i], inputs[i].first, inputs[i].second, cudaMemcpyHostToDevice, stream),
                             "cudaMemcpyAsync");
    cuda_check_error(cudaEventRecord(ev[2], stream), "cudaEventRecord");
    launch(d_in, d_out, stream);
    cuda_check_error(cudaEventRecord(ev[3], stream), "cudaEventRecord");
    for (size_t i = 0; i < outputs.size(); ++i)
        if (outputs[i].second)
            cuda_check_error(cudaMemcpyAsync(outputs[i].first, d_out[i], outputs[i].second, cudaMemcpyDeviceToHost, stream),
                             "cudaMemcpyAsync");
    cuda_check_error(cudaEventRecord(ev[4], stream), "cudaEventRecord");
    for (void* p : d_in)
        if (p) cuda_check_error(cudaFreeAsync(p, stream), "cudaFreeAsync");
    for (void* p : d_out)
        if (p) cuda_check_error(cudaFreeAsync(p, stream), "cudaFreeAsync");
    cuda_check_error(cudaEventRecord(ev[5], stream), "cudaEventRecord");
    cuda_check_error(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    for (int i = 0; i < 5; ++i) cuda_check_error(cudaEventElapsedTime(&steps.ms[i], ev[i], ev[i + 1]), "cudaEventElapsedTime");
    for (auto& e : ev) cuda_check_error(cudaEventDestroy(e), "cudaEventDestroy");
    cuda_check_error(cudaStreamDestroy(stream), "cudaStreamDestroy");
    return steps;
}

inline bool memory_fits(size_t bytes, long gpu_mem_gb) {
    const double gb = double(bytes) / (1024.0 * 1024.0 * 1024.0);
    if (gb > double(gpu_mem_gb)) {
        std::cerr << "[ERROR] GPU memory size is less than the required size" << std::endl;
        return false;
    }
    return true;
}

}  // namespace bench_detail

template <TENSOR3D_KERNEL_3IN_1OUT Kernel>
class Benchmark_Tensor3D_3In_1Out {
   public:
    using Kernel_spec = typename Kernel::Kernel_spec;
    using Numbers = detect::Numbers<Kernel>;
    using A = typename Numbers::A;
    using B = typename Numbers::B;
    using C = typename Numbers::C;
    using D = typename Numbers::D;
    using Temp = typename Numbers::Temp;
    using Tolerance = typename Numbers::Tolerance;

    const Kernel_spec spec;
    const bench_detail::Common common;
    Kernel kernel;

    template <typename... Args>
    Benchmark_Tensor3D_3In_1Out(const Kernel_spec spec_, const cxxopts::Options& options,
                                const cxxopts::ParseResult& parsed, Args&... args)
        : spec(spec_), common(bench_detail::read_common<Tolerance>(options, parsed)), kernel(spec_, args...) {}

    int run() {
        using namespace bench_detail;
        const auto t0 = Clock::now();
        Tensor3D<A> ta(spec.n_cols_A_, spec.n_rows_A_, spec.n_sheets_A_, A(0));
        Tensor3D<B> tb(spec.n_cols_B_, spec.n_rows_B_, spec.n_sheets_B_, B(0));
        Tensor3D<C> tc(spec.n_cols_C_, spec.n_rows_C_, spec.n_sheets_C_, C(0));
        Tensor3D<D> td(spec.n_cols_D_, spec.n_rows_D_, spec.n_sheets_D_, D(0));
        Tensor3D<Temp> tt(spec.n_cols_temp_, spec.n_rows_temp_, spec.n_sheets_temp_, Temp(0));
        const size_t in_bytes = bytes_of(ta) + bytes_of(tb) + bytes_of(tc);
        print_dims("Input tensor3d A dimensions : ", ta);
        print_dims("Input tensor3d B dimensions : ", tb);
        print_dims("Input tensor3d C dimensions : ", tc);
        print_dims("Output tensor3d dimensions  : ", td);
        print_dims("Temp tensor3d dimensions    : ", tt);
        std::cout << "Input size                  : " << in_bytes << " bytes\n"
                  << "Output size                 : " << bytes_of(td) << " bytes\n"
                  << "Temp size                   : " << bytes_of(tt) << " bytes\n" << std::endl;
        if (!memory_fits(in_bytes + bytes_of(td) + bytes_of(tt), common.gpu_mem)) return 1;
        std::cout << "SETUP:" << std::endl;
        init_tensor(ta, common.init_method, common.seed);
        init_tensor(tb, common.init_method, common.seed + 1);
        init_tensor(tc, common.init_method, common.seed + 2);
        std::cout << "  - Initializing tensors (" << common.init_method << "): " << ms_since(t0, Clock::now()) << " ms" << std::endl;

        std::cout << "Tensor3D_Kernel_3In_1Out:" << std::endl;
        const DeviceSteps steps = run_device(
            {{ta.data(), bytes_of(ta)}, {tb.data(), bytes_of(tb)}, {tc.data(), bytes_of(tc)}},
            {{td.data(), bytes_of(td)}, {tt.data(), bytes_of(tt)}},
            [&](const std::vector<void*>& in, const std::vector<void*>& out, cudaStream_t s) {
                kernel.run_device_kernel(static_cast<const A*>(in[0]), static_cast<const B*>(in[1]),
                                         static_cast<const C*>(in[2]), static_cast<D*>(out[0]),
                                         static_cast<Temp*>(out[1]), s);
            });
        steps.print();

        std::cout << "CHECK WITH CPU:" << std::endl;
        const auto c0 = Clock::now();
        const Tensor3D<D> cpu = kernel.run_host_kernel(ta, tb, tc);
        const double cpu_ms = ms_since(c0, Clock::now());
        std::cout << " - Compute result with CPU: " << cpu_ms << " ms" << std::endl;
        const Errors e = compare(td, cpu, common.errors);
        if (common.verbose) {
            std::cout << "A    :\n";
            ta.print(std::cout);
            std::cout << "B    :\n";
            tb.print(std::cout);
            std::cout << "C    :\n";
            tc.print(std::cout);
            std::cout << "D_gpu:\n";
            td.print(std::cout);
            std::cout << "D_cpu:\n";
            cpu.print(std::cout);
        }
        print_summary<Tolerance>(ms_since(t0, Clock::now()), e, common.tol_bits, cpu_ms, steps);
        return 0;
    }
};

template <TENSOR3D_KERNEL_2IN_1OUT Kernel>
class Benchmark_Tensor3D_2In_1Out {
   public:
    using Kernel_spec = typename Kernel::Kernel_spec;
    using Numbers = detect::Numbers<Kernel>;
    using A = typename Numbers::A;
    using B = typename Numbers::B;
    using C = typename Numbers::C;
    using Temp = typename Numbers::Temp;
    using Tolerance = typename Numbers::Tolerance;

    const Kernel_spec spec;
    const bench_detail::Common common;
    Kernel kernel;

    template <typename... Args>
    Benchmark_Tensor3D_2In_1Out(const Kernel_spec spec_, const cxxopts::Options& options,
                                const cxxopts::ParseResult& parsed, Args&... args)
        : spec(spec_), common(bench_detail::read_common<Tolerance>(options, parsed)), kernel(spec_, args...) {}

    int run() {
        using namespace bench_detail;
        const auto t0 = Clock::now();
        Tensor3D<A> ta(spec.n_cols_A_, spec.n_rows_A_, spec.n_sheets_A_, A(0));
        Tensor3D<B> tb(spec.n_cols_B_, spec.n_rows_B_, spec.n_sheets_B_, B(0));
        Tensor3D<C> tc(spec.n_cols_C_, spec.n_rows_C_, spec.n_sheets_C_, C(0));
        Tensor3D<Temp> tt(spec.n_cols_temp_, spec.n_rows_temp_, spec.n_sheets_temp_, Temp(0));
        const size_t in_bytes = bytes_of(ta) + bytes_of(tb);
        print_dims("Input tensor3d A dimensions : ", ta);
        print_dims("Input tensor3d B dimensions : ", tb);
        print_dims("Output tensor3d dimensions  : ", tc);
        print_dims("Temp tensor3d dimensions    : ", tt);
        std::cout << "Input size                  : " << in_bytes << " bytes\n"
                  << "Output size                 : " << bytes_of(tc) << " bytes\n" << std::endl;
        if (!memory_fits(in_bytes + bytes_of(tc) + bytes_of(tt), common.gpu_mem)) return 1;
        std::cout << "SETUP:" << std::endl;
        init_tensor(ta, common.init_method, common.seed);
        init_tensor(tb, common.init_method, common.seed + 1);
        std::cout << "  - Initializing tensors (" << common.init_method << "): " << ms_since(t0, Clock::now()) << " ms" << std::endl;

        std::cout << "Tensor3D_Kernel_2In_1Out:" << std::endl;
        const DeviceSteps steps = run_device(
            {{ta.data(), bytes_of(ta)}, {tb.data(), bytes_of(tb)}},
            {{tc.data(), bytes_of(tc)}, {tt.data(), bytes_of(tt)}},
            [&](const std::vector<void*>& in, const std::vector<void*>& out, cudaStream_t s) {
                kernel.run_device_kernel(static_cast<const A*>(in[0]), static_cast<const B*>(in[1]),
                                         static_cast<C*>(out[0]), static_cast<Temp*>(out[1]), s);
            });
        steps.print();

        std::cout << "CHECK WITH CPU:" << std::endl;
        const auto c0 = Clock::now();
        const Tensor3D<C> cpu = kernel.run_host_kernel(ta, tb);
        const double cpu_ms = ms_since(c0, Clock::now());
        std::cout << " - Compute result with CPU: " << cpu_ms << " ms" << std::endl;
        const Errors e = compare(tc, cpu, common.errors);
        if (common.verbose) {
            std::cout << "A    :\n";
            ta.print(std::cout);
            std::cout << "B    :\n";
            tb.print(std::cout);
            std::cout << "C_gpu:\n";
            tc.print(std::cout);
            std::cout << "C_cpu:\n";
            cpu.print(std::cout);
        }
        print_summary<Tolerance>(ms_since(t0, Clock::now()), e, common.tol_bits, cpu_ms, steps);
        return 0;
    }
};
