// glm_gradient_naive -- unregularised GLM gradient on the B200, checked
// against the host computation.
#include "cuda/kernels/glm/glm_gradient_naive.cuh"
#include "glm_main.cuh"

int main(int argc, char** argv) {
    return glm_main<Glm_gradient_naive_spec, Benchmark_Tensor3D_3In_1Out, Glm_gradient_naive_kernel>(
        "glm_gradient_naive", "Evaluate linear model", argc, argv);
}
