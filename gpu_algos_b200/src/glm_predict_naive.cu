// glm_predict_naive -- GLM prediction on the B200, checked against the host
// computation.
#include "cuda/kernels/glm/glm_predict_naive.cuh"
#include "glm_main.cuh"

int main(int argc, char** argv) {
    return glm_main<Glm_predict_naive_spec, Benchmark_Tensor3D_2In_1Out, Glm_predict_naive_kernel>(
        "glm_predict_naive", "Evaluate linear model", argc, argv);
}
