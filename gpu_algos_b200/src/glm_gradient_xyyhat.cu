// glm_gradient_xyyhat -- regularised GLM gradient (with Yhat) on the B200,
// checked against the host computation.
#include "cuda/kernels/glm/glm_gradient_xyyhat.cuh"
#include "glm_main.cuh"

int main(int argc, char** argv) {
    return glm_main<Glm_gradient_xyyhat_spec, Benchmark_Tensor3D_3In_1Out, Glm_gradient_xyyhat_kernel>(
        "glm_gradient_xyyhat", "Evaluate linear model", argc, argv);
}
