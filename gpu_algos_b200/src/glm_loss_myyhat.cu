// glm_loss_myyhat -- the GLM objective on the B200, checked against the host
// computation.
#include "cuda/kernels/glm/glm_loss_myyhat.cuh"
#include "glm_main.cuh"

int main(int argc, char** argv) {
    return glm_main<Glm_loss_myyhat_spec, Benchmark_Tensor3D_3In_1Out, Glm_loss_myyhat_kernel>(
        "glm_loss_myyhat", "Loss of a linear model", argc, argv);
}
