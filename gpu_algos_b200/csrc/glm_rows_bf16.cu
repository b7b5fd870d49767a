// bfloat16 instantiation of the fused rows kernel (see glm_rows.cuh).
#include "glm_rows_impl.cuh"

namespace glmb {
GLMB_INSTANTIATE_ROWS(__nv_bfloat16)
}  // namespace glmb
