// glm_peer.cuh -- peer-memory exchange of the sharded gradient (glm_peer.cu).
#pragma once

#include "glm_common.cuh"

namespace glmb {

int peer_group_create(int rank, int world, int64_t max_elems, double timeout_ms, glmb_peer_group** out,
                      void* handle_out);
int peer_group_connect(glmb_peer_group* g, const void* handles, void* const* local_ptrs);
int peer_group_status(glmb_peer_group* g, int* status, int reset);
int peer_group_destroy(glmb_peer_group* g);
void* peer_group_buffer(glmb_peer_group* g);

// Sums part[e*nparts + c] over c, exchanges the rank partials through the
// group's peer buffers and writes grad (2*sum + elastic-net term) or, with
// partial_out, the summed partial.  local_status (optional): a status word of
// the partial kernel; when set, the outputs become NaN.
template <typename T>
int exchange_launch(glmb_peer_group* g, const double* part, int64_t nparts, int64_t total, const T* M, T* grad,
                    double* partial_out, double lambda, double alpha, bool reg, const int* local_status,
                    cudaStream_t stream);

}  // namespace glmb
