"""B200-native (sm_100a) GLM path of gpu_algos: predict, gradient and the
elastic-net proximal-gradient fit, behind a C ABI (include/glm_b200.h).

Submodules
----------
capi      ctypes binding of libglm_b200.so (raw pointers)
glm       torch-tensor wrappers of the same entry points
sharded   observation-sharded evaluation across ranks (torch.distributed)
"""
__all__ = ["capi", "glm"]
