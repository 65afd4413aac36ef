/*
 * CPU ORACLE BUILD SUPPORT — test infrastructure only.
 *
 * ggml_backend_tensor_get as the reference's per-token scorer uses it: a copy
 * of `size` bytes at `offset` of a host tensor (the scorer calls it only for a
 * mask that is not device memory). Defined by oracle/ref_cuda_shim.cu.
 */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

void ggml_backend_tensor_get(const struct ggml_tensor* tensor, void* data, size_t offset, size_t size);

#ifdef __cplusplus
}
#endif
