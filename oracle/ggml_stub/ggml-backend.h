/*
 * CPU ORACLE BUILD SUPPORT — test infrastructure only.
 *
 * ggml_backend_tensor_get / _set and ggml_backend_buffer_is_host as the
 * reference's per-token scorer and stage-in headers use them: copies of `size`
 * bytes at `offset` of a host tensor (the scorer reads only a mask that is not
 * device memory). Defined by oracle/ref_cuda_shim.cu.
 */
#pragma once
#include <stdbool.h>

#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

void ggml_backend_tensor_get(const struct ggml_tensor* tensor, void* data, size_t offset, size_t size);
void ggml_backend_tensor_set(struct ggml_tensor* tensor, const void* data, size_t offset, size_t size);
bool ggml_backend_buffer_is_host(ggml_backend_buffer_t buffer);

#ifdef __cplusplus
}
#endif
