/*
 * CPU ORACLE BUILD SUPPORT — test infrastructure only.
 *
 * The smallest set of ggml declarations that the reference's per-token page
 * scorer (src/adapter/llama-kvmem-attention-cuda.{h,cu}) and its stage-in
 * code (src/adapter/llama-kvmem-stagein.cu) need to compile: the ggml_type
 * values they test, a tensor with type / ne / nb / data / buffer / view_src, and
 * ggml_time_us. ggml itself is an un-vendored submodule of the reference
 * (llama.cpp @ cd959bae99ff4bed22bef2604f45241c09bbb8c8), absent here.
 *
 * The enum values are ggml's (they are part of the GGUF file format, so they
 * must match for the reference's comparisons to mean what they say). The
 * tensor struct holds only the fields the scorer reads; the reference's code
 * and oracle/ref_cuda_shim.cu are compiled against this same header, so its
 * layout only has to agree with itself.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_BF16 = 30,
};

struct ggml_backend_buffer;
typedef struct ggml_backend_buffer* ggml_backend_buffer_t;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4]; /* elements per dimension */
    size_t nb[4];  /* byte stride per dimension */
    void* data;
    struct ggml_backend_buffer* buffer;
    struct ggml_tensor* view_src;
};

/* Microseconds of a monotonic clock. Defined by oracle/ref_cuda_shim.cu. */
int64_t ggml_time_us(void);

/* Bytes of `ne` elements of `type` (ne a multiple of the block size). Defined
 * by oracle/ref_cuda_shim.cu. */
size_t ggml_row_size(enum ggml_type type, int64_t ne);

#ifdef __cplusplus
}
#endif
