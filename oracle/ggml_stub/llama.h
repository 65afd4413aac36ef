/*
 * CPU ORACLE BUILD SUPPORT — test infrastructure only.
 *
 * The llama.cpp declarations that the reference's adapter headers
 * (src/adapter/llama-kvmem-hooks.h, included by its stage-in code) name:
 * LLAMA_API, the position / token / sequence id types and the opaque structs
 * its hook API passes around. None of them is used by the stage-in functions
 * compiled here. llama.cpp is an un-vendored submodule of the reference, absent
 * here.
 */
#pragma once
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "ggml.h"

#define LLAMA_API
typedef int32_t llama_pos;
typedef int32_t llama_token;
typedef int32_t llama_seq_id;
struct llama_context;
struct llama_model;
struct llama_vocab;
struct llama_batch;
typedef struct ggml_backend_device* ggml_backend_dev_t;
struct ggml_backend_sched;
struct ggml_context;
struct ggml_cgraph;
