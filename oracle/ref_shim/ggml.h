/* Minimal stand-in for ggml.h, written for this repository so that the
 * reference engine's kernel sources compile without the (un-vendored,
 * unpinned) ggml library. Only the names those sources use are declared;
 * enum values are the GGML file-format type ids. Test infrastructure only. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#define GGML_MAX_DIMS 4

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_COUNT = 40,
};

struct ggml_context;
struct ggml_tensor;

#ifdef __cplusplus
extern "C" {
#endif
void ggml_free(struct ggml_context* ctx);
#ifdef __cplusplus
}
#endif
