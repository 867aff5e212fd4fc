/*
 * Minimal stand-in for the parts of ggml.h that the reference's
 * src/arch/kokoro/lstm_fused.{h,cpp} touch, so that file compiles unchanged
 * without ggml (which the reference fetches from the network at configure
 * time). Oracle build only; never part of the product.
 */
#pragma once
#include <cassert>
#include <cstddef>
#include <cstdint>

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1 };

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    void *data;
};

#define GGML_ASSERT(x) assert(x)
