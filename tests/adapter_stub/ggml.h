// Stand-in for the few public ggml names the op-hook adapter uses
// (ggml_tensor's type/ne/nb/op/src/data, two type ids, GGML_OP_MUL_MAT and
// ggml_is_contiguous).  Test infrastructure: the real header comes with the
// reference's ggml fork, which is not part of this repository.
#pragma once
#include <cstddef>
#include <cstdint>
enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q8_0 = 8 };
enum ggml_op { GGML_OP_NONE = 0, GGML_OP_ADD = 2, GGML_OP_MUL_MAT = 29 };
#define GGML_MAX_SRC 10
struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    enum ggml_op op;
    struct ggml_tensor * src[GGML_MAX_SRC];
    void * data;
};
extern "C" bool ggml_is_contiguous(const struct ggml_tensor * t);   // ggml.h declares its API with C linkage
