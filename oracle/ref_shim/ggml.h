/*
 * Declaration-only stand-in for the parts of ggml.h that the reference's
 * host-side sources touch, so that src/arch/kokoro/lstm_fused.cpp,
 * audio_utils.cpp and kokoro.cpp compile unchanged without ggml (which the
 * reference fetches from the network at configure time). Oracle build only;
 * never part of the product.
 *
 * Nothing here is defined: the oracle's glue (oracle/ref_glue_*.cpp) calls
 * only the reference's pure host functions (the harmonic source and STFT,
 * the Kokoro iSTFT conversion, the duration rounding and mask), and the
 * build drops every function that would build a ggml graph (hidden
 * visibility plus --gc-sections), so none of these declarations is ever
 * resolved. The parameter lists follow the reference's call sites.
 */
#pragma once
#include <cassert>
#include <cstddef>
#include <cstdint>

#define GGML_MAX_DIMS 4
#define GGML_DEFAULT_GRAPH_SIZE 2048
#define GGML_ASSERT(x) assert(x)

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_I32 = 26 };
enum ggml_op { GGML_OP_NONE = 0, GGML_OP_NORM, GGML_OP_RMS_NORM, GGML_OP_SOFT_MAX };
enum ggml_prec { GGML_PREC_DEFAULT = 0, GGML_PREC_F32 = 10 };
enum ggml_status { GGML_STATUS_SUCCESS = 0, GGML_STATUS_FAILED = -1 };

struct ggml_backend_buffer;

/* The fields the reference reads; lstm_fused.cpp reads type, ne, nb, data. */
struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer *buffer;
    int64_t ne[4];
    size_t nb[4];
    enum ggml_op op;
    struct ggml_tensor *src[10];
    struct ggml_tensor *view_src;
    void *data;
    char name[64];
};

struct ggml_context;
struct ggml_cgraph;
struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_context *ggml_init(struct ggml_init_params params);
void ggml_free(struct ggml_context *ctx);
int64_t ggml_time_us(void);
size_t ggml_tensor_overhead(void);
size_t ggml_graph_overhead_custom(size_t size, bool grads);
size_t ggml_nbytes(const struct ggml_tensor *t);
int64_t ggml_nelements(const struct ggml_tensor *t);
struct ggml_tensor *ggml_set_name(struct ggml_tensor *t, const char *name);
void ggml_set_input(struct ggml_tensor *t);
void ggml_set_output(struct ggml_tensor *t);
void ggml_prec_set_acc(struct ggml_tensor *t, enum ggml_prec prec);
struct ggml_tensor *ggml_get_first_tensor(const struct ggml_context *ctx);
struct ggml_tensor *ggml_get_next_tensor(const struct ggml_context *ctx, struct ggml_tensor *t);

struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_new_tensor_3d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1,
                                       int64_t ne2);
struct ggml_tensor *ggml_view_1d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, size_t offset);
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1,
                                 size_t offset);
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                    int64_t ne2);
struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int ax0, int ax1, int ax2, int ax3);
struct ggml_tensor *ggml_transpose(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cont_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_cont_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1,
                                 int64_t ne2);
struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_repeat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_concat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, int dim);
struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_exp(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_sin(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cos(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_clamp(struct ggml_context *ctx, struct ggml_tensor *a, float min, float max);
struct ggml_tensor *ggml_gelu_erf(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_get_rows(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_gelu(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_soft_max_ext(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *mask,
                                      float scale, float max_bias);
struct ggml_tensor *ggml_pad_reflect_1d(struct ggml_context *ctx, struct ggml_tensor *a, int p0, int p1);

struct ggml_cgraph *ggml_new_graph_custom(struct ggml_context *ctx, size_t size, bool grads);
void ggml_build_forward_expand(struct ggml_cgraph *cgraph, struct ggml_tensor *tensor);
int ggml_graph_size(struct ggml_cgraph *cgraph);
int ggml_graph_n_nodes(struct ggml_cgraph *cgraph);
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *cgraph, int i);

#ifdef __cplusplus
}
#endif
