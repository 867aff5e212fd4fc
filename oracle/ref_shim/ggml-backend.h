/*
 * Declaration-only stand-in for the parts of ggml-backend.h that the
 * reference's src/backend/backend.h names (reached through
 * src/arch/kokoro/kokoro.h). Oracle build only; nothing here is defined or
 * resolved (see ggml.h beside this file).
 */
#pragma once
#include "ggml.h"

typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_sched *ggml_backend_sched_t;

#ifdef __cplusplus
extern "C" {
#endif

void ggml_backend_tensor_set(struct ggml_tensor *tensor, const void *data, size_t offset, size_t size);
void ggml_backend_tensor_get(const struct ggml_tensor *tensor, void *data, size_t offset, size_t size);
void ggml_backend_tensor_memset(struct ggml_tensor *tensor, uint8_t value, size_t offset, size_t size);
ggml_backend_sched_t ggml_backend_sched_new(ggml_backend_t *backends, ggml_backend_buffer_type_t *bufts,
                                            int n_backends, size_t graph_size, bool parallel, bool op_offload);
void ggml_backend_sched_free(ggml_backend_sched_t sched);
void ggml_backend_sched_reset(ggml_backend_sched_t sched);
bool ggml_backend_sched_alloc_graph(ggml_backend_sched_t sched, struct ggml_cgraph *graph);
enum ggml_status ggml_backend_sched_graph_compute(ggml_backend_sched_t sched, struct ggml_cgraph *graph);
void ggml_backend_sched_set_tensor_backend(ggml_backend_sched_t sched, struct ggml_tensor *node,
                                           ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
