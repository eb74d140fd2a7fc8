/* omni_abi.h -- the outer C ABI of omni-tokenizer, implemented by
 * libomni_b200.so on B200 GPUs.
 *
 * Same 15 entry points, status codes and structures as the reference's
 * include/omni/omni.h:18-87, so that the reference's Python binding
 * (python/omni_tokenizer/native.py:36-139, loaded through OMNI_LIBRARY) and C
 * callers can use this library unchanged.  Only the CUDA backend (OMNI_CUDA)
 * exists here; OMNI_CPU is answered with OMNI_UNSUPPORTED.  Model files are the
 * reference's OMNIVQ01 format (src/model.cpp:96-205).
 *
 * Behaviour kept from the reference (src/runtime.cpp):
 *   - error text is thread local, valid until the next call on that thread;
 *   - a context retains its model after omni_model_free;
 *   - one inference per context at a time (a concurrent call fails with
 *     OMNI_INVALID_ARGUMENT); contexts share a model's weights;
 *   - omni_context_cancel is an atomic store checked between layers;
 *   - *count is set on success, or to the required capacity;
 *   - omni_encode_image with codes == NULL, capacity == 0 reports the count
 *     with OMNI_INVALID_ARGUMENT without reading pixels. */
#ifndef OMNI_B200_ABI_H
#define OMNI_B200_ABI_H

#include <stddef.h>
#include <stdint.h>

#define OMNI_ABI_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

typedef struct omni_model omni_model;
typedef struct omni_context omni_context;
typedef void (*omni_trace_callback)(void *user, const char *stage, const float *values, size_t rows,
                                    size_t columns);

enum omni_status {
    OMNI_OK = 0,
    OMNI_INVALID_ARGUMENT = 1,
    OMNI_IO_ERROR = 2,
    OMNI_INVALID_MODEL = 3,
    OMNI_UNSUPPORTED = 4,
    OMNI_OUT_OF_MEMORY = 5,
    OMNI_CANCELLED = 6,
    OMNI_INTERNAL_ERROR = 7
};
enum omni_backend { OMNI_CPU = 0, OMNI_CUDA = 1 };
enum omni_kind { OMNI_AUDIO = 1, OMNI_IMAGE = 2 };

typedef struct omni_model_info {
    uint32_t struct_size;
    uint32_t kind;
    uint32_t layers;
    uint32_t width;
    uint32_t heads;
    uint32_t code_dim;
    uint32_t vocabulary_size;
    uint32_t backend;
    uint64_t weight_bytes;
} omni_model_info;

OMNI_ABI_API const char *omni_last_error(void);
OMNI_ABI_API const char *omni_version(void);
OMNI_ABI_API int omni_has_cuda(void);
OMNI_ABI_API int omni_model_load(const char *path, int backend, int device, omni_model **out);
OMNI_ABI_API void omni_model_free(omni_model *model);
OMNI_ABI_API int omni_model_get_info(const omni_model *model, omni_model_info *out);
OMNI_ABI_API int omni_context_create(omni_model *model, omni_context **out);
OMNI_ABI_API void omni_context_free(omni_context *context);
OMNI_ABI_API void omni_context_cancel(omni_context *context);
OMNI_ABI_API void omni_context_reset_cancel(omni_context *context);
OMNI_ABI_API int omni_context_set_trace(omni_context *context, omni_trace_callback callback,
                                        void *user);
/* mel: [mel_channels, frames] fp32, frames % 8 == 0, frames <= 3000;
 * codes_needed = ceil(valid_frames / 8). */
OMNI_ABI_API int omni_encode_audio(omni_context *context, const float *mel, uint32_t frames,
                                   uint32_t valid_frames, uint16_t *codes, size_t capacity,
                                   size_t *count);
/* pixels: RGB CHW fp32 in [-1, 1]; height and width multiples of the patch size;
 * codes in row-major (height / patch, width / patch) order. */
OMNI_ABI_API int omni_encode_image(omni_context *context, const float *pixels, uint32_t height,
                                   uint32_t width, uint16_t *codes, size_t capacity,
                                   size_t *count);
/* The last pre-VQ features as fp32 [code_count, code_dim] (image: L2 normalised). */
OMNI_ABI_API int omni_context_copy_features(omni_context *context, float *output, size_t capacity,
                                            size_t *count);
/* Peak device workspace of the context (activations and scratch; not weights). */
OMNI_ABI_API uint64_t omni_context_peak_workspace(const omni_context *context);

/* Batched extension of this library (not part of the reference's omni.h):
 * `items` inputs of one shape per call, stacked into large GEMMs and one
 * attention launch per layer; results equal the per-item calls'.  Inputs may be
 * host or device memory (device memory of the model's device is read in
 * place).  Codes are each item's codes concatenated in item order (*count =
 * their total); omni_context_copy_features then returns all items' features
 * stacked the same way.  Non-finite input fails with OMNI_INVALID_ARGUMENT.
 *
 * mel: [items, mel_channels, frames] fp32; valid_frames[items], each in
 * (0, frames]; item i has ceil(valid_frames[i] / 8) codes. */
OMNI_ABI_API int omni_b200_encode_audio_batch(omni_context *context, const float *mel, uint32_t items,
                                              uint32_t frames, const uint32_t *valid_frames,
                                              uint16_t *codes, size_t capacity, size_t *count);
/* pixels: [items, 3, height, width] fp32; (height / patch) * (width / patch)
 * codes per image. */
OMNI_ABI_API int omni_b200_encode_images(omni_context *context, const float *pixels, uint32_t items,
                                         uint32_t height, uint32_t width, uint16_t *codes,
                                         size_t capacity, size_t *count);

/* Repeated batched calls run as a CUDA graph: when a call has the same entry
 * point, shapes, valid lengths and input address as the previous call, and
 * its input is device memory or page-locked host memory, and no trace
 * callback is set, the context captures the call's device work into a graph
 * (outputs in buffers the graph keeps) and replays that graph for later calls
 * with the same key -- the whole graph is recomputed from the input each time.
 * Cancellation is checked before a replay starts and by the VQ kernels inside
 * it.  OMNI_B200_GRAPHS=0 (read when the context is created) keeps every call
 * eager.  This counter is the number of graph launches of the context. */
OMNI_ABI_API uint64_t omni_b200_context_graph_launches(const omni_context *context);

#ifdef __cplusplus
}
#endif
#endif
