/* omni_b200.h -- op-level C ABI of the B200 (sm_100a) hot path.
 *
 * Plain pointers and sizes only.  Device pointers are CUDA device addresses on
 * the caller's current device; `stream` is a cudaStream_t passed as void*
 * (NULL = the legacy default stream).  Every function returns an
 * omni_status code (include/omni/omni.h: 0 OK, 1 INVALID_ARGUMENT,
 * 4 UNSUPPORTED, 5 OUT_OF_MEMORY, 7 INTERNAL_ERROR) and leaves a message in
 * omni_b200_last_error() (thread local, valid until the next call on that
 * thread).  Launches are asynchronous; kernel-side failures (a bounded
 * pipeline wait that gave up) are reported by omni_b200_sync_check().
 *
 * These entry points are the batched/op-level form of the reference's inner
 * backend interface omni::Ops (omni-tokenizer src/internal.h:52-90); the
 * reference exposes that interface only to C++ (make_cuda(), used by
 * tests/native_cuda_attention.cpp:24-41).  A consumer binds them the same way
 * the reference's python/omni_tokenizer/native.py binds omni.h: one ctypes (or
 * cgo / JNI) declaration per entry point, status codes checked after each call.
 */
#ifndef OMNI_B200_H
#define OMNI_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define OMNI_B200_API __declspec(dllexport)
#else
#define OMNI_B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of tensors crossing this ABI. */
enum omni_b200_dtype { OMNI_B200_F32 = 0, OMNI_B200_BF16 = 1, OMNI_B200_F16 = 2 };

OMNI_B200_API const char *omni_b200_last_error(void);
OMNI_B200_API const char *omni_b200_version(void);

/* Synchronises `stream`, then reads and clears the current device's kernel
 * error word.  Returns OMNI_INTERNAL_ERROR (7) if any kernel gave up a wait. */
OMNI_B200_API int omni_b200_sync_check(void *stream);

/* Batched attention on head-major tensors q, k, v, out of shape
 * [batch, heads, L, head_dim], dtype BF16 or F16 (out may also be F32):
 *   out[b,h,t,:] = softmax(scale * q[b,h,t,:] . k[b,h,s,:]) over s < limit(b,t)
 * with limit(b,t) = min(L, lengths[b] (or L when lengths == NULL),
 *                       block > 0 ? (t/block + 1)*block : inf).
 * scale <= 0 selects head_dim^-1/2.  lengths is a DEVICE int32[batch]
 * (key-padding mask for variable-length segments).  With skip_padded_queries
 * != 0, 256-row query blocks lying wholly at or beyond lengths[b] are not
 * computed and their output rows are left untouched.
 * Generalises Ops::attention (omni-tokenizer src/internal.h:81-82) from one
 * sequence of heads*head_dim columns to a batch of head-major sequences;
 * head_dim 1..128 (64, 72 and 96 on the fast path with no repacking). */
OMNI_B200_API int omni_b200_attention_bhld(const void *q, const void *k, const void *v, void *out,
                                           int batch, int heads, int L, int head_dim, int dtype,
                                           int out_dtype, const int32_t *lengths, int block,
                                           int skip_padded_queries, float scale, void *stream);

/* Ops::attention (omni-tokenizer src/internal.h:81-82, semantics of
 * src/cpu.cpp:122-172) on the reference's row-major Value layout:
 *   unfused: q, k, v are [n, heads*head_dim];
 *   fused:   q is [n, 3*heads*head_dim] holding Q|K|V column blocks, k = v = NULL.
 * out is [n, heads*head_dim] of out_dtype.  dtype F32 inputs (the audio fp32
 * profile) and layouts that TMA cannot address directly are repacked into
 * `workspace` first.  With 16-bit operands and fewer (query block, head)
 * items than fill the last round of SMs, the kernel also splits
 * that round's items along the keys and merges the parts in a second pass,
 * using scratch after the repacked operands.  omni_b200_attention_rows_workspace()
 * gives the bytes for both (0 when neither is needed); a smaller workspace,
 * or none, runs without the split and with the same results up to rounding. */
OMNI_B200_API size_t omni_b200_attention_rows_workspace(size_t n, int heads, int head_dim,
                                                        int dtype, int fused);
OMNI_B200_API int omni_b200_attention_rows(const void *q, const void *k, const void *v, void *out,
                                           size_t n, int heads, int head_dim, size_t block,
                                           size_t valid, int fused, int dtype, int out_dtype,
                                           void *workspace, size_t workspace_bytes,
                                           void *stream);

/* `batch` sequences of n tokens stacked as batch*n rows (the layout above per
 * sequence), the keys of sequence b limited to lengths[b] (device int32; NULL:
 * `valid` for every sequence) and to the block window: what the encoder graphs
 * run for a batch of audio segments or images.  Workspace as above, from
 * omni_b200_attention_rows_batch_workspace(). */
OMNI_B200_API size_t omni_b200_attention_rows_batch_workspace(size_t n, int batch, int heads,
                                                              int head_dim, int dtype, int fused);
OMNI_B200_API int omni_b200_attention_rows_batch(const void *q, const void *k, const void *v,
                                                 void *out, size_t n, int batch, int heads,
                                                 int head_dim, size_t block, size_t valid,
                                                 const int32_t *lengths, int fused, int dtype,
                                                 int out_dtype, void *workspace,
                                                 size_t workspace_bytes, void *stream);

/* Ops::gelu (omni-tokenizer src/internal.h:77, semantics of src/cpu.cpp:91-96),
 * in place on n elements of dtype (F32 or BF16): x = r(0.5 x (1 + erf(x *
 * 0.70710678...))), each step an fp32 operation, r the rounding to bf16 for
 * BF16.  bf16 inputs are looked up in a table built once per device from that
 * expression (the first call on a device builds it and synchronises the stream). */
OMNI_B200_API int omni_b200_gelu(void *x, size_t n, int dtype, void *stream);

/* Ops::squares (omni-tokenizer src/internal.h:86, semantics of
 * src/cpu.cpp:216-226): out[r] = sum over columns in order of x[r,j]^2, with
 * every square and the total rounded to bf16 when dtype is BF16.  x is
 * [rows, cols] of dtype (F32 or BF16); out is [rows] of out_dtype. */
OMNI_B200_API int omni_b200_squares(const void *x, void *out, size_t rows, size_t cols, int dtype,
                                    int out_dtype, void *stream);

/* Ops::quantize (omni-tokenizer src/internal.h:87-88, semantics of
 * src/cpu.cpp:227-287): ids[r] = argmin over codes c of the profile's
 * expanded L2 distance between x[r,:] and codebook[c,:], smallest id on ties.
 * profile BF16: x, codebook and cbnorm (= squares(codebook), see above) are
 * bf16; dist = bf16(bf16(|x|^2 + |c|^2) - bf16(2 bf16(x.c))); dim % 8 == 0.
 * profile F32: x, codebook and cbnorm are fp32 (cbnorm = squares(codebook));
 * the result is the reference's: the code with the smallest direct fp64
 * distance sum_k (x_k - c_k)^2 among the codes whose expanded-L2 distance lies
 * within the error bound of the best one (src/cpu.cpp:260-283); dim % 4 == 0.
 * ids are uint16 (ids_u16 != 0, as the reference returns) or int32.
 * workspace: omni_b200_vq_workspace() bytes of device memory (BF16 with
 * dim <= 128: 8 per row; BF16 with larger dim: 12 per row; F32: 144 per row).
 * x, codebook, cbnorm must be 16-byte aligned; codes <= 65536, dim <= 65536. */
OMNI_B200_API size_t omni_b200_vq_workspace(size_t rows, size_t dim, size_t codes, int profile);
OMNI_B200_API int omni_b200_vq_argmin(const void *x, const void *codebook, const void *cbnorm,
                                      void *ids, size_t rows, size_t dim, size_t codes,
                                      int profile, int ids_u16, void *workspace,
                                      size_t workspace_bytes, void *stream);

/* omni_b200_vq_argmin with the reference's cancellation contract
 * (Ops::quantize(x, cb, cbnorm, std::atomic<bool>& cancel), omni-tokenizer
 * src/internal.h:87-88; its CUDA backend polls the flag before every 1024-code
 * tile, src/cuda.cu:946-948).  cancel points at an int the device can read --
 * mapped pinned host memory (cudaHostAlloc with cudaHostAllocMapped; pass the
 * device pointer from cudaHostGetDevicePointer) or device memory -- that the
 * caller sets to nonzero to cancel; NULL behaves as omni_b200_vq_argmin.  With
 * a flag, the wide (dim > 128) and fp32 passes run the codebook in windows of
 * 4096 codes (a multiple of 4096 when the rows are too few for one window to
 * give every SM two units of work), one launch each; the flag is copied to the
 * workspace in stream order before each window, and a window whose copy is
 * nonzero is skipped.  The call is asynchronous like the others: after
 * synchronising, a caller that set the flag discards ids and reports
 * OMNI_CANCELLED, as Ops::quantize throws Error(OMNI_CANCELLED). */
OMNI_B200_API int omni_b200_vq_argmin_cancellable(const void *x, const void *codebook, const void *cbnorm,
                                                  void *ids, size_t rows, size_t dim, size_t codes,
                                                  int profile, int ids_u16, void *workspace,
                                                  size_t workspace_bytes, const int *cancel, void *stream);

/* omni_b200_vq_argmin without caller-provided scratch.  No counterpart in the
 * reference (its Ops::quantize allocates from the context's Pool).  For callers
 * that cannot allocate device memory: processes whose HBM is owned by another
 * allocator (a caching allocator or an engine that reserves nearly all of it),
 * and streaming callers that must not call cudaMalloc/cudaFree in their serving
 * loop.  The 8-byte-per-row scratch lives in a fixed device array of 65536
 * rows (512 KiB per device, held by every GPU that loads this library until
 * exit); more rows are rejected with INVALID_ARGUMENT.  The caller still passes
 * x, codebook, cbnorm and ids (same meaning as omni_b200_vq_argmin; BF16
 * profile with dim <= 128 only, other shapes are rejected).  The first
 * call on a device looks up that device's address of the array
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Every call shares the one array: the launch re-initialises the rows it uses,
 * but calls that overlap on the GPU (other streams or threads) race on it. */
OMNI_B200_API int omni_b200_vq_argmin_noalloc(const void *x, const void *codebook,
                                              const void *cbnorm, void *ids, size_t rows,
                                              size_t dim, size_t codes, int profile,
                                              int ids_u16, void *stream);

/* ---- Diagnostics (failure detection without a GPU fault) ----------------
 * Every pipeline wait in this library's kernels is bounded: a wait that has
 * not completed after 2 s records a bit in the current device's kernel error
 * word and lets the kernel end, so a broken pipeline shows up as
 * OMNI_INTERNAL_ERROR from omni_b200_sync_check instead of a hang.  The word
 * is per device, not per call or context: a check on any stream of the device
 * reads and clears it.  No counterpart in the reference (its kernels are
 * library templates without device-side waits).
 *
 * omni_b200_wait_selftest runs that bounded wait on a barrier that nothing
 * completes, with a limit of limit_us microseconds (1 .. 2000000): the kernel
 * gives up, records bit 0x200 and returns; the next omni_b200_sync_check on
 * `stream` reports OMNI_INTERNAL_ERROR, and the device stays usable.
 *
 * omni_b200_debug_fail_allocations makes the next `count` device allocations
 * of this library (host-buffer contexts, encoder contexts and model loads)
 * fail as out of memory without reaching the allocator (0 turns it off).  The
 * encoder contexts trim their memory pool and retry a failed allocation once,
 * as the reference's Pool does (src/cuda.cu:515-527), so one injected failure
 * is absorbed and two surface as OMNI_OUT_OF_MEMORY. */
OMNI_B200_API int omni_b200_wait_selftest(unsigned limit_us, void *stream);
OMNI_B200_API void omni_b200_debug_fail_allocations(int count);

/* ---- Host-buffer entry points -------------------------------------------
 * A context owns one CUDA device, one stream and grow-only device buffers
 * (the role of omni_context in omni-tokenizer src/runtime.cpp:200-211).  The
 * *_host calls take HOST pointers (pinned memory gives full copy bandwidth),
 * copy inputs to the device, run the kernel, copy results back and
 * synchronise.  One call per context at a time: a concurrent call fails with
 * INVALID_ARGUMENT, as in src/runtime.cpp:152-163. */
typedef struct omni_b200_context omni_b200_context;
OMNI_B200_API int omni_b200_context_create(int device, omni_b200_context **out);
OMNI_B200_API void omni_b200_context_free(omni_b200_context *context);
/* Peak bytes of device buffers this context has held. */
OMNI_B200_API uint64_t omni_b200_context_peak_workspace(const omni_b200_context *context);
/* omni_b200_attention_bhld on host tensors; lengths (optional) is a HOST int32[batch]. */
OMNI_B200_API int omni_b200_attention_bhld_host(omni_b200_context *context, const void *q,
                                                const void *k, const void *v, void *out,
                                                int batch, int heads, int L, int head_dim,
                                                int dtype, int out_dtype, const int32_t *lengths,
                                                int block, int skip_padded_queries, float scale);
/* omni_b200_vq_argmin on host tensors; cbnorm may be NULL (computed on the device). */
OMNI_B200_API int omni_b200_vq_argmin_host(omni_b200_context *context, const void *x,
                                           const void *codebook, const void *cbnorm, void *ids,
                                           size_t rows, size_t dim, size_t codes, int profile,
                                           int ids_u16);

#ifdef __cplusplus
}
#endif
#endif
