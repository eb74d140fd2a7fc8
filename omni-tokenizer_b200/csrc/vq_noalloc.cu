// vq_noalloc.cu -- a VQ argmin entry point that allocates nothing.
//
// omni_b200_vq_argmin() needs 8 bytes of device scratch per row, which its
// caller passes in.  Some callers cannot obtain that memory themselves:
//   * processes whose device memory is owned by a caching allocator or an
//     inference engine that reserves nearly all of HBM up front (PyTorch's
//     caching allocator, vLLM-style KV-cache reservations) -- a raw cudaMalloc
//     from inside such a process either fails or fragments the pool, and the
//     C caller has no handle on the owning allocator;
//   * latency-bound streaming callers (live audio tokenisation) that must not
//     call cudaMalloc/cudaFree in their serving loop, because those calls can
//     block on, and cudaFree can synchronise, the whole device.
// For them this file keeps the scratch in a file-scope device array that
// every GPU loading the library holds until process exit, and
// omni_b200_vq_argmin_noalloc() runs the same kernels as
// omni_b200_vq_argmin() against it.  Nothing here calls cudaMalloc, cudaFree
// or an allocating library routine.
#include "omni_b200.h"
#include "vq.h"

#include <cuda_runtime.h>
#include <mutex>
#include <string>

namespace omni_b200 {
int ctx_fail(int code, const char *msg);
void ctx_clear();
int *kernel_error_word();
int launch_status(int rc, const char *what);

namespace {
// Fixed scratch: one 64-bit (distance, id) key per row, 512 KiB per device.
constexpr size_t kNoAllocMaxRows = 65536;
static __device__ __align__(256) unsigned long long g_noalloc_keys[kNoAllocMaxRows];

constexpr int kMaxDevices = 64;
void *g_noalloc_ptr[kMaxDevices];
std::mutex g_noalloc_mutex;

// In host code `g_noalloc_keys` only names a host-side stand-in for the
// symbol; the device address must be queried per device, with that device
// current.  Done once per device, on that device's first call.
void *noalloc_scratch(int *status) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = ctx_fail(4, "vq_argmin_noalloc: no usable CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> guard(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_keys);
        if (e != cudaSuccess || !p) {
            *status = ctx_fail(7, (std::string("vq_argmin_noalloc: cudaGetSymbolAddress failed: ") +
                                   cudaGetErrorString(e))
                                      .c_str());
            return nullptr;
        }
        g_noalloc_ptr[dev] = p;
    }
    *status = 0;
    return g_noalloc_ptr[dev];
}
} // namespace
} // namespace omni_b200

using namespace omni_b200;

extern "C" int omni_b200_vq_argmin_noalloc(const void *x, const void *codebook,
                                           const void *cbnorm, void *ids, size_t rows,
                                           size_t dim, size_t codes, int profile, int ids_u16,
                                           void *stream) {
    ctx_clear();
    if (!x || !codebook || !cbnorm || !ids)
        return ctx_fail(1, "vq_argmin_noalloc: null pointer");
    if (rows == 0)
        return 0;
    if (rows > kNoAllocMaxRows)
        return ctx_fail(1, ("vq_argmin_noalloc: " + std::to_string(rows) +
                            " rows exceed the fixed scratch of " +
                            std::to_string(kNoAllocMaxRows) +
                            " rows; split the batch or use omni_b200_vq_argmin")
                               .c_str());
    if (dim == 0 || codes == 0 || codes > 65536)
        return ctx_fail(1, "vq_argmin_noalloc: need dim > 0 and 0 < codes <= 65536");
    if (profile != OMNI_B200_BF16)
        return ctx_fail(4, "vq_argmin_noalloc: only the BF16 profile runs without scratch; use omni_b200_vq_argmin");
    if (dim % 8 != 0 || dim > 128)
        return ctx_fail(4, "vq_argmin_noalloc: dim must be a multiple of 8 and at most 128");
    const uintptr_t align = reinterpret_cast<uintptr_t>(x) |
                            reinterpret_cast<uintptr_t>(codebook) |
                            reinterpret_cast<uintptr_t>(cbnorm);
    if (align % 16 != 0)
        return ctx_fail(1, "vq_argmin_noalloc: x, codebook and cbnorm must be 16-byte aligned");
    int status = 0;
    void *keys = noalloc_scratch(&status);
    if (!keys)
        return status;
    VqArgs a;
    a.x = x;
    a.codebook = codebook;
    a.cbnorm = cbnorm;
    a.rows = static_cast<int>(rows);
    a.dim = static_cast<int>(dim);
    a.codes = static_cast<int>(codes);
    a.keys = keys; // re-initialised to "no candidate" by the launch before use
    a.ids = ids;
    a.ids_u16 = ids_u16 ? 1 : 0;
    a.err = kernel_error_word();
    if (!a.err)
        return ctx_fail(7, "vq_argmin_noalloc: no CUDA device");
    return launch_status(vq_bf16_launch(a, static_cast<cudaStream_t>(stream)),
                         "vq_argmin_noalloc");
}
