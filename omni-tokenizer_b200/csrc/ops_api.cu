// ops_api.cu -- extern "C" op-level entry points declared in include/omni_b200.h.
#include "omni_b200.h"

#include "fmha.h"
#include "graph_kernels.h"
#include "norms.h"
#include "pack.h"
#include "sm100.cuh"
#include "vq.h"

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cuda_runtime.h>
#include <mutex>
#include <string>

namespace omni_b200 {

// Per-device kernel error word: a kernel whose bounded wait gives up ORs a bit
// into it.  File-scope device storage, so no allocation is needed.
__device__ int g_kernel_error;

namespace {
thread_local std::string g_error;

int fail(int code, const std::string &msg) {
    g_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    g_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? 5 : 7;
}

constexpr int kMaxDevices = 64;
int *g_err_ptr[kMaxDevices];
std::mutex g_err_mutex;
} // namespace

// Device address of the error word on the current device.
int *kernel_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return nullptr;
    std::lock_guard<std::mutex> guard(g_err_mutex);
    if (!g_err_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_kernel_error) != cudaSuccess)
            return nullptr;
        g_err_ptr[dev] = static_cast<int *>(p);
    }
    return g_err_ptr[dev];
}

// Test hook: the next g_fail_allocations device allocations made by this
// library report cudaErrorMemoryAllocation without reaching the allocator.
std::atomic<int> g_fail_allocations{0};
bool injected_allocation_failure() {
    int n = g_fail_allocations.load();
    while (n > 0 && !g_fail_allocations.compare_exchange_weak(n, n - 1)) {
    }
    return n > 0;
}

// The pipeline kernels' bounded wait on an mbarrier that nothing completes: it
// gives up after limit_ns, records kErrWaitSelfTest in the error word and
// returns (no trap, no fault, no hang).
__global__ void wait_selftest_kernel(int *err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    mbar_wait(&bar, 0, err, kErrWaitSelfTest, limit_ns);
    __syncthreads();
}

int ctx_fail(int code, const char *msg) { return fail(code, msg); }
// Clears this thread's error message (every entry point starts with it).
void ctx_clear() { g_error.clear(); }

int launch_status(int rc, const char *what) {
    if (rc == 0)
        return 0;
    if (rc == -2)
        return fail(4, std::string(what) + ": unsupported head dimension");
    if (rc == -1)
        return fail(7, std::string(what) + ": cuTensorMapEncodeTiled is unavailable");
    if (rc >= 1000)
        return fail(7, std::string(what) + ": tensor map encoding failed (CUresult " +
                           std::to_string(rc - 1000) + ")");
    return cuda_fail(static_cast<cudaError_t>(rc), what);
}

} // namespace omni_b200


namespace omni_b200 {

size_t attention_rows_workspace(size_t rows, int heads, int head_dim, int dtype, int fused) {
    if (heads <= 0 || rows == 0)
        return 0;
    const long long d = static_cast<long long>(heads) * head_dim;
    const long long s_token = fused ? 3 * d : d;
    if (dtype == OMNI_B200_F32) {
        // fp32 kernel: TMA reads rows whose head slices start on 16 bytes.
        const int hdp = padded_head_dim_f32(head_dim);
        if (hdp < 0 || (head_dim % 4 == 0 && head_dim >= 32 && s_token % 4 == 0))
            return 0;
        const size_t one = (rows * static_cast<size_t>(heads) * hdp * 4 + 255) / 256 * 256;
        return 3 * one;
    }
    const int hdp = padded_head_dim(head_dim);
    if (hdp < 0)
        return 0;
    const bool direct = head_dim % 8 == 0 && s_token % 8 == 0;
    if (direct)
        return 0;
    const size_t one = (rows * static_cast<size_t>(heads) * hdp * 2 + 255) / 256 * 256;
    return 3 * one;
}

// fp32 operands: the split-precision kernel (no conversion to 16-bit types),
// reading the rows in place or from an fp32 packed copy.
int attention_rows_f32(const void *qp, const void *kp, const void *vp, void *out, size_t n, int batch,
                       int heads, int head_dim, long long s_token, size_t block, size_t valid,
                       const int *lengths, int out_dtype, void *workspace, size_t workspace_bytes,
                       cudaStream_t s) {
    const int hdp = padded_head_dim_f32(head_dim);
    if (hdp < 0)
        return fail(4, "attention_rows: fp32 head_dim above 128 is not supported");
    const size_t rows = n * static_cast<size_t>(batch);
    const long long d = static_cast<long long>(heads) * head_dim;
    TensorView view;
    view.d = head_dim;
    view.tokens = static_cast<int>(n);
    view.heads = heads;
    view.batch = batch;
    view.s_token = s_token;
    view.s_head = head_dim;
    view.s_batch = s_token * static_cast<long long>(n);
    FmhaArgs a;
    // In place when every 32-column box starts inside the head (head_dim >= 32)
    // and the rows are 16-byte aligned; otherwise an fp32 packed copy.
    const bool direct = head_dim % 4 == 0 && head_dim >= 32 && tma_view_ok_f32(qp, view) &&
                        tma_view_ok_f32(kp, view) && tma_view_ok_f32(vp, view);
    if (direct) {
        a.q_ptr = qp;
        a.k_ptr = kp;
        a.v_ptr = vp;
        a.q = a.k = a.v = view;
    } else {
        const size_t one = (rows * static_cast<size_t>(heads) * hdp * 4 + 255) / 256 * 256;
        if (!workspace || workspace_bytes < 3 * one)
            return fail(1, "attention_rows: workspace too small (need " + std::to_string(3 * one) + " bytes)");
        char *w = static_cast<char *>(workspace);
        const void *src[3] = {qp, kp, vp};
        for (int i = 0; i < 3; ++i) {
            const int rc = pack_heads_f32(static_cast<const float *>(src[i]), s_token, head_dim,
                                          static_cast<int>(rows), heads, head_dim, hdp,
                                          reinterpret_cast<float *>(w + i * one), s);
            if (rc)
                return cuda_fail(static_cast<cudaError_t>(rc), "attention_rows: pack");
        }
        TensorView pv;
        pv.d = hdp;
        pv.tokens = static_cast<int>(n);
        pv.heads = heads;
        pv.batch = batch;
        pv.s_token = hdp;
        pv.s_head = static_cast<long long>(rows) * hdp;
        pv.s_batch = static_cast<long long>(n) * hdp;
        a.q_ptr = w;
        a.k_ptr = w + one;
        a.v_ptr = w + 2 * one;
        a.q = a.k = a.v = pv;
    }
    a.out = out;
    a.out_dtype = out_dtype;
    a.o_st = d;
    a.o_sh = head_dim;
    a.o_sb = d * static_cast<long long>(n);
    a.lengths = lengths;
    a.valid = valid > n || valid == 0 ? static_cast<int>(n) : static_cast<int>(valid);
    a.block = block > n ? static_cast<int>(n) : static_cast<int>(block);
    a.skip_padded_q = 0;
    a.scale = 1.0 / std::sqrt(static_cast<double>(head_dim));
    a.out_d = head_dim;
    a.err = kernel_error_word();
    if (!a.err)
        return fail(7, "attention_rows: no CUDA device");
    return launch_status(fmha_f32_launch(a, s), "attention_rows");
}

// `batch` sequences of n tokens stacked as batch*n rows.  Items are contiguous
// along the token axis, so the packed copy [heads, batch*n, hdp] is also a
// (hdp, n, heads, batch) view with s_batch = n*hdp.
size_t attention_rows_split_workspace(size_t n, int batch, int heads, int head_dim, size_t block,
                                      size_t valid, int dtype) {
    if (dtype == OMNI_B200_F32 || n == 0 || n > (1u << 30))
        return 0;
    const int ni = static_cast<int>(n);
    return fmha_split_workspace(batch, heads, ni, head_dim,
                                valid > n || valid == 0 ? ni : static_cast<int>(valid),
                                block > n ? ni : static_cast<int>(block), 0);
}

// Repacking bytes (attention_rows_workspace) rounded up to 256, then the key
// split scratch: the layout of the workspace that the C ABI's queries size.
size_t rows_workspace_total(size_t n, int batch, int heads, int head_dim, int dtype, int fused) {
    const size_t pack = attention_rows_workspace(n * static_cast<size_t>(batch), heads, head_dim, dtype, fused);
    const size_t split = attention_rows_split_workspace(n, batch, heads, head_dim, 0, n, dtype);
    return split ? (pack + 255) / 256 * 256 + split : pack;
}

int attention_rows(const void *q, const void *k, const void *v, void *out, size_t n, int batch,
                   int heads, int head_dim, size_t block, size_t valid, const int *lengths,
                   int fused, int dtype, int out_dtype, void *workspace, size_t workspace_bytes,
                   cudaStream_t s, void *split_ws, size_t split_ws_bytes) {
    g_error.clear();
    if (!q || !out || (!fused && (!k || !v)))
        return fail(1, "attention_rows: null tensor pointer");
    if (n == 0 || batch <= 0 || heads <= 0 || head_dim <= 0 || (valid == 0 && !lengths) ||
        n * static_cast<size_t>(batch) > (1u << 30))
        return fail(1, "attention_rows: sizes must be positive");
    if (dtype < OMNI_B200_F32 || dtype > OMNI_B200_F16 || out_dtype < OMNI_B200_F32 ||
        out_dtype > OMNI_B200_F16)
        return fail(1, "attention_rows: invalid dtype");
    const size_t rows = n * static_cast<size_t>(batch);
    const long long d = static_cast<long long>(heads) * head_dim;
    const long long s_token = fused ? 3 * d : d;
    const void *qp = q, *kp = fused ? static_cast<const char *>(q) + d * (dtype ? 2 : 4) : k,
               *vp = fused ? static_cast<const char *>(q) + 2 * d * (dtype ? 2 : 4) : v;
    if (dtype == OMNI_B200_F32)
        return attention_rows_f32(qp, kp, vp, out, n, batch, heads, head_dim, s_token, block, valid, lengths,
                                  out_dtype, workspace, workspace_bytes, s);
    const int hdp = padded_head_dim(head_dim);
    if (hdp < 0)
        return fail(4, "attention_rows: head_dim above 128 is not supported");
    FmhaArgs a;
    TensorView view;
    view.d = head_dim;
    view.tokens = static_cast<int>(n);
    view.heads = heads;
    view.batch = batch;
    view.s_token = s_token;
    view.s_head = head_dim;
    view.s_batch = s_token * static_cast<long long>(n);
    const size_t need = attention_rows_workspace(rows, heads, head_dim, dtype, fused);
    const bool direct = need == 0 && tma_view_ok(qp, view) && tma_view_ok(kp, view) &&
                        tma_view_ok(vp, view);
    size_t used = 0; // workspace bytes taken by the repacked operands
    if (direct) {
        a.q_ptr = qp;
        a.k_ptr = kp;
        a.v_ptr = vp;
        a.q = a.k = a.v = view;
        a.bf16 = dtype == OMNI_B200_BF16;
    } else {
        const size_t one = (rows * static_cast<size_t>(heads) * hdp * 2 + 255) / 256 * 256;
        if (!workspace || workspace_bytes < 3 * one)
            return fail(1, "attention_rows: workspace too small (need " +
                               std::to_string(3 * one) + " bytes)");
        char *w = static_cast<char *>(workspace);
        used = 3 * one;
        const void *src[3] = {qp, kp, vp};
        for (int i = 0; i < 3; ++i) {
            const int rc = pack_heads(src[i], dtype, s_token, head_dim, static_cast<int>(rows), heads,
                                      head_dim, hdp, w + i * one, s);
            if (rc)
                return cuda_fail(static_cast<cudaError_t>(rc), "attention_rows: pack");
        }
        TensorView pv;
        pv.d = hdp;
        pv.tokens = static_cast<int>(n);
        pv.heads = heads;
        pv.batch = batch;
        pv.s_token = hdp;
        pv.s_head = static_cast<long long>(rows) * hdp;
        pv.s_batch = static_cast<long long>(n) * hdp;
        a.q_ptr = w;
        a.k_ptr = w + one;
        a.v_ptr = w + 2 * one;
        a.q = a.k = a.v = pv;
        a.bf16 = dtype == OMNI_B200_BF16;
    }
    a.out = out;
    a.out_dtype = out_dtype;
    a.o_st = d;
    a.o_sh = head_dim;
    a.o_sb = d * static_cast<long long>(n);
    a.lengths = lengths;
    a.valid = valid > n || valid == 0 ? static_cast<int>(n) : static_cast<int>(valid);
    a.block = block > n ? static_cast<int>(n) : static_cast<int>(block);
    a.skip_padded_q = 0;
    a.scale = 1.0 / std::sqrt(static_cast<double>(head_dim));
    a.out_d = head_dim; // packed operands are hdp wide; the output keeps head_dim
    a.err = kernel_error_word();
    a.split_ws = split_ws;
    a.split_ws_bytes = split_ws_bytes;
    if (!split_ws && workspace) {
        // The key split scratch follows the repacking bytes when the caller's
        // workspace has room for it (sized by rows_workspace_total).
        const size_t at = (used + 255) / 256 * 256;
        if (workspace_bytes > at) {
            a.split_ws = static_cast<char *>(workspace) + at;
            a.split_ws_bytes = workspace_bytes - at;
        }
    }
    if (!a.err)
        return fail(7, "attention_rows: no CUDA device");
    return launch_status(fmha_launch(a, s), "attention_rows");
}

} // namespace omni_b200

using namespace omni_b200;

extern "C" {

const char *omni_b200_last_error(void) { return g_error.c_str(); }

int omni_b200_wait_selftest(unsigned limit_us, void *stream) {
    g_error.clear();
    if (limit_us == 0 || limit_us > 2000000u)
        return fail(1, "wait_selftest: limit_us must be in [1, 2000000]");
    int *err = kernel_error_word();
    if (!err)
        return fail(7, "wait_selftest: no CUDA device");
    wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(err, 1000ull * limit_us);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(e, "wait_selftest");
}

void omni_b200_debug_fail_allocations(int count) { g_fail_allocations.store(count < 0 ? 0 : count); }
const char *omni_b200_version(void) { return "0.1.0+b200"; }

int omni_b200_sync_check(void *stream) {
    g_error.clear();
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess)
        return cuda_fail(e, "stream synchronize");
    int word = 0;
    e = cudaMemcpyFromSymbol(&word, g_kernel_error, sizeof(int));
    if (e != cudaSuccess)
        return cuda_fail(e, "read kernel error word");
    if (word != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_kernel_error, &zero, sizeof(int));
        return fail(7, "a kernel pipeline wait timed out (error bits 0x" + [&] {
            char buf[16];
            snprintf(buf, sizeof buf, "%x", word);
            return std::string(buf);
        }() + ")");
    }
    return 0;
}

int omni_b200_attention_bhld(const void *q, const void *k, const void *v, void *out, int batch,
                             int heads, int L, int head_dim, int dtype, int out_dtype,
                             const int32_t *lengths, int block, int skip_padded_queries,
                             float scale, void *stream) {
    g_error.clear();
    if (!q || !k || !v || !out)
        return fail(1, "attention_bhld: null tensor pointer");
    if (batch <= 0 || heads <= 0 || L <= 0 || head_dim <= 0 || block < 0)
        return fail(1, "attention_bhld: sizes must be positive");
    if (dtype != OMNI_B200_BF16 && dtype != OMNI_B200_F16 && dtype != OMNI_B200_F32)
        return fail(1, "attention_bhld: dtype must be BF16, F16 or F32");
    if (out_dtype < OMNI_B200_F32 || out_dtype > OMNI_B200_F16)
        return fail(1, "attention_bhld: invalid out_dtype");
    const bool f32 = dtype == OMNI_B200_F32;
    if (head_dim > 128 || head_dim % (f32 ? 4 : 8) != 0)
        return fail(4, f32 ? "attention_bhld: fp32 head_dim must be a multiple of 4 in [4, 128]"
                           : "attention_bhld: head_dim must be a multiple of 8 in [8, 128]");
    FmhaArgs a;
    a.q_ptr = q;
    a.k_ptr = k;
    a.v_ptr = v;
    TensorView view;
    view.d = head_dim;
    view.tokens = L;
    view.heads = heads;
    view.batch = batch;
    view.s_token = head_dim;
    view.s_head = static_cast<long long>(L) * head_dim;
    view.s_batch = view.s_head * heads;
    a.q = a.k = a.v = view;
    if (f32 ? (!tma_view_ok_f32(q, view) || !tma_view_ok_f32(k, view) || !tma_view_ok_f32(v, view))
            : (!tma_view_ok(q, view) || !tma_view_ok(k, view) || !tma_view_ok(v, view)))
        return fail(1, "attention_bhld: q, k and v must be 16-byte aligned");
    a.bf16 = dtype == OMNI_B200_BF16;
    a.out = out;
    a.out_dtype = out_dtype;
    a.o_st = head_dim;
    a.o_sh = view.s_head;
    a.o_sb = view.s_batch;
    a.lengths = lengths;
    a.valid = L;
    a.block = block;
    a.skip_padded_q = skip_padded_queries ? 1 : 0;
    a.scale = scale;
    a.err = kernel_error_word();
    if (!a.err)
        return fail(7, "attention_bhld: no CUDA device");
    if (f32)
        return launch_status(fmha_f32_launch(a, static_cast<cudaStream_t>(stream)), "attention_bhld");
    return launch_status(fmha_launch(a, static_cast<cudaStream_t>(stream)), "attention_bhld");
}

size_t omni_b200_attention_rows_workspace(size_t n, int heads, int head_dim, int dtype, int fused) {
    return rows_workspace_total(n, 1, heads, head_dim, dtype, fused);
}

int omni_b200_attention_rows(const void *q, const void *k, const void *v, void *out, size_t n,
                             int heads, int head_dim, size_t block, size_t valid, int fused,
                             int dtype, int out_dtype, void *workspace, size_t workspace_bytes,
                             void *stream) {
    return attention_rows(q, k, v, out, n, 1, heads, head_dim, block, valid, nullptr, fused, dtype,
                          out_dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t omni_b200_attention_rows_batch_workspace(size_t n, int batch, int heads, int head_dim, int dtype,
                                                int fused) {
    if (batch <= 0)
        return 0;
    return rows_workspace_total(n, batch, heads, head_dim, dtype, fused);
}

int omni_b200_attention_rows_batch(const void *q, const void *k, const void *v, void *out, size_t n,
                                   int batch, int heads, int head_dim, size_t block, size_t valid,
                                   const int32_t *lengths, int fused, int dtype, int out_dtype,
                                   void *workspace, size_t workspace_bytes, void *stream) {
    return attention_rows(q, k, v, out, n, batch, heads, head_dim, block, valid, lengths, fused, dtype,
                          out_dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int omni_b200_gelu(void *x, size_t n, int dtype, void *stream) {
    g_error.clear();
    if (!x && n)
        return fail(1, "gelu: null pointer");
    if (dtype != OMNI_B200_F32 && dtype != OMNI_B200_BF16)
        return fail(1, "gelu: dtype must be F32 or BF16");
    if (n == 0)
        return 0;
    const int rc = graph::gelu(x, dtype == OMNI_B200_BF16, n, static_cast<cudaStream_t>(stream));
    return rc ? cuda_fail(static_cast<cudaError_t>(rc), "gelu") : 0;
}

int omni_b200_squares(const void *x, void *out, size_t rows, size_t cols, int dtype, int out_dtype,
                      void *stream) {
    g_error.clear();
    if (!x || !out)
        return fail(1, "squares: null pointer");
    if ((dtype != OMNI_B200_F32 && dtype != OMNI_B200_BF16) ||
        (out_dtype != OMNI_B200_F32 && out_dtype != OMNI_B200_BF16))
        return fail(1, "squares: dtype must be F32 or BF16");
    const int rc = squares_launch(x, out, static_cast<long long>(rows), static_cast<long long>(cols),
                                  dtype == OMNI_B200_BF16, out_dtype == OMNI_B200_BF16,
                                  static_cast<cudaStream_t>(stream));
    return rc ? cuda_fail(static_cast<cudaError_t>(rc), "squares") : 0;
}

size_t omni_b200_vq_workspace(size_t rows, size_t dim, size_t codes, int profile) {
    (void)codes;
    if (profile == OMNI_B200_F32)
        return vq_stream_workspace(rows, 1);
    if (dim > 128)
        return vq_stream_workspace(rows, 0);
    return (rows * 8 + 255) / 256 * 256;
}

int omni_b200_vq_argmin(const void *x, const void *codebook, const void *cbnorm, void *ids,
                        size_t rows, size_t dim, size_t codes, int profile, int ids_u16,
                        void *workspace, size_t workspace_bytes, void *stream) {
    return vq_argmin(x, codebook, cbnorm, ids, rows, dim, codes, profile, ids_u16, workspace, workspace_bytes,
                     nullptr, static_cast<cudaStream_t>(stream));
}

int omni_b200_vq_argmin_cancellable(const void *x, const void *codebook, const void *cbnorm, void *ids,
                                    size_t rows, size_t dim, size_t codes, int profile, int ids_u16,
                                    void *workspace, size_t workspace_bytes, const int *cancel, void *stream) {
    return vq_argmin(x, codebook, cbnorm, ids, rows, dim, codes, profile, ids_u16, workspace, workspace_bytes,
                     cancel, static_cast<cudaStream_t>(stream));
}

} // extern "C"

namespace omni_b200 {

int vq_argmin(const void *x, const void *codebook, const void *cbnorm, void *ids, size_t rows, size_t dim,
              size_t codes, int profile, int ids_u16, void *workspace, size_t workspace_bytes,
              const volatile int *cancel, cudaStream_t stream, const float *xnorm) {
    g_error.clear();
    if (!x || !codebook || !cbnorm || !ids)
        return fail(1, "vq_argmin: null pointer");
    if (rows == 0)
        return 0;
    if (dim == 0 || codes == 0 || codes > 65536 || rows > (1u << 30))
        return fail(1, "vq_argmin: need dim > 0 and 0 < codes <= 65536");
    if (profile != OMNI_B200_BF16 && profile != OMNI_B200_F32)
        return fail(1, "vq_argmin: profile must be OMNI_B200_BF16 or OMNI_B200_F32");
    const bool fp32 = profile == OMNI_B200_F32;
    if (fp32 ? dim % 4 != 0 : dim % 8 != 0)
        return fail(4, fp32 ? "vq_argmin: fp32 profile needs dim % 4 == 0 (16-byte rows)"
                            : "vq_argmin: bf16 profile needs dim % 8 == 0 (16-byte rows)");
    if (dim > 65536)
        return fail(4, "vq_argmin: dim must be at most 65536");
    const uintptr_t align = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(codebook) |
                            reinterpret_cast<uintptr_t>(cbnorm);
    if (align % 16 != 0)
        return fail(1, "vq_argmin: x, codebook and cbnorm must be 16-byte aligned");
    const size_t need = omni_b200_vq_workspace(rows, dim, codes, profile);
    if (!workspace || workspace_bytes < need)
        return fail(1, "vq_argmin: workspace too small (need " + std::to_string(need) + " bytes)");
    VqArgs a;
    a.x = x;
    a.codebook = codebook;
    a.cbnorm = cbnorm;
    a.rows = static_cast<int>(rows);
    a.dim = static_cast<int>(dim);
    a.codes = static_cast<int>(codes);
    a.keys = workspace;
    a.ids = ids;
    a.ids_u16 = ids_u16 ? 1 : 0;
    a.cancel = cancel;
    a.xnorm = fp32 ? xnorm : nullptr;
    a.err = kernel_error_word();
    if (!a.err)
        return fail(7, "vq_argmin: no CUDA device");
    if (fp32 || dim > 128)
        return launch_status(vq_stream_launch(a, fp32 ? 1 : 0, stream), "vq_argmin");
    return launch_status(vq_bf16_launch(a, stream), "vq_argmin");
}

} // namespace omni_b200
