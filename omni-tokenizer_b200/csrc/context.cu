// context.cu -- host-buffer entry points: an omni_b200_context owns one CUDA
// device, one non-blocking stream and grow-only device buffers, mirroring how
// the reference's omni_context owns a Cuda backend with its stream and Pool
// (omni-tokenizer src/runtime.cpp:200-211, src/cuda.cu:448-551).  Each call
// copies host inputs in, runs the kernel, copies results out and synchronises,
// like omni_encode_image / omni_encode_audio do around the graph.
#include "omni_b200.h"

#include <atomic>
#include <cuda_runtime.h>
#include <new>
#include <string>

namespace omni_b200 {
int ctx_fail(int code, const char *msg);
bool injected_allocation_failure();
} // namespace omni_b200

// Batch chunks of the pipelined host-buffer attention call.
constexpr int kMaxChunks = 8;

struct omni_b200_context {
    int device = 0;
    cudaStream_t stream = nullptr;               // copies in (and every other call)
    cudaStream_t s_compute = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {};
    void *buf[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t cap[6] = {0, 0, 0, 0, 0, 0};
    std::atomic_flag running = ATOMIC_FLAG_INIT;
    uint64_t peak = 0, live = 0;
};

namespace {
int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess)
        return 0;
    return omni_b200::ctx_fail(e == cudaErrorMemoryAllocation ? 5 : 7,
                               (std::string(what) + ": " + cudaGetErrorString(e)).c_str());
}

// Ensures buffer i holds at least `bytes` (grow-only, 256-byte granular).
int reserve(omni_b200_context *c, int i, size_t bytes) {
    if (c->cap[i] >= bytes)
        return 0;
    bytes = (bytes + 255) / 256 * 256;
    if (c->buf[i]) {
        cudaFree(c->buf[i]);
        c->live -= c->cap[i];
        c->buf[i] = nullptr;
        c->cap[i] = 0;
    }
    if (omni_b200::injected_allocation_failure())
        return cuda_status(cudaErrorMemoryAllocation, "device buffer");
    if (int rc = cuda_status(cudaMalloc(&c->buf[i], bytes), "device buffer"))
        return rc;
    c->cap[i] = bytes;
    c->live += bytes;
    if (c->live > c->peak)
        c->peak = c->live;
    return 0;
}

struct Busy {
    omni_b200_context *c;
    bool ok;
    explicit Busy(omni_b200_context *ctx) : c(ctx), ok(!ctx->running.test_and_set()) {}
    ~Busy() {
        if (ok)
            c->running.clear();
    }
};

size_t elem_size(int dtype) { return dtype == OMNI_B200_F32 ? 4 : 2; }
} // namespace

extern "C" {

int omni_b200_context_create(int device, omni_b200_context **out) {
    if (!out)
        return omni_b200::ctx_fail(1, "context_create: null output handle");
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
        return omni_b200::ctx_fail(4, "context_create: no such CUDA device");
    auto *c = new (std::nothrow) omni_b200_context;
    if (!c)
        return omni_b200::ctx_fail(5, "context_create: allocation failed");
    c->device = device;
    if (int rc = cuda_status(cudaSetDevice(device), "set device")) {
        delete c;
        return rc;
    }
    int rc = cuda_status(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking),
                         "stream create");
    if (!rc)
        rc = cuda_status(cudaStreamCreateWithFlags(&c->s_compute, cudaStreamNonBlocking),
                         "stream create");
    if (!rc)
        rc = cuda_status(cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking),
                         "stream create");
    for (int k = 0; !rc && k < kMaxChunks; ++k) {
        rc = cuda_status(cudaEventCreateWithFlags(&c->ev_in[k], cudaEventDisableTiming), "event");
        if (!rc)
            rc = cuda_status(cudaEventCreateWithFlags(&c->ev_done[k], cudaEventDisableTiming),
                             "event");
    }
    if (rc) {
        omni_b200_context_free(c);
        return rc;
    }
    *out = c;
    return 0;
}

void omni_b200_context_free(omni_b200_context *c) {
    if (!c)
        return;
    cudaSetDevice(c->device);
    for (cudaStream_t st : {c->stream, c->s_compute, c->s_out})
        if (st)
            cudaStreamSynchronize(st);
    for (void *b : c->buf)
        if (b)
            cudaFree(b);
    for (int k = 0; k < kMaxChunks; ++k) {
        if (c->ev_in[k])
            cudaEventDestroy(c->ev_in[k]);
        if (c->ev_done[k])
            cudaEventDestroy(c->ev_done[k]);
    }
    for (cudaStream_t st : {c->stream, c->s_compute, c->s_out})
        if (st)
            cudaStreamDestroy(st);
    delete c;
}

uint64_t omni_b200_context_peak_workspace(const omni_b200_context *c) { return c ? c->peak : 0; }

int omni_b200_attention_bhld_host(omni_b200_context *c, const void *q, const void *k,
                                  const void *v, void *out, int batch, int heads, int L,
                                  int head_dim, int dtype, int out_dtype,
                                  const int32_t *lengths, int block, int skip_padded_queries,
                                  float scale) {
    if (!c || !q || !k || !v || !out)
        return omni_b200::ctx_fail(1, "attention_bhld_host: null pointer");
    if (batch <= 0 || heads <= 0 || L <= 0 || head_dim <= 0)
        return omni_b200::ctx_fail(1, "attention_bhld_host: sizes must be positive");
    Busy busy(c);
    if (!busy.ok)
        return omni_b200::ctx_fail(1, "attention_bhld_host: context is already executing");
    if (int rc = cuda_status(cudaSetDevice(c->device), "set device"))
        return rc;
    const size_t n = static_cast<size_t>(batch) * heads * L * head_dim;
    const size_t in_bytes = n * elem_size(dtype), out_bytes = n * elem_size(out_dtype);
    for (int i = 0; i < 3; ++i)
        if (int rc = reserve(c, i, in_bytes))
            return rc;
    if (int rc = reserve(c, 3, out_bytes))
        return rc;
    if (lengths)
        if (int rc = reserve(c, 4, sizeof(int32_t) * batch))
            return rc;
    // Pipelined over batch chunks: chunk k's inputs are copied in on `stream`
    // while chunk k-1 runs on `s_compute` and chunk k-2's output is copied out
    // on `s_out` (host-to-device and device-to-host copies use separate copy
    // engines), so the call costs about one pass over the inputs at PCIe rate.
    const int chunks = batch < kMaxChunks ? batch : kMaxChunks;
    // The last chunk is small: after the last input copy only its attention and
    // output copy remain (the tail of the call).  The other chunks share the
    // rest evenly.
    const int last = chunks > 1 ? (batch / (4 * chunks) > 1 ? batch / (4 * chunks) : 1) : batch;
    auto bound = [&](int ck) { // first item of chunk ck (ck <= chunks)
        if (ck >= chunks)
            return batch;
        return static_cast<int>(static_cast<long long>(batch - last) * ck / (chunks - 1 > 0 ? chunks - 1 : 1));
    };
    const size_t item_elems = static_cast<size_t>(heads) * L * head_dim;
    const size_t in_es = elem_size(dtype), out_es = elem_size(out_dtype);
    if (lengths)
        if (int rc = cuda_status(cudaMemcpyAsync(c->buf[4], lengths, sizeof(int32_t) * batch,
                                                 cudaMemcpyHostToDevice, c->stream),
                                 "copy lengths"))
            return rc;
    const void *src[3] = {q, k, v};
    int rc = 0;
    for (int ck = 0; ck < chunks && !rc; ++ck) {
        const int b0 = bound(ck), b1 = bound(ck + 1);
        const size_t off_in = b0 * item_elems * in_es, len_in = (b1 - b0) * item_elems * in_es;
        const size_t off_out = b0 * item_elems * out_es, len_out = (b1 - b0) * item_elems * out_es;
        for (int i = 0; i < 3 && !rc; ++i)
            rc = cuda_status(cudaMemcpyAsync(static_cast<char *>(c->buf[i]) + off_in,
                                             static_cast<const char *>(src[i]) + off_in, len_in,
                                             cudaMemcpyHostToDevice, c->stream),
                             "copy in");
        if (!rc)
            rc = cuda_status(cudaEventRecord(c->ev_in[ck], c->stream), "event record");
        if (!rc)
            rc = cuda_status(cudaStreamWaitEvent(c->s_compute, c->ev_in[ck], 0), "stream wait");
        if (!rc)
            rc = omni_b200_attention_bhld(
                static_cast<char *>(c->buf[0]) + off_in, static_cast<char *>(c->buf[1]) + off_in,
                static_cast<char *>(c->buf[2]) + off_in, static_cast<char *>(c->buf[3]) + off_out,
                b1 - b0, heads, L, head_dim, dtype, out_dtype,
                lengths ? static_cast<const int32_t *>(c->buf[4]) + b0 : nullptr, block,
                skip_padded_queries, scale, c->s_compute);
        if (!rc)
            rc = cuda_status(cudaEventRecord(c->ev_done[ck], c->s_compute), "event record");
        if (!rc)
            rc = cuda_status(cudaStreamWaitEvent(c->s_out, c->ev_done[ck], 0), "stream wait");
        if (!rc)
            rc = cuda_status(cudaMemcpyAsync(static_cast<char *>(out) + off_out,
                                             static_cast<char *>(c->buf[3]) + off_out, len_out,
                                             cudaMemcpyDeviceToHost, c->s_out),
                             "copy out");
    }
    // Drain every stream before returning (also on errors), then report.
    const int rc_in = cuda_status(cudaStreamSynchronize(c->stream), "copy in");
    const int rc_k = omni_b200_sync_check(c->s_compute);
    const int rc_out = cuda_status(cudaStreamSynchronize(c->s_out), "copy out");
    if (rc)
        return rc;
    return rc_in ? rc_in : rc_k ? rc_k : rc_out;
}

int omni_b200_vq_argmin_host(omni_b200_context *c, const void *x, const void *codebook,
                             const void *cbnorm, void *ids, size_t rows, size_t dim, size_t codes,
                             int profile, int ids_u16) {
    if (!c || !x || !codebook || !ids)
        return omni_b200::ctx_fail(1, "vq_argmin_host: null pointer");
    Busy busy(c);
    if (!busy.ok)
        return omni_b200::ctx_fail(1, "vq_argmin_host: context is already executing");
    if (int rc = cuda_status(cudaSetDevice(c->device), "set device"))
        return rc;
    const size_t es = profile == OMNI_B200_F32 ? 4 : 2;
    const size_t ws = omni_b200_vq_workspace(rows, dim, codes, profile);
    int rc = 0;
    if ((rc = reserve(c, 0, rows * dim * es)) || (rc = reserve(c, 1, codes * dim * es)) ||
        (rc = reserve(c, 2, codes * es)) || (rc = reserve(c, 3, rows * (ids_u16 ? 2 : 4))) ||
        (rc = reserve(c, 5, ws)))
        return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(c->buf[0], x, rows * dim * es, cudaMemcpyHostToDevice,
                                          c->stream),
                          "copy x")) ||
        (rc = cuda_status(cudaMemcpyAsync(c->buf[1], codebook, codes * dim * es,
                                          cudaMemcpyHostToDevice, c->stream),
                          "copy codebook")))
        return rc;
    if (cbnorm) {
        if ((rc = cuda_status(cudaMemcpyAsync(c->buf[2], cbnorm, codes * es,
                                              cudaMemcpyHostToDevice, c->stream),
                              "copy norms")))
            return rc;
    } else if ((rc = omni_b200_squares(c->buf[1], c->buf[2], codes, dim, profile, profile,
                                       c->stream))) {
        return rc;
    }
    if ((rc = omni_b200_vq_argmin(c->buf[0], c->buf[1], c->buf[2], c->buf[3], rows, dim, codes,
                                  profile, ids_u16, c->buf[5], c->cap[5], c->stream)))
        return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(ids, c->buf[3], rows * (ids_u16 ? 2 : 4),
                                          cudaMemcpyDeviceToHost, c->stream),
                          "copy ids")))
        return rc;
    return omni_b200_sync_check(c->stream);
}

} // extern "C"
