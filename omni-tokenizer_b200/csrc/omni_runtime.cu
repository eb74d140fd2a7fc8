// omni_runtime.cu -- the reference's outer C ABI (include/omni_abi.h) on B200:
// OMNIVQ01 model loading, the audio and image encoder graphs, and the 15
// omni_* entry points, so that omni-tokenizer's Python Tokenizer and C callers
// can load this library through OMNI_LIBRARY.
//
// Graph semantics follow omni-tokenizer src/runtime.cpp:30-130 (audio, image),
// the loader src/model.cpp:96-205, the operator semantics src/cpu.cpp and the
// C API behaviour src/runtime.cpp:131-288.  Hot operators run on this
// library's sm_100a kernels (attention: fmha_sm100.cu; VQ argmin:
// vq_sm100.cu / vq_stream_sm100.cu; norms: norms.cu); linears are cuBLAS
// GEMMs (fp32 in the audio profile, bf16 x bf16 -> fp32 in the image profile)
// followed by the bias / bf16-rounding epilogue; the remaining operators are
// graph_kernels.cu.  Audio-profile attention stays fp32 (the reference's audio
// kernels are fp32-accurate 3xTF32): fp32 cuBLAS GEMMs for the scores and the
// weighted values around a masked-softmax kernel.  OMNI_B200_AUDIO_BF16=1
// selects this library's bf16 audio mode instead: bf16 weights (converted once
// per model) and activations with the reference's bf16 rounding points, the
// tcgen05 attention kernel, fp32 VQ.
#include "fmha.h"
#include "graph_kernels.h"
#include "omni_abi.h"
#include "omni_b200.h"
#include "vq.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <array>
#include <cublasLt.h>
#include <cublas_v2.h>
#include <map>
#include <mutex>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <fstream>
#include <limits>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace omni_b200 {
bool injected_allocation_failure();
namespace rt {

struct Fail : std::runtime_error {
    int code;
    Fail(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};
void require(bool ok, const std::string &msg, int code = OMNI_INVALID_ARGUMENT) {
    if (!ok)
        throw Fail(code, msg);
}
void cuda_ok(cudaError_t e, const char *what) {
    if (e != cudaSuccess)
        throw Fail(e == cudaErrorMemoryAllocation ? OMNI_OUT_OF_MEMORY : OMNI_INTERNAL_ERROR,
                   std::string(what) + ": " + cudaGetErrorString(e));
}
void op_ok(int rc, const char *what) {
    if (rc == 0)
        return;
    const char *msg = omni_b200_last_error();
    throw Fail(rc > 0 && rc <= 7 ? rc : OMNI_INTERNAL_ERROR,
               std::string(what) + ": " + (msg && *msg ? msg : "device error " + std::to_string(rc)));
}
void blas_ok(cublasStatus_t st, const char *what) {
    if (st != CUBLAS_STATUS_SUCCESS)
        throw Fail(st == CUBLAS_STATUS_ALLOC_FAILED ? OMNI_OUT_OF_MEMORY : OMNI_INTERNAL_ERROR,
                   std::string(what) + ": cuBLAS status " + std::to_string(static_cast<int>(st)));
}

// Device bytes a context holds (activations, scratch); the peak is reported
// by omni_context_peak_workspace.
struct Memory {
    std::atomic<uint64_t> live{0}, peak{0};
    void add(uint64_t n) {
        const uint64_t v = live.fetch_add(n) + n;
        uint64_t p = peak.load();
        while (v > p && !peak.compare_exchange_weak(p, v)) {
        }
    }
};

// A row-major device matrix of fp32 or bf16 values.
struct Tensor {
    std::shared_ptr<void> mem;
    size_t rows = 0, cols = 0;
    bool bf16 = false;
    void *data() const { return mem.get(); }
    size_t size() const { return rows * cols; }
    size_t bytes() const { return size() * (bf16 ? 2 : 4); }
};

Tensor weight_tensor(size_t rows, size_t cols, bool bf16) {
    Tensor t;
    t.rows = rows;
    t.cols = cols;
    t.bf16 = bf16;
    void *p = nullptr;
    cuda_ok(injected_allocation_failure() ? cudaErrorMemoryAllocation : cudaMalloc(&p, t.bytes() ? t.bytes() : 1),
            "weight allocation");
    t.mem = std::shared_ptr<void>(p, [](void *q) { cudaFree(q); });
    return t;
}

struct Config {
    uint32_t kind = 0, layers = 0, width = 0, heads = 0, ffn = 0, input_channels = 0,
             patch_size = 0, pool_size = 0, block_size = 0, pos_height = 0, pos_width = 0,
             code_dim = 0, vocab_size = 0;
};

struct Model {
    Config cfg;
    int backend = OMNI_CUDA, device = 0;
    uint64_t weight_bytes = 0;
    std::unordered_map<std::string, Tensor> w;
    std::unordered_map<std::string, std::vector<uint64_t>> shapes;
    Tensor cbnorm;
    const Tensor &get(const std::string &name) const {
        auto it = w.find(name);
        require(it != w.end(), "Missing tensor: " + name, OMNI_INVALID_MODEL);
        return it->second;
    }
    const Tensor *opt(const std::string &name) const {
        auto it = w.find(name);
        return it == w.end() ? nullptr : &it->second;
    }
    // bf16 copies of an fp32 (audio) model's tensors for the bf16 audio mode,
    // made once, by the first context that asks for them (all but the codebook).
    std::unordered_map<std::string, Tensor> w16;
    std::once_flag w16_once;
    const Tensor &get(const std::string &name, bool bf16) const {
        if (!bf16)
            return get(name);
        auto it = w16.find(name);
        require(it != w16.end(), "Missing tensor: " + name, OMNI_INVALID_MODEL);
        return it->second;
    }
    const Tensor *opt(const std::string &name, bool bf16) const {
        if (!bf16)
            return opt(name);
        auto it = w16.find(name);
        return it == w16.end() ? nullptr : &it->second;
    }
    // Tensors that are views into another tensor of `w` (the audio layers'
    // q/k/v projections inside their stacked qkv weight); not converted for
    // the bf16 audio mode.
    std::set<std::string> views;
};

// ------------------------------------------------------------------ loader
namespace {
uint32_t rd32(std::istream &f) {
    unsigned char b[4];
    f.read(reinterpret_cast<char *>(b), 4);
    require(static_cast<bool>(f), "Truncated model index", OMNI_INVALID_MODEL);
    return uint32_t(b[0]) | uint32_t(b[1]) << 8 | uint32_t(b[2]) << 16 | uint32_t(b[3]) << 24;
}
uint64_t rd64(std::istream &f) {
    const uint64_t lo = rd32(f);
    return lo | uint64_t(rd32(f)) << 32;
}
struct Entry {
    std::string name;
    uint32_t dtype = 0;
    uint64_t offset = 0, bytes = 0;
    std::vector<uint64_t> shape;
};

void expect_shape(const Model &m, const std::string &name, std::vector<uint64_t> s) {
    auto it = m.shapes.find(name);
    require(it != m.shapes.end(), "Missing tensor: " + name, OMNI_INVALID_MODEL);
    require(it->second == s, "Incorrect shape for " + name, OMNI_INVALID_MODEL);
}

// The fixed tensor set of each model kind (src/model.cpp:33-94).
void check_layout(const Model &m) {
    const Config &c = m.cfg;
    const uint64_t W = c.width, F = c.ffn;
    if (c.kind == OMNI_AUDIO) {
        expect_shape(m, "conv1.weight", {W, c.input_channels, 3});
        expect_shape(m, "conv1.bias", {W});
        expect_shape(m, "conv2.weight", {W, W, 3});
        expect_shape(m, "conv2.bias", {W});
        expect_shape(m, "embed_positions.weight", {c.pos_height, W});
        expect_shape(m, "codebook.weight", {c.vocab_size, W});
        require(c.pool_size == 4 && c.patch_size == 0 && c.code_dim == c.width && c.block_size > 0,
                "Invalid audio configuration", OMNI_INVALID_MODEL);
        for (uint32_t l = 0; l < c.layers; ++l) {
            const std::string p = "layers." + std::to_string(l) + ".";
            for (const char *n : {"self_attn_layer_norm", "final_layer_norm"}) {
                expect_shape(m, p + n + ".weight", {W});
                expect_shape(m, p + n + ".bias", {W});
            }
            for (const char *n : {"q_proj", "k_proj", "v_proj", "out_proj"})
                expect_shape(m, p + "self_attn." + n + ".weight", {W, W});
            for (const char *n : {"q_proj", "v_proj", "out_proj"})
                expect_shape(m, p + "self_attn." + n + ".bias", {W});
            expect_shape(m, p + "fc1.weight", {F, W});
            expect_shape(m, p + "fc1.bias", {F});
            expect_shape(m, p + "fc2.weight", {W, F});
            expect_shape(m, p + "fc2.bias", {W});
        }
    } else {
        require(c.input_channels == 3 && c.patch_size > 0 && c.patch_size <= 64 &&
                    c.pos_height == c.pos_width,
                "Invalid image configuration", OMNI_INVALID_MODEL);
        const uint64_t P = c.patch_size;
        expect_shape(m, "patch_embed.proj.weight", {W, 3, P, P});
        expect_shape(m, "patch_embed.proj.bias", {W});
        expect_shape(m, "pos_embed", {1, uint64_t(c.pos_height) * c.pos_width, W});
        expect_shape(m, "quant_conv.weight", {c.code_dim, W, 1, 1});
        expect_shape(m, "quant_conv.bias", {c.code_dim});
        expect_shape(m, "quantize.embedding.weight", {c.vocab_size, c.code_dim});
        for (uint32_t l = 0; l < c.layers; ++l) {
            const std::string p = "blocks." + std::to_string(l) + ".";
            for (const char *n : {"norm1", "norm2"}) {
                expect_shape(m, p + n + ".weight", {W});
                expect_shape(m, p + n + ".bias", {W});
            }
            expect_shape(m, p + "attn.qkv.weight", {3 * W, W});
            expect_shape(m, p + "attn.qkv.bias", {3 * W});
            expect_shape(m, p + "attn.proj.weight", {W, W});
            expect_shape(m, p + "attn.proj.bias", {W});
            expect_shape(m, p + "mlp.fc1.weight", {F, W});
            expect_shape(m, p + "mlp.fc1.bias", {F});
            expect_shape(m, p + "mlp.fc2.weight", {W, F});
            expect_shape(m, p + "mlp.fc2.bias", {W});
        }
    }
}
} // namespace

std::shared_ptr<Model> load_model(const char *path, int backend, int device) {
    require(path && *path, "Model path must not be empty");
    require(backend == OMNI_CUDA,
            "This library implements the CUDA backend only (OMNI_CPU is unsupported)",
            OMNI_UNSUPPORTED);
    int devices = 0;
    require(cudaGetDeviceCount(&devices) == cudaSuccess && device >= 0 && device < devices,
            "Requested CUDA device is unavailable", OMNI_UNSUPPORTED);
    cuda_ok(cudaSetDevice(device), "set device");
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    require(static_cast<bool>(f), "Cannot open model file", OMNI_IO_ERROR);
    const uint64_t file_bytes = static_cast<uint64_t>(f.tellg());
    require(file_bytes >= 68, "Model file is too short", OMNI_INVALID_MODEL);
    f.seekg(0);
    char magic[8];
    f.read(magic, 8);
    require(static_cast<bool>(f) && std::memcmp(magic, "OMNIVQ01", 8) == 0, "Invalid model magic",
            OMNI_INVALID_MODEL);
    require(rd32(f) == 1, "Unsupported model version", OMNI_INVALID_MODEL);
    auto m = std::make_shared<Model>();
    m->backend = backend;
    m->device = device;
    Config &c = m->cfg;
    c.kind = rd32(f);
    for (uint32_t *fld : {&c.layers, &c.width, &c.heads, &c.ffn, &c.input_channels, &c.patch_size,
                          &c.pool_size, &c.block_size, &c.pos_height, &c.pos_width, &c.code_dim,
                          &c.vocab_size})
        *fld = rd32(f);
    require((c.kind == OMNI_AUDIO || c.kind == OMNI_IMAGE) && c.layers > 0 && c.layers <= 80 &&
                c.width > 0 && c.width <= 8192 && c.heads > 0 && c.width % c.heads == 0 &&
                c.ffn > 0 && c.ffn <= 32768 && c.code_dim > 0 && c.code_dim <= 8192 &&
                c.vocab_size > 0 && c.vocab_size <= 16384 && c.input_channels > 0 &&
                c.input_channels <= 512 && c.pos_height > 0 && c.pos_height <= 16384 &&
                c.pos_width <= 16384,
            "Model configuration exceeds supported bounds", OMNI_INVALID_MODEL);
    const uint32_t count = rd32(f);
    require(count == 6 + c.layers * (c.kind == OMNI_AUDIO ? 15u : 12u),
            "Unexpected tensor count for the fixed model", OMNI_INVALID_MODEL);
    std::vector<Entry> entries;
    std::set<std::string> names;
    const uint32_t want_dtype = c.kind == OMNI_AUDIO ? 1u : 2u; // 1 = fp32, 2 = bf16
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t len = rd32(f), dtype = rd32(f), rank = rd32(f), reserved = rd32(f);
        Entry e;
        e.dtype = dtype;
        e.offset = rd64(f);
        e.bytes = rd64(f);
        require(len > 0 && len <= 1024 && dtype == want_dtype && rank > 0 && rank <= 4 &&
                    reserved == 0,
                "Invalid tensor record or precision profile", OMNI_INVALID_MODEL);
        uint64_t elements = 1;
        for (uint32_t r = 0; r < rank; ++r) {
            const uint64_t d = rd64(f);
            require(d > 0 && d <= (uint64_t(1) << 24) &&
                        elements <= std::numeric_limits<uint64_t>::max() / d,
                    "Tensor dimensions overflow", OMNI_INVALID_MODEL);
            elements *= d;
            e.shape.push_back(d);
        }
        require(elements <= std::numeric_limits<uint64_t>::max() / 4 &&
                    e.bytes == elements * (dtype == 1 ? 4 : 2) && e.offset % 64 == 0 &&
                    e.offset <= file_bytes && e.bytes <= file_bytes - e.offset,
                "Invalid tensor data bounds", OMNI_INVALID_MODEL);
        e.name.resize(len);
        f.read(&e.name[0], len);
        require(static_cast<bool>(f) && e.name.find('\0') == std::string::npos &&
                    names.insert(e.name).second,
                "Invalid or duplicate tensor name", OMNI_INVALID_MODEL);
        entries.push_back(std::move(e));
    }
    // Tensor data must not overlap each other or the index.
    {
        std::vector<std::pair<uint64_t, uint64_t>> spans;
        for (const Entry &e : entries)
            spans.emplace_back(e.offset, e.bytes);
        std::sort(spans.begin(), spans.end());
        uint64_t end = static_cast<uint64_t>(f.tellg());
        for (auto &s : spans) {
            require(s.first >= end, "Overlapping model tensors/index", OMNI_INVALID_MODEL);
            end = s.first + s.second;
        }
    }
    for (const Entry &e : entries)
        m->shapes[e.name] = e.shape;
    check_layout(*m);
    const bool bf16 = c.kind == OMNI_IMAGE;
    for (const Entry &e : entries) {
        std::vector<unsigned char> raw(static_cast<size_t>(e.bytes));
        f.seekg(static_cast<std::streamoff>(e.offset));
        f.read(reinterpret_cast<char *>(raw.data()), static_cast<std::streamsize>(e.bytes));
        require(static_cast<bool>(f), "Truncated tensor data", OMNI_IO_ERROR);
        size_t rows = static_cast<size_t>(e.shape[0]), cols = 1;
        for (size_t r = 1; r < e.shape.size(); ++r)
            cols *= static_cast<size_t>(e.shape[r]);
        if (e.name == "pos_embed") {
            rows = static_cast<size_t>(e.shape[1]);
            cols = static_cast<size_t>(e.shape[2]);
        }
        if (c.kind == OMNI_IMAGE && e.name == "patch_embed.proj.weight") {
            // [width, 3, p, p] -> [width, p*p*8]: pixel-major, channels padded
            // to 8, matching the patch layout the graph builds.
            const size_t px = size_t(c.patch_size) * c.patch_size;
            std::vector<unsigned char> packed(rows * px * 8 * 2, 0);
            for (size_t o = 0; o < rows; ++o)
                for (size_t q = 0; q < px; ++q)
                    for (size_t ch = 0; ch < 3; ++ch)
                        std::memcpy(&packed[(o * px * 8 + q * 8 + ch) * 2],
                                    &raw[(o * 3 * px + ch * px + q) * 2], 2);
            raw.swap(packed);
            cols = px * 8;
        }
        Tensor t = weight_tensor(rows, cols, bf16);
        cuda_ok(cudaMemcpy(t.data(), raw.data(), t.bytes(), cudaMemcpyHostToDevice), "weight upload");
        m->weight_bytes += t.bytes();
        m->w.emplace(e.name, std::move(t));
    }
    if (c.kind == OMNI_AUDIO) {
        // The three attention projections of an audio layer read the same
        // input: stack them as one [3 width, width] weight (and a [3 width]
        // bias with zeros where a projection has none) so that the graph runs
        // one GEMM whose output is the fused Q|K|V layout.  The separate
        // tensors stay available as views into the stacked ones.
        const size_t W = c.width;
        for (uint32_t i = 0; i < c.layers; ++i) {
            const std::string p = "layers." + std::to_string(i) + ".self_attn.";
            Tensor qkv = weight_tensor(3 * W, W, false), bias = weight_tensor(3 * W, 1, false);
            cuda_ok(cudaMemset(bias.data(), 0, bias.bytes()), "qkv bias");
            const char *proj[3] = {"q_proj", "k_proj", "v_proj"};
            for (int j = 0; j < 3; ++j) {
                const std::string wn = p + proj[j] + ".weight", bn = p + proj[j] + ".bias";
                Tensor &wt = m->w.at(wn);
                char *dst = static_cast<char *>(qkv.data()) + j * W * W * 4;
                cuda_ok(cudaMemcpy(dst, wt.data(), W * W * 4, cudaMemcpyDeviceToDevice), "qkv weight");
                wt.mem = std::shared_ptr<void>(qkv.mem, dst);
                m->views.insert(wn);
                auto b = m->w.find(bn);
                if (b != m->w.end()) {
                    char *bdst = static_cast<char *>(bias.data()) + j * W * 4;
                    cuda_ok(cudaMemcpy(bdst, b->second.data(), W * 4, cudaMemcpyDeviceToDevice), "qkv bias");
                    b->second.mem = std::shared_ptr<void>(bias.mem, bdst);
                    m->views.insert(bn);
                }
            }
            m->weight_bytes += bias.bytes();
            m->w.emplace(p + "qkv.weight", std::move(qkv));
            m->w.emplace(p + "qkv.bias", std::move(bias));
        }
    }
    const char *cb_name = c.kind == OMNI_AUDIO ? "codebook.weight" : "quantize.embedding.weight";
    Tensor &cb = m->w.at(cb_name);
    if (c.kind == OMNI_IMAGE) {
        // The image codebook is L2-normalised once at load (src/model.cpp:203-204).
        Tensor n = weight_tensor(cb.rows, cb.cols, true);
        cuda_ok(static_cast<cudaError_t>(graph::normalize(cb.data(), n.data(), true, cb.rows, cb.cols, 0)),
                "codebook normalise");
        cb = std::move(n);
    }
    m->cbnorm = weight_tensor(cb.rows, 1, bf16);
    op_ok(omni_b200_squares(cb.data(), m->cbnorm.data(), cb.rows, cb.cols, bf16 ? OMNI_B200_BF16 : OMNI_B200_F32,
                            bf16 ? OMNI_B200_BF16 : OMNI_B200_F32, nullptr),
          "codebook norms");
    cuda_ok(cudaDeviceSynchronize(), "model load");
    return m;
}

// ------------------------------------------------------------------ context
struct Context {
    std::shared_ptr<Model> model;
    cudaStream_t stream = nullptr;
    cublasHandle_t blas = nullptr;
    // Activations come from this context's own stream-ordered pool, which keeps
    // its memory between calls (a pool with the default release threshold
    // returns it at every synchronisation and re-maps it on the next call).
    cudaMemPool_t pool = nullptr;
    std::shared_ptr<Memory> memory = std::make_shared<Memory>();
    std::atomic<bool> cancelled{false};
    // The same flag in mapped pinned host memory, read by the VQ kernels when
    // they start (cancellation between codebook windows of the VQ pass).
    int *cancel_host = nullptr;
    int *cancel_dev = nullptr;
    std::atomic_flag running = ATOMIC_FLAG_INIT;
    Tensor features;
    omni_trace_callback trace = nullptr;
    void *trace_user = nullptr;
    bool audio_bf16 = false;
    // fp32-profile GEMMs through cuBLAS's BF16x9 emulation of fp32 on the tensor
    // cores instead of fp32 on the CUDA cores.
    bool fp32_emulated = false;
    cublasComputeType_t fp32_compute() const {
        return fp32_emulated ? CUBLAS_COMPUTE_32F_EMULATED_16BFX9 : CUBLAS_COMPUTE_32F_PEDANTIC;
    }
    // Host inputs are copied on `copy` into two staging buffers (events
    // ready[i] / done[i]), overlapping the graph of the previous chunk.
    cudaStream_t copy = nullptr;
    cudaEvent_t ready[2] = {}, done[2] = {}, start = nullptr;
    // cuBLASLt linears: handle, workspace and the chosen algorithm per shape
    // (m, n, k, bf16, fused bias).
    cublasLtHandle_t lt = nullptr;
    void *lt_ws = nullptr;
    size_t lt_ws_bytes = 0;
    std::map<std::array<long long, 5>, std::pair<bool, cublasLtMatmulAlgo_t>> lt_algos;
    // cuBLAS workspace, set explicitly so that captured GEMMs allocate nothing.
    void *blas_ws = nullptr;
    // CUDA-graph replay of repeated batched calls: the second call with the
    // same key (entry point, shapes, valid lengths, input address) is captured
    // into a graph whose outputs live in persistent buffers, and later calls
    // with that key replay it.
    struct Replay {
        std::vector<uint64_t> key;
        cudaGraphExec_t exec = nullptr;
        Tensor flag, features, ids, keys;
    };
    Replay replay;
    std::vector<uint64_t> last_key;
    uint64_t graph_launches = 0;
    bool capturing = false; // inside a stream capture: no synchronising retries
    bool graphs = true;     // OMNI_B200_GRAPHS=0 turns replay off
    void drop_replay() {
        if (replay.exec)
            cudaGraphExecDestroy(replay.exec);
        replay = Replay{};
    }

    ~Context() {
        features = {};
        if (stream) {
            cudaSetDevice(model ? model->device : 0);
            cudaStreamSynchronize(stream);
        }
        drop_replay();
        if (copy)
            cudaStreamSynchronize(copy);
        for (cudaEvent_t e : {ready[0], ready[1], done[0], done[1], start})
            if (e)
                cudaEventDestroy(e);
        if (blas)
            cublasDestroy(blas);
        if (lt)
            cublasLtDestroy(lt);
        if (lt_ws)
            cudaFree(lt_ws);
        if (blas_ws)
            cudaFree(blas_ws);
        if (copy)
            cudaStreamDestroy(copy);
        if (stream)
            cudaStreamDestroy(stream);
        if (pool)
            cudaMemPoolDestroy(pool);
        if (cancel_host)
            cudaFreeHost(cancel_host);
    }
    void check() const {
        if (cancelled.load())
            throw Fail(OMNI_CANCELLED, "Inference cancelled");
    }
    // Stream-ordered activation memory, counted in the workspace peak.
    Tensor make(size_t rows, size_t cols, bool bf16) {
        Tensor t;
        t.rows = rows;
        t.cols = cols;
        t.bf16 = bf16;
        const size_t bytes = t.bytes() ? t.bytes() : 1;
        void *p = nullptr;
        // Out of memory: release the pool's idle memory and retry once (the
        // reference's Pool trims its cache and retries, src/cuda.cu:515-527).
        cudaError_t e = injected_allocation_failure() ? cudaErrorMemoryAllocation
                                                      : cudaMallocFromPoolAsync(&p, bytes, pool, stream);
        if (e == cudaErrorMemoryAllocation && !capturing) {
            cudaGetLastError(); // take the failed call out of the runtime's last-error state
            cuda_ok(cudaStreamSynchronize(stream), "activation allocation");
            cuda_ok(cudaMemPoolTrimTo(pool, 0), "activation allocation");
            e = injected_allocation_failure() ? cudaErrorMemoryAllocation
                                              : cudaMallocFromPoolAsync(&p, bytes, pool, stream);
        }
        cuda_ok(e, "activation allocation");
        memory->add(bytes);
        auto mem = memory;
        cudaStream_t s = stream;
        t.mem = std::shared_ptr<void>(p, [mem, s, bytes](void *q) {
            cudaFreeAsync(q, s);
            mem->live.fetch_sub(bytes);
        });
        return t;
    }
    void *scratch(size_t bytes, Tensor &holder) {
        holder = make((bytes + 3) / 4, 1, false);
        return holder.data();
    }
};

namespace {
// One cuBLASLt matmul D = x W^T (+ bias in the epilogue) in the tensor's
// own type (fp32 accumulate; bf16 results rounded once, after the bias).
// Returns false when cuBLASLt offers no algorithm for the shape.
bool lt_linear(Context &c, const Tensor &x, const Tensor &w, const void *bias, Tensor &y) {
    const size_t m = x.rows, n = w.rows, k = x.cols;
    const std::array<long long, 5> key{static_cast<long long>(m), static_cast<long long>(n),
                                       static_cast<long long>(k), x.bf16 ? 1 : 0, bias ? 1 : 0};
    const cudaDataType_t t = x.bf16 ? CUDA_R_16BF : CUDA_R_32F;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
    auto cleanup = [&] {
        if (la)
            cublasLtMatrixLayoutDestroy(la);
        if (lb)
            cublasLtMatrixLayoutDestroy(lb);
        if (lc)
            cublasLtMatrixLayoutDestroy(lc);
        if (op)
            cublasLtMatmulDescDestroy(op);
    };
    // Column-major view: D^T [n, m] = W [k, n]^T * X^T [k, m].
    blas_ok(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F), "matmul desc");
    const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof ta);
    cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof tb);
    if (bias) {
        const cublasLtEpilogue_t ep = CUBLASLT_EPILOGUE_BIAS;
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &ep, sizeof ep);
        cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof bias);
    }
    cublasLtMatrixLayoutCreate(&la, t, k, n, k);
    cublasLtMatrixLayoutCreate(&lb, t, k, m, k);
    cublasLtMatrixLayoutCreate(&lc, t, n, m, n);
    auto it = c.lt_algos.find(key);
    if (it == c.lt_algos.end()) {
        cublasLtMatmulPreference_t pref = nullptr;
        cublasLtMatmulPreferenceCreate(&pref);
        cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &c.lt_ws_bytes,
                                             sizeof c.lt_ws_bytes);
        cublasLtMatmulHeuristicResult_t res{};
        int found = 0;
        const cublasStatus_t st = cublasLtMatmulAlgoGetHeuristic(c.lt, op, la, lb, lc, lc, pref, 1, &res, &found);
        cublasLtMatmulPreferenceDestroy(pref);
        it = c.lt_algos.emplace(key, std::make_pair(st == CUBLAS_STATUS_SUCCESS && found > 0, res.algo)).first;
    }
    if (!it->second.first) {
        cleanup();
        return false;
    }
    const float one = 1.f, zero = 0.f;
    const cublasStatus_t st = cublasLtMatmul(c.lt, op, &one, w.data(), la, x.data(), lb, &zero, y.data(), lc,
                                             y.data(), lc, &it->second.second, c.lt_ws, c.lt_ws_bytes, c.stream);
    cleanup();
    blas_ok(st, "linear");
    return true;
}

// y = x W^T (+ b).  bias_after_round: the reference's image_conv -- r(r(x W^T) + b).
// cuBLASLt with the bias in its epilogue when it has an algorithm; otherwise a
// cuBLAS GEMM into fp32 followed by the bias / rounding epilogue kernel.
Tensor linear(Context &c, const Tensor &x, const Tensor &w, const Tensor *b,
              bool bias_after_round = false) {
    require(x.cols == w.cols, "Linear dimensions disagree", OMNI_INVALID_MODEL);
    const size_t m = x.rows, n = w.rows, k = x.cols;
    Tensor y = c.make(m, n, x.bf16);
    if (m == 0)
        return y;
    const bool fused_bias = b && !bias_after_round;
    const bool lt_ok = c.lt && w.bf16 == x.bf16 && (!fused_bias || b->bf16 == x.bf16) &&
                       (x.bf16 || !c.fp32_emulated) && lt_linear(c, x, w, fused_bias ? b->data() : nullptr, y);
    if (!lt_ok) {
        Tensor acc_holder;
        float *acc = x.bf16 ? static_cast<float *>(c.scratch(m * n * 4, acc_holder))
                            : static_cast<float *>(y.data());
        const float one = 1.f, zero = 0.f;
        blas_ok(cublasGemmEx(c.blas, CUBLAS_OP_T, CUBLAS_OP_N, static_cast<int>(n), static_cast<int>(m),
                             static_cast<int>(k), &one, w.data(), x.bf16 ? CUDA_R_16BF : CUDA_R_32F,
                             static_cast<int>(k), x.data(), x.bf16 ? CUDA_R_16BF : CUDA_R_32F,
                             static_cast<int>(k), &zero, acc, CUDA_R_32F, static_cast<int>(n),
                             x.bf16 ? CUBLAS_COMPUTE_32F : c.fp32_compute(), CUBLAS_GEMM_DEFAULT),
                "linear");
        cuda_ok(static_cast<cudaError_t>(graph::linear_epilogue(acc, fused_bias ? b->data() : nullptr,
                                                                b ? b->bf16 : false, y.data(), y.bf16, m,
                                                                n, c.stream)),
                "linear epilogue");
    }
    if (b && bias_after_round)
        cuda_ok(static_cast<cudaError_t>(graph::bias(y.data(), b->data(), y.bf16, m, n, c.stream)),
                "bias");
    return y;
}

// x = r(x + z) in place (when z is given; the residual), then the layer norm of x.
Tensor add_norm(Context &c, Tensor &x, const Tensor *z, const Tensor &w, const Tensor &b, float eps) {
    require(!z || (z->cols == x.cols && z->rows >= x.rows && z->bf16 == x.bf16), "Residual dimensions disagree",
            OMNI_INTERNAL_ERROR);
    Tensor y = c.make(x.rows, x.cols, x.bf16);
    cuda_ok(static_cast<cudaError_t>(graph::add_layer_norm(x.data(), z ? z->data() : nullptr, w.data(), b.data(),
                                                           y.data(), x.bf16, x.rows, x.cols, eps, c.stream)),
            "layer norm");
    return y;
}

void add_in_place(Context &c, Tensor &x, const Tensor &y) {
    require(x.cols == y.cols && y.rows >= x.rows && x.bf16 == y.bf16, "Residual dimensions disagree",
            OMNI_INTERNAL_ERROR);
    cuda_ok(static_cast<cudaError_t>(graph::add(x.data(), y.data(), x.bf16, x.size(), c.stream)), "add");
}

void gelu_in_place(Context &c, Tensor &x) {
    cuda_ok(static_cast<cudaError_t>(graph::gelu(x.data(), x.bf16, x.size(), c.stream)), "gelu");
}

// Ops::attention on `batch` stacked sequences of [n, heads*hd] rows (fused:
// [n, 3*heads*hd]); keys of sequence b limited to valid[b] (valid_dev: the
// same counts as device int32, or null when every count is n).
Tensor attention(Context &c, const Tensor &q, const Tensor *k, const Tensor *v, size_t heads,
                 size_t block, bool fused, size_t batch, const std::vector<int> &valid,
                 const int *valid_dev) {
    const size_t rows = q.rows, n = rows / batch, d = fused ? q.cols / 3 : q.cols, hd = d / heads;
    Tensor y = c.make(rows, d, q.bf16);
    if (!q.bf16 && !c.audio_bf16 && padded_head_dim_f32(static_cast<int>(hd)) < 0) {
        // fp32 profile with head dims beyond the fused kernel's 128: per item,
        // S = scale Q K^T for all heads (one strided batched fp32 GEMM), masked
        // softmax in place, O = P V.  Head dims up to 128 take the fused
        // split-precision kernel through attention_rows below.
        // Q, K, V rows are `ld` floats apart (d, or 3 d in the fused layout).
        const size_t ld = fused ? 3 * d : d;
        const long long nn = static_cast<long long>(n) * n;
        Tensor scores = c.make(batch * heads * n, n, false);
        float *S = static_cast<float *>(scores.data());
        const float scale = 1.f / std::sqrt(static_cast<float>(hd)), one = 1.f, zero = 0.f;
        const float *Q = static_cast<const float *>(q.data());
        const float *K = fused ? Q + d : static_cast<const float *>(k->data());
        const float *V = fused ? Q + 2 * d : static_cast<const float *>(v->data());
        float *O = static_cast<float *>(y.data());
        const int ni = static_cast<int>(n), di = static_cast<int>(d), li = static_cast<int>(ld),
                  hi = static_cast<int>(hd);
        for (size_t b = 0; b < batch; ++b)
            blas_ok(cublasGemmStridedBatchedEx(c.blas, CUBLAS_OP_T, CUBLAS_OP_N, ni, ni, hi, &scale,
                                               K + b * n * ld, CUDA_R_32F, li, static_cast<long long>(hd),
                                               Q + b * n * ld, CUDA_R_32F, li, static_cast<long long>(hd), &zero,
                                               S + b * heads * nn, CUDA_R_32F, ni, nn, static_cast<int>(heads),
                                               c.fp32_compute(), CUBLAS_GEMM_DEFAULT),
                    "attention scores");
        cuda_ok(static_cast<cudaError_t>(graph::softmax_rows(S, batch, heads, n, valid_dev,
                                                             static_cast<size_t>(valid[0]), block, c.stream)),
                "attention softmax");
        for (size_t b = 0; b < batch; ++b)
            blas_ok(cublasGemmStridedBatchedEx(c.blas, CUBLAS_OP_N, CUBLAS_OP_N, hi, ni, ni, &one, V + b * n * ld,
                                               CUDA_R_32F, li, static_cast<long long>(hd), S + b * heads * nn,
                                               CUDA_R_32F, ni, nn, &zero, O + b * n * d, CUDA_R_32F, di,
                                               static_cast<long long>(hd), static_cast<int>(heads),
                                               c.fp32_compute(), CUBLAS_GEMM_DEFAULT),
                    "attention values");
        return y;
    }
    const int dt = q.bf16 ? OMNI_B200_BF16 : OMNI_B200_F32;
    const size_t ws_bytes = attention_rows_workspace(rows, static_cast<int>(heads), static_cast<int>(hd), dt,
                                                     fused ? 1 : 0);
    Tensor ws_holder, split_holder;
    void *ws = ws_bytes ? c.scratch(ws_bytes, ws_holder) : nullptr;
    // Scratch for the key split of a partial last round (small batches).
    const size_t split_bytes = attention_rows_split_workspace(
        n, static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(hd), block,
        valid_dev ? 0 : static_cast<size_t>(valid[0]), dt);
    void *split = split_bytes ? c.scratch(split_bytes, split_holder) : nullptr;
    op_ok(attention_rows(q.data(), fused ? nullptr : k->data(), fused ? nullptr : v->data(), y.data(), n,
                         static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(hd), block,
                         valid_dev ? 0 : static_cast<size_t>(valid[0]), valid_dev, fused ? 1 : 0, dt, dt, ws,
                         ws_bytes, c.stream, split, split_bytes),
          "attention");
    return y;
}

// Ops::quantize (src/cuda.cu:934-973).  Cancellation: the reference polls its
// flag before every codebook tile (:946-948); here the VQ kernels read the
// context's mapped flag when they start, the wide and fp32 passes run the
// codebook in windows of kVqCancelWindow codes, and the call reports
// OMNI_CANCELLED once the stream is drained.
// Launch part: uint16 ids of x's rows into `ids` (device), asynchronously.
void quantize_launch(Context &c, const Tensor &x, const Tensor &cb, const Tensor &cbnorm, void *ids,
                     const float *xnorm = nullptr) {
    const int profile = x.bf16 ? OMNI_B200_BF16 : OMNI_B200_F32;
    const size_t ws_bytes = omni_b200_vq_workspace(x.rows, x.cols, cb.rows, profile);
    Tensor ws_holder;
    void *ws = c.scratch(ws_bytes, ws_holder);
    op_ok(vq_argmin(x.data(), cb.data(), cbnorm.data(), ids, x.rows, x.cols, cb.rows, profile, 1, ws, ws_bytes,
                    c.cancel_dev, c.stream, xnorm),
          "quantize");
}

// Reads `rows` uint16 ids back once the stream has drained; kernel errors and
// a cancellation that arrived meanwhile are reported here.
std::vector<uint16_t> read_ids(Context &c, const Tensor &ids, size_t rows) {
    std::vector<uint16_t> out(rows);
    if (rows)
        cuda_ok(cudaMemcpyAsync(out.data(), ids.data(), rows * 2, cudaMemcpyDeviceToHost, c.stream), "ids");
    cuda_ok(cudaStreamSynchronize(c.stream), "quantize");
    op_ok(omni_b200_sync_check(c.stream), "quantize");
    c.check();
    return out;
}

std::vector<float> download(Context &c, const Tensor &t) {
    std::vector<float> out(t.size());
    if (t.size() == 0)
        return out;
    Tensor tmp;
    const float *src = static_cast<const float *>(t.data());
    if (t.bf16) {
        tmp = c.make(t.rows, t.cols, false);
        cuda_ok(static_cast<cudaError_t>(graph::to_float(t.data(), static_cast<float *>(tmp.data()), true,
                                                         t.size(), c.stream)),
                "download");
        src = static_cast<const float *>(tmp.data());
    }
    cuda_ok(cudaMemcpyAsync(out.data(), src, t.size() * 4, cudaMemcpyDeviceToHost, c.stream), "download");
    cuda_ok(cudaStreamSynchronize(c.stream), "download");
    return out;
}

void trace(Context &c, const Tensor &x, const std::string &stage) {
    if (c.trace) {
        const std::vector<float> v = download(c, x);
        c.trace(c.trace_user, stage.c_str(), v.data(), x.rows, x.cols);
    }
}

// True when `p` is device (or managed) memory; such inputs are read in place.
bool device_input(const void *p, int device) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (at.type == cudaMemoryTypeManaged)
        return true;
    if (at.type == cudaMemoryTypeDevice) {
        require(at.device == device, "Input is in another device's memory");
        return true;
    }
    return false;
}

// Activation rows one chunk of a batched call holds at most.
constexpr size_t kChunkRows = 98304;

// Runs body(first_item, items, device_input) over chunks of `chunk` items.
// Host input goes through two device staging buffers: the copy of chunk i+1
// (on c.copy) overlaps the graph of chunk i (on c.stream).
template <class Body>
void for_chunks(Context &c, const float *input, size_t count, size_t item_floats, size_t chunk,
                Body body) {
    const bool on_device = device_input(input, c.model->device);
    const size_t chunks = (count + chunk - 1) / chunk;
    Tensor stage[2];
    auto upload = [&](size_t ci) {
        const int slot = static_cast<int>(ci & 1);
        const size_t i0 = ci * chunk, items = std::min(chunk, count - i0);
        if (ci >= 2)
            cuda_ok(cudaStreamWaitEvent(c.copy, c.done[slot], 0), "copy order");
        cuda_ok(cudaMemcpyAsync(stage[slot].data(), input + i0 * item_floats, items * item_floats * 4,
                                cudaMemcpyHostToDevice, c.copy),
                "upload");
        cuda_ok(cudaEventRecord(c.ready[slot], c.copy), "copy order");
    };
    if (!on_device) {
        for (int i = 0; i < (chunks > 1 ? 2 : 1); ++i)
            stage[i] = c.make(chunk * item_floats, 1, false);
        cuda_ok(cudaEventRecord(c.start, c.stream), "copy order"); // the staging allocations
        cuda_ok(cudaStreamWaitEvent(c.copy, c.start, 0), "copy order");
        upload(0);
    }
    for (size_t ci = 0; ci < chunks; ++ci) {
        c.check();
        const int slot = static_cast<int>(ci & 1);
        const size_t i0 = ci * chunk, items = std::min(chunk, count - i0);
        const float *src = input + i0 * item_floats;
        if (!on_device) {
            cuda_ok(cudaStreamWaitEvent(c.stream, c.ready[slot], 0), "copy order");
            src = static_cast<const float *>(stage[slot].data());
        }
        body(i0, items, src);
        if (!on_device) {
            cuda_ok(cudaEventRecord(c.done[slot], c.stream), "copy order");
            if (ci + 1 < chunks)
                upload(ci + 1);
        }
    }
}

size_t chunk_items(size_t count, size_t rows_per_item) {
    const size_t per = std::max<size_t>(1, kChunkRows / std::max<size_t>(rows_per_item, 1));
    const size_t chunks = (count + per - 1) / per;
    return (count + chunks - 1) / chunks;
}

// Reads the non-finite flag the graph raised (after the stream has drained).
void finite_or_fail(Context &c, const Tensor &flag) {
    int v = 0;
    cuda_ok(cudaMemcpyAsync(&v, flag.data(), sizeof v, cudaMemcpyDeviceToHost, c.stream), "input check");
    cuda_ok(cudaStreamSynchronize(c.stream), "input check");
    require(v == 0, "Input contains a non-finite value");
}

// Inputs a captured graph can read again at replay: device memory, or host
// memory that is page-locked (copies from pageable memory cannot be captured).
bool replayable_input(const void *p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged || at.type == cudaMemoryTypeHost;
}

// Buffers that outlive one batched call's device work: the non-finite flag,
// the features (what omni_context_copy_features returns), the uint16 ids and
// per-item key limits.
struct Bufs {
    Tensor flag, features, ids, keys;
};

// Captures work(b) on the context's stream into a graph, instantiates and
// launches it, and keeps it as the context's replay.  Returns false (nothing
// launched) when the work cannot be captured; a cancellation propagates.
template <class Work> bool capture_and_launch(Context &c, const std::vector<uint64_t> &key, const Bufs &b, Work &work) {
    if (cudaStreamBeginCapture(c.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    c.capturing = true;
    cudaGraph_t g = nullptr;
    try {
        work(b);
    } catch (const Fail &f) {
        c.capturing = false;
        if (cudaStreamEndCapture(c.stream, &g) == cudaSuccess && g)
            cudaGraphDestroy(g);
        cudaGetLastError();
        if (f.code == OMNI_CANCELLED)
            throw;
        c.graphs = false; // this context runs its calls eagerly from now on
        return false;
    }
    c.capturing = false;
    cudaError_t e = cudaStreamEndCapture(c.stream, &g);
    cudaGraphExec_t exec = nullptr;
    if (e == cudaSuccess)
        e = cudaGraphInstantiate(&exec, g, 0);
    if (g)
        cudaGraphDestroy(g);
    if (e == cudaSuccess)
        e = cudaGraphLaunch(exec, c.stream);
    if (e != cudaSuccess) {
        if (exec)
            cudaGraphExecDestroy(exec);
        cudaGetLastError();
        c.graphs = false;
        return false;
    }
    ++c.graph_launches;
    c.replay.key = key;
    c.replay.exec = exec;
    c.replay.flag = b.flag;
    c.replay.features = b.features;
    c.replay.ids = b.ids;
    c.replay.keys = b.keys;
    return true;
}

// One batched call: work(b) (all device work, writing b.flag, b.features and
// b.ids) runs eagerly, or as a CUDA graph when the call repeats -- inputs in
// device or page-locked host memory, no trace callback, the same key as the
// previous call (captured then) or as the captured graph (replayed).  A replay
// checks cancellation before its launch; inside it, the VQ kernels read the
// context's mapped flag as in the eager graph.  Then the ids are read back.
template <class Alloc, class Work>
std::vector<uint16_t> run_batch(Context &c, const std::vector<uint64_t> &key, bool eligible, size_t id_rows,
                                Alloc alloc, Work work) {
    eligible = eligible && c.graphs && !c.trace;
    Bufs b;
    if (eligible && c.replay.exec && c.replay.key == key) {
        c.check();
        cuda_ok(cudaGraphLaunch(c.replay.exec, c.stream), "graph launch");
        ++c.graph_launches;
        b.flag = c.replay.flag;
        b.features = c.replay.features;
        b.ids = c.replay.ids;
        b.keys = c.replay.keys;
    } else {
        if (eligible && key == c.last_key)
            c.drop_replay(); // its buffers go back to the pool before the new ones are made
        b = alloc();
        const bool captured = eligible && key == c.last_key && capture_and_launch(c, key, b, work);
        if (!captured)
            work(b);
    }
    c.last_key = eligible ? key : std::vector<uint64_t>{};
    auto ids = read_ids(c, b.ids, id_rows);
    finite_or_fail(c, b.flag);
    c.features = b.features;
    return ids;
}
} // namespace

// Audio graph (src/runtime.cpp:30-75) over `count` log-mel segments
// [count, mel, frames] (host or device memory) with valid[i] frames each:
// causal conv stem, pre-norm encoder layers with block-causal attention,
// mean-pool by 4, fp32 VQ.  Segments stack as rows; each keeps its own conv
// padding, positions and key limit.  Codes of segment i are its first
// ceil(valid[i] / 8), concatenated in segment order.
std::vector<uint16_t> encode_audio_batch(Context &c, const float *mel, size_t count, uint32_t frames,
                                         const uint32_t *valid) {
    Model &model = *c.model;
    const Model &m = model;
    const Config &cfg = m.cfg;
    c.check();
    // bf16 audio mode (OMNI_B200_AUDIO_BF16=1): weights and activations in bf16
    // with the reference's bf16 rounding points (as its image graph); the VQ
    // stays fp32, on the bf16 features, against the fp32 codebook.
    const bool bf = c.audio_bf16;
    if (bf)
        std::call_once(model.w16_once, [&] {
            for (const auto &kv : model.w) {
                if (kv.first == "codebook.weight" || kv.second.bf16 || model.views.count(kv.first))
                    continue;
                Tensor t = weight_tensor(kv.second.rows, kv.second.cols, true);
                cuda_ok(static_cast<cudaError_t>(graph::convert(static_cast<const float *>(kv.second.data()),
                                                                t.data(), true, t.size(), c.stream)),
                        "bf16 weights");
                model.w16.emplace(kv.first, std::move(t));
            }
            cuda_ok(cudaStreamSynchronize(c.stream), "bf16 weights");
        });
    const size_t C = cfg.input_channels, T = frames, L = (T + 1) / 2, W = cfg.width;
    std::vector<size_t> offset(count + 1, 0);
    for (size_t i = 0; i < count; ++i)
        offset[i + 1] = offset[i] + (valid[i] + 7) / 8;
    std::vector<int> keys(count);
    for (size_t i = 0; i < count; ++i)
        keys[i] = static_cast<int>((valid[i] + 1) / 2);
    const size_t chunk = chunk_items(count, T);
    // Persistent buffers: flag, fp32 features (the VQ input and what
    // omni_context_copy_features returns), ids, and per segment the key limit
    // followed by the first feature row (count + 1 offsets).
    std::vector<int> limits(keys);
    for (size_t i = 0; i <= count; ++i)
        limits.push_back(static_cast<int>(offset[i]));
    auto alloc = [&] {
        Bufs b;
        b.flag = c.make(1, 1, false);
        b.features = c.make(offset[count], W, false);
        b.ids = c.make((offset[count] + 1) / 2, 1, false);
        b.keys = c.make(limits.size(), 1, false);
        cuda_ok(cudaMemcpyAsync(b.keys.data(), limits.data(), limits.size() * 4, cudaMemcpyHostToDevice, c.stream),
                "key counts");
        return b;
    };
    auto work = [&](const Bufs &b) {
        cuda_ok(cudaMemsetAsync(b.flag.data(), 0, 4, c.stream), "input check");
        Tensor flag = b.flag;
        // Squared norms of the feature rows, written with them for the VQ.
        Tensor xn = c.make(offset[count], 1, false);
        const int *row_offsets = static_cast<const int *>(b.keys.data()) + count;
        for_chunks(c, mel, count, C * T, chunk, [&](size_t i0, size_t items, const float *src) {
            cuda_ok(static_cast<cudaError_t>(graph::finite_check(src, items * C * T, static_cast<int *>(flag.data()),
                                                                 c.stream)),
                    "input check");
            Tensor x = c.make(items * T, C, false);
            cuda_ok(static_cast<cudaError_t>(graph::frames_major(src, static_cast<float *>(x.data()), items, C, T,
                                                                 c.stream)),
                    "frames");
            if (bf) {
                Tensor x16 = c.make(items * T, C, true);
                cuda_ok(static_cast<cudaError_t>(graph::convert(static_cast<const float *>(x.data()), x16.data(), true,
                                                                x.size(), c.stream)),
                        "frames");
                x = x16;
            }
            auto conv = [&](const Tensor &in, size_t rows, size_t stride, const char *name) {
                const size_t out_rows = (rows + stride - 1) / stride;
                Tensor g = c.make(items * out_rows, in.cols * 3, in.bf16);
                cuda_ok(static_cast<cudaError_t>(graph::conv_gather(in.data(), g.data(), in.bf16, items, rows,
                                                                    in.cols, stride, c.stream)),
                        "conv gather");
                Tensor y = linear(c, g, m.get(std::string(name) + ".weight", bf),
                                  m.opt(std::string(name) + ".bias", bf));
                gelu_in_place(c, y);
                return y;
            };
            x = conv(x, T, 1, "conv1");
            x = conv(x, T, 2, "conv2");
            const Tensor &pos = m.get("embed_positions.weight", bf);
            cuda_ok(static_cast<cudaError_t>(graph::add_periodic(x.data(), pos.data(), x.bf16, x.size(), L * W,
                                                                 c.stream)),
                    "positions");
            trace(c, x, "embedding");
            const std::vector<int> chunk_keys(keys.begin() + i0, keys.begin() + i0 + items);
            const int *keys_dev = static_cast<const int *>(b.keys.data()) + i0;
            // Each residual add runs fused with the layer norm that follows it; the
            // MLP output `mlp` of layer i joins x at the start of layer i + 1.
            Tensor mlp;
            for (uint32_t i = 0; i < cfg.layers; ++i) {
                c.check();
                const std::string p = "layers." + std::to_string(i) + ".";
                Tensor z = add_norm(c, x, i ? &mlp : nullptr, m.get(p + "self_attn_layer_norm.weight", bf),
                                    m.get(p + "self_attn_layer_norm.bias", bf), 1e-5f);
                if (i)
                    trace(c, x, "layer." + std::to_string(i - 1));
                auto proj = [&](const Tensor &in, const std::string &name) {
                    return linear(c, in, m.get(name + ".weight", bf), m.opt(name + ".bias", bf));
                };
                // Q|K|V from one GEMM (the stacked projections), attended in the
                // fused layout with the unfused scale hd^-1/2.
                Tensor qkv = proj(z, p + "self_attn.qkv");
                z = attention(c, qkv, nullptr, nullptr, cfg.heads, cfg.block_size, true, items, chunk_keys, keys_dev);
                qkv = {};
                z = proj(z, p + "self_attn.out_proj");
                z = add_norm(c, x, &z, m.get(p + "final_layer_norm.weight", bf), m.get(p + "final_layer_norm.bias", bf),
                             1e-5f);
                z = proj(z, p + "fc1");
                gelu_in_place(c, z);
                mlp = proj(z, p + "fc2");
            }
            if (cfg.layers) {
                add_in_place(c, x, mlp);
                trace(c, x, "layer." + std::to_string(cfg.layers - 1));
            }
            // The next cancellation point is the VQ pass (src/runtime.cpp:47-66).
            // Pre-VQ epilogue in one pass (src/runtime.cpp:64-66): mean-pool by
            // pool_size per segment, keep each segment's ceil(valid / 8) rows as
            // fp32 features (bf16 mode: the bf16 pooled values), and write their
            // squared norms for the fp32 VQ.  Pooling the stacked rows equals
            // pooling per segment: L is a multiple of the pool size (frames % 8
            // == 0), so no group straddles two segments.
            cuda_ok(static_cast<cudaError_t>(graph::pool_features(
                        x.data(), x.bf16, items, L, W, cfg.pool_size, row_offsets + i0,
                        static_cast<float *>(b.features.data()), static_cast<float *>(xn.data()), c.stream)),
                    "pool");
        });
        quantize_launch(c, b.features, m.get("codebook.weight"), m.cbnorm, b.ids.data(),
                        static_cast<const float *>(xn.data()));
    };
    std::vector<uint64_t> key{1, reinterpret_cast<uintptr_t>(mel), count, frames, bf ? 1u : 0u};
    key.insert(key.end(), valid, valid + count);
    return run_batch(c, key, replayable_input(mel), offset[count], alloc, work);
}

// Image graph (src/runtime.cpp:76-130) over `count` CHW images of one size
// (host or device memory): patch embedding, interpolated positions, pre-norm
// blocks with fused-QKV attention, 1x1 projection, L2 normalisation, bf16 VQ.
// Images stack as rows; attention runs per image.  Codes in image order.
std::vector<uint16_t> encode_images(Context &c, const float *pixels, size_t count, uint32_t height,
                                    uint32_t width) {
    const Model &m = *c.model;
    const Config &cfg = m.cfg;
    c.check();
    const size_t P = cfg.patch_size, gh = height / P, gw = width / P, n = gh * gw;
    const size_t item_floats = size_t(3) * height * width;
    auto alloc = [&] {
        Bufs b;
        b.flag = c.make(1, 1, false);
        b.features = c.make(count * n, cfg.code_dim, true);
        b.ids = c.make((count * n + 1) / 2, 1, false);
        return b;
    };
    auto work = [&](const Bufs &b) {
        cuda_ok(cudaMemsetAsync(b.flag.data(), 0, 4, c.stream), "input check");
        const Tensor &flag = b.flag, &features = b.features;
        Tensor pos = c.make(n, cfg.width, true);
        cuda_ok(static_cast<cudaError_t>(graph::interpolate(m.get("pos_embed").data(), pos.data(), true,
                                                            cfg.pos_height, gh, gw, cfg.width, c.stream)),
                "interpolate");
        const std::vector<int> all_keys(1, static_cast<int>(n));
        const size_t chunk = chunk_items(count, n);
        for_chunks(c, pixels, count, item_floats, chunk, [&](size_t i0, size_t items, const float *src) {
            cuda_ok(static_cast<cudaError_t>(graph::finite_check(src, items * item_floats,
                                                                 static_cast<int *>(flag.data()), c.stream)),
                    "input check");
            Tensor patches = c.make(items * n, 8 * P * P, true);
            cuda_ok(static_cast<cudaError_t>(graph::image_patches(src, patches.data(), items, height, width, P,
                                                                  c.stream)),
                    "patches");
            Tensor x = linear(c, patches, m.get("patch_embed.proj.weight"), &m.get("patch_embed.proj.bias"), true);
            patches = {};
            trace(c, x, "patch");
            if (i0 == 0)
                trace(c, pos, "position");
            cuda_ok(static_cast<cudaError_t>(graph::add_periodic(x.data(), pos.data(), true, x.size(), pos.size(),
                                                                 c.stream)),
                    "positions");
            trace(c, x, "embedding");
            // Residual adds fused with the following norm, as in the audio graph.
            Tensor mlp;
            for (uint32_t i = 0; i < cfg.layers; ++i) {
                c.check();
                const std::string p = "blocks." + std::to_string(i) + ".";
                auto proj = [&](const Tensor &in, const std::string &name) {
                    return linear(c, in, m.get(name + ".weight"), m.opt(name + ".bias"));
                };
                Tensor z = add_norm(c, x, i ? &mlp : nullptr, m.get(p + "norm1.weight"), m.get(p + "norm1.bias"),
                                    1e-6f);
                if (i)
                    trace(c, x, "layer." + std::to_string(i - 1));
                if (i == 0)
                    trace(c, z, "norm1.0");
                z = proj(z, p + "attn.qkv");
                if (i == 0)
                    trace(c, z, "qkv.0");
                z = attention(c, z, nullptr, nullptr, cfg.heads, 0, true, items, all_keys, nullptr);
                if (i == 0)
                    trace(c, z, "attention.0");
                z = proj(z, p + "attn.proj");
                z = add_norm(c, x, &z, m.get(p + "norm2.weight"), m.get(p + "norm2.bias"), 1e-6f);
                if (i == 0)
                    trace(c, x, "residual1.0");
                z = proj(z, p + "mlp.fc1");
                if (i == 0)
                    trace(c, z, "fc1.0");
                gelu_in_place(c, z);
                if (i == 0)
                    trace(c, z, "gelu.0");
                mlp = proj(z, p + "mlp.fc2");
                if (i == 0)
                    trace(c, mlp, "fc2.0");
            }
            if (cfg.layers) {
                add_in_place(c, x, mlp);
                trace(c, x, "layer." + std::to_string(cfg.layers - 1));
            }
            c.check();
            void *feat = static_cast<__nv_bfloat16 *>(features.data()) + i0 * n * cfg.code_dim;
            if (c.trace) { // the "projected" stage needs image_conv's output on its own
                x = linear(c, x, m.get("quant_conv.weight"), &m.get("quant_conv.bias"), true);
                trace(c, x, "projected");
                cuda_ok(static_cast<cudaError_t>(graph::normalize(x.data(), feat, true, x.rows, x.cols, c.stream)),
                        "normalize");
            } else {
                // image_conv's bias (added after the rounded GEMM) and the L2
                // normalisation in one pass over the projected rows.
                x = linear(c, x, m.get("quant_conv.weight"), nullptr);
                cuda_ok(static_cast<cudaError_t>(graph::bias_normalize(x.data(), m.get("quant_conv.bias").data(), feat,
                                                                       x.rows, x.cols, c.stream)),
                        "normalize");
            }
        });
        quantize_launch(c, features, m.get("quantize.embedding.weight"), m.cbnorm, b.ids.data());
    };
    const std::vector<uint64_t> key{2, reinterpret_cast<uintptr_t>(pixels), count, height, width};
    return run_batch(c, key, replayable_input(pixels), count * n, alloc, work);
}

} // namespace rt
} // namespace omni_b200

// --------------------------------------------------------------- C ABI
struct omni_model {
    std::shared_ptr<omni_b200::rt::Model> impl;
};
struct omni_context {
    omni_b200::rt::Context impl;
};

namespace {
thread_local std::string g_abi_error;
template <class F> int guarded(F f) {
    try {
        g_abi_error.clear();
        f();
        return OMNI_OK;
    } catch (const omni_b200::rt::Fail &e) {
        g_abi_error = e.what();
        return e.code;
    } catch (const std::bad_alloc &) {
        g_abi_error = "Allocation failed";
        return OMNI_OUT_OF_MEMORY;
    } catch (const std::exception &e) {
        g_abi_error = e.what();
        return OMNI_INTERNAL_ERROR;
    } catch (...) {
        g_abi_error = "Unknown native failure";
        return OMNI_INTERNAL_ERROR;
    }
}
struct Running {
    omni_b200::rt::Context &c;
    explicit Running(omni_b200::rt::Context &ctx) : c(ctx) {
        omni_b200::rt::require(!c.running.test_and_set(), "Context is already executing");
    }
    ~Running() { c.running.clear(); }
};
} // namespace

using omni_b200::rt::require;

extern "C" {
const char *omni_last_error(void) { return g_abi_error.c_str(); }
const char *omni_version(void) { return "0.1.0+b200"; }
int omni_has_cuda(void) {
    int n = 0;
    return cudaGetDeviceCount(&n) == cudaSuccess && n > 0 ? 1 : 0;
}
int omni_model_load(const char *path, int backend, int device, omni_model **out) {
    if (out)
        *out = nullptr;
    return guarded([&] {
        require(out != nullptr, "Output handle is null");
        auto m = omni_b200::rt::load_model(path, backend, device);
        *out = new omni_model{std::move(m)};
    });
}
void omni_model_free(omni_model *m) { delete m; }
int omni_model_get_info(const omni_model *m, omni_model_info *out) {
    return guarded([&] {
        require(m && out && out->struct_size >= sizeof(omni_model_info), "Invalid model info arguments");
        const auto &c = m->impl->cfg;
        *out = {sizeof(omni_model_info), c.kind, c.layers, c.width, c.heads, c.code_dim, c.vocab_size,
                uint32_t(m->impl->backend), m->impl->weight_bytes};
    });
}
int omni_context_create(omni_model *m, omni_context **out) {
    if (out)
        *out = nullptr;
    return guarded([&] {
        require(m && out, "Invalid context arguments");
        auto c = std::make_unique<omni_context>();
        c->impl.model = m->impl;
        omni_b200::rt::cuda_ok(cudaSetDevice(m->impl->device), "set device");
        omni_b200::rt::cuda_ok(cudaStreamCreateWithFlags(&c->impl.stream, cudaStreamNonBlocking),
                               "stream create");
        omni_b200::rt::blas_ok(cublasCreate(&c->impl.blas), "cuBLAS handle");
        omni_b200::rt::blas_ok(cublasSetStream(c->impl.blas, c->impl.stream), "cuBLAS stream");
        omni_b200::rt::cuda_ok(cudaMalloc(&c->impl.blas_ws, size_t(32) << 20), "cuBLAS workspace");
        omni_b200::rt::blas_ok(cublasSetWorkspace(c->impl.blas, c->impl.blas_ws, size_t(32) << 20), "cuBLAS workspace");
        const char *graphs = std::getenv("OMNI_B200_GRAPHS");
        c->impl.graphs = !(graphs && *graphs == '0');
        omni_b200::rt::cuda_ok(cudaStreamCreateWithFlags(&c->impl.copy, cudaStreamNonBlocking), "stream create");
        omni_b200::rt::cuda_ok(cudaHostAlloc(reinterpret_cast<void **>(&c->impl.cancel_host), sizeof(int),
                                             cudaHostAllocMapped),
                               "cancel flag");
        *c->impl.cancel_host = 0;
        omni_b200::rt::cuda_ok(cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->impl.cancel_dev),
                                                        c->impl.cancel_host, 0),
                               "cancel flag");
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = m->impl->device;
        omni_b200::rt::cuda_ok(cudaMemPoolCreate(&c->impl.pool, &props), "memory pool");
        uint64_t keep = ~uint64_t(0);
        omni_b200::rt::cuda_ok(cudaMemPoolSetAttribute(c->impl.pool, cudaMemPoolAttrReleaseThreshold, &keep),
                               "memory pool");
        const char *lt = std::getenv("OMNI_B200_CUBLASLT");
        if (!(lt && *lt == '0')) {
            omni_b200::rt::blas_ok(cublasLtCreate(&c->impl.lt), "cuBLASLt handle");
            c->impl.lt_ws_bytes = size_t(32) << 20;
            omni_b200::rt::cuda_ok(cudaMalloc(&c->impl.lt_ws, c->impl.lt_ws_bytes), "cuBLASLt workspace");
        }
        for (cudaEvent_t *e : {&c->impl.ready[0], &c->impl.ready[1], &c->impl.done[0], &c->impl.done[1],
                               &c->impl.start})
            omni_b200::rt::cuda_ok(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "event create");
        const char *fast = std::getenv("OMNI_B200_AUDIO_BF16");
        c->impl.audio_bf16 = fast && *fast && *fast != '0';
        // fp32-profile GEMMs: BF16x9 emulation when the process's cuBLAS has it
        // (resolved at run time: a process may have loaded an older cuBLAS 12,
        // same soname, before this library).  OMNI_B200_FP32_EMULATION=0 keeps
        // plain fp32; =1 requires the emulation.
        const char *emu = std::getenv("OMNI_B200_FP32_EMULATION");
        const bool off = emu && *emu == '0', required = emu && *emu && *emu != '0';
        using SetStrategy = cublasStatus_t (*)(cublasHandle_t, cublasEmulationStrategy_t);
        SetStrategy set = nullptr;
        if (void *h = dlopen("libcublas.so.12", RTLD_LAZY | RTLD_NOLOAD)) { // the copy already bound
            set = reinterpret_cast<SetStrategy>(dlsym(h, "cublasSetEmulationStrategy"));
            dlclose(h);
        }
        require(set != nullptr || !required, "OMNI_B200_FP32_EMULATION needs cuBLAS 12.9 or newer in this process",
                OMNI_UNSUPPORTED);
        if (set && !off) {
            omni_b200::rt::blas_ok(set(c->impl.blas, CUBLAS_EMULATION_STRATEGY_EAGER), "cuBLAS emulation strategy");
            c->impl.fp32_emulated = true;
        }
        *out = c.release();
    });
}
void omni_context_free(omni_context *c) { delete c; }
void omni_context_cancel(omni_context *c) {
    if (c) {
        c->impl.cancelled.store(true);
        if (c->impl.cancel_host)
            *reinterpret_cast<volatile int *>(c->impl.cancel_host) = 1;
    }
}
void omni_context_reset_cancel(omni_context *c) {
    if (c) {
        if (c->impl.cancel_host)
            *reinterpret_cast<volatile int *>(c->impl.cancel_host) = 0;
        c->impl.cancelled.store(false);
    }
}
int omni_context_set_trace(omni_context *c, omni_trace_callback callback, void *user) {
    return guarded([&] {
        require(c != nullptr, "Invalid context");
        Running guard(c->impl);
        c->impl.trace = callback;
        c->impl.trace_user = user;
    });
}
int omni_encode_audio(omni_context *c, const float *mel, uint32_t frames, uint32_t valid,
                      uint16_t *codes, size_t capacity, size_t *count) {
    return omni_b200_encode_audio_batch(c, mel, 1, frames, &valid, codes, capacity, count);
}
int omni_encode_image(omni_context *c, const float *pixels, uint32_t height, uint32_t width,
                      uint16_t *codes, size_t capacity, size_t *count) {
    return omni_b200_encode_images(c, pixels, 1, height, width, codes, capacity, count);
}
int omni_b200_encode_audio_batch(omni_context *c, const float *mel, uint32_t items, uint32_t frames,
                                 const uint32_t *valid, uint16_t *codes, size_t capacity, size_t *count) {
    return guarded([&] {
        require(c && mel && valid && count, "Invalid audio pointers");
        const auto &cfg = c->impl.model->cfg;
        require(cfg.kind == OMNI_AUDIO, "Model is not an audio tokenizer");
        require(items > 0, "Invalid audio batch size");
        require(frames > 0 && frames % 8 == 0 && frames <= 3000 && frames / 2 <= cfg.pos_height,
                "Invalid audio frame lengths");
        size_t total = 0;
        for (uint32_t i = 0; i < items; ++i) {
            require(valid[i] > 0 && valid[i] <= frames, "Invalid audio frame lengths");
            total += (valid[i] + 7) / 8;
        }
        *count = total;
        require(codes && capacity >= *count, "Output capacity is too small");
        Running guard(c->impl);
        omni_b200::rt::cuda_ok(cudaSetDevice(c->impl.model->device), "set device");
        c->impl.features = {};
        const auto ids = omni_b200::rt::encode_audio_batch(c->impl, mel, items, frames, valid);
        std::copy(ids.begin(), ids.end(), codes);
    });
}
int omni_b200_encode_images(omni_context *c, const float *pixels, uint32_t items, uint32_t height,
                            uint32_t width, uint16_t *codes, size_t capacity, size_t *count) {
    return guarded([&] {
        require(c && pixels && count, "Invalid image pointers");
        const auto &cfg = c->impl.model->cfg;
        require(cfg.kind == OMNI_IMAGE, "Model is not an image tokenizer");
        require(items > 0, "Invalid image batch size");
        require(height > 0 && width > 0 && height % cfg.patch_size == 0 && width % cfg.patch_size == 0,
                "Invalid image dimensions");
        const uint64_t patches = uint64_t(height / cfg.patch_size) * (width / cfg.patch_size);
        // Activation, patch, attention and VQ buffers stay within int-indexed BLAS
        // dimensions (the reference's capacity rule, src/runtime.cpp:253-262); a
        // batch is processed in chunks of whole images, so the rule is per image.
        const uint64_t columns = std::max({uint64_t(8) * cfg.patch_size * cfg.patch_size,
                                          uint64_t(3) * cfg.width, uint64_t(cfg.ffn),
                                          uint64_t(cfg.code_dim), uint64_t(256) * cfg.heads,
                                          uint64_t(1024)});
        const uint64_t elements = std::min(uint64_t(std::numeric_limits<int>::max()),
                                          uint64_t(std::numeric_limits<size_t>::max() / sizeof(float)));
        require(patches <= elements / columns, "Image dimensions exceed native tensor indexing capacity");
        require(patches * items <= uint64_t(std::numeric_limits<int>::max()), "Image batch is too large");
        *count = static_cast<size_t>(patches * items);
        require(codes && capacity >= *count, "Output capacity is too small");
        Running guard(c->impl);
        omni_b200::rt::cuda_ok(cudaSetDevice(c->impl.model->device), "set device");
        c->impl.features = {};
        const auto ids = omni_b200::rt::encode_images(c->impl, pixels, items, height, width);
        std::copy(ids.begin(), ids.end(), codes);
    });
}
int omni_context_copy_features(omni_context *c, float *out, size_t capacity, size_t *count) {
    return guarded([&] {
        require(c && count, "Invalid feature pointers");
        Running guard(c->impl);
        *count = c->impl.features.size();
        require(*count > 0, "No completed feature tensor");
        require(out && capacity >= *count, "Feature output capacity is too small");
        omni_b200::rt::cuda_ok(cudaSetDevice(c->impl.model->device), "set device");
        const auto v = omni_b200::rt::download(c->impl, c->impl.features);
        std::copy(v.begin(), v.end(), out);
    });
}
uint64_t omni_context_peak_workspace(const omni_context *c) {
    return c ? c->impl.memory->peak.load() : 0;
}
uint64_t omni_b200_context_graph_launches(const omni_context *c) { return c ? c->impl.graph_launches : 0; }
} // extern "C"
