// vq.h -- host-side interface of the sm_100a VQ argmin kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace omni_b200 {

struct VqParams {
    CUtensorMap tx0, tx1, tc0, tc1; // x / codebook tile maps, chunk 0 and chunk 1
    const void *x;                  // bf16 [rows, dim]
    const void *cbnorm;             // bf16 [codes] (|c|^2 in the bf16 profile)
    void *keys;                     // uint64 [rows]: (order bits of dist) << 32 | id
    int rows, dim, codes;
    int slices, slice_codes;
    int *err;
};

struct VqArgs {
    const void *x = nullptr, *codebook = nullptr, *cbnorm = nullptr;
    int rows = 0, dim = 0, codes = 0;
    void *keys = nullptr; // scratch: 8 bytes per row
    void *ids = nullptr;  // output ids
    int ids_u16 = 0;      // 1: uint16 ids, 0: int32 ids
    int *err = nullptr;
    // Optional cancellation flag the device can read (mapped pinned host memory
    // or device memory): the streamed kernels run the codebook in windows of
    // kVqCancelWindow codes (a multiple of it when the rows are too few to fill
    // the GPU), one launch each; the flag is copied to device memory in stream
    // order just before each window's launch, and a launch whose copy is
    // nonzero skips its window (the ids are then incomplete; the caller reports
    // the cancellation).
    const volatile int *cancel = nullptr;
    // fp32 profile: the rows' squared norms when the caller produced them with
    // x (any fp32 summation order: they enter only the approximate search,
    // whose window bounds fp32 rounding of the sum); the squares pass is then
    // skipped.
    const float *xnorm = nullptr;
};

constexpr int kVqCancelWindow = 4096; // codes per launch when a cancel flag is given

int vq_padded_dim(int dim);
int vq_bf16_launch(const VqArgs &args, cudaStream_t stream);

// ---- streamed kernels (vq_stream_sm100.cu): bf16 profile with dim > 128 and
// the fp32 profile.
constexpr int kVqCandCap = 32; // fp32 profile: candidates kept per row
enum VqsMode { kVqsBf16 = 0, kVqsApprox = 1, kVqsCand = 2 };

struct VqsParams {
    CUtensorMap tx, tc;           // x / codebook maps, 128-byte column chunks
    const float *xn;              // [rows] |x|^2 (bf16 profile: the bf16 value)
    const void *cbnorm;           // bf16 [codes] (bf16 profile) or f32 [codes]
    unsigned long long *keys;     // [rows] (order bits of dist) << 32 | id
    unsigned *cand_count;         // fp32 profile: [rows]
    unsigned *cand;               // fp32 profile: [rows][kVqCandCap]
    int rows, dim, codes, chunks;
    int code_lo, code_hi;         // codebook window of this launch, [code_lo, code_hi)
    int slices, slice_codes;      // the window split into slices of slice_codes codes
    float win_a, win_c, win_s;    // fp32 profile: window a |x||c| + c |c|^2 + s (|x|^2 + |c|^2)
    const volatile int *cancel;   // device copy of the flag: nonzero skips the window
    int *err;
};

// omni_b200_vq_argmin with an optional cancellation flag (see VqArgs::cancel);
// the encoder graphs pass their context's flag.
int vq_argmin(const void *x, const void *codebook, const void *cbnorm, void *ids, size_t rows, size_t dim,
              size_t codes, int profile, int ids_u16, void *workspace, size_t workspace_bytes,
              const volatile int *cancel, cudaStream_t stream, const float *xnorm = nullptr);

// Scratch bytes for vq_stream_launch (VqArgs::keys points at it).
size_t vq_stream_workspace(size_t rows, int profile_fp32);
int vq_stream_launch(const VqArgs &args, int profile_fp32, cudaStream_t stream);

} // namespace omni_b200
