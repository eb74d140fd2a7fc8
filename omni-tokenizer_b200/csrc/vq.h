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
};

int vq_padded_dim(int dim);
int vq_bf16_launch(const VqArgs &args, cudaStream_t stream);

} // namespace omni_b200
