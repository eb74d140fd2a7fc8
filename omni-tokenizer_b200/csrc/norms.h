// norms.h -- per-row squared norms (reference Ops::squares semantics).
#pragma once
#include <cuda_runtime.h>

namespace omni_b200 {
// x is [rows, cols] of bf16 (bf16 != 0) or f32; out is [rows] of bf16 or f32.
int squares_launch(const void *x, void *out, long long rows, long long cols, int bf16, int out_bf16,
                   cudaStream_t stream);
} // namespace omni_b200
