// tma.h -- tensor-map helpers (2- or 4-byte elements, swizzle chosen from the box row bytes:
// 128 B -> 128B swizzle, 64 B -> 64B, 32 B -> 32B).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace omni_b200 {
// Returns 0, -1 (no driver entry point) or 1000 + CUresult.  swizzle_bytes
// (32, 64 or 128) overrides the swizzle implied by the box row bytes.
int encode_tiled(CUtensorMap *map, const void *base, bool bf16, int rank, const uint64_t *dims,
                 const uint64_t *byte_strides, const uint32_t *box, int swizzle_bytes = 0);
// swizzle_bytes value selecting the 128-byte swizzle of 32-byte atoms (the only
// shared-memory layout the tensor cores read for MN-major tf32 operands).
constexpr int kSwizzle128Atom32 = -32;
// fp32 elements; the swizzle follows the box row bytes like encode_tiled unless
// swizzle_bytes selects one (32, 64, 128 or kSwizzle128Atom32).
int encode_tiled_f32(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
                     const uint64_t *byte_strides, const uint32_t *box, int swizzle_bytes = 0);
// Row-major [rows, cols] matrix; box of box_w columns x box_rows rows.
int make_map_2d(CUtensorMap *map, const void *base, int cols, long long rows, int box_w,
                int box_rows, bool bf16 = true);
// Row-major fp32 [rows, cols] matrix; box of box_w columns x box_rows rows
// (box_w * 4 bytes = 32, 64 or 128 selects the swizzle).
int make_map_2d_f32(CUtensorMap *map, const void *base, int cols, long long rows, int box_w,
                    int box_rows);
} // namespace omni_b200
