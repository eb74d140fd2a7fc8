// tma.cu -- TMA tensor-map encoding shared by the kernels.  The driver's
// cuTensorMapEncodeTiled is fetched through the runtime's entry-point query,
// so the library has no link-time dependency on libcuda.
#include "tma.h"

#include <mutex>

namespace omni_b200 {
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

CUtensorMapSwizzle swizzle_for(int row_bytes) {
    return row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
           : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                             : CU_TENSOR_MAP_SWIZZLE_32B;
}
} // namespace

namespace {
// swizzle_bytes: 32, 64 or 128 (16-byte atoms), kSwizzle128Atom32 (128-byte span of
// 32-byte atoms), or 0 to follow the box row bytes.
int encode_typed(CUtensorMap *map, const void *base, CUtensorMapDataType type, int elem_bytes,
                 int rank, const uint64_t *dims, const uint64_t *byte_strides,
                 const uint32_t *box, int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn)
        return -1;
    cuuint64_t d[5];
    cuuint64_t s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank)
            s[i] = byte_strides[i];
    }
    const CUresult r =
        fn(map, type, static_cast<cuuint32_t>(rank), const_cast<void *>(base), d, s, b, e,
           CU_TENSOR_MAP_INTERLEAVE_NONE,
           swizzle_bytes == kSwizzle128Atom32
               ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
               : swizzle_for(swizzle_bytes > 0 ? swizzle_bytes : static_cast<int>(box[0]) * elem_bytes),
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r) + 1000;
}
} // namespace

int encode_tiled(CUtensorMap *map, const void *base, bool bf16, int rank, const uint64_t *dims,
                 const uint64_t *byte_strides, const uint32_t *box, int swizzle_bytes) {
    return encode_typed(map, base,
                        bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        rank, dims, byte_strides, box, swizzle_bytes);
}

int encode_tiled_f32(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
                     const uint64_t *byte_strides, const uint32_t *box, int swizzle_bytes) {
    return encode_typed(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rank, dims, byte_strides, box,
                        swizzle_bytes);
}

int make_map_2d_f32(CUtensorMap *map, const void *base, int cols, long long rows, int box_w,
                    int box_rows) {
    const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(cols) * 4};
    const uint32_t box[2] = {static_cast<uint32_t>(box_w), static_cast<uint32_t>(box_rows)};
    return encode_typed(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 2, dims, strides, box, 0);
}

int make_map_2d(CUtensorMap *map, const void *base, int cols, long long rows, int box_w,
                int box_rows, bool bf16) {
    const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(cols) * 2};
    const uint32_t box[2] = {static_cast<uint32_t>(box_w), static_cast<uint32_t>(box_rows)};
    return encode_tiled(map, base, bf16, 2, dims, strides, box);
}

} // namespace omni_b200
