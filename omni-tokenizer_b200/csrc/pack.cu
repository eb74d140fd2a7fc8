// pack.cu -- repacks attention operands that TMA cannot read directly (head
// dims whose rows are not 16-byte multiples, unaligned strides) into a
// head-major [heads, n, HDP] buffer with zero padding beyond head_dim: bf16 or
// fp16 for the 2-byte kernel, fp32 (unchanged values) for the split-precision
// fp32 kernel.  Replaces the role of pack_kernel in
// omni-tokenizer src/cuda.cu:226-238 (which fed cuBLAS fp32 SGEMMs).
#include "pack.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace omni_b200 {

__device__ __forceinline__ float load_elem(const void *p, long long i, int dtype) {
    if (dtype == 0)
        return static_cast<const float *>(p)[i];
    if (dtype == 1)
        return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    return __half2float(static_cast<const __half *>(p)[i]);
}

// One thread per output pair (two consecutive padded head-dim elements).
// fp16 sources stay fp16 (the kernel then runs kind::f16 with fp16 operands);
// fp32 and bf16 sources become bf16.
__global__ void pack_heads_kernel(const void *src, int dtype, long long s_token, long long s_head,
                                  int n, int heads, int hd, int hdp, uint32_t *dst) {
    const long long pairs = static_cast<long long>(heads) * n * (hdp / 2);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < pairs;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int e = static_cast<int>(i % (hdp / 2)) * 2;
        const long long row = i / (hdp / 2); // h * n + t
        const int t = static_cast<int>(row % n), h = static_cast<int>(row / n);
        const long long base = t * s_token + h * s_head;
        const float a = e < hd ? load_elem(src, base + e, dtype) : 0.f;
        const float b = e + 1 < hd ? load_elem(src, base + e + 1, dtype) : 0.f;
        if (dtype == 2) {
            __half2 v = __floats2half2_rn(a, b);
            dst[i] = *reinterpret_cast<uint32_t *>(&v);
        } else {
            __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
            dst[i] = *reinterpret_cast<uint32_t *>(&v);
        }
    }
}

// fp32 copy for the split-precision kernel: one thread per output element.
__global__ void pack_heads_f32_kernel(const float *src, long long s_token, long long s_head, int n,
                                      int heads, int hd, int hdp, float *dst) {
    const long long total = static_cast<long long>(heads) * n * hdp;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int e = static_cast<int>(i % hdp);
        const long long row = i / hdp; // h * n + t
        const int t = static_cast<int>(row % n), h = static_cast<int>(row / n);
        dst[i] = e < hd ? src[t * s_token + h * s_head + e] : 0.f;
    }
}

int pack_heads_f32(const float *src, long long s_token, long long s_head, int n, int heads, int hd,
                   int hdp, float *dst, cudaStream_t stream) {
    const long long total = static_cast<long long>(heads) * n * hdp;
    if (total == 0)
        return 0;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16)
        blocks = 148 * 16;
    pack_heads_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, s_token, s_head, n, heads,
                                                                             hd, hdp, dst);
    return static_cast<int>(cudaGetLastError());
}

int pack_heads(const void *src, int dtype, long long s_token, long long s_head, int n, int heads,
               int hd, int hdp, void *dst, cudaStream_t stream) {
    const long long pairs = static_cast<long long>(heads) * n * (hdp / 2);
    if (pairs == 0)
        return 0;
    long long blocks = (pairs + 255) / 256;
    if (blocks > 148 * 16)
        blocks = 148 * 16;
    pack_heads_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        src, dtype, s_token, s_head, n, heads, hd, hdp, static_cast<uint32_t *>(dst));
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
