// norms.cu -- per-row squared norms with the reference's profile rounding.
//
// omni-tokenizer src/cpu.cpp:216-226 (Cpu::squares): n = sum over columns, in
// column order, of x^2 (each square rounded to bf16 in the bf16 profile), then
// n is rounded to bf16 in the bf16 profile.  One thread per row keeps that
// exact order (the reference's GPU kernel, src/cuda.cu:215-225, sums in a tree
// and so can differ from its own CPU path in the last bf16 bit).
// __fmul_rn/__fadd_rn keep the compiler from contracting into an FMA.
#include "norms.h"

#include <cuda_bf16.h>
#include <stdint.h>

namespace omni_b200 {

__global__ void squares_kernel(const void *x, void *out, long long rows, long long cols, int bf16,
                               int out_bf16) {
    for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < rows;
         r += static_cast<long long>(gridDim.x) * blockDim.x) {
        float n = 0.f;
        if (bf16) {
            const __nv_bfloat16 *xr = static_cast<const __nv_bfloat16 *>(x) + r * cols;
            for (long long j = 0; j < cols; ++j) {
                const float v = __bfloat162float(xr[j]);
                n = __fadd_rn(n, __bfloat162float(__float2bfloat16_rn(__fmul_rn(v, v))));
            }
            n = __bfloat162float(__float2bfloat16_rn(n));
        } else {
            const float *xr = static_cast<const float *>(x) + r * cols;
            for (long long j = 0; j < cols; ++j)
                n = __fadd_rn(n, __fmul_rn(xr[j], xr[j]));
        }
        if (out_bf16)
            static_cast<__nv_bfloat16 *>(out)[r] = __float2bfloat16_rn(n);
        else
            static_cast<float *>(out)[r] = n;
    }
}

int squares_launch(const void *x, void *out, long long rows, long long cols, int bf16, int out_bf16,
                   cudaStream_t stream) {
    if (rows <= 0)
        return 0;
    long long blocks = (rows + 127) / 128;
    if (blocks > 148 * 8)
        blocks = 148 * 8;
    squares_kernel<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(x, out, rows, cols, bf16,
                                                                      out_bf16);
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
