// norms.cu -- per-row squared norms with the reference's profile rounding.
//
// omni-tokenizer src/cpu.cpp:216-226 (Cpu::squares): n = sum over columns, in
// column order, of x^2 (each square rounded to bf16 in the bf16 profile), then
// n is rounded to bf16 in the bf16 profile.  One thread per row keeps that
// exact order (the reference's GPU kernel, src/cuda.cu:215-225, sums in a tree
// and so can differ from its own CPU path in the last bf16 bit).
// __fmul_rn/__fadd_rn keep the compiler from contracting into an FMA.
//
// squares_rows8 (16-byte aligned rows): one warp per 8 rows.  Per step the
// warp reads an [8 rows x 32 VEC columns] tile with one coalesced 16-byte load
// per lane and row, writes the products (squared, rounded as the profile says)
// to shared memory, and lane r < 8 adds row r's products in column order while
// the next tile's loads are in flight.  Columns past the end count as +0
// products, which leave a sum of squares unchanged bit for bit.  Other layouts
// take squares_kernel (one thread per row).
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

constexpr int kSqWarps = 4;

template <bool BF16> __global__ void __launch_bounds__(kSqWarps * 32)
    squares_rows8(const void *x, void *out, long long rows, long long cols, int out_bf16) {
    constexpr int VEC = BF16 ? 8 : 4; // elements per 16-byte load
    constexpr int TW = 32 * VEC;      // tile width (columns)
    __shared__ float prod[kSqWarps][8][TW + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long groups = (rows + 7) / 8;
    const int esize = BF16 ? 2 : 4;
    const long long pitch = cols * esize; // bytes per row (a multiple of 16)
    const char *base = static_cast<const char *>(x);
    for (long long grp = blockIdx.x * static_cast<long long>(kSqWarps) + warp; grp < groups;
         grp += static_cast<long long>(gridDim.x) * kSqWarps) {
        const long long r0 = grp * 8;
        const int nr = rows - r0 < 8 ? static_cast<int>(rows - r0) : 8;
        uint4 v[8];
        auto load = [&](long long c0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const long long c = c0 + static_cast<long long>(lane) * VEC;
                v[i] = (i < nr && c < cols)
                           ? __ldg(reinterpret_cast<const uint4 *>(base + (r0 + i) * pitch + c * esize))
                           : make_uint4(0u, 0u, 0u, 0u);
            }
        };
        float n = 0.f;
        load(0);
        for (long long c0 = 0; c0 < cols; c0 += TW) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float *dst = &prod[warp][i][lane * VEC];
                const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if constexpr (BF16) {
                        const float lo = __uint_as_float(w[e] << 16), hi = __uint_as_float(w[e] & 0xffff0000u);
                        dst[2 * e] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(lo, lo)));
                        dst[2 * e + 1] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(hi, hi)));
                    } else {
                        const float f = __uint_as_float(w[e]);
                        dst[e] = __fmul_rn(f, f);
                    }
                }
            }
            __syncwarp();
            if (c0 + TW < cols)
                load(c0 + TW); // in flight during the sums below
            if (lane < 8) {
                const float *row = prod[warp][lane];
#pragma unroll 16
                for (int j = 0; j < TW; ++j)
                    n = __fadd_rn(n, row[j]);
            }
            __syncwarp();
        }
        if (lane < nr) {
            if (BF16)
                n = __bfloat162float(__float2bfloat16_rn(n));
            if (out_bf16)
                static_cast<__nv_bfloat16 *>(out)[r0 + lane] = __float2bfloat16_rn(n);
            else
                static_cast<float *>(out)[r0 + lane] = n;
        }
    }
}

int squares_launch(const void *x, void *out, long long rows, long long cols, int bf16, int out_bf16,
                   cudaStream_t stream) {
    if (rows <= 0)
        return 0;
    const int esize = bf16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(x) % 16 == 0 && (cols * esize) % 16 == 0 && cols >= 64) {
        const long long groups = (rows + 7) / 8;
        long long blocks = (groups + kSqWarps - 1) / kSqWarps;
        if (blocks > 148 * 16)
            blocks = 148 * 16;
        if (bf16)
            squares_rows8<true><<<static_cast<unsigned>(blocks), kSqWarps * 32, 0, stream>>>(x, out, rows, cols,
                                                                                            out_bf16);
        else
            squares_rows8<false><<<static_cast<unsigned>(blocks), kSqWarps * 32, 0, stream>>>(x, out, rows, cols,
                                                                                             out_bf16);
        return static_cast<int>(cudaGetLastError());
    }
    long long blocks = (rows + 127) / 128;
    if (blocks > 148 * 8)
        blocks = 148 * 8;
    squares_kernel<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(x, out, rows, cols, bf16,
                                                                      out_bf16);
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
