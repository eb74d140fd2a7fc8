// graph_kernels.cu -- the non-hot operators of the encoder graphs.
//
// Each kernel restates one operator of omni-tokenizer's CPU backend
// (src/cpu.cpp) with the same rounding points: in the bf16 profile a result is
// rounded to bf16 exactly once, where Cpu applies r(x, true).  Products and
// sums use __fmul_rn / __fadd_rn where the reference's order matters, so that
// the compiler does not contract them into FMAs the reference does not use.
#include "graph_kernels.h"
#include "sm100.cuh"

#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>
#include <algorithm>
#include <mutex>

namespace omni_b200 {
namespace graph {
namespace {

__device__ __forceinline__ float ld(const void *p, size_t i, bool bf16) {
    return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i])
                : static_cast<const float *>(p)[i];
}
__device__ __forceinline__ void st(void *p, size_t i, float v, bool bf16) {
    if (bf16)
        static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else
        static_cast<float *>(p)[i] = v;
}
// The value a bf16-profile result holds after rounding (fp32 otherwise).
__device__ __forceinline__ float rnd(float v, bool bf16) {
    return bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

unsigned blocks_for(size_t n, unsigned threads) {
    size_t b = (n + threads - 1) / threads;
    return static_cast<unsigned>(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}
int status() { return static_cast<int>(cudaGetLastError()); }

#define GRID_STRIDE(i, n)                                                                          \
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < (n);         \
         i += static_cast<size_t>(gridDim.x) * blockDim.x)

// 16-byte vectors: 8 bf16 or 4 fp32 values.
template <bool BF16> constexpr int kVec = BF16 ? 8 : 4;

template <bool BF16> __device__ __forceinline__ void vload(const void *p, size_t i, float *v) {
    const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const char *>(p) + i * (BF16 ? 2 : 4));
    if constexpr (BF16) {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(h[k]);
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
        }
    } else {
        v[0] = __uint_as_float(u.x);
        v[1] = __uint_as_float(u.y);
        v[2] = __uint_as_float(u.z);
        v[3] = __uint_as_float(u.w);
    }
}

template <bool BF16> __device__ __forceinline__ void vstore(void *p, size_t i, const float *v) {
    uint4 u;
    if constexpr (BF16) {
        __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    } else {
        u = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
    }
    *reinterpret_cast<uint4 *>(static_cast<char *>(p) + i * (BF16 ? 2 : 4)) = u;
}

__device__ __forceinline__ float gelu_erf(float z) {
    return __fmul_rn(__fmul_rn(0.5f, z), __fadd_rn(1.f, erff(__fmul_rn(z, 0.7071067811865475244f))));
}

// Elementwise kernels keep two 16-byte vectors per thread in flight: both are
// loaded before either is computed or stored.
template <bool BF16> __global__ void k_gelu_vec(void *__restrict__ x, size_t nvec) {
    constexpr int N = kVec<BF16>;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nvec; i += 2 * stride) {
        const size_t j = i + stride;
        float v[2][N];
        vload<BF16>(x, i * N, v[0]);
        if (j < nvec)
            vload<BF16>(x, j * N, v[1]);
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int k = 0; k < N; ++k)
                v[u][k] = gelu_erf(v[u][k]);
        vstore<BF16>(x, i * N, v[0]);
        if (j < nvec)
            vstore<BF16>(x, j * N, v[1]);
    }
}

// bf16 GELU by table: the input of the bf16 profile's GELU is a bf16 value, so
// the result is a function of its 16 bits.  g_gelu_bf16[bits] holds exactly
// what k_gelu_vec<true> stores for that input (built on the device with the
// same gelu_erf and rounding), and the table kernel looks it up from shared memory.
__device__ uint16_t g_gelu_bf16[65536];

__global__ void k_gelu_table_build() {
    GRID_STRIDE(i, 65536) {
        const float v = __uint_as_float(static_cast<uint32_t>(i) << 16);
        g_gelu_bf16[i] = __bfloat16_as_ushort(__float2bfloat16_rn(gelu_erf(v)));
    }
}

// The table kernel keeps only the common part of the table in shared memory:
// bf16 inputs with exponent field in [kGeluE0, kGeluE1] (|z| in [2^-25, 16)),
// both signs -- two contiguous slices of g_gelu_bf16, 14.8 KB -- and reads the
// rare rest (tiny or large |z|, zeros, infinities, NaN) from the full table in
// global memory.  So every result is the full table's entry, bit for bit.
// (The whole 128 KB table per block cost as much traffic as the data itself on
// small activations.)
constexpr int kGeluE0 = 102, kGeluE1 = 130, kGeluNE = kGeluE1 - kGeluE0 + 1;
constexpr int kGeluSlice = kGeluNE * 128; // entries per sign
constexpr int kGeluTableThreads = 1024;

__global__ void __launch_bounds__(kGeluTableThreads, 1) k_gelu_table(uint4 *__restrict__ x, size_t nvec) {
    __shared__ __align__(16) uint16_t table[2 * kGeluSlice];
    static_assert((kGeluE0 * 128) % 8 == 0 && kGeluSlice % 8 == 0, "16-byte slices");
    const uint4 *lo = reinterpret_cast<const uint4 *>(g_gelu_bf16 + kGeluE0 * 128);
    const uint4 *hi = reinterpret_cast<const uint4 *>(g_gelu_bf16 + 0x8000 + kGeluE0 * 128);
    uint4 *t4 = reinterpret_cast<uint4 *>(table);
    for (int i = threadIdx.x; i < kGeluSlice / 8; i += kGeluTableThreads) {
        t4[i] = lo[i];
        t4[kGeluSlice / 8 + i] = hi[i];
    }
    __syncthreads();
    auto look = [&](uint32_t b) -> uint32_t {
        const uint32_t e = (b >> 7) & 0xffu;
        const uint32_t k = e - kGeluE0; // wraps for e < kGeluE0
        if (k < static_cast<uint32_t>(kGeluNE))
            return table[(b >> 15) * kGeluSlice + k * 128 + (b & 127u)];
        return __ldg(g_gelu_bf16 + b);
    };
    const size_t stride = static_cast<size_t>(gridDim.x) * kGeluTableThreads;
    constexpr int U = 4; // vectors in flight per thread
    for (size_t i = blockIdx.x * static_cast<size_t>(kGeluTableThreads) + threadIdx.x; i < nvec; i += U * stride) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i + u * stride < nvec)
                v[u] = x[i + u * stride];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            uint32_t *w = reinterpret_cast<uint32_t *>(&v[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                w[k] = look(w[k] & 0xffffu) | (look(w[k] >> 16) << 16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i + u * stride < nvec)
                x[i + u * stride] = v[u];
    }
}

template <bool BF16> __global__ void k_add_vec(void *__restrict__ x, const void *__restrict__ y, size_t nvec) {
    constexpr int N = kVec<BF16>;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nvec; i += 2 * stride) {
        const size_t j = i + stride;
        const bool two = j < nvec;
        float a[2][N], b[2][N];
        vload<BF16>(x, i * N, a[0]);
        vload<BF16>(y, i * N, b[0]);
        if (two) {
            vload<BF16>(x, j * N, a[1]);
            vload<BF16>(y, j * N, b[1]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int k = 0; k < N; ++k)
                a[u][k] = __fadd_rn(a[u][k], b[u][k]);
        vstore<BF16>(x, i * N, a[0]);
        if (two)
            vstore<BF16>(x, j * N, a[1]);
    }
}

// x[r, c] = r(x[r, c] + b[c]) over whole vectors (cols % vector == 0).
template <bool BF16>
__global__ void k_bias_vec(void *__restrict__ x, const void *__restrict__ b, size_t nvec, size_t cols) {
    constexpr int N = kVec<BF16>;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nvec; i += 2 * stride) {
        const size_t j = i + stride;
        const bool two = j < nvec;
        float a[2][N], c[2][N];
        vload<BF16>(x, i * N, a[0]);
        vload<BF16>(b, (i * N) % cols, c[0]);
        if (two) {
            vload<BF16>(x, j * N, a[1]);
            vload<BF16>(b, (j * N) % cols, c[1]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int k = 0; k < N; ++k)
                a[u][k] = __fadd_rn(a[u][k], c[u][k]);
        vstore<BF16>(x, i * N, a[0]);
        if (two)
            vstore<BF16>(x, j * N, a[1]);
    }
}

// One warp per row, the row in registers (VPL vectors per lane): optionally
// x = r(x + z) written back (the residual), then y = r(((x - mean) inv) w + b)
// with mean and var as the reference's norm (fp32, biased variance).
template <bool BF16, int VPL>
__global__ void k_add_norm(void *__restrict__ x, const void *__restrict__ z, const void *__restrict__ w,
                           const void *__restrict__ b, void *__restrict__ y, size_t rows, int cols, float eps) {
    constexpr int N = kVec<BF16>;
    const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows)
        return;
    const size_t base = row * static_cast<size_t>(cols);
    float v[VPL][N];
    // All of the row's loads are issued before any arithmetic or store.
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * N;
        if (c < cols)
            vload<BF16>(x, base + c, v[i]);
    }
    if (z) {
        float t[VPL][N];
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int c = (i * 32 + lane) * N;
            if (c < cols)
                vload<BF16>(z, base + c, t[i]);
        }
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int c = (i * 32 + lane) * N;
            if (c < cols) {
#pragma unroll
                for (int k = 0; k < N; ++k)
                    v[i][k] = rnd(__fadd_rn(v[i][k], t[i][k]), BF16);
                vstore<BF16>(x, base + c, v[i]);
            }
        }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * N;
        if (c < cols) {
#pragma unroll
            for (int k = 0; k < N; ++k)
                s = __fadd_rn(s, v[i][k]);
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float mean = s / static_cast<float>(cols);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * N;
        if (c < cols) {
#pragma unroll
            for (int k = 0; k < N; ++k) {
                const float d = __fsub_rn(v[i][k], mean);
                q = __fadd_rn(q, __fmul_rn(d, d));
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, o));
    const float inv = 1.f / sqrtf(q / static_cast<float>(cols) + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * N;
        if (c < cols) {
            float wv[N], bv[N];
            vload<BF16>(w, c, wv);
            vload<BF16>(b, c, bv);
#pragma unroll
            for (int k = 0; k < N; ++k)
                v[i][k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i][k], mean), inv), wv[k]), bv[k]);
            vstore<BF16>(y, base + c, v[i]);
        }
    }
}

__global__ void k_linear_epilogue(const float *acc, const void *b, bool bbf16, void *y, bool bf16,
                                  size_t rows, size_t cols) {
    GRID_STRIDE(i, rows * cols) {
        const float bv = b ? ld(b, i % cols, bbf16) : 0.f;
        st(y, i, __fadd_rn(acc[i], bv), bf16);
    }
}

// One block per row; the two reductions follow the row in column order per
// thread (stride blockDim) and combine in a fixed tree.
__global__ void k_layer_norm(const void *x, const void *w, const void *b, void *y, bool bf16,
                             size_t cols, float eps) {
    __shared__ float red[32];
    const size_t row = blockIdx.x;
    const size_t base = row * cols;
    auto block_sum = [&](float v) {
        for (int o = 16; o > 0; o >>= 1)
            v += __shfl_xor_sync(0xffffffffu, v, o);
        if ((threadIdx.x & 31) == 0)
            red[threadIdx.x >> 5] = v;
        __syncthreads();
        float t = 0.f;
        if (threadIdx.x < 32) {
            t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
            for (int o = 16; o > 0; o >>= 1)
                t += __shfl_xor_sync(0xffffffffu, t, o);
            if (threadIdx.x == 0)
                red[0] = t;
        }
        __syncthreads();
        t = red[0];
        __syncthreads();
        return t;
    };
    float s = 0.f;
    for (size_t j = threadIdx.x; j < cols; j += blockDim.x)
        s = __fadd_rn(s, ld(x, base + j, bf16));
    const float mean = block_sum(s) / static_cast<float>(cols);
    float v = 0.f;
    for (size_t j = threadIdx.x; j < cols; j += blockDim.x) {
        const float z = __fsub_rn(ld(x, base + j, bf16), mean);
        v = __fadd_rn(v, __fmul_rn(z, z));
    }
    const float var = block_sum(v);
    const float inv = 1.f / sqrtf(var / static_cast<float>(cols) + eps);
    for (size_t j = threadIdx.x; j < cols; j += blockDim.x) {
        const float z = __fmul_rn(__fmul_rn(__fsub_rn(ld(x, base + j, bf16), mean), inv), ld(w, j, bf16));
        st(y, base + j, __fadd_rn(z, ld(b, j, bf16)), bf16);
    }
}

__global__ void k_gelu(void *x, bool bf16, size_t n) {
    GRID_STRIDE(i, n) {
        st(x, i, gelu_erf(ld(x, i, bf16)), bf16);
    }
}

__global__ void k_add(void *x, const void *y, bool bf16, size_t n) {
    GRID_STRIDE(i, n) { st(x, i, __fadd_rn(ld(x, i, bf16), ld(y, i, bf16)), bf16); }
}

__global__ void k_bias(void *x, const void *b, bool bf16, size_t rows, size_t cols) {
    GRID_STRIDE(i, rows * cols) { st(x, i, __fadd_rn(ld(x, i, bf16), ld(b, i % cols, bf16)), bf16); }
}

// Segments of `rows` input rows each; every segment has its own left padding.
__global__ void k_conv_gather(const void *x, void *y, bool bf16, size_t segments, size_t rows,
                              size_t cols, size_t stride, size_t out_rows) {
    GRID_STRIDE(i, segments * out_rows * cols * 3) {
        const size_t seg = i / (out_rows * cols * 3), ti = i % (out_rows * cols * 3);
        const size_t t = ti / (cols * 3), rem = ti % (cols * 3), c = rem / 3, k = rem % 3;
        const long long s = static_cast<long long>(t * stride + k) - 2;
        const float v = s >= 0 && s < static_cast<long long>(rows)
                            ? ld(x, (seg * rows + static_cast<size_t>(s)) * cols + c, bf16)
                            : 0.f;
        st(y, i, v, bf16);
    }
}

__global__ void k_add_periodic(void *x, const void *y, bool bf16, size_t n, size_t period) {
    GRID_STRIDE(i, n) { st(x, i, __fadd_rn(ld(x, i, bf16), ld(y, i % period, bf16)), bf16); }
}

__global__ void k_finite(const float *x, size_t n, int *flag) {
    bool bad = false;
    GRID_STRIDE(i, n) { bad |= !isfinite(x[i]); }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0)
        atomicOr(flag, 1);
}

// [count, channels, frames] -> [count * frames, channels], 32x32 tiles through shared memory.
__global__ void k_frames_major(const float *x, float *y, size_t channels, size_t frames) {
    __shared__ float tile[32][33];
    const size_t item = blockIdx.z;
    const size_t t0 = static_cast<size_t>(blockIdx.x) * 32, c0 = static_cast<size_t>(blockIdx.y) * 32;
    const float *src = x + item * channels * frames;
    float *dst = y + item * channels * frames;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t c = c0 + r, t = t0 + threadIdx.x;
        if (c < channels && t < frames)
            tile[r][threadIdx.x] = src[c * frames + t];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t t = t0 + r, c = c0 + threadIdx.x;
        if (c < channels && t < frames)
            dst[t * channels + c] = tile[threadIdx.x][r];
    }
}

__global__ void k_pool(const void *x, void *y, bool bf16, size_t rows, size_t cols, size_t factor,
                       size_t out_rows) {
    GRID_STRIDE(i, out_rows * cols) {
        const size_t t = i / cols, j = i % cols;
        float sum = 0.f;
        for (size_t k = 0; k < factor && t * factor + k < rows; ++k)
            sum = __fadd_rn(sum, ld(x, (t * factor + k) * cols + j, bf16));
        st(y, i, sum / static_cast<float>(factor), bf16);
    }
}

__global__ void k_interpolate(const void *x, void *y, bool bf16, size_t source, size_t height,
                              size_t width, size_t cols) {
    GRID_STRIDE(idx, height * width * cols) {
        const size_t c = idx % cols, ij = idx / cols, i = ij / width, j = ij % width;
        const float sy = fmaxf(0.f, __fsub_rn(__fmul_rn(static_cast<float>(i) + .5f,
                                                       static_cast<float>(source) / static_cast<float>(height)),
                                             .5f));
        const float sx = fmaxf(0.f, __fsub_rn(__fmul_rn(static_cast<float>(j) + .5f,
                                                       static_cast<float>(source) / static_cast<float>(width)),
                                             .5f));
        const size_t y0 = static_cast<size_t>(sy), x0 = static_cast<size_t>(sx);
        const size_t y1 = y0 + 1 < source ? y0 + 1 : source - 1, x1 = x0 + 1 < source ? x0 + 1 : source - 1;
        const float fy = sy - static_cast<float>(y0), fx = sx - static_cast<float>(x0);
        const float a = fmaf(1.f - fx, ld(x, (y0 * source + x0) * cols + c, bf16),
                             __fmul_rn(fx, ld(x, (y0 * source + x1) * cols + c, bf16)));
        const float b = fmaf(1.f - fx, ld(x, (y1 * source + x0) * cols + c, bf16),
                             __fmul_rn(fx, ld(x, (y1 * source + x1) * cols + c, bf16)));
        st(y, idx, fmaf(1.f - fy, a, __fmul_rn(fy, b)), bf16);
    }
}

// One thread per row (column order as the reference).
__global__ void k_normalize(const void *x, void *y, bool bf16, size_t rows, size_t cols) {
    GRID_STRIDE(r, rows) {
        float n = 0.f;
        for (size_t j = 0; j < cols; ++j) {
            const float v = ld(x, r * cols + j, bf16);
            n = __fadd_rn(n, __fmul_rn(v, v));
        }
        n = fmaxf(rnd(sqrtf(n), bf16), rnd(1e-12f, bf16));
        for (size_t j = 0; j < cols; ++j)
            st(y, r * cols + j, ld(x, r * cols + j, bf16) / n, bf16);
    }
}

// One warp per pooled row; per step each lane reads `FACTOR` 16-byte vectors
// (unconditional loads from valid rows, so that all of a step's loads are in
// flight together), forms VEC pooled values (the group's rows added in order,
// then / factor, rounded in the bf16 profile) and stores them as fp32.  The
// squared norm is a warp reduction of the lanes' partial sums: the fp32 VQ
// uses it only in its approximate search, whose candidate window bounds the
// fp32 rounding of a sum of squares in any order.
template <bool BF16, int FACTOR>
__global__ void __launch_bounds__(128) k_pool_features(const void *x, size_t items, size_t rows_per_item,
                                                       size_t cols, const int *out_offset, float *features,
                                                       float *xn) {
    constexpr int VEC = kVec<BF16>, TW = 32 * VEC;
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const size_t pooled = (rows_per_item + FACTOR - 1) / FACTOR;
    for (size_t w = static_cast<size_t>(blockIdx.x) * warps + (threadIdx.x >> 5); w < items * pooled;
         w += static_cast<size_t>(gridDim.x) * warps) {
        const size_t b = w / pooled, t = w % pooled;
        if (t >= static_cast<size_t>(out_offset[b + 1] - out_offset[b]))
            continue;
        const size_t out_row = static_cast<size_t>(out_offset[b]) + t, r0 = b * rows_per_item + t * FACTOR;
        float part = 0.f;
#pragma unroll 2
        for (size_t c = static_cast<size_t>(lane) * VEC; c < cols; c += TW) {
            float v[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e)
                v[e] = 0.f;
            float a[FACTOR][VEC];
#pragma unroll
            for (int k = 0; k < FACTOR; ++k) {
                const bool ok = t * FACTOR + k < rows_per_item;
                vload<BF16>(x, (ok ? r0 + k : r0) * cols + c, a[k]);
                if (!ok)
#pragma unroll
                    for (int e = 0; e < VEC; ++e)
                        a[k][e] = 0.f;
            }
#pragma unroll
            for (int k = 0; k < FACTOR; ++k)
#pragma unroll
                for (int e = 0; e < VEC; ++e)
                    v[e] = __fadd_rn(v[e], a[k][e]);
            float *dst = features + out_row * cols + c;
#pragma unroll
            for (int e = 0; e < VEC; e += 4) {
                float4 q;
                q.x = rnd(v[e] / static_cast<float>(FACTOR), BF16);
                q.y = rnd(v[e + 1] / static_cast<float>(FACTOR), BF16);
                q.z = rnd(v[e + 2] / static_cast<float>(FACTOR), BF16);
                q.w = rnd(v[e + 3] / static_cast<float>(FACTOR), BF16);
                *reinterpret_cast<float4 *>(dst + e) = q;
                part = fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, fmaf(q.w, q.w, part))));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0)
            xn[out_row] = part;
    }
}

__global__ void k_bias_normalize(const __nv_bfloat16 *x, const __nv_bfloat16 *bias, __nv_bfloat16 *y,
                                 size_t rows, size_t cols) {
    GRID_STRIDE(r, rows) {
        float n = 0.f;
        for (size_t j = 0; j < cols; ++j) {
            const float v = rnd(__fadd_rn(__bfloat162float(x[r * cols + j]), __bfloat162float(bias[j])), true);
            n = __fadd_rn(n, __fmul_rn(v, v));
        }
        n = fmaxf(rnd(sqrtf(n), true), rnd(1e-12f, true));
        for (size_t j = 0; j < cols; ++j) {
            const float v = rnd(__fadd_rn(__bfloat162float(x[r * cols + j]), __bfloat162float(bias[j])), true);
            y[r * cols + j] = __float2bfloat16_rn(v / n);
        }
    }
}

__global__ void k_image_patches(const float *px, __nv_bfloat16 *y, size_t count, size_t height,
                                size_t width, size_t patch) {
    const size_t gw = width / patch, pd = 8 * patch * patch, cells = (height / patch) * gw;
    GRID_STRIDE(i, count * cells * pd) {
        const size_t item = i / (cells * pd), cell = (i / pd) % cells, rem = i % pd, pix = rem / 8,
                     ch = rem % 8;
        float v = 0.f;
        if (ch < 3) {
            const size_t gy = cell / gw, gx = cell % gw, dy = pix / patch, dx = pix % patch;
            v = px[(item * 3 + ch) * height * width + (gy * patch + dy) * width + gx * patch + dx];
        }
        y[i] = __float2bfloat16_rn(v);
    }
}

__global__ void k_convert(const float *x, void *y, bool bf16, size_t n) {
    GRID_STRIDE(i, n) { st(y, i, x[i], bf16); }
}
__global__ void k_to_float(const void *x, float *y, bool bf16, size_t n) {
    GRID_STRIDE(i, n) { y[i] = ld(x, i, bf16); }
}

// Scores -> probabilities in place, one warp per score row.  Rows are
// [items, heads, n] of n scores each; row t of item b keeps keys below
// limit = min(n, valid[b]) (and the block window), p = exp(z - max) / total as
// the reference's Ops::attention; masked keys become 0.
// The same with 16-byte accesses (n % 4 == 0): lane owns columns
// 4 (lane + 32 i) .. +3.
template <int VEC_PER_LANE>
__global__ void k_softmax_rows4(float *__restrict__ s, size_t items, size_t heads, size_t n, const int *valid,
                                size_t valid_all, size_t block) {
    const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= items * heads * n)
        return;
    const size_t b = row / (heads * n), t = row % n;
    size_t limit = valid ? static_cast<size_t>(valid[b] > 0 ? valid[b] : 0) : valid_all;
    limit = limit < n ? limit : n;
    if (block)
        limit = limit < (t / block + 1) * block ? limit : (t / block + 1) * block;
    float4 *z = reinterpret_cast<float4 *>(s + row * n);
    float4 v[VEC_PER_LANE];
#pragma unroll
    for (int i = 0; i < VEC_PER_LANE; ++i) {
        const size_t c = 4 * (lane + 32 * static_cast<size_t>(i));
        v[i] = c < n ? z[c / 4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < VEC_PER_LANE; ++i) {
        const size_t c = 4 * (lane + 32 * static_cast<size_t>(i));
        float *e = &v[i].x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            e[k] = c + k < limit ? e[k] : -INFINITY;
            mx = fmaxf(mx, e[k]);
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < VEC_PER_LANE; ++i) {
        const size_t c = 4 * (lane + 32 * static_cast<size_t>(i));
        float *e = &v[i].x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            e[k] = c + k < limit ? expf(e[k] - mx) : 0.f;
            total += e[k];
        }
    }
    for (int o = 16; o > 0; o >>= 1)
        total += __shfl_xor_sync(0xffffffffu, total, o);
    // One reciprocal per row instead of an IEEE division per score (within an
    // ulp of p / total; the division was a third of the kernel's instructions).
    const float inv = 1.f / total;
#pragma unroll
    for (int i = 0; i < VEC_PER_LANE; ++i) {
        const size_t c = 4 * (lane + 32 * static_cast<size_t>(i));
        if (c < n) {
            float4 w = v[i];
            w.x *= inv;
            w.y *= inv;
            w.z *= inv;
            w.w *= inv;
            z[c / 4] = w;
        }
    }
}

template <int PER_LANE>
__global__ void k_softmax_rows(float *s, size_t items, size_t heads, size_t n, const int *valid,
                               size_t valid_all, size_t block) {
    const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= items * heads * n)
        return;
    const size_t b = row / (heads * n), t = row % n;
    size_t limit = valid ? static_cast<size_t>(valid[b] > 0 ? valid[b] : 0) : valid_all;
    limit = limit < n ? limit : n;
    if (block)
        limit = limit < (t / block + 1) * block ? limit : (t / block + 1) * block;
    float *z = s + row * n;
    float v[PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const size_t c = lane + 32 * static_cast<size_t>(i);
        v[i] = c < limit ? z[c] : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
    for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const size_t c = lane + 32 * static_cast<size_t>(i);
        v[i] = c < limit ? expf(v[i] - mx) : 0.f;
        total += v[i];
    }
    for (int o = 16; o > 0; o >>= 1)
        total += __shfl_xor_sync(0xffffffffu, total, o);
    const float inv = 1.f / total;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
        const size_t c = lane + 32 * static_cast<size_t>(i);
        if (c < n)
            z[c] = v[i] * inv;
    }
}

} // namespace

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int bias(void *x, const void *b, bool bf16, size_t rows, size_t cols, cudaStream_t s);

int linear_epilogue(const float *acc, const void *b, bool bbf16, void *y, bool bf16, size_t rows,
                    size_t cols, cudaStream_t s) {
    if (static_cast<const void *>(acc) == y && !bf16) { // fp32 in place: only the bias
        if (!b)
            return 0;
        if (!bbf16)
            return bias(y, b, false, rows, cols, s);
    }
    k_linear_epilogue<<<blocks_for(rows * cols, 256), 256, 0, s>>>(acc, b, bbf16, y, bf16, rows, cols);
    return status();
}
int layer_norm(const void *x, const void *w, const void *b, void *y, bool bf16, size_t rows,
               size_t cols, float eps, cudaStream_t s) {
    if (rows)
        k_layer_norm<<<static_cast<unsigned>(rows), 256, 0, s>>>(x, w, b, y, bf16, cols, eps);
    return status();
}
namespace {
// The table is built once per device.
std::atomic<unsigned long long> g_gelu_table_ready{0};
std::mutex g_gelu_mutex;

bool gelu_table(cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return false;
    const unsigned long long bit = 1ull << dev;
    if (g_gelu_table_ready.load() & bit)
        return true;
    std::lock_guard<std::mutex> guard(g_gelu_mutex);
    if (!(g_gelu_table_ready.load() & bit)) {
        k_gelu_table_build<<<64, 1024, 0, s>>>();
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
            return false;
        g_gelu_table_ready.fetch_or(bit);
    }
    return true;
}
} // namespace

int gelu(void *x, bool bf16, size_t n, cudaStream_t s) {
    const size_t N = bf16 ? 8 : 4, nvec = aligned16(x) ? n / N : 0, done = nvec * N;
    if (nvec) {
        if (bf16 && gelu_table(s)) {
            int sms = 148, dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            // One block per SM, each loading the 14.8 KB of table once.
            const size_t want = (nvec + kGeluTableThreads - 1) / kGeluTableThreads;
            const size_t cap = static_cast<size_t>(sms);
            const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
            k_gelu_table<<<grid, kGeluTableThreads, 0, s>>>(static_cast<uint4 *>(x), nvec);
        } else if (bf16) {
            k_gelu_vec<true><<<blocks_for(nvec, 256), 256, 0, s>>>(x, nvec);
        } else {
            k_gelu_vec<false><<<blocks_for(nvec, 256), 256, 0, s>>>(x, nvec);
        }
    }
    if (done < n)
        k_gelu<<<blocks_for(n - done, 256), 256, 0, s>>>(static_cast<char *>(x) + done * (bf16 ? 2 : 4), bf16,
                                                         n - done);
    return status();
}
int add(void *x, const void *y, bool bf16, size_t n, cudaStream_t s) {
    const size_t N = bf16 ? 8 : 4, nvec = aligned16(x) && aligned16(y) ? n / N : 0, done = nvec * N;
    const size_t es = bf16 ? 2 : 4;
    if (nvec) {
        if (bf16)
            k_add_vec<true><<<blocks_for(nvec, 256), 256, 0, s>>>(x, y, nvec);
        else
            k_add_vec<false><<<blocks_for(nvec, 256), 256, 0, s>>>(x, y, nvec);
    }
    if (done < n)
        k_add<<<blocks_for(n - done, 256), 256, 0, s>>>(static_cast<char *>(x) + done * es,
                                                        static_cast<const char *>(y) + done * es, bf16, n - done);
    return status();
}

namespace {
template <bool BF16, int VPL>
void launch_add_norm(void *x, const void *z, const void *w, const void *b, void *y, size_t rows, size_t cols,
                     float eps, cudaStream_t s) {
    constexpr int kRows = 4; // warps (rows) per block
    k_add_norm<BF16, VPL><<<static_cast<unsigned>((rows + kRows - 1) / kRows), kRows * 32, 0, s>>>(
        x, z, w, b, y, rows, static_cast<int>(cols), eps);
}
template <bool BF16>
bool add_norm_vec(void *x, const void *z, const void *w, const void *b, void *y, size_t rows, size_t cols,
                  float eps, cudaStream_t s) {
    const size_t per = 32 * static_cast<size_t>(kVec<BF16>), need = (cols + per - 1) / per;
    if (need <= 1)
        launch_add_norm<BF16, 1>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 2)
        launch_add_norm<BF16, 2>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 4)
        launch_add_norm<BF16, 4>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 6)
        launch_add_norm<BF16, 6>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 8)
        launch_add_norm<BF16, 8>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 12)
        launch_add_norm<BF16, 12>(x, z, w, b, y, rows, cols, eps, s);
    else if (need <= 16)
        launch_add_norm<BF16, 16>(x, z, w, b, y, rows, cols, eps, s);
    else
        return false;
    return true;
}
} // namespace

int add_layer_norm(void *x, const void *z, const void *w, const void *b, void *y, bool bf16, size_t rows,
                   size_t cols, float eps, cudaStream_t s) {
    if (rows == 0)
        return 0;
    const size_t N = bf16 ? 8 : 4;
    const bool vec = cols % N == 0 && aligned16(x) && (!z || aligned16(z)) && aligned16(w) && aligned16(b) &&
                     aligned16(y);
    if (vec && (bf16 ? add_norm_vec<true>(x, z, w, b, y, rows, cols, eps, s)
                     : add_norm_vec<false>(x, z, w, b, y, rows, cols, eps, s)))
        return status();
    if (z) {
        const int rc = add(x, z, bf16, rows * cols, s);
        if (rc)
            return rc;
    }
    return layer_norm(x, w, b, y, bf16, rows, cols, eps, s);
}
int bias(void *x, const void *b, bool bf16, size_t rows, size_t cols, cudaStream_t s) {
    const size_t N = bf16 ? 8 : 4, n = rows * cols;
    if (cols % N == 0 && aligned16(x) && aligned16(b)) {
        if (n) {
            if (bf16)
                k_bias_vec<true><<<blocks_for(n / N, 256), 256, 0, s>>>(x, b, n / N, cols);
            else
                k_bias_vec<false><<<blocks_for(n / N, 256), 256, 0, s>>>(x, b, n / N, cols);
        }
        return status();
    }
    k_bias<<<blocks_for(n, 256), 256, 0, s>>>(x, b, bf16, rows, cols);
    return status();
}
int conv_gather(const void *x, void *y, bool bf16, size_t segments, size_t rows, size_t cols,
                size_t stride, cudaStream_t s) {
    const size_t out_rows = (rows + stride - 1) / stride;
    k_conv_gather<<<blocks_for(segments * out_rows * cols * 3, 256), 256, 0, s>>>(x, y, bf16, segments, rows,
                                                                                   cols, stride, out_rows);
    return status();
}
int add_periodic(void *x, const void *y, bool bf16, size_t n, size_t period, cudaStream_t s) {
    k_add_periodic<<<blocks_for(n, 256), 256, 0, s>>>(x, y, bf16, n, period);
    return status();
}
int finite_check(const float *x, size_t n, int *flag, cudaStream_t s) {
    if (n)
        k_finite<<<blocks_for(n, 256), 256, 0, s>>>(x, n, flag);
    return status();
}
int frames_major(const float *x, float *y, size_t count, size_t channels, size_t frames, cudaStream_t s) {
    if (count && channels && frames) {
        const dim3 grid(static_cast<unsigned>((frames + 31) / 32), static_cast<unsigned>((channels + 31) / 32),
                        static_cast<unsigned>(count));
        k_frames_major<<<grid, dim3(32, 8), 0, s>>>(x, y, channels, frames);
    }
    return status();
}
int pool(const void *x, void *y, bool bf16, size_t rows, size_t cols, size_t factor,
         cudaStream_t s) {
    const size_t out_rows = (rows + factor - 1) / factor;
    k_pool<<<blocks_for(out_rows * cols, 256), 256, 0, s>>>(x, y, bf16, rows, cols, factor, out_rows);
    return status();
}
int interpolate(const void *x, void *y, bool bf16, size_t source, size_t height, size_t width,
                size_t cols, cudaStream_t s) {
    k_interpolate<<<blocks_for(height * width * cols, 256), 256, 0, s>>>(x, y, bf16, source, height,
                                                                          width, cols);
    return status();
}
int normalize(const void *x, void *y, bool bf16, size_t rows, size_t cols, cudaStream_t s) {
    k_normalize<<<blocks_for(rows, 128), 128, 0, s>>>(x, y, bf16, rows, cols);
    return status();
}
int pool_features(const void *x, bool bf16, size_t items, size_t rows_per_item, size_t cols, size_t factor,
                  const int *out_offset, float *features, float *xn, cudaStream_t s) {
    if (items == 0 || cols == 0)
        return 0;
    // 16-byte vectors of x and of the fp32 feature rows; the reference's pool
    // factor (4; src/model.cpp:43) is compiled in.
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(features) % 16 != 0 ||
        cols % (bf16 ? 8 : 4) != 0 || factor != 4)
        return static_cast<int>(cudaErrorInvalidValue);
    const size_t rows = items * ((rows_per_item + factor - 1) / factor);
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>((rows + 3) / 4, 148 * 32));
    if (bf16)
        k_pool_features<true, 4><<<blocks, 128, 0, s>>>(x, items, rows_per_item, cols, out_offset, features, xn);
    else
        k_pool_features<false, 4><<<blocks, 128, 0, s>>>(x, items, rows_per_item, cols, out_offset, features, xn);
    return status();
}
int bias_normalize(const void *x, const void *b, void *y, size_t rows, size_t cols, cudaStream_t s) {
    k_bias_normalize<<<blocks_for(rows, 128), 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(x),
                                                            static_cast<const __nv_bfloat16 *>(b),
                                                            static_cast<__nv_bfloat16 *>(y), rows, cols);
    return status();
}
int image_patches(const float *pixels, void *y, size_t count, size_t height, size_t width, size_t patch,
                  cudaStream_t s) {
    const size_t n = count * (height / patch) * (width / patch) * 8 * patch * patch;
    k_image_patches<<<blocks_for(n, 256), 256, 0, s>>>(pixels, static_cast<__nv_bfloat16 *>(y), count, height,
                                                        width, patch);
    return status();
}
int convert(const float *x, void *y, bool bf16, size_t n, cudaStream_t s) {
    k_convert<<<blocks_for(n, 256), 256, 0, s>>>(x, y, bf16, n);
    return status();
}
int to_float(const void *x, float *y, bool bf16, size_t n, cudaStream_t s) {
    k_to_float<<<blocks_for(n, 256), 256, 0, s>>>(x, y, bf16, n);
    return status();
}
int softmax_rows(float *scores, size_t items, size_t heads, size_t n, const int *valid, size_t valid_all,
                 size_t block, cudaStream_t s) {
    const size_t rows = items * heads * n;
    if (rows == 0)
        return 0;
    constexpr int kWarps = 8;
    const unsigned grid = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
    if (n % 4 == 0 && aligned16(scores)) {
        if (n <= 512)
            k_softmax_rows4<4><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
        else if (n <= 1536)
            k_softmax_rows4<12><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
        else if (n <= 4096)
            k_softmax_rows4<32><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
        else
            return -2;
        return status();
    }
    if (n <= 512)
        k_softmax_rows<16><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
    else if (n <= 1536)
        k_softmax_rows<48><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
    else if (n <= 4096)
        k_softmax_rows<128><<<grid, kWarps * 32, 0, s>>>(scores, items, heads, n, valid, valid_all, block);
    else
        return -2; // longer rows are not produced by the graphs (audio n <= 1500)
    return status();
}

} // namespace graph
} // namespace omni_b200
