// graph_kernels.h -- the non-hot operators of the encoder graphs (CUDA).
//
// Semantics follow the reference's CPU backend, omni-tokenizer
// src/cpu.cpp:20-221 (Cpu::upload / linear epilogue / norm / gelu / add / bias /
// conv_gather / pool / interpolate / normalize) and the patch layout of
// src/internal.h:57-70 (Ops::image_patches).  A tensor is either fp32 or, in
// the bf16 profile, bf16 in memory: every bf16-profile result is rounded to
// bf16 once, exactly where the reference applies round_bf16.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace omni_b200 {
namespace graph {

// y = r(acc + bias) (bias may be null); acc fp32 [rows, cols]; y fp32 or bf16.
int linear_epilogue(const float *acc, const void *bias, bool bias_bf16, void *y, bool bf16,
                    size_t rows, size_t cols, cudaStream_t s);
// Layer norm over each row: r((x - mean) * inv * w + b), inv = 1/sqrt(var + eps).
int layer_norm(const void *x, const void *w, const void *b, void *y, bool bf16, size_t rows,
               size_t cols, float eps, cudaStream_t s);
// x = r(x + z) in place when z is given, then y = layer norm of x (as above):
// one warp per row with the row in registers (rows up to 2048 columns).
int add_layer_norm(void *x, const void *z, const void *w, const void *b, void *y, bool bf16, size_t rows,
                   size_t cols, float eps, cudaStream_t s);
// In place: x = r(0.5 x (1 + erf(x / sqrt 2))).
int gelu(void *x, bool bf16, size_t n, cudaStream_t s);
// In place: x = r(x + y) over the first n elements.
int add(void *x, const void *y, bool bf16, size_t n, cudaStream_t s);
// In place: x[r, c] = r(x[r, c] + b[c]).
int bias(void *x, const void *b, bool bf16, size_t rows, size_t cols, cudaStream_t s);
// Kernel-3 causal conv input (left pad 2): y[t, 3c + k] = x[t*stride + k - 2, c],
// for `segments` stacked inputs of `rows` rows each (each padded on its own).
int conv_gather(const void *x, void *y, bool bf16, size_t segments, size_t rows, size_t cols,
                size_t stride, cudaStream_t s);
// In place: x[i] = r(x[i] + y[i mod period]) (positions added to stacked items).
int add_periodic(void *x, const void *y, bool bf16, size_t n, size_t period, cudaStream_t s);
// *flag |= 1 when any of x[0..n) is NaN or infinite.
int finite_check(const float *x, size_t n, int *flag, cudaStream_t s);
// [count, channels, frames] -> [count * frames, channels] (log-mel to frame rows).
int frames_major(const float *x, float *y, size_t count, size_t channels, size_t frames, cudaStream_t s);
// Mean of `factor` consecutive rows (the last group may be short; divisor stays factor).
int pool(const void *x, void *y, bool bf16, size_t rows, size_t cols, size_t factor,
         cudaStream_t s);
// Bilinear resize of a [source*source, cols] grid to [height*width, cols].
int interpolate(const void *x, void *y, bool bf16, size_t source, size_t height, size_t width,
                size_t cols, cudaStream_t s);
// Row-wise L2 normalisation with the reference's max(r(sqrt(n)), r(1e-12)) guard.
int normalize(const void *x, void *y, bool bf16, size_t rows, size_t cols, cudaStream_t s);
// Audio graph tail (pre-VQ epilogue in one pass): mean-pool `factor` rows of
// each of `items` stacked sequences of `rows_per_item` rows of x (bf16 or
// fp32), keep the first out_offset[b+1] - out_offset[b] pooled rows of item b
// and write them as fp32 rows out_offset[b] + t of `features` (what pool, the
// per-item row copies and the fp32 conversion wrote one after another), and
// their squared norms xn for the fp32 VQ's approximate search (a warp
// reduction: any fp32 summation order is within that search's window).
// Needs factor 4, 16-byte aligned x and features and cols a multiple of 8
// (bf16) or 4 (fp32); else cudaErrorInvalidValue.
int pool_features(const void *x, bool bf16, size_t items, size_t rows_per_item, size_t cols, size_t factor,
                  const int *out_offset, float *features, float *xn, cudaStream_t s);
// Image graph tail (pre-VQ epilogue in one pass, bf16): per row v = r(x + b),
// then y = r(v / max(r(sqrt(sum v^2)), r(1e-12))) -- image_conv's bias added
// after the rounded GEMM, followed by normalize.
int bias_normalize(const void *x, const void *b, void *y, size_t rows, size_t cols, cudaStream_t s);
// `count` CHW fp32 images -> bf16 patches [count*gh*gw, 8*p*p] (channel-padded to 8
// per pixel).
int image_patches(const float *pixels, void *y, size_t count, size_t height, size_t width, size_t patch,
                  cudaStream_t s);
// fp32 -> bf16 (round to nearest even, NaN quieted) or a copy for fp32.
int convert(const float *x, void *y, bool bf16, size_t n, cudaStream_t s);
// bf16/fp32 -> fp32.
int to_float(const void *x, float *y, bool bf16, size_t n, cudaStream_t s);
// Attention probabilities in place over [items, heads, n, n] fp32 scores:
// row t of item b keeps keys < min(n, valid[b] (or valid_all when valid is
// null), block window end); p = exp(z - max) / total, masked keys 0.  n <= 4096.
int softmax_rows(float *scores, size_t items, size_t heads, size_t n, const int *valid, size_t valid_all,
                 size_t block, cudaStream_t s);

} // namespace graph
} // namespace omni_b200
