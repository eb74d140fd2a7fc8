// pack.h -- operand repacking for the attention kernel.
#pragma once
#include <cuda_runtime.h>

namespace omni_b200 {
// src element (t, h, e) lives at src[t*s_token + h*s_head + e] with dtype
// 0 = f32, 1 = bf16, 2 = f16; dst is [heads, n, hdp] of bf16 (f16 when the
// source is f16), zero for e >= hd.
int pack_heads(const void *src, int dtype, long long s_token, long long s_head, int n, int heads,
               int hd, int hdp, void *dst, cudaStream_t stream);
// fp32 source, fp32 [heads, n, hdp] destination (values copied unchanged).
int pack_heads_f32(const float *src, long long s_token, long long s_head, int n, int heads, int hd,
                   int hdp, float *dst, cudaStream_t stream);
} // namespace omni_b200
