// gemm_sm100.h -- bf16 linear on the tensor cores (gemm_sm100.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace omni_b200 {

// y[M, N] = r(x[M, K] W[N, K]^T (+ b[N])) for bf16 row-major x, W, b and y,
// fp32 accumulation, one rounding to bf16 after the bias (r).  Needs N and K
// multiples of 8 and 16-byte aligned pointers (linear_bf16_supported; b may be
// null).  Returns 0, a CUDA error code, or a negative code when the shape or
// the workspace does not fit.
bool linear_bf16_supported(const void *x, const void *w, const void *b, const void *y, int M, int N, int K);
size_t linear_bf16_workspace(int M, int N, int K, bool bias);
int linear_bf16(const void *x, const void *w, const void *b, void *y, int M, int N, int K, void *workspace,
                size_t workspace_bytes, cudaStream_t s);
// Whether this GEMM is the faster choice for the shape on B200: launches that
// fill at least four waves of SM pairs with 256 x 256 tiles (below that,
// cuBLASLt's smaller tiles keep more SMs busy).
bool linear_bf16_preferred(int M, int N, int K);

} // namespace omni_b200
