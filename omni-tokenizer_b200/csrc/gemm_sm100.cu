// gemm_sm100.cu -- the encoder graphs' bf16 linears on B200 (sm_100a).
//
// Ops::linear of the reference's bf16 profile (semantics of
// src/cpu.cpp:47-69): y = r(x W^T + b), fp32 sums, one rounding to bf16 after
// the bias, x [M, K] and y [M, N] row-major, W [N, K] in the file's layout.
//
// A CUTLASS sm100 kernel built from CuTe/CUTLASS templates: tcgen05.mma with
// cta_group::2 (one 256 x 256 tile per pair of SMs, a cluster of two CTAs
// along M), TMA loads of A and B without cluster multicast (in a 2x1x1
// cluster each CTA of the pair loads its own 128 rows of A and half of B's
// columns), a 6-stage shared-memory ring, fp32 accumulators double-buffered
// in TMEM so that a tile's epilogue overlaps the next tile's main loop, and a
// TMA-store epilogue that adds the bias and rounds.  On the encoders' large
// shapes it runs at 1.46-1.54 PFLOP/s on B200, against 1.14-1.36 for the
// cuBLASLt kernels the library used before (M = 23,328-93,312 rows, N and K
// of 1024-4304).
//
// Tried and not kept: GELU in this epilogue (the fc1 + GELU pair).  The
// epilogue runs four warps, one per sub-partition; the ~40-operation erf per
// element ran as a serial chain (about 0.2 instructions per clock per
// sub-partition) and made the fused GEMM 3.6-4x slower than this GEMM plus
// the separate GELU pass.
#include <cuda_runtime.h>

#include <cute/tensor.hpp>
#include <cutlass/cutlass.h>
#include <cutlass/epilogue/collective/collective_builder.hpp>
#include <cutlass/epilogue/fusion/operations.hpp>
#include <cutlass/gemm/collective/collective_builder.hpp>
#include <cutlass/gemm/device/gemm_universal_adapter.h>
#include <cutlass/gemm/dispatch_policy.hpp>
#include <cutlass/gemm/kernel/gemm_universal.hpp>
#include <cutlass/numeric_types.h>

#include <atomic>

#include "gemm_sm100.h"

namespace omni_b200 {
namespace {

using bf16 = cutlass::bfloat16_t;
constexpr int kAlign = 8; // 16 bytes of bf16
constexpr int kTileM = 256, kTileN = 256;

template <bool BIAS> struct LinearGemm {
    using MmaTileShape = cute::Shape<cute::Int<kTileM>, cute::Int<kTileN>, cute::_64>;
    using ClusterShape = cute::Shape<cute::_2, cute::_1, cute::_1>;
    using FusionOp = cute::conditional_t<BIAS, cutlass::epilogue::fusion::LinCombPerColBias<bf16, float, bf16, bf16, float>,
                                         cutlass::epilogue::fusion::LinearCombination<bf16, float, bf16, float>>;
    using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTileShape, ClusterShape,
        cutlass::epilogue::collective::EpilogueTileAuto, float, float, void, cutlass::layout::RowMajor, kAlign,
        bf16, cutlass::layout::RowMajor, kAlign, cutlass::epilogue::TmaWarpSpecialized2Sm, FusionOp>::CollectiveOp;
    using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, bf16, cutlass::layout::RowMajor, kAlign, bf16,
        cutlass::layout::ColumnMajor, kAlign, float, MmaTileShape, ClusterShape,
        cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
        cutlass::gemm::KernelTmaWarpSpecialized2SmSm100>::CollectiveOp;
    using Kernel = cutlass::gemm::kernel::GemmUniversal<cute::Shape<int, int, int, int>, Mainloop, Epilogue, void>;
    using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;

    static typename Gemm::Arguments args(const void *x, const void *w, const void *b, void *y, int M, int N, int K,
                                         int sms) {
        using StrideA = typename Gemm::GemmKernel::StrideA;
        using StrideB = typename Gemm::GemmKernel::StrideB;
        using StrideC = typename Gemm::GemmKernel::StrideC;
        using StrideD = typename Gemm::GemmKernel::StrideD;
        // A = x [M, K] row-major; B = W [N, K] row-major (K-major: CUTLASS's
        // column-major B); D = y [M, N] row-major.
        StrideA sa = cute::make_stride(static_cast<int64_t>(K), cute::Int<1>{}, static_cast<int64_t>(M) * K);
        StrideB sb = cute::make_stride(static_cast<int64_t>(K), cute::Int<1>{}, static_cast<int64_t>(N) * K);
        StrideC sc = cute::make_stride(static_cast<int64_t>(N), cute::Int<1>{}, static_cast<int64_t>(M) * N);
        StrideD sd = sc;
        typename Gemm::Arguments a{cutlass::gemm::GemmUniversalMode::kGemm,
                                   {M, N, K, 1},
                                   {static_cast<const bf16 *>(x), sa, static_cast<const bf16 *>(w), sb},
                                   {{}, nullptr, sc, static_cast<bf16 *>(y), sd}};
        a.epilogue.thread.alpha = 1.f;
        a.epilogue.thread.beta = 0.f;
        if constexpr (BIAS)
            a.epilogue.thread.bias_ptr = static_cast<const bf16 *>(b);
        int dev = 0;
        cudaGetDevice(&dev);
        a.hw_info.device_id = dev;
        a.hw_info.sm_count = sms;
        return a;
    }

    static int run(const void *x, const void *w, const void *b, void *y, int M, int N, int K, int sms,
                   void *workspace, size_t workspace_bytes, cudaStream_t s) {
        Gemm gemm;
        auto a = args(x, w, b, y, M, N, K, sms);
        if (gemm.can_implement(a) != cutlass::Status::kSuccess)
            return -3;
        if (Gemm::get_workspace_size(a) > workspace_bytes)
            return -4;
        if (gemm.initialize(a, workspace, s) != cutlass::Status::kSuccess)
            return -5;
        if (gemm.run(s) != cutlass::Status::kSuccess)
            return -6;
        return static_cast<int>(cudaGetLastError());
    }
    static size_t workspace(int M, int N, int K, int sms) {
        return Gemm::get_workspace_size(args(nullptr, nullptr, nullptr, nullptr, M, N, K, sms));
    }
};

int sm_count() {
    static std::atomic<int> sms{0};
    int n = sms.load();
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        sms.store(n);
    }
    return n;
}

} // namespace

bool linear_bf16_supported(const void *x, const void *w, const void *b, const void *y, int M, int N, int K) {
    auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return M > 0 && N > 0 && K > 0 && N % kAlign == 0 && K % kAlign == 0 && a16(x) && a16(w) && (!b || a16(b)) &&
           a16(y);
}

bool linear_bf16_preferred(int M, int N, int K) {
    const long long tiles = static_cast<long long>((M + kTileM - 1) / kTileM) * ((N + kTileN - 1) / kTileN);
    return K >= 256 && tiles >= 4LL * (sm_count() / 2);
}

size_t linear_bf16_workspace(int M, int N, int K, bool bias) {
    return bias ? LinearGemm<true>::workspace(M, N, K, sm_count()) : LinearGemm<false>::workspace(M, N, K, sm_count());
}

int linear_bf16(const void *x, const void *w, const void *b, void *y, int M, int N, int K, void *workspace,
                size_t workspace_bytes, cudaStream_t s) {
    if (!linear_bf16_supported(x, w, b, y, M, N, K))
        return -2;
    return b ? LinearGemm<true>::run(x, w, b, y, M, N, K, sm_count(), workspace, workspace_bytes, s)
             : LinearGemm<false>::run(x, w, b, y, M, N, K, sm_count(), workspace, workspace_bytes, s);
}

} // namespace omni_b200
