// vq_stream_sm100.cu -- VQ argmin with the code dimension streamed through
// shared memory (sm_100a): the bf16 profile for wide codes (dim > 128, e.g.
// the production 1280 / 2048) and the exact fp32 profile for every dim.
//
// Reference semantics (omni-tokenizer src/cpu.cpp:227-287, Cpu::quantize):
//   bf16 profile  dist = bf16(bf16(|x|^2 + |c|^2) - bf16(2 x.c)), smallest
//                 dist wins, ties -> smallest id (same epilogue arithmetic as
//                 vq_sm100.cu);
//   fp32 profile  approximate search with dist = fma(-2, x.c, |x|^2 + |c|^2),
//                 then every code whose approximate distance lies within the
//                 error bound of the best one is re-scored with the direct
//                 fp64 sum  sum_k (double(x_k) - double(c_k))^2  in column
//                 order; the smallest direct distance wins, ties -> smallest
//                 id (src/cpu.cpp:260-283, src/internal.h:13-18).
//
// fp32 profile on B200.  The tensor cores have no fp32 MMA, so the
// approximate distances come from kind::tf32 (inputs truncated to 10 mantissa
// bits).  The candidate window is therefore a bound written for this kernel,
// not the reference's fp32 gamma.  approx(c) = fma(-2, dot(c), xn + cn(c)) uses
// the same fp32 row norm xn for every code of the row, so the error of xn is
// a common offset d: approx(c) = exact(c) + d + e(c), and only the per-code
// part needs a bound:
//   |e(c)| <= w(c) = a |x| |c| + bc |c|^2 + bs (|x|^2 + |c|^2),
//   a = 2^-7 + (dim + 1) 2^-21,   bc = dim 2^-22,   bs = 2^-20
// The dot product carries the tf32 truncation, at most 2^-10 per factor, so
// 2|x.c - tf32 dot| <= (2^-8 + 2^-19) sum_k |x_k c_k| <= (2^-8 + 2^-19)|x||c|
// (Cauchy-Schwarz), plus the fp32 accumulation, at most dim 2^-23 per unit of
// sum |x_k c_k|; the codebook norm cn (fp32, in column order) is within
// (dim - 1) 2^-24 |c|^2; the sum xn + cn and the final fma round twice, at most
// 3 2^-24 (|x|^2 + |c|^2) together, and evaluating the test below rounds lo(c)
// and the threshold once each (distances are at most 2 (|x|^2 + |c|^2), so at
// most 2 2^-24 (|x|^2 + |c|^2) each).  a, bc and bs carry a factor of two of
// slack over these, and |x| |c| is taken as sqrt(|x|^2) sqrt(|c|^2) of the fp32
// norms.
// (The row norm may come from any fp32 summation order: its error is the common
// d.)  With b* the code of the smallest approximate distance, the exact nearest
// code c* satisfies approx(c*) - w(c*) <= exact(c*) + d <= exact(b*) + d <=
// approx(b*) + w(b*),
// so the candidate set {c : approx(c) - w(c) <= approx(b*) + w(b*)} contains c*
// and every code whose direct distance ties with it.  The reference's own
// candidate set also contains c* (its gamma bound), and both pick the smallest
// (direct distance, id) among candidates, so the ids agree.  Non-finite
// approximate distances are always candidates; a row with more than
// kVqCandCap candidates is scored against every code (vq_brute_fp64).
//
// Passes (one launch each):
//   kVqsBf16    bf16 profile, keys[row] = (order bits of dist) << 32 | id
//   kVqsApprox  fp32 profile, keys[row] = approximate best (same key form)
//   kVqsCand    fp32 profile, appends candidates to cand[row][kVqCandCap]
// followed by vq_refine_fp64 and vq_brute_fp64 (fp32) or vqs_finish (bf16).
//
// Kernel layout: persistent grid over units (128-row tile, codebook slice);
// warp 4 TMA producer, warp 5 TMEM owner and tcgen05.mma issuer, warps 0-3
// epilogue (thread r owns TMEM lane r = row r of the tile).  Each 256-code
// tile accumulates over 128-byte column chunks of x (128 rows) and of the
// codebook (256 codes) that stream through a 4-stage ring; TMEM holds two
// 256-column fp32 accumulators so the epilogue of one code tile overlaps the
// MMAs of the next.
#include "norms.h"
#include "sm100.cuh"
#include "tma.h"
#include "vq.h"

#include <cuda_bf16.h>
#include <cmath>
#include <mutex>

namespace omni_b200 {

template <bool TF32> struct VqsShape {
    static constexpr int EB = TF32 ? 4 : 2;      // bytes per element
    static constexpr int KC = 128 / EB;          // elements per 128-byte column chunk
    static constexpr int X_CHUNK = 128 * 128;    // 128 rows x 128 bytes
    static constexpr int C_CHUNK = 256 * 128;    // 256 codes x 128 bytes
    static constexpr int STAGE = X_CHUNK + C_CHUNK;
    static constexpr int STAGES = 4;
    static constexpr int SMEM_BYTES = STAGES * STAGE + 512 + 1024;
};

constexpr int kVqsThreads = 192;

__device__ __forceinline__ uint32_t vqs_order_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u)
        return 0xffffffffu; // NaN never wins
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float vqs_from_order_bits(uint32_t b) {
    return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}

__device__ __noinline__ void vqs_wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicOr(err, kErrWaitDrain);
            return;
        }
    }
}

template <bool TF32, int MODE>
__global__ void __launch_bounds__(kVqsThreads, 1) vq_stream_kernel(const __grid_constant__ VqsParams p) {
    using S = VqsShape<TF32>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S::STAGES * S::STAGE);
    uint64_t *full = bars;                  // [STAGES]
    uint64_t *empty = full + S::STAGES;     // [STAGES]
    uint64_t *acc_full = empty + S::STAGES; // [2]
    uint64_t *acc_empty = acc_full + 2;     // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;
    const int row_tiles = (p.rows + 127) / 128;
    const int units = row_tiles * p.slices;
    // Cancellation (the reference polls its flag before every codebook tile,
    // src/cuda.cu:946-948): a CTA that starts after the flag was set skips its
    // part of this launch's codebook window, before it allocates anything.
    if (p.cancel && __syncthreads_or(threadIdx.x == 0 ? *p.cancel != 0 : 0))
        return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc_full[0], 1);
        mbar_init(&acc_full[1], 1);
        mbar_init(&acc_empty[0], 4); // one arrive per epilogue warp
        mbar_init(&acc_empty[1], 4);
        mbar_init(drain, 1);
        fence_mbarrier_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 4) {
        // ------------------------------------------------------ TMA producer
        if (elect_one()) {
            tma_prefetch_desc(&p.tx);
            tma_prefetch_desc(&p.tc);
        }
        int n = 0; // stage fills issued
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
            const int rt = u / p.slices, sl = u % p.slices;
            const int c_begin = p.code_lo + sl * p.slice_codes;
            const int c_end = min(p.code_hi, c_begin + p.slice_codes);
            for (int c = c_begin; ok && c < c_end; c += 256) {
                for (int kc = 0; kc < p.chunks; ++kc, ++n) {
                    const int st = n % S::STAGES;
                    ok = __all_sync(0xffffffffu, mbar_wait(&empty[st], ((n / S::STAGES) & 1) ^ 1,
                                                           err, kErrWaitEmpty));
                    if (!ok)
                        break;
                    if (elect_one()) {
                        uint8_t *dst = smem + st * S::STAGE;
                        mbar_arrive_expect_tx(&full[st], S::STAGE);
                        tma_load_2d(dst, &p.tx, &full[st], kc * S::KC, rt * 128);
                        tma_load_2d(dst + S::X_CHUNK, &p.tc, &full[st], kc * S::KC, c);
                    }
                    __syncwarp();
                }
            }
        }
        // Every issued fill must land before the CTA may exit.
        for (int j = n - S::STAGES < 0 ? 0 : n - S::STAGES; j < n; ++j)
            vqs_wait_drain(&full[j % S::STAGES], (j / S::STAGES) & 1, err);
    } else if (warp == 5) {
        // ------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = TF32 ? make_idesc_tf32(128, 256) : make_idesc_f16(128, 256, true, false);
        const uint32_t leader = elect_one() ? 1u : 0u;
        const uint32_t sbase = smem_u32(smem);
        int n = 0, n_acc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
            const int sl = u % p.slices;
            const int c_begin = p.code_lo + sl * p.slice_codes;
            const int c_end = min(p.code_hi, c_begin + p.slice_codes);
            for (int c = c_begin; ok && c < c_end; c += 256, ++n_acc) {
                const int buf = n_acc & 1;
                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], ((n_acc >> 1) & 1) ^ 1,
                                                             err, kErrWaitAcc))))
                    break;
                const uint32_t d = tmem + buf * 256;
                for (int kc = 0; kc < p.chunks; ++kc, ++n) {
                    const int st = n % S::STAGES;
                    if (!(ok = __all_sync(0xffffffffu,
                                          mbar_wait(&full[st], (n / S::STAGES) & 1, err, kErrWaitK))))
                        break;
                    tc_fence_after();
                    const uint32_t xs = sbase + st * S::STAGE;
                    const uint64_t ad = make_smem_desc(xs, 16, 1024, kLayoutSW128);
                    const uint64_t bd = make_smem_desc(xs + S::X_CHUNK, 16, 1024, kLayoutSW128);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) { // 32 bytes of K per MMA
                        const uint32_t acc = (kc > 0 || kk > 0) ? 1u : 0u;
                        if constexpr (TF32)
                            umma_ss_tf32_if(leader, d, ad + 2 * kk, bd + 2 * kk, idesc, acc);
                        else
                            umma_ss_if(leader, d, ad + 2 * kk, bd + 2 * kk, idesc, acc);
                    }
                    tc_commit_if(leader, &empty[st]);
                }
                if (!ok)
                    break;
                tc_commit_if(leader, &acc_full[buf]);
            }
        }
        tc_commit_if(leader, drain);
        __syncwarp();
        vqs_wait_drain(drain, 0, err);
    } else {
        // --------------------------------------------------------- epilogue
        const int r = (warp << 5) + lane; // TMEM lane == row within the tile
        const uint32_t lane_base = static_cast<uint32_t>(warp << 5) << 16;
        int n_acc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
            const int rt = u / p.slices, sl = u % p.slices;
            const int c_begin = p.code_lo + sl * p.slice_codes;
            const int c_end = min(p.code_hi, c_begin + p.slice_codes);
            const int row = rt * 128 + r;
            const bool live = row < p.rows;
            const float xn = live ? p.xn[row] : 0.f;
            // kVqsCand: the row's approximate best and its window edge.
            float thr = INFINITY;
            if (MODE == kVqsCand && live) {
                const unsigned long long key = p.keys[row];
                if (key != ~0ull) {
                    const int b = static_cast<int>(key & 0xffffffffu);
                    const float best = vqs_from_order_bits(static_cast<uint32_t>(key >> 32));
                    const float cb = static_cast<const float *>(p.cbnorm)[b];
                    thr = best + p.win_a * sqrtf(xn) * sqrtf(cb) + p.win_c * cb + p.win_s * (xn + cb);
                }
                if (!(thr < INFINITY)) // non-finite: every code is a candidate
                    thr = INFINITY;
            }
            const float sx = MODE == kVqsCand ? p.win_a * sqrtf(xn) : 0.f;
            const __nv_bfloat162 x2 = __float2bfloat162_rn(xn);
            const __nv_bfloat162 neg2 = __floats2bfloat162_rn(-2.f, -2.f);
            float best = INFINITY;
            int best_id = 0;
            for (int c = c_begin; c < c_end; c += 256, ++n_acc) {
                const int buf = n_acc & 1;
                // The code tile's norms: lane l holds codes c + 8 l .. c + 8 l + 7
                // (one coalesced 16- or 32-byte load per lane, issued before the
                // accumulator wait), handed to every row thread by shuffles.
                // Codes past the end hold +inf (bf16 profile: 0, masked below).
                const int kl = c + 8 * lane;
                uint4 cw = make_uint4(0u, 0u, 0u, 0u);
                float cf[8];
                if constexpr (MODE == kVqsBf16) {
                    const unsigned short *cs = static_cast<const unsigned short *>(p.cbnorm);
                    if (kl + 8 <= p.codes) {
                        cw = *reinterpret_cast<const uint4 *>(cs + kl);
                    } else {
                        unsigned short h[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            h[e] = kl + e < p.codes ? cs[kl + e] : 0;
                        cw = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                                        h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
                    }
                } else {
                    const float *cn = static_cast<const float *>(p.cbnorm);
                    if (kl + 8 <= p.codes) {
                        const float4 a = *reinterpret_cast<const float4 *>(cn + kl);
                        const float4 b = *reinterpret_cast<const float4 *>(cn + kl + 4);
                        cf[0] = a.x, cf[1] = a.y, cf[2] = a.z, cf[3] = a.w;
                        cf[4] = b.x, cf[5] = b.y, cf[6] = b.z, cf[7] = b.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            cf[e] = kl + e < p.codes ? cn[kl + e] : INFINITY;
                    }
                }
                // kVqsCand: sqrt(|c|^2) once per code, by the lane that holds it.
                float cr[8];
                if constexpr (MODE == kVqsCand) {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        cr[e] = sqrtf(cf[e]);
                }
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&acc_full[buf], (n_acc >> 1) & 1, err, kErrWaitS));
                if (!ok)
                    break;
                tc_fence_after();
#pragma unroll 1
                for (int ch = 0; ch < 8; ++ch) {
                    uint32_t dv[32];
                    tmem_ld32(tmem + lane_base + buf * 256 + ch * 32, dv);
                    const int code0 = c + ch * 32;
                    tmem_wait_ld();
                    if (code0 >= p.codes) // warp-uniform
                        continue;
                    if constexpr (MODE == kVqsBf16) {
                        float cmin = INFINITY;
                        float dist[32];
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            // Codes code0 + 2q, 2q + 1: lane 4 ch + q / 4, word q % 4.
                            const uint32_t w = q % 4 == 0 ? cw.x : q % 4 == 1 ? cw.y : q % 4 == 2 ? cw.z : cw.w;
                            const uint32_t cwq = __shfl_sync(0xffffffffu, w, 4 * ch + q / 4);
                            const int k0 = code0 + 2 * q;
                            const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162 *>(&cwq);
                            const __nv_bfloat162 dd = __floats2bfloat162_rn(__uint_as_float(dv[2 * q]),
                                                                            __uint_as_float(dv[2 * q + 1]));
                            const __nv_bfloat162 s2 = __hadd2(x2, c2);
                            const __nv_bfloat162 t = __hfma2(dd, neg2, s2);
                            dist[2 * q] = k0 < p.codes ? __bfloat162float(t.x) : INFINITY;
                            dist[2 * q + 1] = k0 + 1 < p.codes ? __bfloat162float(t.y) : INFINITY;
                            cmin = fminf(cmin, fminf(dist[2 * q], dist[2 * q + 1]));
                        }
                        if (live && cmin < best) {
                            best = cmin;
#pragma unroll
                            for (int e = 31; e >= 0; --e)
                                if (dist[e] == cmin)
                                    best_id = code0 + e;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            const int k = code0 + e;
                            // Code code0 + e: lane 4 ch + e / 8, element e % 8.
                            const float cnk = __shfl_sync(0xffffffffu, cf[e % 8], 4 * ch + e / 8);
                            const float dist = fmaf(-2.f, __uint_as_float(dv[e]), xn + cnk);
                            if constexpr (MODE == kVqsApprox) {
                                if (k < p.codes && dist < best) {
                                    best = dist;
                                    best_id = k;
                                }
                            } else {
                                const float crk = __shfl_sync(0xffffffffu, cr[e % 8], 4 * ch + e / 8);
                                if (!live || k >= p.codes)
                                    continue;
                                // Candidate unless provably outside the window.
                                const float lo = dist - (sx * crk + p.win_c * cnk + p.win_s * (xn + cnk));
                                if (!(lo <= thr) && isfinite(lo) && thr < INFINITY)
                                    continue;
                                const unsigned slot = atomicAdd(p.cand_count + row, 1u);
                                if (slot < static_cast<unsigned>(kVqCandCap))
                                    p.cand[static_cast<long long>(row) * kVqCandCap + slot] =
                                        static_cast<unsigned>(k);
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&acc_empty[buf]);
            }
            if (MODE != kVqsCand && ok && live && best < INFINITY) {
                const unsigned long long key =
                    (static_cast<unsigned long long>(vqs_order_bits(best)) << 32) |
                    static_cast<unsigned>(best_id);
                atomicMin(p.keys + row, key);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5)
        tmem_dealloc(tmem, 512);
}

__device__ __forceinline__ void vq_write_id(void *ids, int row, double best, unsigned best_id, int ids_u16) {
    const unsigned id = best < INFINITY ? best_id : 0u;
    if (ids_u16)
        static_cast<uint16_t *>(ids)[row] = static_cast<uint16_t>(id);
    else
        static_cast<int32_t *>(ids)[row] = static_cast<int32_t>(id);
}

// Exact fp64 re-scoring of the candidates, one warp per row (rows whose list
// overflowed are left to vq_brute_fp64).  The winner is the smallest (direct
// distance, id) with a distance below +inf (src/cpu.cpp:272-282); a row
// without one keeps id 0.
__global__ void vq_refine_fp64(const float *x, const float *codebook, const unsigned *cand_count,
                               const unsigned *cand, void *ids, int rows, int dim, int codes,
                               int ids_u16) {
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int lane = threadIdx.x & 31;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
        const unsigned n = cand_count[row];
        if (n > static_cast<unsigned>(kVqCandCap))
            continue;
        const int count = static_cast<int>(n);
        const float *xr = x + static_cast<long long>(row) * dim;
        double best = INFINITY;
        unsigned best_id = 0xffffffffu;
        for (int j = lane; j < count; j += 32) {
            const unsigned code = cand[static_cast<long long>(row) * kVqCandCap + j];
            const float *cr = codebook + static_cast<long long>(code) * dim;
            double direct = 0.0;
            for (int k = 0; k < dim; ++k) {
                const double delta = static_cast<double>(xr[k]) - static_cast<double>(cr[k]);
                direct = __dadd_rn(direct, __dmul_rn(delta, delta));
            }
            if (direct < best || (direct == best && code < best_id)) {
                best = direct;
                best_id = code;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const double ob = __shfl_xor_sync(0xffffffffu, best, off);
            const unsigned oi = __shfl_xor_sync(0xffffffffu, best_id, off);
            if (ob < best || (ob == best && oi < best_id)) {
                best = ob;
                best_id = oi;
            }
        }
        if (lane == 0)
            vq_write_id(ids, row, best, best_id, ids_u16);
    }
}

// Rows whose candidate list overflowed: every code scored with the same direct
// fp64 sum, one block per row.  Each thread owns codes j = t, t + 256, ... and
// sums its code's terms in column order; x streams through shared memory in
// 1024-column pieces.
constexpr int kBruteThreads = 256, kBrutePiece = 1024;
__global__ void __launch_bounds__(kBruteThreads) vq_brute_fp64(const float *x, const float *codebook,
                                                               const unsigned *cand_count, void *ids, int rows,
                                                               int dim, int codes, int ids_u16) {
    __shared__ double xs[kBrutePiece];
    __shared__ double red_d[kBruteThreads / 32];
    __shared__ unsigned red_i[kBruteThreads / 32];
    constexpr int kPerThread = 8; // codes per pass of a thread
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
        if (cand_count[row] <= static_cast<unsigned>(kVqCandCap))
            continue; // uniform over the block
        const float *xr = x + static_cast<long long>(row) * dim;
        double best = INFINITY;
        unsigned best_id = 0xffffffffu;
        for (int c0 = 0; c0 < codes; c0 += kBruteThreads * kPerThread) {
            double acc[kPerThread];
#pragma unroll
            for (int i = 0; i < kPerThread; ++i)
                acc[i] = 0.0;
            for (int k0 = 0; k0 < dim; k0 += kBrutePiece) {
                const int kn = min(kBrutePiece, dim - k0);
                __syncthreads();
                for (int k = threadIdx.x; k < kn; k += kBruteThreads)
                    xs[k] = static_cast<double>(xr[k0 + k]);
                __syncthreads();
#pragma unroll
                for (int i = 0; i < kPerThread; ++i) {
                    const int code = c0 + i * kBruteThreads + threadIdx.x;
                    if (code >= codes)
                        continue;
                    const float *cr = codebook + static_cast<long long>(code) * dim + k0;
                    double a = acc[i];
                    for (int k = 0; k < kn; ++k) {
                        const double delta = xs[k] - static_cast<double>(__ldg(cr + k));
                        a = __dadd_rn(a, __dmul_rn(delta, delta));
                    }
                    acc[i] = a;
                }
            }
#pragma unroll
            for (int i = 0; i < kPerThread; ++i) {
                const int code = c0 + i * kBruteThreads + threadIdx.x;
                if (code < codes && (acc[i] < best || (acc[i] == best && static_cast<unsigned>(code) < best_id))) {
                    best = acc[i];
                    best_id = static_cast<unsigned>(code);
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const double ob = __shfl_xor_sync(0xffffffffu, best, off);
            const unsigned oi = __shfl_xor_sync(0xffffffffu, best_id, off);
            if (ob < best || (ob == best && oi < best_id)) {
                best = ob;
                best_id = oi;
            }
        }
        if ((threadIdx.x & 31) == 0) {
            red_d[threadIdx.x >> 5] = best;
            red_i[threadIdx.x >> 5] = best_id;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kBruteThreads / 32; ++w)
                if (red_d[w] < best || (red_d[w] == best && red_i[w] < best_id)) {
                    best = red_d[w];
                    best_id = red_i[w];
                }
            vq_write_id(ids, row, best, best_id, ids_u16);
        }
    }
}

__global__ void vqs_finish(const unsigned long long *keys, void *ids, int rows, int ids_u16) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
        const unsigned long long k = keys[i];
        // An untouched key means every distance was NaN: the reference keeps id 0.
        const unsigned id = k == ~0ull ? 0u : static_cast<unsigned>(k & 0xffffffffu);
        if (ids_u16)
            static_cast<uint16_t *>(ids)[i] = static_cast<uint16_t>(id);
        else
            static_cast<int32_t *>(ids)[i] = static_cast<int32_t>(id);
    }
}

__global__ void vqs_init(unsigned long long *keys, unsigned *cand_count, int rows) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
        keys[i] = ~0ull;
        if (cand_count)
            cand_count[i] = 0u;
    }
}

// ------------------------------------------------------------------ host side
namespace {
template <bool TF32, int MODE> int vqs_launch_typed(const VqsParams &p, int grid, cudaStream_t stream) {
    using S = VqsShape<TF32>;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr = set_smem_limit(reinterpret_cast<const void *>(vq_stream_kernel<TF32, MODE>),
                                            S::SMEM_BYTES, done);
    if (attr != cudaSuccess)
        return static_cast<int>(attr);
    vq_stream_kernel<TF32, MODE><<<grid, kVqsThreads, S::SMEM_BYTES, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

int sm_count() {
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// Units = 128-row tiles x slices of the launch's codebook window, about 8
// units per SM.
int plan_units(VqsParams &p) {
    const int sms = sm_count();
    const int row_tiles = (p.rows + 127) / 128;
    const int code_tiles = (p.code_hi - p.code_lo + 255) / 256;
    int slices = (8 * sms + row_tiles - 1) / row_tiles;
    slices = slices < 1 ? 1 : slices > code_tiles ? code_tiles : slices;
    const int tiles_per_slice = (code_tiles + slices - 1) / slices;
    p.slice_codes = tiles_per_slice * 256;
    p.slices = (code_tiles + tiles_per_slice - 1) / tiles_per_slice;
    const long long units = static_cast<long long>(row_tiles) * p.slices;
    return static_cast<int>(units < sms ? units : sms);
}
} // namespace

size_t vq_stream_workspace(size_t rows, int profile_fp32) {
    // keys (8) + xn (4) [+ candidate count (4) + candidate list] per row, then
    // 256 bytes for the device copy of a cancellation flag.
    const size_t per_row = profile_fp32 ? 16 + 4 * static_cast<size_t>(kVqCandCap) : 12;
    return (rows * per_row + 255) / 256 * 256 + 256;
}

int vq_stream_launch(const VqArgs &a, int profile_fp32, cudaStream_t stream) {
    VqsParams p{};
    const bool tf32 = profile_fp32 != 0;
    const int kc = tf32 ? 32 : 64;
    int rc = tf32 ? make_map_2d_f32(&p.tx, a.x, a.dim, a.rows, kc, 128)
                  : make_map_2d(&p.tx, a.x, a.dim, a.rows, kc, 128);
    if (rc)
        return rc;
    rc = tf32 ? make_map_2d_f32(&p.tc, a.codebook, a.dim, a.codes, kc, 256)
              : make_map_2d(&p.tc, a.codebook, a.dim, a.codes, kc, 256);
    if (rc)
        return rc;
    // Workspace carve: keys | xn | cand_count | cand.
    uint8_t *ws = static_cast<uint8_t *>(a.keys);
    const size_t rows = static_cast<size_t>(a.rows);
    p.keys = reinterpret_cast<unsigned long long *>(ws);
    float *xn_ws = reinterpret_cast<float *>(ws + 8 * rows);
    p.xn = xn_ws;
    if (tf32) {
        p.cand_count = reinterpret_cast<unsigned *>(ws + 12 * rows);
        p.cand = reinterpret_cast<unsigned *>(ws + 16 * rows);
    }
    // The cancellation flag is copied to device memory before each window's
    // launch and the CTAs read that copy: the flag usually lives in mapped
    // pinned host memory, and 148 CTAs reading host memory as they start made
    // each launch about four times slower (44 -> 179 us at 750 x 1024 fp32).
    int *flag_dev = reinterpret_cast<int *>(ws + (rows * (tf32 ? 16 + 4 * static_cast<size_t>(kVqCandCap) : 12) + 255) /
                                                     256 * 256);
    p.cbnorm = a.cbnorm;
    p.rows = a.rows;
    p.dim = a.dim;
    p.codes = a.codes;
    p.chunks = (a.dim + kc - 1) / kc;
    // Window coefficients (see the top of this file), rounded up by 1e-4 for
    // the fp32 evaluation of the window itself.
    p.win_a = static_cast<float>((std::ldexp(1.0, -7) + (a.dim + 1.0) * std::ldexp(1.0, -21)) * 1.0001);
    p.win_c = static_cast<float>(a.dim * std::ldexp(1.0, -22) * 1.0001);
    p.win_s = static_cast<float>(std::ldexp(1.0, -20) * 1.0001);
    p.err = a.err;
    p.cancel = a.cancel ? flag_dev : nullptr;
    const int threads = 256;
    const int kb = (a.rows + threads - 1) / threads;
    vqs_init<<<kb < 4096 ? kb : 4096, threads, 0, stream>>>(p.keys, p.cand_count, a.rows);
    // |x|^2 per row in the profile's arithmetic (bf16 profile: the bf16 value),
    // unless the caller wrote the fp32 norms alongside x.
    if (tf32 && a.xnorm)
        p.xn = a.xnorm;
    else if ((rc = squares_launch(a.x, xn_ws, a.rows, a.dim, tf32 ? 0 : 1, 0, stream)))
        return rc;
    // One launch per codebook window: the whole codebook, or (when the caller
    // can cancel) windows of kVqCancelWindow codes, widened in multiples of it
    // until one window gives two units per SM (few rows: a 4096-code window of
    // three row tiles would occupy 48 SMs).  The keys merge by atomicMin across
    // launches, so windows compose exactly.
    int window = a.codes;
    if (a.cancel) {
        const long long row_tiles = (a.rows + 127) / 128;
        const long long tiles = (2LL * sm_count() + row_tiles - 1) / row_tiles;
        const long long w = (tiles * 256 + kVqCancelWindow - 1) / kVqCancelWindow * kVqCancelWindow;
        window = w < a.codes ? static_cast<int>(w) : a.codes;
    }
    auto pass = [&](auto launch) {
        for (int lo = 0; lo < a.codes; lo += window) {
            if (a.cancel) {
                const cudaError_t e = cudaMemcpyAsync(flag_dev, const_cast<const int *>(a.cancel), sizeof(int),
                                                      cudaMemcpyDefault, stream);
                if (e != cudaSuccess)
                    return static_cast<int>(e);
            }
            p.code_lo = lo;
            p.code_hi = lo + window < a.codes ? lo + window : a.codes;
            if (int e = launch(plan_units(p)))
                return e;
        }
        return 0;
    };
    if (!tf32) {
        if ((rc = pass([&](int grid) { return vqs_launch_typed<false, kVqsBf16>(p, grid, stream); })))
            return rc;
        vqs_finish<<<kb < 4096 ? kb : 4096, threads, 0, stream>>>(p.keys, a.ids, a.rows, a.ids_u16);
        return static_cast<int>(cudaGetLastError());
    }
    if ((rc = pass([&](int grid) { return vqs_launch_typed<true, kVqsApprox>(p, grid, stream); })) ||
        (rc = pass([&](int grid) { return vqs_launch_typed<true, kVqsCand>(p, grid, stream); })))
        return rc;
    const int rb = (a.rows * 32 + threads - 1) / threads;
    vq_refine_fp64<<<rb < 8192 ? rb : 8192, threads, 0, stream>>>(
        static_cast<const float *>(a.x), static_cast<const float *>(a.codebook), p.cand_count,
        p.cand, a.ids, a.rows, a.dim, a.codes, a.ids_u16);
    vq_brute_fp64<<<a.rows < 4 * sm_count() ? a.rows : 4 * sm_count(), kBruteThreads, 0, stream>>>(
        static_cast<const float *>(a.x), static_cast<const float *>(a.codebook), p.cand_count, a.ids, a.rows,
        a.dim, a.codes, a.ids_u16);
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
