// vq_sm100.cu -- fused VQ codebook nearest-neighbour argmin for B200 (sm_100a).
//
// Replaces omni-tokenizer's Cuda::quantize (src/cuda.cu:934-973), which for
// every 1024-code tile wrote a dots[rows x 1024] matrix to HBM with cuBLASLt
// and re-read it in argmin_kernel (src/cuda.cu:336-384).  Here the distance
// GEMM runs on tcgen05 into TMEM and the argmin is the GEMM's epilogue: only
// one 64-bit (distance, id) key per row ever reaches global memory.
//
// bf16 profile arithmetic (omni-tokenizer src/cpu.cpp:246-259,
// src/cuda.cu:343-349):
//   D    = bf16(x . c)                      (fp32 accumulation, rounded once)
//   S    = bf16(|x|^2 + |c|^2)
//   dist = bf16(S - bf16(2 D))
// and the smallest id wins among equal distances.  The epilogue evaluates S
// with add.rn.bf16x2 and dist with fma.rn.bf16x2(D, -2, S): both operands are
// bf16 values, so fp32 arithmetic followed by one bf16 rounding (the
// reference) and a single correctly rounded bf16 operation give the same
// result (the fp32 step is exact unless the exponents differ by more than 15,
// in which case both round to the larger operand).
// |x|^2 is summed per row in column order exactly as src/cpu.cpp:216-226.
//
// Work is split into units (128-row tile, slice of the codebook) spread over a
// persistent grid; each unit ends with one atomicMin per row on
//   key = (order-preserving bits of dist) << 32 | id,
// whose minimum is the smallest distance and, among equal distances, the
// smallest id -- the reference's tie rule.
//
// Roles: warp 16 TMA producer, warp 17 TMEM owner + tcgen05.mma issuer,
// warps 0-15 epilogue: warp w reads TMEM lane quarter w % 4 (rows
// 32 (w % 4) .. +31 of the tile) and accumulator columns [64 (w / 4), +64), so
// each sub-partition runs four epilogue warps and hides the TMEM-load and
// norm-load latency; every warp keeps its own running best per row and ends
// a unit with one atomicMin per row.
// TMEM: two 256-column fp32 accumulators (512 columns).
#include "sm100.cuh"
#include "tma.h"
#include "vq.h"

#include <cmath>
#include <mutex>

namespace omni_b200 {

template <int DP> struct VqShape {
    static constexpr int C0 = DP < 64 ? DP : 64;
    static constexpr int C1 = DP - C0;
    static constexpr int ROW0 = C0 * 2, ROW1 = C1 * 2;
    static constexpr int X_BYTES = 128 * DP * 2;
    static constexpr int XCH0 = 128 * ROW0;
    static constexpr int C_BYTES = 256 * DP * 2;
    static constexpr int CCH0 = 256 * ROW0;
    static constexpr int BUDGET = 200 * 1024;
    static constexpr int STAGES_RAW = (BUDGET - X_BYTES) / C_BYTES;
    static constexpr int STAGES = STAGES_RAW > 6 ? 6 : STAGES_RAW;
    static constexpr int KSTEPS = DP / 16;
    // At least 120 KB so that one CTA (which allocates all 512 TMEM columns)
    // occupies an SM by itself.
    static constexpr int SMEM_RAW = X_BYTES + STAGES * C_BYTES + 512 + 1024;
    static constexpr int SMEM_BYTES = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
    static_assert(STAGES >= 2, "codebook ring needs two stages");
    static_assert(C1 == 0 || C1 == 16 || C1 == 32 || C1 == 64, "unsupported dim padding");
};

constexpr int kVqThreads = 576;
constexpr int kVqEpiWarps = 16;
constexpr int kVqProducerWarp = 16;
constexpr int kVqMmaWarp = 17;

__device__ __forceinline__ uint32_t order_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u)
        return 0xffffffffu; // NaN never wins (the reference's `dist < best` is false)
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __noinline__ void vq_wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicOr(err, kErrWaitDrain);
            return;
        }
    }
}

template <int DP>
__global__ void __launch_bounds__(kVqThreads, 1) vq_bf16_kernel(const __grid_constant__ VqParams p) {
    using S = VqShape<DP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sX = smem;
    uint8_t *sC = sX + S::X_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sC + S::STAGES * S::C_BYTES);
    uint64_t *x_full = bars;
    uint64_t *x_empty = bars + 1;
    uint64_t *c_full = bars + 2;
    uint64_t *c_empty = c_full + S::STAGES;
    uint64_t *acc_full = c_empty + S::STAGES; // [2]
    uint64_t *acc_empty = acc_full + 2;       // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;
    const int row_tiles = (p.rows + 127) / 128;
    const int units = row_tiles * p.slices;

    if (threadIdx.x == 0) {
        mbar_init(x_full, 1);
        mbar_init(x_empty, 1);
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&c_full[s], 1);
            mbar_init(&c_empty[s], 1);
        }
        mbar_init(&acc_full[0], 1);
        mbar_init(&acc_full[1], 1);
        mbar_init(&acc_empty[0], kVqEpiWarps); // one arrive per epilogue warp
        mbar_init(&acc_empty[1], kVqEpiWarps);
        mbar_init(drain, 1);
        fence_mbarrier_init();
    }
    if (warp == kVqMmaWarp) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == kVqProducerWarp) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&p.tx0);
            tma_prefetch_desc(&p.tc0);
            int x_loads = 0, n_c = 0; // loads issued so far
            bool ok = true;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
                const int rt = u / p.slices, sl = u % p.slices;
                const int c_begin = sl * p.slice_codes;
                const int c_end = min(p.codes, c_begin + p.slice_codes);
                if (!(ok = mbar_wait(x_empty, (x_loads & 1) ^ 1, err, kErrWaitEmpty)))
                    break;
                mbar_arrive_expect_tx(x_full, S::X_BYTES);
                tma_load_2d(sX, &p.tx0, x_full, 0, rt * 128);
                if constexpr (S::C1 > 0)
                    tma_load_2d(sX + S::XCH0, &p.tx1, x_full, S::C0, rt * 128);
                ++x_loads;
                for (int c = c_begin; c < c_end; c += 256) {
                    const int st = n_c % S::STAGES;
                    const uint32_t ph = (n_c / S::STAGES) & 1;
                    if (!(ok = mbar_wait(&c_empty[st], ph ^ 1, err, kErrWaitEmpty)))
                        break;
                    uint8_t *dst = sC + st * S::C_BYTES;
                    mbar_arrive_expect_tx(&c_full[st], S::C_BYTES);
                    tma_load_2d(dst, &p.tc0, &c_full[st], 0, c);
                    if constexpr (S::C1 > 0)
                        tma_load_2d(dst + S::CCH0, &p.tc1, &c_full[st], S::C0, c);
                    ++n_c;
                }
            }
            // Drain: the last X load and the last load of every ring slot must
            // land before the CTA may exit.
            if (x_loads > 0)
                vq_wait_drain(x_full, (x_loads - 1) & 1, err);
            for (int j = n_c - S::STAGES < 0 ? 0 : n_c - S::STAGES; j < n_c; ++j)
                vq_wait_drain(&c_full[j % S::STAGES], (j / S::STAGES) & 1, err);
        }
        __syncwarp();
    } else if (warp == kVqMmaWarp) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc_f16(128, 256, true, false);
            constexpr uint32_t lay0 = layout_for_row_bytes(S::ROW0);
            constexpr uint32_t lay1 = layout_for_row_bytes(S::ROW1 > 0 ? S::ROW1 : 32);
            const uint32_t sx = smem_u32(sX), sc = smem_u32(sC);
            int n_x = 0, n_c = 0, n_acc = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++n_x) {
                const int sl = u % p.slices;
                const int c_begin = sl * p.slice_codes;
                const int c_end = min(p.codes, c_begin + p.slice_codes);
                if (!(ok = mbar_wait(x_full, n_x & 1, err, kErrWaitQ)))
                    break;
                for (int c = c_begin; c < c_end; c += 256, ++n_c, ++n_acc) {
                    const int st = n_c % S::STAGES;
                    const uint32_t ph = (n_c / S::STAGES) & 1;
                    const int buf = n_acc & 1;
                    if (!(ok = mbar_wait(&acc_empty[buf], ((n_acc >> 1) & 1) ^ 1, err, kErrWaitAcc)))
                        break;
                    if (!(ok = mbar_wait(&c_full[st], ph, err, kErrWaitK)))
                        break;
                    tc_fence_after();
                    const uint32_t cb = sc + st * S::C_BYTES;
#pragma unroll
                    for (int kk = 0; kk < S::KSTEPS; ++kk) {
                        const int e = kk * 16;
                        const bool c1 = e >= S::C0;
                        const uint32_t rowb = c1 ? S::ROW1 : S::ROW0;
                        const uint32_t xoff = (c1 ? S::XCH0 : 0) + (e - (c1 ? S::C0 : 0)) * 2;
                        const uint32_t coff = (c1 ? S::CCH0 : 0) + (e - (c1 ? S::C0 : 0)) * 2;
                        const uint64_t ad = make_smem_desc(sx + xoff, 16, 8 * rowb, c1 ? lay1 : lay0);
                        const uint64_t bd = make_smem_desc(cb + coff, 16, 8 * rowb, c1 ? lay1 : lay0);
                        umma_ss(tmem + buf * 256, ad, bd, idesc, kk > 0 ? 1u : 0u);
                    }
                    tc_commit(&c_empty[st]);
                    tc_commit(&acc_full[buf]);
                }
                tc_commit(x_empty);
            }
            tc_commit(drain);
            vq_wait_drain(drain, 0, err);
        }
        __syncwarp();
    } else {
        // --------------------------------------------------------- epilogue
        const int qd = warp & 3, cg = warp >> 2;   // lane quarter, 64-column group
        const int r = (qd << 5) + lane;            // TMEM lane == row within the tile
        const uint32_t lane_base = static_cast<uint32_t>(qd << 5) << 16;
        const __nv_bfloat16 *x = static_cast<const __nv_bfloat16 *>(p.x);
        const uint4 *cn = static_cast<const uint4 *>(p.cbnorm);
        const __nv_bfloat162 neg2 = __floats2bfloat162_rn(-2.f, -2.f);
        int n_acc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
            const int rt = u / p.slices, sl = u % p.slices;
            const int c_begin = sl * p.slice_codes;
            const int c_end = min(p.codes, c_begin + p.slice_codes);
            const int row = rt * 128 + r;
            // |x|^2 in column order (src/cpu.cpp:216-226), bf16 profile: the
            // row is fetched with independent 16-byte loads (dim % 8 == 0),
            // then summed sequentially; padding columns add +0.
            float xn = 0.f;
            if (row < p.rows) {
                const uint4 *xr =
                    reinterpret_cast<const uint4 *>(x + static_cast<long long>(row) * p.dim);
                uint4 xw[DP / 8];
#pragma unroll
                for (int q = 0; q < DP / 8; ++q)
                    xw[q] = q * 8 < p.dim ? __ldg(xr + q) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int q = 0; q < DP / 8; ++q) {
                    const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&xw[q]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 v = __bfloat1622float2(h2[e]);
                        xn = __fadd_rn(xn, __bfloat162float(__float2bfloat16_rn(__fmul_rn(v.x, v.x))));
                        xn = __fadd_rn(xn, __bfloat162float(__float2bfloat16_rn(__fmul_rn(v.y, v.y))));
                    }
                }
            }
            const __nv_bfloat162 x2 = __float2bfloat162_rn(xn); // rounds: bf16(sum)
            float best = INFINITY;
            int best_id = 0;
            for (int c = c_begin; c < c_end; c += 256, ++n_acc) {
                const int buf = n_acc & 1;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(&acc_full[buf], (n_acc >> 1) & 1, err, kErrWaitS));
                if (!ok)
                    break;
                tc_fence_after();
                const bool partial = c + 256 > p.codes;
                uint32_t dd2[2][32];
                tmem_ld32(tmem + lane_base + buf * 256 + cg * 64, dd2[0]);
                tmem_ld32(tmem + lane_base + buf * 256 + cg * 64 + 32, dd2[1]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int ch = cg * 2 + h;
                    uint32_t *d = dd2[h];
                    const int code0 = c + ch * 32;
                    uint4 cnv[4];
                    if (!partial) {
#pragma unroll
                        for (int w = 0; w < 4; ++w)
                            cnv[w] = __ldg(cn + (code0 >> 3) + w);
                    } else {
                        // Last tile: read only norms that exist.
                        const unsigned short *cs = static_cast<const unsigned short *>(p.cbnorm);
                        unsigned short hv[32];
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            hv[e] = code0 + e < p.codes ? cs[code0 + e] : 0;
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            cnv[w].x = hv[8 * w] | (static_cast<uint32_t>(hv[8 * w + 1]) << 16);
                            cnv[w].y = hv[8 * w + 2] | (static_cast<uint32_t>(hv[8 * w + 3]) << 16);
                            cnv[w].z = hv[8 * w + 4] | (static_cast<uint32_t>(hv[8 * w + 5]) << 16);
                            cnv[w].w = hv[8 * w + 6] | (static_cast<uint32_t>(hv[8 * w + 7]) << 16);
                        }
                    }
                    if (h == 0)
                        tmem_wait_ld();
                    __nv_bfloat162 dist[16];
                    __nv_bfloat162 m2 = __floats2bfloat162_rn(INFINITY, INFINITY);
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const __nv_bfloat162 dd =
                            __floats2bfloat162_rn(__uint_as_float(d[2 * q]), __uint_as_float(d[2 * q + 1]));
                        const uint32_t cw = (&cnv[q >> 2].x)[q & 3];
                        const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162 *>(&cw);
                        const __nv_bfloat162 s2 = __hadd2(x2, c2);
                        dist[q] = __hfma2(dd, neg2, s2);
                        m2 = __hmin2(m2, dist[q]);
                    }
                    if (partial) {
                        // Codes past the end were zero-filled by TMA: never candidates.
                        m2 = __floats2bfloat162_rn(INFINITY, INFINITY);
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            if (code0 + 2 * q >= p.codes)
                                dist[q].x = __float2bfloat16_rn(INFINITY);
                            if (code0 + 2 * q + 1 >= p.codes)
                                dist[q].y = __float2bfloat16_rn(INFINITY);
                            m2 = __hmin2(m2, dist[q]);
                        }
                    }
                    const float cmin = fminf(__bfloat162float(m2.x), __bfloat162float(m2.y));
                    if (cmin < best) {
                        best = cmin;
#pragma unroll
                        for (int q = 15; q >= 0; --q) {
                            if (__bfloat162float(dist[q].y) == cmin)
                                best_id = code0 + 2 * q + 1;
                            if (__bfloat162float(dist[q].x) == cmin)
                                best_id = code0 + 2 * q;
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&acc_empty[buf]);
            }
            if (ok && row < p.rows) {
                const unsigned long long key =
                    (static_cast<unsigned long long>(order_bits(best)) << 32) |
                    static_cast<unsigned>(best_id);
                atomicMin(static_cast<unsigned long long *>(p.keys) + row, key);
            }
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kVqMmaWarp)
        tmem_dealloc(tmem, 512);
}

__global__ void vq_keys_init(unsigned long long *keys, int rows) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x)
        keys[i] = ~0ull;
}

__global__ void vq_keys_finish(const unsigned long long *keys, void *ids, int rows, int ids_u16) {
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

// ------------------------------------------------------------------ host side
int vq_padded_dim(int dim) {
    if (dim <= 16)
        return 16;
    if (dim <= 32)
        return 32;
    if (dim <= 64)
        return 64;
    if (dim <= 80)
        return 80;
    if (dim <= 96)
        return 96;
    if (dim <= 128)
        return 128;
    return -1;
}

template <int DP> int vq_launch_typed(VqParams &p, int grid, cudaStream_t stream) {
    using S = VqShape<DP>;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr =
        set_smem_limit(reinterpret_cast<const void *>(vq_bf16_kernel<DP>), S::SMEM_BYTES, done);
    if (attr != cudaSuccess)
        return static_cast<int>(attr);
    vq_bf16_kernel<DP><<<grid, kVqThreads, S::SMEM_BYTES, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

int vq_bf16_launch(const VqArgs &a, cudaStream_t stream) {
    const int dp = vq_padded_dim(a.dim);
    if (dp < 0)
        return -2;
    VqParams p{};
    const int w0 = dp < 64 ? dp : 64, w1 = dp - w0;
    int rc = 0;
    if ((rc = make_map_2d(&p.tx0, a.x, a.dim, a.rows, w0, 128)) ||
        (rc = make_map_2d(&p.tc0, a.codebook, a.dim, a.codes, w0, 256)))
        return rc;
    if (w1 > 0 && ((rc = make_map_2d(&p.tx1, a.x, a.dim, a.rows, w1, 128)) ||
                   (rc = make_map_2d(&p.tc1, a.codebook, a.dim, a.codes, w1, 256))))
        return rc;
    p.x = a.x;
    p.cbnorm = a.cbnorm;
    p.keys = a.keys;
    p.rows = a.rows;
    p.dim = a.dim;
    p.codes = a.codes;
    p.err = a.err;
    // Units = row tiles x codebook slices; aim for ~8 units per SM.
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int row_tiles = (a.rows + 127) / 128;
    const int code_tiles = (a.codes + 255) / 256;
    int slices = (8 * sms + row_tiles - 1) / row_tiles;
    slices = slices < 1 ? 1 : slices > code_tiles ? code_tiles : slices;
    const int tiles_per_slice = (code_tiles + slices - 1) / slices;
    p.slice_codes = tiles_per_slice * 256;
    p.slices = (code_tiles + tiles_per_slice - 1) / tiles_per_slice;
    const long long units = static_cast<long long>(row_tiles) * p.slices;
    const int grid = static_cast<int>(units < sms ? units : sms);
    const int threads = 256;
    const int kb = (a.rows + threads - 1) / threads;
    vq_keys_init<<<kb < 4096 ? kb : 4096, threads, 0, stream>>>(
        static_cast<unsigned long long *>(a.keys), a.rows);
    switch (dp) {
    case 16:
        rc = vq_launch_typed<16>(p, grid, stream);
        break;
    case 32:
        rc = vq_launch_typed<32>(p, grid, stream);
        break;
    case 64:
        rc = vq_launch_typed<64>(p, grid, stream);
        break;
    case 80:
        rc = vq_launch_typed<80>(p, grid, stream);
        break;
    case 96:
        rc = vq_launch_typed<96>(p, grid, stream);
        break;
    case 128:
        rc = vq_launch_typed<128>(p, grid, stream);
        break;
    default:
        return -2;
    }
    if (rc)
        return rc;
    vq_keys_finish<<<kb < 4096 ? kb : 4096, threads, 0, stream>>>(
        static_cast<const unsigned long long *>(a.keys), a.ids, a.rows, a.ids_u16);
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
