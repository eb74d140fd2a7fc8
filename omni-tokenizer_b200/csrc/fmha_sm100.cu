// fmha_sm100.cu -- encoder self-attention forward for B200 (sm_100a).
//
// Replaces omni-tokenizer's attention path (src/cuda.cu:832-907, which calls
// the Sm80 mem-efficient kernel of src/audio_attention.cu, the Sm80
// FlashAttention-2 kernel of src/flash_attention.cu, or a cuBLAS SGEMM +
// softmax fallback).  Semantics follow src/cpu.cpp:122-172: per head,
// O = softmax(scale * Q K^T + mask) V with scale = hd^-1/2 and the key limit
// limit(t) = min(L, valid[, (t/block + 1) * block]).
//
// One CTA owns 256 query rows of one (batch, head) as two 128-row tiles and
// streams the key/value sequence once in 128-key tiles:
//   warp 8      TMA producer: Q tiles once, then K_j / V_j into a ring of
//               STAGES shared-memory slots (mbarrier full/empty pairs);
//   warp 9      TMEM owner and single-thread tcgen05.mma issuer:
//               S_i = Q_i K_j^T (smem x smem -> TMEM) and
//               O_i += P_i V_j (P from TMEM x V from smem -> TMEM);
//   warps 0-7   two softmax warpgroups, one per query tile; thread r owns
//               TMEM lane r = query row r: it loads its S row, applies the
//               mask, keeps the running max / sum, rescales O in TMEM only
//               when the max grew by more than 2^8 (lazy rescale), writes P
//               (bf16/fp16 pairs) over the first 64 columns of its S row and
//               finally normalises O and stores it to global memory.
// The MMA issue order S_0(j+1) after O_0 += P_0(j) (and likewise for tile 1)
// lets the tensor core work on one tile while the other tile's softmax runs.
//
// TMEM columns (512 allocated): S_0 [0,128), S_1 [128,256),
// O_0 [256, 256+HDP), O_1 [384, 384+HDP).
//
// Head dims: HDP in {16, 32, 64, 80, 96, 128} is the padded head dim; a head
// of hd <= HDP is loaded with TMA zero fill beyond hd, so the padding lanes
// contribute nothing.  Each 128-row tile is stored as chunk 0 (64 columns,
// 128-byte swizzle; or the whole tile when HDP < 64) followed by chunk 1
// (HDP - 64 columns: 16 -> 32-byte swizzle, 32 -> 64-byte, 64 -> 128-byte).
#include "fmha.h"
#include "sm100.cuh"
#include "tma.h"

#include <cmath>
#include <cstdio>
#include <mutex>

namespace omni_b200 {

template <int HDP> struct FmhaShape {
    static constexpr int C0 = HDP < 64 ? HDP : 64; // chunk 0 width (elements)
    static constexpr int C1 = HDP - C0;            // chunk 1 width: 0, 16, 32 or 64
    static constexpr int ROW0 = C0 * 2;            // bytes per row of chunk 0
    static constexpr int ROW1 = C1 * 2;
    static constexpr int CH0_BYTES = 128 * ROW0;
    static constexpr int TILE_BYTES = 128 * HDP * 2; // one 128-row tile
    static constexpr int STAGES = HDP <= 96 ? 3 : 2;
    static constexpr int KSTEPS = HDP / 16;
    static constexpr int BAR_BYTES = 256;
    // At least 120 KB so that one CTA (which allocates all 512 TMEM columns)
    // occupies an SM by itself.
    static constexpr int SMEM_RAW = (2 + 2 * STAGES) * TILE_BYTES + BAR_BYTES + 1024;
    static constexpr int SMEM_BYTES = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
    static_assert(C1 == 0 || C1 == 16 || C1 == 32 || C1 == 64, "unsupported head dim padding");
    static_assert(HDP % 16 == 0, "head dim padding must be a multiple of 16");
};

constexpr int kThreads = 320;

// Loads one 128-row tile (both chunks) of a (token, head, batch) tensor.
template <int HDP>
__device__ __forceinline__ void load_tile(uint8_t *dst, const CUtensorMap *m0,
                                          const CUtensorMap *m1, uint64_t *bar, int row, int head,
                                          int batch) {
    using S = FmhaShape<HDP>;
    tma_load_4d(dst, m0, bar, 0, row, head, batch);
    if constexpr (S::C1 > 0)
        tma_load_4d(dst + S::CH0_BYTES, m1, bar, S::C0, row, head, batch);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
    if (bf16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    }
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// Drain wait: bounded by time only (does not give up early on other threads'
// errors), used so that no TMA write or MMA is still in flight when the CTA
// releases its shared memory and TMEM.
__device__ __noinline__ void wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicOr(err, kErrWaitDrain);
            return;
        }
    }
}

template <int HDP, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) fmha_fwd_kernel(const __grid_constant__ FmhaParams p) {
    using S = FmhaShape<HDP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sQ = smem;
    uint8_t *sK = sQ + 2 * S::TILE_BYTES;
    uint8_t *sV = sK + S::STAGES * S::TILE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sV + S::STAGES * S::TILE_BYTES);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1;
    uint64_t *k_empty = k_full + S::STAGES;
    uint64_t *v_full = k_empty + S::STAGES;
    uint64_t *v_empty = v_full + S::STAGES;
    uint64_t *s_full = v_empty + S::STAGES; // [2]
    uint64_t *p_full = s_full + 2;          // [2]
    uint64_t *o_done = p_full + 2;
    uint64_t *drain = o_done + 1;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, b = blockIdx.z;
    const int L = p.L;
    const int q0 = blockIdx.x * 256;
    int valid = p.lengths ? p.lengths[b] : p.valid;
    valid = valid < L ? valid : L;
    if (valid < 0)
        valid = 0;
    if (q0 >= L || (p.skip_padded_q && q0 >= valid))
        return; // uniform for the whole CTA, before any barrier or TMEM use

    // Keys this CTA needs: the largest limit(t) over its rows (limit grows with t).
    const int last_row = min(q0 + 255, L - 1);
    int kv_limit = valid;
    if (p.block > 0)
        kv_limit = min(kv_limit, (last_row / p.block + 1) * p.block);
    const int T = (kv_limit + 127) / 128;
    int *err = p.err;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(&p_full[0], 128);
        mbar_init(&p_full[1], 128);
        mbar_init(o_done, 1);
        mbar_init(drain, 1);
        fence_mbarrier_init();
    }
    if (warp == 9) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 8) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && T > 0) {
            tma_prefetch_desc(&p.tq0);
            tma_prefetch_desc(&p.tk0);
            tma_prefetch_desc(&p.tv0);
            mbar_arrive_expect_tx(q_full, 2 * S::TILE_BYTES);
            load_tile<HDP>(sQ, &p.tq0, &p.tq1, q_full, q0, h, b);
            load_tile<HDP>(sQ + S::TILE_BYTES, &p.tq0, &p.tq1, q_full, q0 + 128, h, b);
            int issued_k = 0, issued_v = 0;
            for (int j = 0; j < T; ++j) {
                const int st = j % S::STAGES;
                const uint32_t ph = (j / S::STAGES) & 1;
                if (!mbar_wait(&k_empty[st], ph ^ 1, err, kErrWaitEmpty))
                    break;
                mbar_arrive_expect_tx(&k_full[st], S::TILE_BYTES);
                load_tile<HDP>(sK + st * S::TILE_BYTES, &p.tk0, &p.tk1, &k_full[st], j * 128, h, b);
                issued_k = j + 1;
                if (!mbar_wait(&v_empty[st], ph ^ 1, err, kErrWaitEmpty))
                    break;
                mbar_arrive_expect_tx(&v_full[st], S::TILE_BYTES);
                load_tile<HDP>(sV + st * S::TILE_BYTES, &p.tv0, &p.tv1, &v_full[st], j * 128, h, b);
                issued_v = j + 1;
            }
            // Every issued copy must land before the CTA may exit.
            wait_drain(q_full, 0, err);
            for (int j = issued_k - S::STAGES < 0 ? 0 : issued_k - S::STAGES; j < issued_k; ++j)
                wait_drain(&k_full[j % S::STAGES], (j / S::STAGES) & 1, err);
            for (int j = issued_v - S::STAGES < 0 ? 0 : issued_v - S::STAGES; j < issued_v; ++j)
                wait_drain(&v_full[j % S::STAGES], (j / S::STAGES) & 1, err);
        }
        __syncwarp();
    } else if (warp == 9) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0 && T > 0) {
            constexpr uint32_t idesc_qk = make_idesc_f16(128, 128, BF16, false);
            constexpr uint32_t idesc_pv0 = make_idesc_f16(128, S::C0, BF16, true);
            constexpr uint32_t idesc_pv1 = make_idesc_f16(128, S::C1 > 0 ? S::C1 : 16, BF16, true);
            constexpr uint32_t lay0 = layout_for_row_bytes(S::ROW0);
            constexpr uint32_t lay1 = layout_for_row_bytes(S::ROW1 > 0 ? S::ROW1 : 32);
            const uint32_t sq = smem_u32(sQ), sk = smem_u32(sK), sv = smem_u32(sV);
            auto qk = [&](int i, int st) {
                const uint32_t d = tmem + i * 128;
#pragma unroll
                for (int kk = 0; kk < S::KSTEPS; ++kk) {
                    const int e = kk * 16;
                    const bool c1 = e >= S::C0;
                    const uint32_t rowb = c1 ? S::ROW1 : S::ROW0;
                    const uint32_t off = (c1 ? S::CH0_BYTES : 0) + (e - (c1 ? S::C0 : 0)) * 2;
                    const uint64_t ad = make_smem_desc(sq + i * S::TILE_BYTES + off, 16, 8 * rowb,
                                                       c1 ? lay1 : lay0);
                    const uint64_t bd = make_smem_desc(sk + st * S::TILE_BYTES + off, 16, 8 * rowb,
                                                       c1 ? lay1 : lay0);
                    umma_ss(d, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
                }
            };
            auto pv = [&](int i, int st, bool accumulate) {
                const uint32_t d = tmem + 256 + i * 128;
                const uint32_t a = tmem + i * 128;
                const uint32_t vb = sv + st * S::TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t acc = (accumulate || kk > 0) ? 1u : 0u;
                    const uint64_t b0 = make_smem_desc(vb + kk * 16 * S::ROW0, S::CH0_BYTES,
                                                       8 * S::ROW0, lay0);
                    umma_ts(d, a + kk * 8, b0, idesc_pv0, acc);
                    if constexpr (S::C1 > 0) {
                        const uint64_t b1 = make_smem_desc(vb + S::CH0_BYTES + kk * 16 * S::ROW1,
                                                           S::TILE_BYTES, 8 * S::ROW1, lay1);
                        umma_ts(d + S::C0, a + kk * 8, b1, idesc_pv1, acc);
                    }
                }
            };
            bool ok = mbar_wait(q_full, 0, err, kErrWaitQ) && mbar_wait(&k_full[0], 0, err, kErrWaitK);
            if (ok) {
                tc_fence_after();
                qk(0, 0);
                tc_commit(&s_full[0]);
                qk(1, 0);
                tc_commit(&s_full[1]);
                tc_commit(&k_empty[0]);
            }
            for (int j = 0; ok && j < T; ++j) {
                const int st = j % S::STAGES;
                const uint32_t ph = (j / S::STAGES) & 1;
                const int j1 = j + 1, st1 = j1 % S::STAGES;
                const uint32_t ph1 = (j1 / S::STAGES) & 1;
                if (!(ok = mbar_wait(&v_full[st], ph, err, kErrWaitV)))
                    break;
                if (!(ok = mbar_wait(&p_full[0], j & 1, err, kErrWaitP)))
                    break;
                tc_fence_after();
                pv(0, st, j > 0);
                if (j1 < T) {
                    if (!(ok = mbar_wait(&k_full[st1], ph1, err, kErrWaitK)))
                        break;
                    tc_fence_after();
                    qk(0, st1);
                    tc_commit(&s_full[0]);
                }
                if (!(ok = mbar_wait(&p_full[1], j & 1, err, kErrWaitP)))
                    break;
                tc_fence_after();
                pv(1, st, j > 0);
                tc_commit(&v_empty[st]);
                if (j1 < T) {
                    qk(1, st1);
                    tc_commit(&s_full[1]);
                    tc_commit(&k_empty[st1]);
                }
            }
            tc_commit(o_done);
            tc_commit(drain);
            wait_drain(drain, 0, err);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------- softmax warpgroups
        const int i = warp >> 2;                    // query tile
        const int r = ((warp & 3) << 5) + lane;     // TMEM lane == row in tile
        const int t = q0 + i * 128 + r;             // query token
        int limit = valid;
        if (p.block > 0)
            limit = min(limit, (t / p.block + 1) * p.block);
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) << 5) << 16;
        const uint32_t tS = tmem + lane_base + i * 128;
        const uint32_t tO = tmem + lane_base + 256 + i * 128;
        const float sl2 = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < T; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[i], j & 1, err, kErrWaitS));
            if (!ok)
                break;
            tc_fence_after();
            uint32_t sraw[128];
            tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&sraw[0]));
            tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sraw[32]));
            tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&sraw[64]));
            tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&sraw[96]));
            tmem_wait_ld();
            float *s = reinterpret_cast<float *>(sraw);
            const int kv0 = j * 128;
            if (kv0 + 128 > limit) {
#pragma unroll
                for (int c = 0; c < 128; ++c)
                    if (kv0 + c >= limit)
                        s[c] = -INFINITY;
            }
            float mt = s[0];
#pragma unroll
            for (int c = 1; c < 128; ++c)
                mt = fmaxf(mt, s[c]);
            const float mnew = fmaxf(m, mt * sl2);
            // Lazy rescale: a row keeps its stale max while P stays below 2^8.
            const bool grow = mnew > m + 8.0f;
            const float alpha = (grow && j > 0) ? ex2_approx(m - mnew) : 1.f;
            if (grow) {
                l *= alpha;
                m = mnew;
            }
            // tcgen05.ld/st are warp-collective: rescale the warp's O rows
            // together (alpha == 1 for rows whose max did not grow).
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
                for (int c = 0; c < HDP; c += 16) {
                    uint32_t o[16];
                    tmem_ld16(tO + c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tmem_st16(tO + c, o);
                }
            }
            const float neg_m = -m;
            float sum = 0.f;
            uint32_t pk[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float p0 = ex2_approx(fmaf(s[2 * c], sl2, neg_m));
                const float p1 = ex2_approx(fmaf(s[2 * c + 1], sl2, neg_m));
                sum += p0 + p1;
                pk[c] = pack2(p0, p1, BF16);
            }
            l += sum;
            __syncwarp();
            tmem_st32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
            tmem_st32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[i]);
        }
        if (ok && T > 0)
            ok = __all_sync(0xffffffffu, mbar_wait(o_done, 0, err, kErrWaitO));
        if (ok) {
            tc_fence_after();
            const float inv = (T > 0 && l > 0.f) ? 1.f / l : 0.f;
            const bool store = t < L;
            const long long base = b * p.o_sb + h * p.o_sh + static_cast<long long>(t) * p.o_st;
#pragma unroll
            for (int c = 0; c < HDP; c += 16) {
                uint32_t o[16];
                if (T > 0) {
                    tmem_ld16(tO + c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        o[e] = 0u;
                }
                if (!store)
                    continue;
                float v[16];
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    v[e] = __uint_as_float(o[e]) * inv;
                if (p.out_dtype == kOutF32) {
                    float *out = static_cast<float *>(p.out) + base;
                    if (p.out_vec && c + 16 <= p.hd) {
#pragma unroll
                        for (int e = 0; e < 16; e += 4)
                            *reinterpret_cast<float4 *>(out + c + e) =
                                make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                    } else {
                        for (int e = 0; e < 16 && c + e < p.hd; ++e)
                            out[c + e] = v[e];
                    }
                } else {
                    const bool bf = p.out_dtype == kOutBF16;
                    uint16_t *out = static_cast<uint16_t *>(p.out) + base;
                    if (p.out_vec && c + 16 <= p.hd) {
                        uint4 w0, w1;
                        w0.x = pack2(v[0], v[1], bf);
                        w0.y = pack2(v[2], v[3], bf);
                        w0.z = pack2(v[4], v[5], bf);
                        w0.w = pack2(v[6], v[7], bf);
                        w1.x = pack2(v[8], v[9], bf);
                        w1.y = pack2(v[10], v[11], bf);
                        w1.z = pack2(v[12], v[13], bf);
                        w1.w = pack2(v[14], v[15], bf);
                        *reinterpret_cast<uint4 *>(out + c) = w0;
                        *reinterpret_cast<uint4 *>(out + c + 8) = w1;
                    } else if (p.out_vec && c + 8 <= p.hd) {
                        uint4 w0;
                        w0.x = pack2(v[0], v[1], bf);
                        w0.y = pack2(v[2], v[3], bf);
                        w0.z = pack2(v[4], v[5], bf);
                        w0.w = pack2(v[6], v[7], bf);
                        *reinterpret_cast<uint4 *>(out + c) = w0;
                    } else {
                        for (int e = 0; e < 16 && c + e < p.hd; ++e) {
                            const uint32_t w = pack2(v[e], 0.f, bf);
                            out[c + e] = static_cast<uint16_t>(w & 0xffffu);
                        }
                    }
                }
            }
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 9)
        tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host side
// Builds a 4-D (d, token, head, batch) tiled map with a box of
// box_w x box_rows x 1 x 1 elements.
int make_map(CUtensorMap *map, const void *base, bool bf16, const TensorView &v, int box_w,
             int box_rows) {
    const uint64_t dims[4] = {static_cast<uint64_t>(v.d), static_cast<uint64_t>(v.tokens),
                              static_cast<uint64_t>(v.heads), static_cast<uint64_t>(v.batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(v.s_token) * 2,
                                 static_cast<uint64_t>(v.s_head) * 2,
                                 static_cast<uint64_t>(v.s_batch) * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(box_w), static_cast<uint32_t>(box_rows), 1, 1};
    return encode_tiled(map, base, bf16, 4, dims, strides, box);
}

bool tma_view_ok(const void *base, const TensorView &v) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    // 16-byte aligned base and 16-byte multiple strides (2-byte elements).
    return (a % 16) == 0 && (v.s_token % 8) == 0 && (v.s_head % 8) == 0 &&
           (v.batch == 1 || (v.s_batch % 8) == 0) && v.d >= 1;
}

int padded_head_dim(int hd) {
    if (hd <= 16)
        return 16;
    if (hd <= 32)
        return 32;
    if (hd <= 64)
        return 64;
    if (hd <= 80)
        return 80;
    if (hd <= 96)
        return 96;
    if (hd <= 128)
        return 128;
    return -1;
}

template <int HDP, bool BF16> int launch_typed(FmhaParams &p, int grid_x, cudaStream_t stream) {
    using S = FmhaShape<HDP>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(fmha_fwd_kernel<HDP, BF16>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
    });
    if (attr != cudaSuccess)
        return static_cast<int>(attr);
    dim3 grid(grid_x, p.heads, p.batch);
    fmha_fwd_kernel<HDP, BF16><<<grid, kThreads, S::SMEM_BYTES, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

template <int HDP> int launch_hdp(FmhaParams &p, bool bf16, int grid_x, cudaStream_t stream) {
    return bf16 ? launch_typed<HDP, true>(p, grid_x, stream)
                : launch_typed<HDP, false>(p, grid_x, stream);
}

int fmha_launch(const FmhaArgs &a, cudaStream_t stream) {
    const int hdp = padded_head_dim(a.q.d);
    if (hdp < 0)
        return -2;
    FmhaParams p{};
    const int w0 = hdp < 64 ? hdp : 64, w1 = hdp - w0;
    int rc = 0;
    if ((rc = make_map(&p.tq0, a.q_ptr, a.bf16, a.q, w0, 128)) ||
        (rc = make_map(&p.tk0, a.k_ptr, a.bf16, a.k, w0, 128)) ||
        (rc = make_map(&p.tv0, a.v_ptr, a.bf16, a.v, w0, 128)))
        return rc;
    if (w1 > 0) {
        if ((rc = make_map(&p.tq1, a.q_ptr, a.bf16, a.q, w1, 128)) ||
            (rc = make_map(&p.tk1, a.k_ptr, a.bf16, a.k, w1, 128)) ||
            (rc = make_map(&p.tv1, a.v_ptr, a.bf16, a.v, w1, 128)))
            return rc;
    }
    p.out = a.out;
    p.o_sb = a.o_sb;
    p.o_sh = a.o_sh;
    p.o_st = a.o_st;
    p.lengths = a.lengths;
    p.batch = a.q.batch;
    p.heads = a.q.heads;
    p.L = a.q.tokens;
    p.hd = a.out_d > 0 ? a.out_d : a.q.d;
    p.valid = a.valid;
    p.block = a.block;
    p.skip_padded_q = a.skip_padded_q;
    p.out_dtype = a.out_dtype;
    const int esize = a.out_dtype == kOutF32 ? 4 : 2;
    const uintptr_t oa = reinterpret_cast<uintptr_t>(a.out);
    const int vec_elems = 16 / esize;
    p.out_vec = (oa % 16 == 0) && (a.o_st % vec_elems == 0) && (a.o_sh % vec_elems == 0) &&
                (p.batch == 1 || a.o_sb % vec_elems == 0) && (p.hd % 8 == 0);
    const double scale = a.scale > 0 ? a.scale : 1.0 / std::sqrt(static_cast<double>(p.hd));
    p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
    p.err = a.err;
    const int grid_x = (p.L + 255) / 256;
    switch (hdp) {
    case 16:
        return launch_hdp<16>(p, a.bf16, grid_x, stream);
    case 32:
        return launch_hdp<32>(p, a.bf16, grid_x, stream);
    case 64:
        return launch_hdp<64>(p, a.bf16, grid_x, stream);
    case 80:
        return launch_hdp<80>(p, a.bf16, grid_x, stream);
    case 96:
        return launch_hdp<96>(p, a.bf16, grid_x, stream);
    case 128:
        return launch_hdp<128>(p, a.bf16, grid_x, stream);
    }
    return -2;
}

} // namespace omni_b200
