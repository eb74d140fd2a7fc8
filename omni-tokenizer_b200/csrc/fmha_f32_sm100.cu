// fmha_f32_sm100.cu -- fp32 encoder self-attention for B200 (sm_100a).
//
// The reference's production audio profile runs attention in fp32: the Sm80
// mem-efficient kernel with 3xTF32 tensor-core products (src/audio_attention.cu
// :10-38, dispatched from src/cuda.cu:836-842), held by its own GPU test to
// 3e-6 per element against a float64 scalar attention
// (tests/native_cuda_attention.cpp:88).  Semantics are those of
// src/cpu.cpp:122-172: O = softmax(scale Q K^T + mask) V per head, scale =
// hd^-1/2, key limit limit(t) = min(L, valid[, (t/block + 1) block]).
//
// Split-precision products on the tcgen05 tensor cores.  An fp32 operand x is
// written as hi + lo with a tf32 hi and a tf32 lo (10 explicit mantissa bits
// each), and a b = ah bh + ah bl + al bh + al bl, of which this kernel issues
// the first three as MMAs of kind::tf32 accumulating in fp32 in TMEM.
//   * Q (split in registers once per item, stored to TMEM): hi = x rounded
//     to the nearest tf32 value, lo = x - hi (exact) rounded to the nearest
//     tf32 value, so |lo| <= 2^-11 |x| with a random sign.
//   * K, V and P: the tensor cores read an fp32 operand by dropping its low
//     13 bits (truncation, measured on B200), so the fp32 value itself serves
//     as hi = trunc(x), and only lo = x - trunc(x) (exact, |lo| < 2^-10 |x|)
//     rounded to the nearest tf32 value is written beside it: K and V tiles
//     are read once in shared memory and never rewritten, P is stored to TMEM
//     as computed plus its lo part.
// A product then drops al bl (at most 2^-21 |a b| in QK, where Q's lo has a
// random sign; at most 2^-20 |a b| in PV) and the rounding of the lo parts
// (at most 2^-21 relative each): a relative error of a few 1e-7 per product.
//
// One CTA owns 128 query rows of one (batch, head) per work item and streams
// the keys in NK-key tiles (persistent grid, one CTA per SM):
//   warp 8      TMA producer: raw fp32 K_j / V_j into a ring of STAGES slots;
//   warps 4-7   converters: write the lo part of each raw K / V tile beside
//               it (identical swizzled layouts, so the split is
//               position-independent); per item they
//               also load the 128 query rows (thread = row = TMEM lane),
//               split them and store Q hi / lo into TMEM;
//   warp 9      TMEM owner and tcgen05.mma issuer:
//                 S = Q K^T        (Q from TMEM x K from smem, 3 MMAs per
//                                   8-wide K step),
//                 O += P V         (P from TMEM x V from smem, V MN-major as
//                                   loaded, 3 MMAs per 8-key step);
//               issue order QK(g+1) before PV(g), so the next scores are
//               computed while the softmax works on the current ones;
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r), its running
//               max and sum; it masks, exponentiates (MUFU ex2), splits P into
//               hi/lo and stores both to TMEM, rescales O in TMEM when its max
//               grew by more than 2^8 (lazy rescale), and finally normalises
//               and stores its row of O.
// TMEM (512 columns at head_dim 64): Q hi | Q lo | S | P_0 hi, lo | P_1 hi, lo
// | O.  Keeping Q in TMEM leaves shared memory to the K/V ring (3 stages of
// 64 keys at head_dim 64), which hides the latency of a tile's load and split.
// P is double-buffered by the parity of the global step g (single-buffered
// where TMEM is short, head_dim 128); the barriers of each buffer are separate
// so that every parity wait refers to the barrier's most recent phase.
#include "fmha.h"
#include "sm100.cuh"
#include "tma.h"

#include <cmath>

namespace omni_b200 {
namespace f32attn {

template <int HDP, int NK> struct Shape {
    static constexpr int CH = HDP / 32;             // 128-byte column chunks (32 fp32)
    static constexpr int KV_CHUNK = NK * 128;       // bytes of one K or V chunk (NK rows)
    static constexpr int KV_BYTES = CH * KV_CHUNK;  // one of K hi / K lo / V hi / V lo
    static constexpr int STAGE_BYTES = 4 * KV_BYTES;
    static constexpr int BAR_BYTES = 1024;
    static constexpr int BUDGET = 227 * 1024 - BAR_BYTES - 1024;
    static constexpr int STAGES_RAW = BUDGET / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 6 ? 6 : STAGES_RAW;
    static constexpr int SMEM_RAW = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    // At least 120 KB so that one CTA (which allocates all 512 TMEM columns)
    // occupies an SM by itself.
    static constexpr int SMEM_BYTES = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
    // TMEM columns: Q hi at kQ, Q lo at kQ + HDP, S at kS, P_b hi at kP + 2 NK b
    // (lo at + NK), O at kO.
    static constexpr int PBUF = 2 * HDP + NK + 4 * NK + HDP <= 512 ? 2 : 1;
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kS = 2 * HDP;
    static constexpr uint32_t kP = 2 * HDP + NK;
    static constexpr uint32_t kO = kP + 2 * NK * PBUF;
    static_assert(HDP % 32 == 0 && HDP <= 128, "head dim padding must be 32, 64, 96 or 128");
    static_assert(NK % 32 == 0 && NK >= 32 && NK <= 128, "key tile must be 32, 64, 96 or 128");
    static_assert(kO + HDP <= 512, "TMEM budget");
    static_assert(STAGES >= 2, "shared memory budget");
};

constexpr int kSoftWarps = 4;
constexpr int kConvWarp0 = 4;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;

struct Item {
    int b, h, q0, valid, T; // T = KV tiles the item needs (0: output zeros)
    bool skip;              // rows past the end / padded-query skip
};

template <int NK> __device__ __forceinline__ Item decode_item(const FmhaF32Params &p, int u) {
    const int qblocks = (p.L + 127) / 128;
    Item it;
    const int bh = u / qblocks;
    it.q0 = (u - bh * qblocks) * 128;
    it.b = bh / p.heads;
    it.h = bh - it.b * p.heads;
    int valid = p.lengths ? p.lengths[it.b] : p.valid;
    valid = valid < p.L ? valid : p.L;
    it.valid = valid < 0 ? 0 : valid;
    it.skip = it.q0 >= p.L || (p.skip_padded_q && it.q0 >= it.valid);
    const int last_row = min(it.q0 + 127, p.L - 1);
    int kv_limit = it.valid;
    if (p.block > 0)
        kv_limit = min(kv_limit, (last_row / p.block + 1) * p.block);
    it.T = (kv_limit + NK - 1) / NK;
    return it;
}

// The first item at or after u (in steps of the grid) with KV work.
template <int NK> __device__ __forceinline__ int next_work_item(const FmhaF32Params &p, int u, int items) {
    for (; u < items; u += gridDim.x) {
        const Item it = decode_item<NK>(p, u);
        if (!it.skip && it.T > 0)
            break;
    }
    return u;
}

// Round to the nearest tf32 value (ties away from zero): add half of the
// dropped 13-bit field to the magnitude, then clear it.
__device__ __forceinline__ uint32_t tf32_round_bits(uint32_t x) { return (x + 0x1000u) & 0xFFFFE000u; }

// x = hi + lo with hi the nearest tf32 value (Q and P, stored to TMEM).
__device__ __forceinline__ void split_tf32(float x, float &hi, float &lo) {
    hi = __uint_as_float(tf32_round_bits(__float_as_uint(x)));
    lo = __uint_as_float(tf32_round_bits(__float_as_uint(x - hi))); // x - hi is exact
}

// The part of x that the tensor cores drop when they read x as tf32
// (truncation), rounded to the nearest tf32 value.
__device__ __forceinline__ float tf32_lo_of_trunc(float x) {
    const float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    return __uint_as_float(tf32_round_bits(__float_as_uint(x - hi))); // x - hi is exact
}

// Writes the lo parts of a raw fp32 tile of `bytes` bytes at `raw` to the same
// offsets under `lo` (identical swizzled layouts); the raw tile stays as it is
// and serves as the hi operand.  The 128 converter threads stride over its
// 16-byte chunks.
__device__ __forceinline__ void split_tile(const uint8_t *raw, uint8_t *lo, int bytes, int tid) {
    const float4 *r4 = reinterpret_cast<const float4 *>(raw);
    float4 *l4 = reinterpret_cast<float4 *>(lo);
#pragma unroll 4
    for (int i = tid; i < bytes / 16; i += 128) {
        const float4 v = r4[i];
        l4[i] = make_float4(tf32_lo_of_trunc(v.x), tf32_lo_of_trunc(v.y), tf32_lo_of_trunc(v.z),
                            tf32_lo_of_trunc(v.w));
    }
}

__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0)
        mbar_arrive(bar);
}

// Waits bounded by time only (does not give up early on other threads'
// errors): used so that no TMA write or MMA is in flight when the CTA releases
// its shared memory and TMEM.
__device__ __forceinline__ void wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t start = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - start > kWaitLimitNs) {
            atomicOr(err, kErrWaitDrain);
            return;
        }
    }
}

__device__ __forceinline__ bool wait_all(uint64_t *bar, uint32_t parity, int *err, int code) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
}

__device__ __forceinline__ uint32_t pack_out2(float lo, float hi, int out_dtype) {
    if (out_dtype == kOutBF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    }
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

template <int HDP, int NK>
__global__ void __launch_bounds__(kThreads, 1) fmha_f32_kernel(const __grid_constant__ FmhaF32Params p) {
    using S = Shape<HDP, NK>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sKV = smem;                 // [STAGES] x (K hi, K lo, V hi, V lo)
    uint64_t *bars = reinterpret_cast<uint64_t *>(sKV + S::STAGES * S::STAGE_BYTES);
    uint64_t *q_full = bars;             // Q hi / lo stored in TMEM (4 converter warps)
    uint64_t *q_free = bars + 1;         // every QK of the item done (commit)
    uint64_t *k_full = bars + 2;         // [STAGES] K tile landed
    uint64_t *k_ready = k_full + 6;      // [STAGES] K tile split
    uint64_t *k_empty = k_ready + 6;     // [STAGES] QK done with the slot (commit)
    uint64_t *v_full = k_empty + 6;      // [STAGES]
    uint64_t *v_ready = v_full + 6;      // [STAGES]
    uint64_t *v_empty = v_ready + 6;     // [STAGES]
    uint64_t *s_full = v_empty + 6;      // S computed (commit)
    uint64_t *s_free = s_full + 1;       // softmax read S (4 warps)
    uint64_t *p_full = s_free + 1;       // [PBUF] P_b stored (4 warps)
    uint64_t *pv_done = p_full + 2;      // [PBUF] O += P_b V complete (commit)
    uint64_t *drain = pv_done + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
    auto k_hi = [&](int st) { return sKV + st * S::STAGE_BYTES; };
    auto k_lo = [&](int st) { return sKV + st * S::STAGE_BYTES + S::KV_BYTES; };
    auto v_hi = [&](int st) { return sKV + st * S::STAGE_BYTES + 2 * S::KV_BYTES; };
    auto v_lo = [&](int st) { return sKV + st * S::STAGE_BYTES + 3 * S::KV_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = p.batch * p.heads * ((p.L + 127) / 128);
    int *err = p.err;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 4);
        mbar_init(q_free, 1);
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_ready[s], 4);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_ready[s], 4);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kSoftWarps);
        for (int b = 0; b < S::PBUF; ++b) {
            mbar_init(&p_full[b], kSoftWarps);
            mbar_init(&pv_done[b], 1);
        }
        mbar_init(drain, 1);
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (tmem != 0) {
        // The MMA issuer, softmax and converters address TMEM from column 0 of lane 0.
        if (threadIdx.x == 0)
            atomicOr(err, kErrWaitDrain);
        __syncthreads();
        if (warp == kMmaWarp)
            tmem_dealloc(tmem, 512);
        return;
    }
    // O += P_gp V of global step gp is complete: pv_done[gp % PBUF] has
    // completed once for every earlier step of the same buffer.
    auto wait_pv = [&](int gp) {
        return wait_all(&pv_done[gp % S::PBUF], (gp / S::PBUF) & 1, err, kErrWaitO);
    };

    if (warp == kProducerWarp) {
        // ------------------------------------------------------ TMA producer
        if (elect_one()) {
            tma_prefetch_desc(&p.tk);
            tma_prefetch_desc(&p.tv);
        }
        int nk = 0, nv = 0; // K loads, V loads issued
        bool ok = true;
        for (int u = next_work_item<NK>(p, blockIdx.x, items); ok && u < items;
             u = next_work_item<NK>(p, u + gridDim.x, items)) {
            const Item it = decode_item<NK>(p, u);
            for (int j = 0; j < it.T; ++j) {
                const int st = nk % S::STAGES;
                const uint32_t ph = (nk / S::STAGES) & 1;
                if (!(ok = wait_all(&k_empty[st], ph ^ 1, err, kErrWaitEmpty)))
                    break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&k_full[st], S::KV_BYTES);
#pragma unroll
                    for (int c = 0; c < S::CH; ++c)
                        tma_load_4d(k_hi(st) + c * S::KV_CHUNK, &p.tk, &k_full[st], 32 * c, j * NK, it.h, it.b);
                }
                __syncwarp();
                ++nk;
                if (!(ok = wait_all(&v_empty[st], ph ^ 1, err, kErrWaitEmpty)))
                    break;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&v_full[st], S::KV_BYTES);
#pragma unroll
                    for (int c = 0; c < S::CH; ++c)
                        tma_load_4d(v_hi(st) + c * S::KV_CHUNK, &p.tv, &v_full[st], 32 * c, j * NK, it.h, it.b);
                }
                __syncwarp();
                ++nv;
            }
        }
        // Every issued copy must land before the CTA may exit.
        for (int m = nk - S::STAGES < 0 ? 0 : nk - S::STAGES; m < nk; ++m)
            wait_drain(&k_full[m % S::STAGES], (m / S::STAGES) & 1, err);
        for (int m = nv - S::STAGES < 0 ? 0 : nv - S::STAGES; m < nv; ++m)
            wait_drain(&v_full[m % S::STAGES], (m / S::STAGES) & 1, err);
    } else if (warp >= kConvWarp0 && warp < kConvWarp0 + 4) {
        // -------------------------------------------------------- converters
        const int tid = threadIdx.x - kConvWarp0 * 32;  // = query row in the tile = TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        int nq = 0, n = 0;
        bool ok = true;
        auto split_k = [&](int g) {
            const int st = g % S::STAGES;
            if (!wait_all(&k_full[st], (g / S::STAGES) & 1, err, kErrWaitK))
                return false;
            split_tile(k_hi(st), k_lo(st), S::KV_BYTES, tid);
            fence_proxy_async_smem();
            warp_arrive(&k_ready[st]);
            return true;
        };
        auto split_v = [&](int g) {
            const int st = g % S::STAGES;
            if (!wait_all(&v_full[st], (g / S::STAGES) & 1, err, kErrWaitV))
                return false;
            split_tile(v_hi(st), v_lo(st), S::KV_BYTES, tid);
            fence_proxy_async_smem();
            warp_arrive(&v_ready[st]);
            return true;
        };
        for (int u = next_work_item<NK>(p, blockIdx.x, items); ok && u < items;
             u = next_work_item<NK>(p, u + gridDim.x, items)) {
            const Item it = decode_item<NK>(p, u);
            // This thread's query row, loaded now so that the global-memory
            // latency overlaps the split of the item's first K tile.
            float qraw[HDP];
            const int t = it.q0 + tid;
            const float *qrow = p.q + it.b * p.q_sb + it.h * p.q_sh + static_cast<long long>(t) * p.q_st;
            if (t < p.L && p.q_vec) {
#pragma unroll
                for (int e = 0; e < HDP; e += 4) {
                    const float4 v = e < p.q_d ? *reinterpret_cast<const float4 *>(qrow + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                    qraw[e] = v.x;
                    qraw[e + 1] = v.y;
                    qraw[e + 2] = v.z;
                    qraw[e + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int e = 0; e < HDP; ++e)
                    qraw[e] = (t < p.L && e < p.q_d) ? qrow[e] : 0.f;
            }
            if (!(ok = split_k(n)))
                break;
            // Q hi / lo into TMEM once every QK of the previous item is done.
            if (nq > 0 && !(ok = wait_all(q_free, (nq - 1) & 1, err, kErrWaitQ)))
                break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < HDP / 16; ++c) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float h, lw;
                    split_tf32(qraw[16 * c + e], h, lw);
                    hi[e] = __float_as_uint(h);
                    lo[e] = __float_as_uint(lw);
                }
                tmem_st16(tmem + lane_base + S::kQ + 16 * c, hi);
                tmem_st16(tmem + lane_base + S::kQ + HDP + 16 * c, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            warp_arrive(q_full);
            ++nq;
            if (!(ok = split_v(n)))
                break;
            ++n;
            for (int j = 1; ok && j < it.T; ++j, ++n)
                ok = split_k(n) && split_v(n);
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------- MMA issuer
        // The whole warp runs the loop with warp-uniform values; one elected
        // lane issues each tcgen05.mma / tcgen05.commit.
        constexpr uint32_t idesc_qk = make_idesc_tf32(128, NK);
        constexpr uint32_t idesc_pv = make_idesc_tf32(128, HDP, true);
        const uint32_t leader = elect_one() ? 1u : 0u;
        auto commit = [&](uint64_t *bar) { tc_commit_if(leader, bar); };
        // Descriptors of stage 0; a stage is STAGE_BYTES further on, and the
        // start-address field (bits 0-13, address >> 4) takes the offset by
        // plain addition (every address stays below 256 KB).  All per-MMA
        // offsets below are compile-time constants, so the issue path is one
        // 64-bit add and one tcgen05.mma per MMA.
        const uint64_t kh0 = make_smem_desc(smem_u32(k_hi(0)), 16, 1024, kLayoutSW128);
        const uint64_t kl0 = make_smem_desc(smem_u32(k_lo(0)), 16, 1024, kLayoutSW128);
        const uint64_t vh0 = make_smem_desc(smem_u32(v_hi(0)), S::KV_CHUNK, 512, kLayoutSW128A32);
        const uint64_t vl0 = make_smem_desc(smem_u32(v_lo(0)), S::KV_CHUNK, 512, kLayoutSW128A32);
        auto stage_off = [](int st) { return static_cast<uint64_t>((st * S::STAGE_BYTES) >> 4); };
        // S = Q K_st^T: Q hi / lo from TMEM (one column per element), K
        // K-major in smem; per 8-wide K step hi*lo, lo*hi, then hi*hi.
        auto qk = [&](int st) {
            const uint64_t bh = kh0 + stage_off(st), bl = kl0 + stage_off(st);
#pragma unroll
            for (int kk = 0; kk < HDP / 8; ++kk) {
                // 128-byte chunk kk / 4, 32-byte step kk % 4 inside it.
                const uint64_t off = static_cast<uint64_t>(((kk >> 2) * S::KV_CHUNK) >> 4) + 2 * (kk & 3);
                umma_ts_tf32_if(leader, S::kS, S::kQ + 8 * kk, bl + off, idesc_qk, kk > 0 ? 1u : 0u);
                umma_ts_tf32_if(leader, S::kS, S::kQ + HDP + 8 * kk, bh + off, idesc_qk, 1u);
                umma_ts_tf32_if(leader, S::kS, S::kQ + 8 * kk, bh + off, idesc_qk, 1u);
            }
        };
        // O (+)= P_b V_st: P hi / lo from TMEM, V MN-major (rows = keys) in the
        // 128-byte swizzle of 32-byte atoms (the tf32 MN-major layout): 32-column
        // chunks KV_CHUNK bytes apart (LBO), 4-row swizzle groups 512 bytes apart
        // (SBO); per 8-key step the descriptor moves 8 rows = 1 KB.
        auto pv = [&](int b, int st, bool accumulate) {
            const uint32_t ph = S::kP + 2 * NK * b, pl = ph + NK;
            const uint64_t vh = vh0 + stage_off(st), vl = vl0 + stage_off(st);
#pragma unroll
            for (int kk = 0; kk < NK / 8; ++kk) {
                const uint64_t off = static_cast<uint64_t>((kk * 8 * 128) >> 4);
                umma_ts_tf32_if(leader, S::kO, ph + 8 * kk, vl + off, idesc_pv, (accumulate || kk > 0) ? 1u : 0u);
                umma_ts_tf32_if(leader, S::kO, pl + 8 * kk, vh + off, idesc_pv, 1u);
                umma_ts_tf32_if(leader, S::kO, ph + 8 * kk, vh + off, idesc_pv, 1u);
            }
        };
        int nq = 0, g = 0;
        bool ok = true;
        bool pending = false; // a PV of step g - 1 still to issue
        bool pending_acc = false;
        // Issues O += P(gp) V(gp).
        auto issue_pv = [&](int gp, bool acc) {
            const int b = gp % S::PBUF, st = gp % S::STAGES;
            if (!wait_all(&p_full[b], (gp / S::PBUF) & 1, err, kErrWaitP))
                return false;
            if (!wait_all(&v_ready[st], (gp / S::STAGES) & 1, err, kErrWaitV))
                return false;
            tc_fence_after();
            pv(b, st, acc);
            commit(&pv_done[b]);
            commit(&v_empty[st]);
            return true;
        };
        for (int u = next_work_item<NK>(p, blockIdx.x, items); ok && u < items;
             u = next_work_item<NK>(p, u + gridDim.x, items)) {
            const Item it = decode_item<NK>(p, u);
            if (!(ok = wait_all(q_full, nq & 1, err, kErrWaitQ)))
                break;
            ++nq;
            for (int j = 0; j < it.T; ++j, ++g) {
                const int st = g % S::STAGES;
                if (g >= 1 && !(ok = wait_all(s_free, (g - 1) & 1, err, kErrWaitS)))
                    break;
                if (!(ok = wait_all(&k_ready[st], (g / S::STAGES) & 1, err, kErrWaitK)))
                    break;
                tc_fence_after();
                qk(st);
                commit(s_full);
                commit(&k_empty[st]);
                if (j + 1 == it.T)
                    commit(q_free); // the item's Q is no longer read
                if (pending && !(ok = issue_pv(g - 1, pending_acc)))
                    break;
                pending = true;
                pending_acc = j > 0;
            }
        }
        if (ok && pending)
            ok = issue_pv(g - 1, pending_acc);
        commit(drain);
        wait_drain(drain, 0, err);
    } else if (warp < kSoftWarps) {
        // ---------------------------------------------------------- softmax
        const int r = warp * 32 + lane;                        // row in the tile = TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const float sl2 = p.scale_log2;
        constexpr int kOch = HDP / 16;
        int g = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < items; u += gridDim.x) {
            const Item it = decode_item<NK>(p, u);
            if (it.skip)
                continue;
            const int t = it.q0 + r;
            int limit = it.valid;
            if (p.block > 0)
                limit = min(limit, (t / p.block + 1) * p.block);
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.T; ++j, ++g) {
                const int b = g % S::PBUF;
                if (!(ok = wait_all(s_full, g & 1, err, kErrWaitS)))
                    break;
                tc_fence_after();
                uint32_t sraw[NK];
#pragma unroll
                for (int c = 0; c < NK / 32; ++c)
                    tmem_ld32(tmem + lane_base + S::kS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sraw[32 * c]));
                tmem_wait_ld();
                tc_fence_before();
                warp_arrive(s_free); // S may be overwritten by QK(g + 1)
                float *s = reinterpret_cast<float *>(sraw);
                const int kv0 = j * NK;
                if (kv0 + NK > limit) {
#pragma unroll
                    for (int c = 0; c < NK; ++c)
                        if (kv0 + c >= limit)
                            s[c] = -INFINITY;
                }
                // Row max: independent 3-input max chains of 16 scores.
                float mc[NK / 16];
#pragma unroll
                for (int q = 0; q < NK / 16; ++q) {
                    const float *sq = s + 16 * q;
                    float v = fmax3(sq[0], sq[1], sq[2]);
#pragma unroll
                    for (int e = 3; e < 15; e += 2)
                        v = fmax3(v, sq[e], sq[e + 1]);
                    mc[q] = fmaxf(v, sq[15]);
                }
#pragma unroll
                for (int w = NK / 32; w > 0; w >>= 1)
#pragma unroll
                    for (int q = 0; q < w; ++q)
                        mc[q] = fmaxf(mc[q], mc[q + w]);
                const float mnew = fmaxf(m, mc[0] * sl2);
                // Lazy rescale: a row keeps its stale max while P stays below 2^8.
                const bool grow = mnew > m + 8.0f;
                const float alpha = (grow && j > 0) ? ex2_approx(m - mnew) : 1.f;
                if (grow) {
                    l *= alpha;
                    m = mnew;
                }
                // P = 2^(s scale - m): packed fp32 FMA, MUFU ex2, packed sums; P
                // overwrites S in place.
                const float neg_m = -m;
                float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
                for (int c = 0; c < NK; c += 4) {
                    float x0, x1, x2, x3;
                    ffma2(x0, x1, s[c], s[c + 1], sl2, sl2, neg_m, neg_m);
                    ffma2(x2, x3, s[c + 2], s[c + 3], sl2, sl2, neg_m, neg_m);
                    x0 = ex2_approx(x0);
                    x1 = ex2_approx(x1);
                    x2 = ex2_approx(x2);
                    x3 = ex2_approx(x3);
                    fadd2(a0, a1, a0, a1, x0, x1);
                    fadd2(b0, b1, b0, b1, x2, x3);
                    s[c] = x0;
                    s[c + 1] = x1;
                    s[c + 2] = x2;
                    s[c + 3] = x3;
                }
                l += (a0 + a1) + (b0 + b1);
                // P_b is free once the previous PV that read it is complete.
                if (g >= S::PBUF && !(ok = wait_pv(g - S::PBUF)))
                    break;
                // O rescale: after O += P V of step g - 1, before that of step g.
                // tcgen05.ld/st are warp-collective, so the warp rescales together
                // (alpha == 1 for rows whose max did not grow).
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
                    if (!(ok = wait_pv(g - 1)))
                        break;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < kOch; ++c) {
                        uint32_t o[16];
                        tmem_ld16(tmem + lane_base + S::kO + 16 * c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st16(tmem + lane_base + S::kO + 16 * c, o);
                    }
                }
                tc_fence_after();
                // P hi = P as computed (the tensor cores truncate it to tf32), P lo =
                // the truncated part rounded to the nearest tf32 value.
#pragma unroll
                for (int c = 0; c < NK / 32; ++c) {
                    tmem_st32(tmem + lane_base + S::kP + 2 * NK * b + 32 * c,
                              *reinterpret_cast<uint32_t(*)[32]>(&sraw[32 * c]));
                    uint32_t lo[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        lo[e] = __float_as_uint(tf32_lo_of_trunc(s[32 * c + e]));
                    tmem_st32(tmem + lane_base + S::kP + 2 * NK * b + NK + 32 * c, lo);
                }
                tmem_wait_st();
                tc_fence_before();
                warp_arrive(&p_full[b]);
            }
            if (!ok)
                break;
            // Epilogue: wait for the item's last O += P V, normalise, store.
            uint32_t oraw[HDP];
            float *o = reinterpret_cast<float *>(oraw);
            if (it.T > 0) {
                if (!(ok = wait_pv(g - 1)))
                    break;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HDP / 32; ++c)
                    tmem_ld32(tmem + lane_base + S::kO + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&oraw[32 * c]));
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < HDP; ++e)
                    oraw[e] = 0u;
            }
            const float inv = (it.T > 0 && l > 0.f) ? 1.f / l : 0.f;
            if (t < p.L) {
                const long long base = it.b * p.o_sb + it.h * p.o_sh + static_cast<long long>(t) * p.o_st;
                if (p.out_dtype == kOutF32) {
                    float *out = static_cast<float *>(p.out) + base;
                    if (p.out_vec) {
#pragma unroll
                        for (int e = 0; e < HDP; e += 4)
                            if (e < p.hd)
                                *reinterpret_cast<float4 *>(out + e) =
                                    make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
                    } else {
#pragma unroll
                        for (int e = 0; e < HDP; ++e)
                            if (e < p.hd)
                                out[e] = o[e] * inv;
                    }
                } else {
                    uint16_t *out = static_cast<uint16_t *>(p.out) + base;
#pragma unroll
                    for (int e = 0; e < HDP; e += 2) {
                        const uint32_t w = pack_out2(o[e] * inv, o[e + 1] * inv, p.out_dtype);
                        if (e < p.hd)
                            out[e] = static_cast<uint16_t>(w & 0xffffu);
                        if (e + 1 < p.hd)
                            out[e + 1] = static_cast<uint16_t>(w >> 16);
                    }
                }
            }
        }
    }
    // Warps 10+ do not exist; every role falls through to the common exit.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        tmem_dealloc(tmem, 512);
}

// 4-D (d, token, head, batch) fp32 map with a box of 32 columns x `rows`
// tokens: 128-byte swizzle (16-byte atoms) for the K-major operands Q and K,
// 128-byte swizzle of 32-byte atoms for V (MN-major in O += P V).
int make_map_f32(CUtensorMap *map, const void *base, const TensorView &v, int rows, bool mn_major = false) {
    const uint64_t dims[4] = {static_cast<uint64_t>(v.d), static_cast<uint64_t>(v.tokens),
                              static_cast<uint64_t>(v.heads), static_cast<uint64_t>(v.batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(v.s_token) * 4, static_cast<uint64_t>(v.s_head) * 4,
                                 static_cast<uint64_t>(v.s_batch) * 4};
    const uint32_t box[4] = {32u, static_cast<uint32_t>(rows), 1u, 1u};
    return encode_tiled_f32(map, base, 4, dims, strides, box, mn_major ? kSwizzle128Atom32 : 128);
}

template <int HDP, int NK> int launch(const FmhaArgs &a, FmhaF32Params &p, cudaStream_t stream) {
    using S = Shape<HDP, NK>;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr =
        set_smem_limit(reinterpret_cast<const void *>(fmha_f32_kernel<HDP, NK>), S::SMEM_BYTES, done);
    if (attr != cudaSuccess)
        return static_cast<int>(attr);
    int rc = 0;
    if ((rc = make_map_f32(&p.tk, a.k_ptr, a.k, NK)) || (rc = make_map_f32(&p.tv, a.v_ptr, a.v, NK, true)))
        return rc;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            sms = 148;
    }
    const long long items = static_cast<long long>(p.batch) * p.heads * ((p.L + 127) / 128);
    const int grid = static_cast<int>(items < sms ? items : sms);
    fmha_f32_kernel<HDP, NK><<<grid, kThreads, S::SMEM_BYTES, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

} // namespace f32attn

int padded_head_dim_f32(int hd) {
    if (hd <= 32)
        return 32;
    if (hd <= 64)
        return 64;
    if (hd <= 128)
        return 128;
    return -1;
}

bool tma_view_ok_f32(const void *base, const TensorView &v) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    // 16-byte aligned base and 16-byte multiple strides (4-byte elements).
    return (a % 16) == 0 && (v.s_token % 4) == 0 && (v.s_head % 4) == 0 &&
           (v.batch == 1 || (v.s_batch % 4) == 0) && v.d >= 1;
}

int fmha_f32_launch(const FmhaArgs &a, cudaStream_t stream) {
    const int hdp = padded_head_dim_f32(a.q.d);
    if (hdp < 0)
        return -2;
    FmhaF32Params p{};
    p.q = static_cast<const float *>(a.q_ptr);
    p.q_sb = a.q.s_batch;
    p.q_sh = a.q.s_head;
    p.q_st = a.q.s_token;
    p.q_d = a.q.d;
    p.q_vec = (reinterpret_cast<uintptr_t>(a.q_ptr) % 16 == 0) && (a.q.s_token % 4 == 0) && (a.q.s_head % 4 == 0) &&
              (a.q.batch == 1 || a.q.s_batch % 4 == 0) && (a.q.d % 4 == 0);
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
    const uintptr_t oa = reinterpret_cast<uintptr_t>(a.out);
    p.out_vec = a.out_dtype == kOutF32 && (oa % 16 == 0) && (a.o_st % 4 == 0) && (a.o_sh % 4 == 0) &&
                (p.batch == 1 || a.o_sb % 4 == 0) && (p.hd % 4 == 0);
    const double scale = a.scale > 0 ? a.scale : 1.0 / std::sqrt(static_cast<double>(p.hd));
    p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
    p.err = a.err;
    switch (hdp) {
    case 32:
        return f32attn::launch<32, 64>(a, p, stream);
    case 64:
        return f32attn::launch<64, 64>(a, p, stream);
    case 128:
        return f32attn::launch<128, 32>(a, p, stream);
    }
    return -2;
}

} // namespace omni_b200
