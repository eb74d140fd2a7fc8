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

#ifndef OMNI_FMHA_PT
#define OMNI_FMHA_PT 1
#endif
#ifndef OMNI_FMHA_SEP
#define OMNI_FMHA_SEP 0
#endif
// 1: two softmax warps per query row (each owns 64 of the 128 score columns
// and they exchange row maxima per TMEM lane quarter); 0: one thread per row.
#ifndef OMNI_FMHA_SPLIT
#define OMNI_FMHA_SPLIT 0
#endif

// Columns of one O tile in TMEM (the PV MMA's N).  Head dims <= 64 with the
// SEP layout: exactly the head dim, so that each query tile gets P columns of
// its own.  Otherwise one spare column past the head dim for the row-sum
// column of ones (64 -> 80, 96 -> 112).
__host__ __device__ constexpr int head_out_cols(int hdp) {
    return (OMNI_FMHA_SEP && hdp <= 64) ? hdp : hdp == 64 ? 80 : hdp == 96 ? 112 : hdp;
}
#ifndef OMNI_FMHA_QBUF
#define OMNI_FMHA_QBUF (HDP <= 96 ? 2 : 1)
#endif

template <int HDP> struct FmhaShape {
    static constexpr int C0 = HDP < 64 ? HDP : 64; // chunk 0 width (elements)
    static constexpr int C1 = HDP - C0;            // chunk 1 width: 0, 16, 32 or 64
    static constexpr int ROW0 = C0 * 2;            // bytes per row of chunk 0
    static constexpr int ROW1 = C1 * 2;
    static constexpr int CH0_BYTES = 128 * ROW0;
    static constexpr int TILE_BYTES = 128 * HDP * 2; // one 128-row Q or K tile
    // V tiles keep chunk 1 as a full 64-column 128-byte-swizzle atom (zero
    // filled past the head dim) so that O += P V is ONE MMA of N = HDP per
    // 16-key step: its two MN atoms are LBO = 16 KB apart.
    // PV output width (O_i occupies HDPO <= 128 columns), see head_out_cols.
    static constexpr int HDPO = head_out_cols(HDP);
    static constexpr int V_BYTES = HDPO > 64 ? 2 * 128 * 128 : TILE_BYTES;
    static constexpr int V_CH0 = 128 * ROW0;
    // HDPO <= 80 (PT schedule): P gets TMEM columns of its own, the 48 free
    // columns after each O tile -- keys [0, 64) at kPcol0, [64, 128) at
    // kPcol1 -- shared by the two query tiles.  S_i is then free as soon as
    // the softmax has read it, so the next S_i = Q_i K^T is computed while the
    // softmax still works on the current tile, and the MMAs leave the
    // softmax's critical path.  Wider heads write P over S (no spare columns).
    static constexpr bool PT = OMNI_FMHA_PT && HDPO <= 80;
    static constexpr uint32_t kPcol0 = 256 + 80, kPcol1 = 384 + 80;
    // SEP (head dims <= 64): TMEM = S_0 | S_1 | O_0 | O_1 | P_0 | P_1 with
    // 64-column O and P tiles, so each tile has P columns of its own and
    // waits only for its own previous O += P V before writing P.
    static constexpr bool SEP = PT && OMNI_FMHA_SEP && !OMNI_FMHA_SPLIT && HDP <= 64;
    static constexpr uint32_t O_STRIDE = SEP ? 64 : 128; // O_1 - O_0 in columns
    __host__ __device__ static constexpr uint32_t p_col(int i) { return 384 + 64 * i; }
    static constexpr int QBUF = OMNI_FMHA_QBUF; // Q buffers (2: next item prefetch)
    static constexpr int BUDGET = 226 * 1024 - 12 * 1024;
    static constexpr int STAGES_RAW = (BUDGET - QBUF * 2 * TILE_BYTES) / (TILE_BYTES + V_BYTES);
    static constexpr int STAGES = STAGES_RAW > 4 ? 4 : STAGES_RAW;
    static constexpr int KSTEPS = HDP / 16;
    // Barriers, TMEM handle, (two warps per row) the row-max / row-sum
    // exchange buffers and the sorted item table (kSortMaxBatch sequences).
    static constexpr int BAR_BYTES = 1024 + 8192 + 4096;
    // At least 120 KB so that one CTA (which allocates all 512 TMEM columns)
    // occupies an SM by itself.
    static constexpr int SMEM_RAW =
        QBUF * 2 * TILE_BYTES + STAGES * (TILE_BYTES + V_BYTES) + BAR_BYTES + 1024;
    static constexpr int SMEM_BYTES = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
    static_assert(C1 == 0 || C1 == 16 || C1 == 32 || C1 == 64, "unsupported head dim padding");
    static_assert(HDP % 16 == 0, "head dim padding must be a multiple of 16");
    static_assert(STAGES >= 2, "K/V ring needs two stages");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of one CTA");
};

// Sorted item order (variable-length batches without a block window): the
// sequences ordered by KV tiles, longest first (ties: lower index), their
// items enumerated in that order (head-major, then query block), and rank r
// dealt to CTA c in snake order -- round k covers ranks [kG, kG + G) and
// goes c = 0..G-1 on even k, G-1..0 on odd k -- so every CTA's work is nearly
// the same (a static round-robin over the batch order left one CTA with about
// 25 % more work than the mean on a 64-sequence batch of lengths 100..1500).
// Table in shared memory: seq[rank] = batch index, pre[rank] = items before it.
constexpr int kSortMaxBatch = 496;
// After the table (seq[496], pre[497]): this CTA's split part.  A CTA's slots
// are u = blockIdx.x + k * grid, so its only split slot is v = blockIdx.x,
// decoded once in the prologue: (b, h, q0, valid), (T, kb, skip, 0).
constexpr int kSplitSlot = 1000; // 16-byte aligned (int4 reads)
constexpr int kSplitMaxParts = 8;

// 12 warps: 0-3 softmax tile 0, 4-7 softmax tile 1 (warp w serves TMEM lane
// quarter w % 4; each thread owns one query row, all 128 score columns), 8 TMA
// producer, 9 MMA issuer / TMEM owner, 10-11 output stores of tile 0 / tile 1.
// Registers are rebalanced with setmaxnreg: launch 168/thread; the softmax
// warpgroups grow to 208 and the control warpgroup shrinks to 72
// (8*32*208 + 4*32*72 = 62464 <= 384*168 = 64512 per CTA; 2*208 + 72 = 488
// <= 512 per SM sub-partition).
//
// OMNI_FMHA_SPLIT = 1: 20 warps, 0-7 softmax tile 0 and 8-15 tile 1 (warp w
// serves lane quarter w % 4 and score columns [64 ((w / 4) % 2), +64)), 16-19
// as warps 8-11 above; launch 96 registers, softmax 104, control 64
// (16*32*104 + 4*32*64 = 61440 = 640*96; 4*104 + 64 = 480 per sub-partition).
constexpr int kSplit = OMNI_FMHA_SPLIT;
constexpr int kTileWarps = 4 << kSplit;        // softmax warps per query tile
constexpr int kSoftWarps = 2 * kTileWarps;
constexpr int kThreads = (kSoftWarps + 4) * 32;
constexpr int kSoftmaxRegs = kSplit ? 104 : 208;
constexpr int kControlRegs = kSplit ? 64 : 72;
constexpr int kProducerWarp = kSoftWarps;
constexpr int kMmaWarp = kSoftWarps + 1;

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

// 2^x0, 2^x1 with one packed half-precision MUFU ex2; returns the pair as
// bf16x2 (bf16) or f16x2, low half = x0.
__device__ __forceinline__ uint32_t ex2_pair(float x0, float x1, bool bf16) {
    uint32_t r;
    if (bf16)
        asm("{\n\t.reg .b32 t;\n\tcvt.rn.bf16x2.f32 t, %2, %1;\n\tex2.approx.ftz.bf16x2 %0, t;\n\t}"
            : "=r"(r)
            : "f"(x0), "f"(x1));
    else
        asm("{\n\t.reg .b32 t;\n\tcvt.rn.f16x2.f32 t, %2, %1;\n\tex2.approx.f16x2 %0, t;\n\t}"
            : "=r"(r)
            : "f"(x0), "f"(x1));
    return r;
}

// 2^x on the FMA pipe for a pair of lanes: round-to-nearest range reduction
// (adding 1.5 * 2^23 leaves round(x) in the low mantissa bits), a degree-3
// polynomial for 2^f on [-1/2, 1/2] and exponent insertion by integer add.
// The coefficients are a relative-error fit made for this kernel (weighted
// least squares on Chebyshev nodes); max relative error 7.5e-5, below the
// half-ulp of fp16 and bf16.  Inputs are clamped at -125 so that the exponent
// add cannot wrap (2^-125 is far below any P that reaches the sum); masked
// (-inf) scores never take this path.
__device__ __forceinline__ void exp2_poly2(float &y0, float &y1, float x0, float x1) {
    constexpr float kRound = 12582912.0f; // 1.5 * 2^23
    constexpr float c0 = 0.9999280571937561f, c1 = 0.6932610273361206f;
    constexpr float c2 = 0.2426111102104187f, c3 = 0.05517149344086647f;
    x0 = fmaxf(x0, -125.f);
    x1 = fmaxf(x1, -125.f);
    float t0, t1, j0, j1, f0, f1, p0, p1;
    fadd2(t0, t1, x0, x1, kRound, kRound);
    fadd2(j0, j1, t0, t1, -kRound, -kRound);
    ffma2(f0, f1, j0, j1, -1.f, -1.f, x0, x1);
    ffma2(p0, p1, f0, f1, c3, c3, c2, c2);
    ffma2(p0, p1, p0, p1, f0, f1, c1, c1);
    ffma2(p0, p1, p0, p1, f0, f1, c0, c0);
    y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
    y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Which pairs of a 128-score row use the polynomial (the rest use MUFU ex2):
// 3 of every 8, balancing the MUFU, FMA and issue budgets of a sub-partition.
#ifndef OMNI_FMHA_POLY
#define OMNI_FMHA_POLY 0
#endif
#ifndef OMNI_FMHA_TURN
#define OMNI_FMHA_TURN 0
#endif
__device__ __forceinline__ constexpr bool poly_pair(int pair) {
    return OMNI_FMHA_POLY && ((pair & 7) == 1 || (pair & 7) == 4 || (pair & 7) == 6);
}

template <int N> __device__ __forceinline__ void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N> __device__ __forceinline__ void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Drain wait: bounded by time only (does not give up early on other threads'
// errors), used so that no TMA write or MMA is still in flight when the CTA
// releases its shared memory and TMEM.
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

// One work item = 256 query rows of one (batch, head), or (split keys) one
// part of such an item: KV tiles [kb, kb + T) of the item's T_item tiles.
struct Item {
    int b, h, q0, valid, T; // T = KV tiles the item (part) needs (0: write zeros)
    int kb;                 // first KV tile
    int part;               // split part slot v (>= 0), or -1: a whole item
    bool skip;              // nothing to do (rows past the end / padded-query skip)
};

// Item of rank r (sorted order or batch order), all its KV tiles.
// `tab` is null unless the launch uses the sorted order or split slots.
template <bool SPLIT> __device__ __forceinline__ Item decode_rank(const FmhaParams &p, const int *tab, int r) {
    const int qblocks = (p.L + 255) / 256;
    Item it;
    it.kb = 0;
    it.part = -1;
    if (SPLIT ? p.sorted != 0 : tab != nullptr) {
        const int *seq = tab, *pre = tab + kSortMaxBatch;
        if (r >= pre[p.batch]) {
            it.b = it.h = it.q0 = it.valid = it.T = 0;
            it.skip = true;
            return it;
        }
        int lo = 0, hi = p.batch - 1; // last rank with pre[rank] <= r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= r)
                lo = mid;
            else
                hi = mid - 1;
        }
        const int nq = (pre[lo + 1] - pre[lo]) / p.heads;
        const int off = r - pre[lo];
        it.b = seq[lo];
        it.h = off / nq;
        it.q0 = (off - it.h * nq) * 256;
    } else {
        const int bh = r / qblocks;
        it.q0 = (r - bh * qblocks) * 256;
        it.b = bh / p.heads;
        it.h = bh - it.b * p.heads;
    }
    int valid = p.lengths ? p.lengths[it.b] : p.valid;
    valid = valid < p.L ? valid : p.L;
    it.valid = valid < 0 ? 0 : valid;
    it.skip = it.q0 >= p.L || (p.skip_padded_q && it.q0 >= it.valid);
    const int last_row = min(it.q0 + 255, p.L - 1);
    int kv_limit = it.valid;
    if (p.block > 0)
        kv_limit = min(kv_limit, (last_row / p.block + 1) * p.block);
    it.T = (kv_limit + 127) / 128;
    return it;
}

// Slot u of this CTA.  Whole items: round k = u / grid, position c; sorted
// order deals rank k*G + c (even k) or k*G + G-1-c (odd k).  Split slots
// (u >= split_first): the CTA's one part, decoded in the prologue into
// tab[kSplitSlot..] as (b, h, q0, valid, T, kb, skip).
template <bool SPLIT> __device__ __forceinline__ Item decode_item(const FmhaParams &p, const int *tab, int u) {
    if (SPLIT && u >= p.split_first) {
        Item it;
        const int v = u - p.split_first;
        const int4 a = *reinterpret_cast<const int4 *>(tab + kSplitSlot);
        const int4 b = *reinterpret_cast<const int4 *>(tab + kSplitSlot + 4);
        it.b = a.x;
        it.h = a.y;
        it.q0 = a.z;
        it.valid = a.w;
        it.T = b.x;
        it.kb = b.y;
        it.skip = v >= p.split_tail * p.split_s || b.z != 0;
        it.part = v;
        return it;
    }
    int r = u;
    if (SPLIT ? p.sorted != 0 : tab != nullptr) {
        const int G = gridDim.x, k = u / G, c = u - k * G;
        r = k * G + ((k & 1) ? G - 1 - c : c);
    }
    return decode_rank<SPLIT>(p, tab, r);
}

// The first item at or after u (in steps of the grid) that has KV work, or
// `items` when there is none: the items whose Q, K and V are loaded and whose
// MMAs are issued.
template <bool SPLIT>
__device__ __forceinline__ int next_work_item(const FmhaParams &p, const int *tab, int u, int items) {
    for (; u < items; u += gridDim.x) {
        const Item it = decode_item<SPLIT>(p, tab, u);
        if (!it.skip && it.T > 0)
            break;
    }
    return u;
}

// Loads the two Q tiles of item u into Q slot nq % QBUF once the slot is free.
template <int HDP, bool SPLIT>
__device__ __forceinline__ bool load_q_tiles(const FmhaParams &p, const int *tab, int u, int nq, uint8_t *sQ,
                                             uint64_t *q_full, uint64_t *q_empty, int *err) {
    using S = FmhaShape<HDP>;
    const Item it = decode_item<SPLIT>(p, tab, u);
    const int qs = nq % S::QBUF;
    if (!__all_sync(0xffffffffu,
                    mbar_wait(&q_empty[qs], ((nq / S::QBUF) & 1) ^ 1, err, kErrWaitEmpty)))
        return false;
    uint8_t *qdst = sQ + qs * 2 * S::TILE_BYTES;
    if (elect_one()) {
        mbar_arrive_expect_tx(&q_full[qs], 2 * S::TILE_BYTES);
        load_tile<HDP>(qdst, &p.tq0, &p.tq1, &q_full[qs], it.q0, it.h, it.b);
        load_tile<HDP>(qdst + S::TILE_BYTES, &p.tq0, &p.tq1, &q_full[qs], it.q0 + 128, it.h,
                       it.b);
    }
    __syncwarp();
    return true;
}

// Barriers between the softmax warps of a tile (and their consumers) count
// one arrive per warp: the warp's lanes first synchronise (which orders their
// shared-memory and tensor-memory accesses before lane 0's release), then
// lane 0 arrives.  256 per-thread arrives on one barrier word would serialise
// in the shared-memory atomic unit (~2 clk each, on the softmax critical path).
__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0)
        mbar_arrive(bar);
}

// SPLIT: the launch has split slots (p.split_s > 1); a separate instance so
// that launches without them run code that has no split branch.
template <int HDP, bool BF16, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) fmha_fwd_kernel(const __grid_constant__ FmhaParams p) {
    using S = FmhaShape<HDP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *sQ = smem;                                   // [QBUF][2 tiles]
    uint8_t *sK = sQ + S::QBUF * 2 * S::TILE_BYTES;       // [STAGES]
    uint8_t *sV = sK + S::STAGES * S::TILE_BYTES;         // [STAGES]
    uint64_t *bars = reinterpret_cast<uint64_t *>(sV + S::STAGES * S::V_BYTES);
    uint64_t *q_full = bars;                  // [2]
    uint64_t *q_empty = bars + 2;             // [2]
    uint64_t *k_full = bars + 4;              // [STAGES]
    uint64_t *k_empty = k_full + S::STAGES;   // [STAGES]
    uint64_t *v_full = k_empty + S::STAGES;   // [STAGES]
    uint64_t *v_empty = v_full + S::STAGES;   // [STAGES]
    uint64_t *s_full = v_empty + S::STAGES;   // [2]
    uint64_t *p_full = s_full + 2;            // [2]
    uint64_t *o_full = p_full + 2;
    uint64_t *drain = o_full + 1;
    uint64_t *ebar = drain + 1;               // [2] output tile staged, per tile
    uint64_t *turn = ebar + 2;                // [2] exp-phase hand-off between the tiles
    uint64_t *s_free = turn + 2;              // [2] softmax has read S_i (PT)
    uint64_t *pv_done = s_free + 2;           // [2] O_i += P_i V complete (PT)
    uint64_t *xq = pv_done + 2;               // [2 tiles][4 quarters] row-max exchange (split)
    uint64_t *lq = xq + 8;                    // [2 tiles][4 quarters] row-sum exchange (split)
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(lq + 8);
    // Exchange buffers (split): [2 parity][2 tile][4 quarter][2 half][32 lanes].
    float *xmax = reinterpret_cast<float *>(bars + 128);
    [[maybe_unused]] float *xsum = xmax + 2 * 2 * 4 * 2 * 32;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = p.err;
    // Sorted item table and split slot (after the exchange buffers).
    int *tab = (SPLIT || p.sorted) ? reinterpret_cast<int *>(xsum + 2 * 2 * 4 * 2 * 32) : nullptr;
    static_assert(2 * 2 * 4 * 2 * 32 * 8 + (kSplitSlot + 8) * 4 <= 8192 + 4096, "item table space");
    if (p.sorted) {
        int *seq = tab, *pre = tab + kSortMaxBatch;
        const int qblocks = (p.L + 255) / 256;
        auto kv_tiles = [&](int b) {
            int v = p.lengths[b];
            v = v < p.L ? v : p.L;
            return v < 0 ? 0 : (v + 127) / 128;
        };
        for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
            const int tb = kv_tiles(b);
            int r = 0;
            for (int b2 = 0; b2 < p.batch; ++b2) {
                const int t2 = kv_tiles(b2);
                r += (t2 > tb || (t2 == tb && b2 < b)) ? 1 : 0;
            }
            seq[r] = b;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int acc = 0;
            for (int r = 0; r < p.batch; ++r) {
                pre[r] = acc;
                int v = p.lengths[seq[r]];
                v = v < p.L ? v : p.L;
                v = v < 0 ? 0 : v;
                const int nq = p.skip_padded_q ? (v + 255) / 256 : qblocks;
                acc += p.heads * nq;
            }
            pre[p.batch] = acc;
        }
        __syncthreads();
    }
    const int items = SPLIT ? p.split_items
                      : p.sorted    ? (tab[kSortMaxBatch + p.batch] + gridDim.x - 1) / gridDim.x * gridDim.x
                                    : p.batch * p.heads * ((p.L + 255) / 256);

    if (threadIdx.x == 0) {
        if (SPLIT) {
            // Part q of the tail item of rank split_first + w (v = q * tail + w):
            // KV tiles [q T / s, (q + 1) T / s) of the item's T.
            const int v = blockIdx.x, q = v / p.split_tail, w = v - q * p.split_tail;
            Item it = decode_rank<true>(p, tab, p.split_first + w);
            const int kb = q * it.T / p.split_s, ke = (q + 1) * it.T / p.split_s;
            *reinterpret_cast<int4 *>(tab + kSplitSlot) = make_int4(it.b, it.h, it.q0, it.valid);
            *reinterpret_cast<int4 *>(tab + kSplitSlot + 4) = make_int4(ke - kb, kb, it.skip ? 1 : 0, 0);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            // Released by the MMA warp, or (TMA output) by the two tiles'
            // output stores, which stage O in this Q slot.
            mbar_init(&q_empty[i], p.o_tma ? 2 : 1);
            mbar_init(&ebar[i], kTileWarps);
            mbar_init(&turn[i], kTileWarps);
            mbar_init(&s_free[i], kTileWarps);
            mbar_init(&pv_done[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], kTileWarps);
        }
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int e = 0; e < 8; ++e) {
            mbar_init(&xq[e], 2); // the two warps of one lane quarter
            mbar_init(&lq[e], 2);
        }
        mbar_init(o_full, 1);
        mbar_init(drain, 1);
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_holder, 512);
        tmem_relinquish();
    }
    if constexpr (S::HDPO > 64) {
        // V's second chunk: zeros, except the ones column (row-sum trick).  TMA
        // later rewrites only the first v1_width columns of each row.
        const uint32_t one = BF16 ? 0x3F80u : 0x3C00u;
        for (int idx = threadIdx.x; idx < S::STAGES * 128 * 8; idx += kThreads) {
            const int st = idx / (128 * 8), row = (idx / 8) % 128, c16 = idx % 8;
            uint4 w = make_uint4(0u, 0u, 0u, 0u);
            if (p.ones_col >= 64 && c16 == ((p.ones_col - 64) >> 3))
                w.x = one; // element (ones_col - 64) % 8 == 0 of its 16-byte chunk
            uint8_t *row_base = sV + st * S::V_BYTES + S::V_CH0 + row * 128;
            *reinterpret_cast<uint4 *>(row_base + ((c16 ^ (row & 7)) << 4)) = w;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    if (tmem != 0) {
        // Unexpected: the MMA issuer relies on a whole-TMEM allocation at 0.
        if (threadIdx.x == 0)
            atomicOr(err, kErrWaitDrain);
        __syncthreads();
        if (warp == kMmaWarp)
            tmem_dealloc(tmem, 512);
        return;
    }

    if (warp >= kProducerWarp) {
        setmaxnreg_dec<kControlRegs>();
        if (warp == kProducerWarp) {
            // -------------------------------------------------- TMA producer
            // The whole warp runs this loop (warp-uniform state); one elected
            // lane issues each barrier arrive and TMA copy.
            if (elect_one()) {
                tma_prefetch_desc(&p.tq0);
                tma_prefetch_desc(&p.tk0);
                tma_prefetch_desc(&p.tv0);
            }
            // K and V loads issued by this CTA (Q tiles are loaded by warp 10).
            int nk = 0, nv = 0;
            bool ok = true;
            for (int u = next_work_item<SPLIT>(p, tab, blockIdx.x, items); ok && u < items;
                 u = next_work_item<SPLIT>(p, tab, u + gridDim.x, items)) {
                const Item it = decode_item<SPLIT>(p, tab, u);
                for (int j = 0; j < it.T; ++j) {
                    const int st = nk % S::STAGES;
                    const uint32_t ph = (nk / S::STAGES) & 1;
                    ok = __all_sync(0xffffffffu, mbar_wait(&k_empty[st], ph ^ 1, err, kErrWaitEmpty));
                    if (!ok)
                        break;
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&k_full[st], S::TILE_BYTES);
                        load_tile<HDP>(sK + st * S::TILE_BYTES, &p.tk0, &p.tk1, &k_full[st],
                                       ((SPLIT ? it.kb : 0) + j) * 128, it.h, it.b);
                    }
                    __syncwarp();
                    ++nk;
                    ok = __all_sync(0xffffffffu, mbar_wait(&v_empty[st], ph ^ 1, err, kErrWaitEmpty));
                    if (!ok)
                        break;
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&v_full[st], 128 * 2 * (S::C0 + p.v1_width));
                        uint8_t *vdst = sV + st * S::V_BYTES;
                        const int row = ((SPLIT ? it.kb : 0) + j) * 128;
                        tma_load_4d(vdst, &p.tv0, &v_full[st], 0, row, it.h, it.b);
                        if (S::HDPO > 64 && p.v1_width > 0)
                            tma_load_4d(vdst + S::V_CH0, &p.tv1, &v_full[st], 64, row, it.h, it.b);
                    }
                    __syncwarp();
                    ++nv;
                }
            }
            // Every issued copy must land before the CTA may exit.
            for (int n = nk - S::STAGES < 0 ? 0 : nk - S::STAGES; n < nk; ++n)
                wait_drain(&k_full[n % S::STAGES], (n / S::STAGES) & 1, err);
            for (int n = nv - S::STAGES < 0 ? 0 : nv - S::STAGES; n < nv; ++n)
                wait_drain(&v_full[n % S::STAGES], (n / S::STAGES) & 1, err);
        } else if (warp == kMmaWarp) {
            // ---------------------------------------------------- MMA issuer
            // The whole warp runs this loop with warp-uniform values; one
            // elected lane issues each tcgen05.mma / tcgen05.commit.
            constexpr uint32_t idesc_qk = make_idesc_f16(128, 128, BF16, false);
            constexpr uint32_t idesc_pv = make_idesc_f16(128, S::HDPO, BF16, true);
            constexpr uint32_t lay0 = layout_for_row_bytes(S::ROW0);
            constexpr uint32_t lay1 = layout_for_row_bytes(S::ROW1 > 0 ? S::ROW1 : 32);
            const uint32_t sq = smem_u32(sQ), sk = smem_u32(sK), sv = smem_u32(sV);
            // Descriptors are advanced by adding (byte offset >> 4) to the start
            // address field; the K-step loops are unrolled so that every offset
            // is a compile-time constant (the issue path then runs at the
            // tensor core's rate).
            const uint32_t leader = elect_one() ? 1u : 0u;
            // All 512 TMEM columns belong to this CTA, so the allocation starts
            // at lane 0 / column 0: use the constant (warp-uniform, so MMA
            // operands stay in uniform registers); the start of the kernel
            // checked that the allocator returned exactly that address.
            const uint32_t tmem = 0;
            auto commit = [&](uint64_t *bar) { tc_commit_if(leader, bar); };
            auto qk = [&](uint32_t qbase, int i, int st) {
                const uint32_t d = tmem + i * 128;
                const uint64_t a0 = make_smem_desc(qbase + i * S::TILE_BYTES, 16, 8 * S::ROW0, lay0);
                const uint64_t b0 = make_smem_desc(sk + st * S::TILE_BYTES, 16, 8 * S::ROW0, lay0);
#pragma unroll
                for (int kk = 0; kk < S::C0 / 16; ++kk)
                    umma_ss_if(leader, d, a0 + 2 * kk, b0 + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
                if constexpr (S::C1 > 0) {
                    const uint64_t a1 = make_smem_desc(qbase + i * S::TILE_BYTES + S::CH0_BYTES, 16,
                                                       8 * S::ROW1, lay1);
                    const uint64_t b1 = make_smem_desc(sk + st * S::TILE_BYTES + S::CH0_BYTES, 16,
                                                       8 * S::ROW1, lay1);
#pragma unroll
                    for (int kk = 0; kk < S::C1 / 16; ++kk)
                        umma_ss_if(leader, d, a1 + 2 * kk, b1 + 2 * kk, idesc_qk, 1u);
                }
            };
            auto pv = [&](int i, int st, bool accumulate) {
                const uint32_t d = tmem + 256 + i * 128;
                const uint32_t a = tmem + i * 128;
                const uint32_t vb = sv + st * S::V_BYTES;
                constexpr uint32_t vrow = S::HDPO >= 64 ? 128 : S::ROW0;
                const uint64_t v0 = make_smem_desc(vb, S::V_CH0, 8 * vrow,
                                                   S::HDPO >= 64 ? kLayoutSW128 : lay0);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_ts_if(leader, d, a + kk * 8,
                               v0 + static_cast<uint64_t>((kk * 16 * vrow) >> 4), idesc_pv,
                               (accumulate || kk > 0) ? 1u : 0u);
            };
            // O_i += P_i V_st with P in its own TMEM columns (PT).
            auto pv_pt = [&](int i, int st, bool accumulate) {
                const uint32_t d = tmem + 256 + i * S::O_STRIDE;
                const uint32_t vb = sv + st * S::V_BYTES;
                constexpr uint32_t vrow = S::HDPO >= 64 ? 128 : S::ROW0;
                const uint64_t v0 = make_smem_desc(vb, S::V_CH0, 8 * vrow,
                                                   S::HDPO >= 64 ? kLayoutSW128 : lay0);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_ts_if(leader, d,
                               S::SEP ? tmem + S::p_col(i) + kk * 8
                                      : tmem + (kk < 4 ? S::kPcol0 : S::kPcol1) + (kk & 3) * 8,
                               v0 + static_cast<uint64_t>((kk * 16 * vrow) >> 4), idesc_pv,
                               (accumulate || kk > 0) ? 1u : 0u);
            };
            if constexpr (S::PT) {
                // Per KV tile g: S_0(g+1), S_1(g+1) as soon as the softmax has
                // read S_0(g), S_1(g); then O_0 += P_0(g) V_g and O_1 += P_1(g) V_g
                // as each P arrives.  pv_done[i] fires after O_i += P_i V.  The
                // loop is pipelined across items: during an item's last KV tile
                // the next item's first S goes out (its Q sits in the other Q
                // slot), so the tensor core computes it while the softmax warps
                // finish the item and run its epilogue.
                static_assert(S::QBUF >= 2, "cross-item S issue needs a second Q slot");
                int nq = 0, kv = 0;
                bool ok = true, first_s_issued = false;
                // S_i(g) for both tiles from the Q slot at qb.
                auto issue_s = [&](uint32_t qb, int g, int st) {
                    for (int i = 0; i < 2; ++i) {
                        if (g > 0 && !__all_sync(0xffffffffu, mbar_wait(&s_free[i], (g - 1) & 1, err, kErrWaitS)))
                            return false;
                        tc_fence_after();
                        qk(qb, i, st);
                        commit(&s_full[i]);
                    }
                    commit(&k_empty[st]);
                    return true;
                };
                for (int u = next_work_item<SPLIT>(p, tab, blockIdx.x, items); ok && u < items;) {
                    const Item it = decode_item<SPLIT>(p, tab, u);
                    const int u_next = next_work_item<SPLIT>(p, tab, u + gridDim.x, items);
                    const int qs = nq % S::QBUF;
                    const uint32_t qbase = sq + qs * 2 * S::TILE_BYTES;
                    if (!first_s_issued) { // S_i(g0) for the item's first KV tile g0 = kv
                        const int st = kv % S::STAGES;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[qs], (nq / S::QBUF) & 1, err, kErrWaitQ))))
                            break;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&k_full[st], (kv / S::STAGES) & 1, err, kErrWaitK))))
                            break;
                        if (!(ok = issue_s(qbase, kv, st)))
                            break;
                    }
                    first_s_issued = false;
                    for (int j = 0; ok && j < it.T; ++j) {
                        const int g = kv + j, st = g % S::STAGES;
                        if (j + 1 < it.T || u_next < items) {
                            // The next S: this item's tile j + 1, or the next
                            // item's first tile (global KV tile g + 1 either way).
                            const int st1 = (g + 1) % S::STAGES;
                            uint32_t qb = qbase;
                            if (j + 1 == it.T) {
                                const int qs1 = (nq + 1) % S::QBUF;
                                if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[qs1], ((nq + 1) / S::QBUF) & 1, err, kErrWaitQ))))
                                    break;
                                qb = sq + qs1 * 2 * S::TILE_BYTES;
                                first_s_issued = true;
                            }
                            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&k_full[st1], ((g + 1) / S::STAGES) & 1, err, kErrWaitK))))
                                break;
                            if (!(ok = issue_s(qb, g + 1, st1)))
                                break;
                        }
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&v_full[st], (g / S::STAGES) & 1, err, kErrWaitV))))
                            break;
                        for (int i = 0; i < 2; ++i) {
                            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&p_full[i], g & 1, err, kErrWaitP))))
                                break;
                            tc_fence_after();
                            pv_pt(i, st, j > 0);
                            commit(&pv_done[i]);
                        }
                        if (!ok)
                            break;
                        commit(&v_empty[st]);
                    }
                    if (!ok)
                        break;
                    if (!p.o_tma)
                        commit(&q_empty[qs]); // every MMA reading this Q slot is done
                    kv += it.T;
                    ++nq;
                    u = u_next;
                }
            } else {
                int nq = 0, kv = 0, n_items = 0;
                bool ok = true;
                for (int u = blockIdx.x; ok && u < items; u += gridDim.x) {
                    const Item it = decode_item<SPLIT>(p, tab, u);
                    if (it.skip || it.T == 0)
                        continue;
                    const int qs = nq % S::QBUF;
                    const uint32_t qbase = sq + qs * 2 * S::TILE_BYTES;
                    if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[qs], (nq / S::QBUF) & 1, err, kErrWaitQ))))
                        break;
                    {
                        const int st = kv % S::STAGES;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&k_full[st], (kv / S::STAGES) & 1, err, kErrWaitK))))
                            break;
                        tc_fence_after();
                        qk(qbase, 0, st);
                        commit(&s_full[0]);
                        qk(qbase, 1, st);
                        commit(&s_full[1]);
                        commit(&k_empty[st]);
                    }
                    for (int j = 0; j < it.T; ++j) {
                        const int g = kv + j, st = g % S::STAGES;
                        const uint32_t ph = (g / S::STAGES) & 1;
                        const int g1 = g + 1, st1 = g1 % S::STAGES;
                        const uint32_t ph1 = (g1 / S::STAGES) & 1;
                        const bool more = j + 1 < it.T;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&v_full[st], ph, err, kErrWaitV))))
                            break;
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&p_full[0], g & 1, err, kErrWaitP))))
                            break;
                        tc_fence_after();
                        pv(0, st, j > 0);
                        if (more) {
                            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&k_full[st1], ph1, err, kErrWaitK))))
                                break;
                            tc_fence_after();
                            qk(qbase, 0, st1);
                            commit(&s_full[0]);
                        }
                        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&p_full[1], g & 1, err, kErrWaitP))))
                            break;
                        tc_fence_after();
                        pv(1, st, j > 0);
                        commit(&v_empty[st]);
                        if (more) {
                            qk(qbase, 1, st1);
                            commit(&s_full[1]);
                            commit(&k_empty[st1]);
                        }
                    }
                    if (!ok)
                        break;
                    commit(o_full); // O_0, O_1 of this item are final
                    if (!p.o_tma)
                        commit(&q_empty[qs]); // every MMA reading this Q slot is done
                    kv += it.T;
                    ++nq;
                    ++n_items;
                }
            }
            commit(drain);
            wait_drain(drain, 0, err);
        } else {
            // ------------------------------------- Q loads and output stores
            // Warp 10 + i stores tile i of every item (TMA output): it waits
            // until the four softmax warps of the tile have staged O in the
            // item's Q slot, writes the tile with TMA and waits until the copy
            // has read shared memory before it releases the Q slot.  Warp 10
            // also loads the Q tiles: the first QBUF items' at the start, then
            // item n + QBUF's as soon as item n has released its slot, so that
            // the K/V producer never waits for a Q slot.
            const int i = warp - (kMmaWarp + 1);
            int n_items = 0, nq = 0;
            int uq = next_work_item<SPLIT>(p, tab, blockIdx.x, items); // next item whose Q is due
            bool ok = true;
            if (i == 0) {
                for (int k = 0; ok && k < S::QBUF && uq < items; ++k) {
                    ok = load_q_tiles<HDP, SPLIT>(p, tab, uq, nq, sQ, q_full, q_empty, err);
                    ++nq;
                    uq = next_work_item<SPLIT>(p, tab, uq + gridDim.x, items);
                }
            }
            for (int u = next_work_item<SPLIT>(p, tab, blockIdx.x, items); ok && u < items;
                 u = next_work_item<SPLIT>(p, tab, u + gridDim.x, items)) {
                if (p.o_tma) {
                    const Item it = decode_item<SPLIT>(p, tab, u);
                    const int qs_out = n_items % S::QBUF;
                    ok = __all_sync(0xffffffffu, mbar_wait(&ebar[i], n_items & 1, err, kErrWaitO));
                    if (!ok)
                        break;
                    ++n_items;
                    if (elect_one()) {
                        uint8_t *stile = sQ + (qs_out * 2 + i) * S::TILE_BYTES;
                        const int row0 = it.q0 + i * 128;
                        // A tile wholly past the end stores nothing; a split
                        // part wrote its partial rows to the scratch instead.
                        if (row0 < p.L && (!SPLIT || it.part < 0)) {
                            tma_store_4d(&p.to0, stile, 0, row0, it.h, it.b);
                            if constexpr (S::C1 > 0)
                                tma_store_4d(&p.to1, stile + S::CH0_BYTES, S::C0, row0, it.h,
                                             it.b);
                            tma_store_commit();
                            tma_store_wait_read();
                        }
                        mbar_arrive(&q_empty[qs_out]);
                    }
                    __syncwarp();
                }
                if (i == 0 && uq < items) {
                    if (!(ok = load_q_tiles<HDP, SPLIT>(p, tab, uq, nq, sQ, q_full, q_empty, err)))
                        break;
                    ++nq;
                    uq = next_work_item<SPLIT>(p, tab, uq + gridDim.x, items);
                }
            }
            if (i == 0) {
                // Every issued Q copy must land before the CTA may exit.
                for (int n = nq - S::QBUF < 0 ? 0 : nq - S::QBUF; n < nq; ++n)
                    wait_drain(&q_full[n % S::QBUF], (n / S::QBUF) & 1, err);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------- softmax warpgroups
        // Tile i = warp / kTileWarps; warp w serves TMEM lane quarter w % 4
        // (fixed by the hardware).  One thread per row (kSplit = 0): all 128
        // score columns, the running max / sum and the row of O.  Two warps per
        // row (kSplit = 1): half hh = (w / 4) % 2 owns score columns
        // [64 hh, 64 hh + 64) and half of O's column chunks; the two warps of a
        // lane quarter exchange their row maxima through shared memory.
        setmaxnreg_inc<kSoftmaxRegs>();
        constexpr int kCols = 128 >> kSplit; // score columns per thread
        const int i = warp / kTileWarps, hh = kSplit ? (warp >> 2) & 1 : 0, qd = warp & 3;
        const int r = (qd << 5) + lane; // TMEM lane == row in tile
        const uint32_t lane_base = static_cast<uint32_t>(qd << 5) << 16;
        const uint32_t tS = tmem + lane_base + i * 128 + hh * kCols;
        const uint32_t tO = tmem + lane_base + 256 + i * S::O_STRIDE;
        const float sl2 = p.scale_log2;
        const bool ones = S::HDPO > 64 && p.ones_col >= 0;
        constexpr int kOch = S::HDPO / 16, kEch = HDP / 16;
        // O column chunks this warp rescales / stores.
        constexpr int kOsplit = kSplit ? (kOch + 1) / 2 : kOch, kEsplit = kSplit ? (kEch + 1) / 2 : kEch;
        const int oc_begin = hh ? kOsplit : 0, oc_end = hh ? kOch : kOsplit;
        const int ec_begin = hh ? kEsplit : 0, ec_end = hh ? kEch : kEsplit;
        int g = 0, n_items = 0;
        [[maybe_unused]] int n_sum = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < items; u += gridDim.x) {
            const Item it = decode_item<SPLIT>(p, tab, u);
            if (SPLIT && it.part >= 0 && it.part < p.split_tail && threadIdx.x == 0)
                p.split_hdr[it.part] = make_int4(it.b, it.h, it.q0, it.skip ? 1 : 0); // part 0 of item w
            if (it.skip)
                continue;
            const int t = it.q0 + i * 128 + r; // query token
            int limit = it.valid;
            if (p.block > 0)
                limit = min(limit, (t / p.block + 1) * p.block);
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.T; ++j, ++g) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[i], g & 1, err, kErrWaitS));
                if (!ok)
                    break;
                tc_fence_after();
                uint32_t sraw[kCols];
#pragma unroll
                for (int c = 0; c < kCols / 32; ++c)
                    tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sraw[32 * c]));
                tmem_wait_ld();
                if constexpr (S::PT) {
                    // S_i is in registers: the MMA warp may compute S_i(j+1).
                    tc_fence_before();
                    warp_arrive(&s_free[i]);
                }
                float *s = reinterpret_cast<float *>(sraw);
                const int kv0 = ((SPLIT ? it.kb : 0) + j) * 128 + hh * kCols;
                const bool masked = kv0 + kCols > limit;
                if (masked) {
#pragma unroll
                    for (int c = 0; c < kCols; ++c)
                        if (kv0 + c >= limit)
                            s[c] = -INFINITY;
                }
                // Row max: independent 3-input max chains of 16 scores (short
                // dependency chains; the max is latency-bound).
                float mc[kCols / 16];
#pragma unroll
                for (int q = 0; q < kCols / 16; ++q) {
                    const float *sq = s + 16 * q;
                    float v = fmax3(sq[0], sq[1], sq[2]);
#pragma unroll
                    for (int e = 3; e < 15; e += 2)
                        v = fmax3(v, sq[e], sq[e + 1]);
                    mc[q] = fmaxf(v, sq[15]);
                }
#pragma unroll
                for (int w = kCols / 32; w > 0; w >>= 1)
#pragma unroll
                    for (int q = 0; q < w; ++q)
                        mc[q] = fmaxf(mc[q], mc[q + w]);
                float mt = mc[0];
                if constexpr (kSplit) {
                    // Exchange with the other half of the row (double-buffered
                    // by iteration parity).  After this wait both halves have
                    // read their scores, so P may overwrite S (P-over-S layout).
                    float *xm = xmax + ((((g & 1) * 2 + i) * 4 + qd) * 2) * 32;
                    xm[hh * 32 + lane] = mt;
                    warp_arrive(&xq[i * 4 + qd]);
                    ok = __all_sync(0xffffffffu, mbar_wait(&xq[i * 4 + qd], g & 1, err, kErrWaitP));
                    if (!ok)
                        break;
                    mt = fmaxf(mt, xm[(hh ^ 1) * 32 + lane]);
                }
                const float mnew = fmaxf(m, mt * sl2);
                // Lazy rescale: a row keeps its stale max while P stays below 2^8.
                const bool grow = mnew > m + 8.0f;
                const float alpha = (grow && j > 0) ? ex2_approx(m - mnew) : 1.f;
                if (grow) {
                    l *= alpha;
                    m = mnew;
                }
                float neg_m = -m;
                if constexpr (SPLIT) {
                    // A part past a row's block window: every score of the row
                    // is masked so far (m = -inf) and P must be 0, not 2^NaN.
                    neg_m = m == -INFINITY ? 0.f : neg_m;
                }
                if (OMNI_FMHA_TURN && (i == 1 || g > 0)) {
                    // The tiles take turns for the exp phase: tile 0 runs
                    // iteration g after tile 1 finished g-1, tile 1 after tile 0
                    // finished g.
                    const uint32_t par = i == 1 ? (g & 1) : ((g - 1) & 1);
                    ok = __all_sync(0xffffffffu, mbar_wait(&turn[i], par, err, kErrWaitP));
                    if (!ok)
                        break;
                }
                // P = 2^(s*scale - m) (packed fp32 FMA, MUFU ex2 or the FMA-pipe
                // polynomial); P pair c (keys 2c, 2c+1 of this thread's columns)
                // is written over sraw[c] (its inputs s[2c], s[2c+1] are
                // consumed by then).  Rows of a masked tile use MUFU only (exact
                // zeros for -inf).
                float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
                for (int c = 0; c < kCols / 2; c += 2) {
                    float x0, x1, x2, x3;
                    ffma2(x0, x1, s[2 * c], s[2 * c + 1], sl2, sl2, neg_m, neg_m);
                    ffma2(x2, x3, s[2 * c + 2], s[2 * c + 3], sl2, sl2, neg_m, neg_m);
                    if (poly_pair(c) && !masked) {
                        exp2_poly2(x0, x1, x0, x1);
                    } else {
                        x0 = ex2_approx(x0);
                        x1 = ex2_approx(x1);
                    }
                    if (poly_pair(c + 1) && !masked) {
                        exp2_poly2(x2, x3, x2, x3);
                    } else {
                        x2 = ex2_approx(x2);
                        x3 = ex2_approx(x3);
                    }
                    if (!ones) {
                        fadd2(a0, a1, a0, a1, x0, x1);
                        fadd2(b0, b1, b0, b1, x2, x3);
                    }
                    sraw[c] = pack2(x0, x1, BF16);
                    sraw[c + 1] = pack2(x2, x3, BF16);
                }
                if (!ones)
                    l += (a0 + a1) + (b0 + b1);
                if (OMNI_FMHA_TURN)
                    warp_arrive(&turn[i ^ 1]); // the other tile's turn
                if constexpr (S::SEP) {
                    // Own P columns: P_i(g) overwrites P_i(g-1) once
                    // O_i += P_i(g-1) V is complete (which also allows the O
                    // rescale).
                    if (g > 0) {
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(&pv_done[i], (g - 1) & 1, err, kErrWaitO));
                        if (!ok)
                            break;
                        tc_fence_after();
                    }
                } else if constexpr (S::PT) {
                    // The P columns are shared by the two tiles: tile 0 writes
                    // P(g) once O_1 += P_1(g-1) V is complete, tile 1 once
                    // O_0 += P_0(g) V is.  Each of those MMAs was issued after
                    // this tile's own previous O += P V, so O_i may be rescaled
                    // after the wait too.
                    if (i == 1 || g > 0) {
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait(&pv_done[i ^ 1], i == 0 ? (g - 1) & 1 : g & 1,
                                                  err, kErrWaitO));
                        if (!ok)
                            break;
                        tc_fence_after();
                    }
                }
                // O rescale (after the scores are dead, to keep registers low).
                // tcgen05.ld/st are warp-collective: the warp's rows rescale
                // together (alpha == 1 for rows whose max did not grow).
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int c = 0; c < kOch; ++c) {
                        if (c < oc_begin || c >= oc_end)
                            continue;
                        uint32_t o[16];
                        tmem_ld16(tO + c * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st16(tO + c * 16, o);
                    }
                }
                __syncwarp();
                if constexpr (S::SEP) {
                    tmem_st32(tmem + lane_base + S::p_col(i),
                              *reinterpret_cast<uint32_t(*)[32]>(&sraw[0]));
                    tmem_st32(tmem + lane_base + S::p_col(i) + 32,
                              *reinterpret_cast<uint32_t(*)[32]>(&sraw[32]));
                } else if constexpr (S::PT) {
                    // Keys [0, 64) at kPcol0, [64, 128) at kPcol1.
                    if constexpr (kSplit) {
                        tmem_st32(tmem + lane_base + (hh ? S::kPcol1 : S::kPcol0),
                                  *reinterpret_cast<uint32_t(*)[32]>(&sraw[0]));
                    } else {
                        tmem_st32(tmem + lane_base + S::kPcol0,
                                  *reinterpret_cast<uint32_t(*)[32]>(&sraw[0]));
                        tmem_st32(tmem + lane_base + S::kPcol1,
                                  *reinterpret_cast<uint32_t(*)[32]>(&sraw[32]));
                    }
                } else {
                    // P over the first 64 columns of S_i (all of S_i was read:
                    // by this thread, or by both halves before the exchange).
                    const uint32_t tP = tmem + lane_base + i * 128 + hh * 32;
                    tmem_st32(tP, *reinterpret_cast<uint32_t(*)[32]>(&sraw[0]));
                    if constexpr (!kSplit)
                        tmem_st32(tP + 32, *reinterpret_cast<uint32_t(*)[32]>(&sraw[32]));
                }
                tmem_wait_st(); // P, and the O rescale above
                tc_fence_before();
                warp_arrive(&p_full[i]);
            }
            if (!ok)
                break;
            if (it.T > 0) {
                if constexpr (S::PT)
                    ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[i], (g - 1) & 1, err, kErrWaitO));
                else
                    ok = __all_sync(0xffffffffu, mbar_wait(o_full, n_items & 1, err, kErrWaitO));
                if (!ok)
                    break;
                ++n_items;
                tc_fence_after();
            }
            // One thread per row: the whole O row (and the ones column) in one
            // batch of TMEM loads with a single wait.  Two warps per row (fewer
            // registers): the ones column here, O chunk by chunk below.
            constexpr int kOb = kSplit ? 1 : kOch;
            uint32_t ob[kOb][16];
            if constexpr (kSplit) {
                if (ones && it.T > 0) {
                    tmem_ld16(tO + (p.ones_col & ~15), ob[0]);
                    tmem_wait_ld();
                    float lv = 0.f;
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        lv = e == (p.ones_col & 15) ? __uint_as_float(ob[0][e]) : lv;
                    l = lv;
                }
            } else {
                if (it.T > 0) {
#pragma unroll
                    for (int cq = 0; cq < kOb; ++cq)
                        tmem_ld16(tO + cq * 16, ob[cq]);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int cq = 0; cq < kOb; ++cq)
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            ob[cq][e] = 0u;
                }
                if (ones && it.T > 0) {
                    // Row sum of P = O[:, ones_col] (rescaled together with O).
                    float lv = 0.f;
#pragma unroll
                    for (int cq = 0; cq < kOb; ++cq)
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            lv = cq * 16 + e == p.ones_col ? __uint_as_float(ob[cq][e]) : lv;
                    l = lv;
                }
            }
            // Chunk cq of this thread's O row.
            auto o_chunk = [&](int cq, uint32_t (&tmp)[16]) -> const uint32_t * {
                if constexpr (kSplit) {
                    if (it.T > 0) {
                        tmem_ld16(tO + cq * 16, tmp);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            tmp[e] = 0u;
                    }
                    return tmp;
                } else {
                    return ob[cq < kOb ? cq : 0];
                }
            };
            if constexpr (kSplit) {
                if (!ones && it.T > 0) {
                    // Sum of the two halves' partial row sums (double-buffered
                    // by exchange parity).
                    float *xs = xsum + ((((n_sum & 1) * 2 + i) * 4 + qd) * 2) * 32;
                    xs[hh * 32 + lane] = l;
                    warp_arrive(&lq[i * 4 + qd]);
                    ok = __all_sync(0xffffffffu, mbar_wait(&lq[i * 4 + qd], n_sum & 1, err, kErrWaitO));
                    if (!ok)
                        break;
                    ++n_sum;
                    l += xs[(hh ^ 1) * 32 + lane];
                }
            }
            if constexpr (SPLIT && !kSplit) {
                if (it.part >= 0) {
                    // Split part: the unnormalised O row (all HDP columns), the
                    // row's max (log2 units: P = 2^(s * scale_log2 - m)) and its
                    // sum of P; fmha_split_combine merges the parts.  An empty
                    // part (T = 0) writes m = -inf, l = 0, O = 0.
                    const int prow = it.part * 256 + i * 128 + r;
                    float4 *po = reinterpret_cast<float4 *>(p.split_o + static_cast<size_t>(prow) * HDP);
#pragma unroll
                    for (int cq = 0; cq < kEch; ++cq)
#pragma unroll
                        for (int e = 0; e < 16; e += 4)
                            po[cq * 4 + e / 4] =
                                make_float4(__uint_as_float(ob[cq][e]), __uint_as_float(ob[cq][e + 1]),
                                            __uint_as_float(ob[cq][e + 2]), __uint_as_float(ob[cq][e + 3]));
                    p.split_m[prow] = m;
                    p.split_l[prow] = l;
                    if (p.o_tma && it.T > 0)
                        warp_arrive(&ebar[i]); // the store warp releases the Q slot
                    __syncwarp();
                    continue;
                }
            }
            const float inv = (it.T > 0 && l > 0.f) ? 1.f / l : 0.f;
            if (p.o_tma && it.T > 0) {
                // Stage the row of O in the item's Q slot (the same swizzled
                // chunk layout as a Q tile; every MMA reading Q is complete once
                // O is final), then the tile's store warp writes it with TMA
                // (rows past L and columns past hd clipped).
                const int qs_out = (n_items - 1) % S::QBUF;
                uint8_t *stile = sQ + (qs_out * 2 + i) * S::TILE_BYTES;
#pragma unroll
                for (int cq = 0; cq < kEch; ++cq) {
                    if (cq < ec_begin || cq >= ec_end)
                        continue;
                    const int c = cq * 16;
                    uint32_t otmp[16];
                    const uint32_t *o = o_chunk(cq, otmp);
                    uint4 w0, w1;
                    w0.x = pack2(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv, BF16);
                    w0.y = pack2(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv, BF16);
                    w0.z = pack2(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv, BF16);
                    w0.w = pack2(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv, BF16);
                    w1.x = pack2(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv, BF16);
                    w1.y = pack2(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv, BF16);
                    w1.z = pack2(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv, BF16);
                    w1.w = pack2(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv, BF16);
                    const bool ch1 = c >= S::C0;
                    const int rowb = ch1 ? S::ROW1 : S::ROW0;
                    const int k16 = ((ch1 ? c - S::C0 : c) * 2) >> 4; // 16-byte chunk in the row
                    const int sw = ((r * rowb) >> 7) & ((rowb >> 4) - 1);
                    uint8_t *rowp = stile + (ch1 ? S::CH0_BYTES : 0) + r * rowb;
                    *reinterpret_cast<uint4 *>(rowp + ((k16 ^ sw) << 4)) = w0;
                    *reinterpret_cast<uint4 *>(rowp + (((k16 + 1) ^ sw) << 4)) = w1;
                }
                fence_proxy_async_smem();
                warp_arrive(&ebar[i]); // the tile's store warp takes it from here
                continue;
            }
            const bool store = t < p.L;
            const long long base =
                it.b * p.o_sb + it.h * p.o_sh + static_cast<long long>(t) * p.o_st;
#pragma unroll
            for (int cq = 0; cq < kEch; ++cq) {
                if (cq < ec_begin || cq >= ec_end)
                    continue;
                const int c = cq * 16;
                uint32_t otmp[16];
                const uint32_t *o = o_chunk(cq, otmp);
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
            __syncwarp();
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        tmem_dealloc(tmem, 512);
}

// Merges the parts of the split items: for row t of tail item w with parts
// q = 0..s-1 (slot v = q * tail + w), M = max m_q, a_q = 2^(m_q - M),
// O = (sum a_q O_q) / (sum a_q l_q).  Thread = (row, 8-column group) of one
// item (blockIdx.y = w); every load (the error word, the item header, each
// part's m, l and 8 columns of O) is issued before any is used, so the pass
// costs one round trip to L2, where the parts were just written.
struct FmhaCombineParams {
    const int4 *hdr;
    const float *m, *l, *o;
    void *out;
    long long o_sb, o_sh, o_st;
    int L, hd, hdp, tail, s, out_dtype, out_vec;
    const int *err;
};

// MAXP: the most parts the instance merges (4: 64 registers, four blocks of
// 256 threads per SM, so a two-segment audio layer's 352 blocks fit in one
// wave; 8: twice the registers and blocks).
template <int MAXP>
__global__ void __launch_bounds__(256, MAXP <= 4 ? 4 : 2) fmha_split_combine(const __grid_constant__ FmhaCombineParams c) {
    const int w = blockIdx.y, ng = c.hdp / 8;
    const int unit = blockIdx.x * blockDim.x + threadIdx.x;
    if (unit >= 256 * ng)
        return;
    const int row = unit / ng, c0 = (unit - row * ng) * 8;
    const int e = *c.err;
    const int4 hd4 = c.hdr[w]; // batch, head, first query row, skip
    float mq[MAXP], lq[MAXP];
    float4 oq[MAXP][2];
#pragma unroll
    for (int q = 0; q < MAXP; ++q) {
        if (q < c.s) {
            const int pr = (q * c.tail + w) * 256 + row;
            mq[q] = c.m[pr];
            lq[q] = c.l[pr];
            const float4 *po = reinterpret_cast<const float4 *>(c.o + static_cast<size_t>(pr) * c.hdp + c0);
            oq[q][0] = po[0];
            oq[q][1] = po[1];
        }
    }
    const int t = hd4.z + row;
    // The attention kernel gave up (its parts may be incomplete), a skipped
    // item, rows past the end or columns past the head: nothing to write.
    if (e != 0 || hd4.w || t >= c.L || c0 >= c.hd)
        return;
    float mmax = -INFINITY;
#pragma unroll
    for (int q = 0; q < MAXP; ++q)
        if (q < c.s)
            mmax = fmaxf(mmax, mq[q]);
    float acc[8], l = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        acc[k] = 0.f;
    if (mmax != -INFINITY) {
#pragma unroll
        for (int q = 0; q < MAXP; ++q) {
            if (q < c.s) {
                const float a = exp2f(mq[q] - mmax);
                l = fmaf(a, lq[q], l);
                acc[0] = fmaf(a, oq[q][0].x, acc[0]);
                acc[1] = fmaf(a, oq[q][0].y, acc[1]);
                acc[2] = fmaf(a, oq[q][0].z, acc[2]);
                acc[3] = fmaf(a, oq[q][0].w, acc[3]);
                acc[4] = fmaf(a, oq[q][1].x, acc[4]);
                acc[5] = fmaf(a, oq[q][1].y, acc[5]);
                acc[6] = fmaf(a, oq[q][1].z, acc[6]);
                acc[7] = fmaf(a, oq[q][1].w, acc[7]);
            }
        }
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const long long base = hd4.x * c.o_sb + hd4.y * c.o_sh + static_cast<long long>(t) * c.o_st + c0;
    const bool whole = c.out_vec && c0 + 8 <= c.hd;
    if (c.out_dtype == kOutF32) {
        float *out = static_cast<float *>(c.out) + base;
        if (whole) {
            reinterpret_cast<float4 *>(out)[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
            reinterpret_cast<float4 *>(out)[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
        } else {
            for (int k = 0; k < 8 && c0 + k < c.hd; ++k)
                out[k] = acc[k] * inv;
        }
        return;
    }
    const bool bf = c.out_dtype == kOutBF16;
    uint16_t *out = static_cast<uint16_t *>(c.out) + base;
    uint32_t wv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
        wv[k] = pack2(acc[2 * k] * inv, acc[2 * k + 1] * inv, bf);
    if (whole) {
        *reinterpret_cast<uint4 *>(out) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    } else {
        for (int k = 0; k < 8 && c0 + k < c.hd; ++k)
            out[k] = static_cast<uint16_t>(k & 1 ? wv[k >> 1] >> 16 : wv[k >> 1] & 0xffffu);
    }
}

// ------------------------------------------------------------------ host side
// Builds a 4-D (d, token, head, batch) tiled map with a box of
// box_w x box_rows x 1 x 1 elements.
int make_map(CUtensorMap *map, const void *base, bool bf16, const TensorView &v, int box_w,
             int box_rows, int swizzle_bytes = 0) {
    const uint64_t dims[4] = {static_cast<uint64_t>(v.d), static_cast<uint64_t>(v.tokens),
                              static_cast<uint64_t>(v.heads), static_cast<uint64_t>(v.batch)};
    const uint64_t strides[3] = {static_cast<uint64_t>(v.s_token) * 2,
                                 static_cast<uint64_t>(v.s_head) * 2,
                                 static_cast<uint64_t>(v.s_batch) * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(box_w), static_cast<uint32_t>(box_rows), 1, 1};
    return encode_tiled(map, base, bf16, 4, dims, strides, box, swizzle_bytes);
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

template <int HDP, bool BF16, bool SPLIT> int launch_typed(FmhaParams &p, int grid, cudaStream_t stream) {
    using S = FmhaShape<HDP>;
    static std::atomic<unsigned long long> done{0};
    const cudaError_t attr = set_smem_limit(reinterpret_cast<const void *>(fmha_fwd_kernel<HDP, BF16, SPLIT>),
                                            S::SMEM_BYTES, done);
    if (attr != cudaSuccess)
        return static_cast<int>(attr);
    fmha_fwd_kernel<HDP, BF16, SPLIT><<<grid, kThreads, S::SMEM_BYTES, stream>>>(p);
    return static_cast<int>(cudaGetLastError());
}

// Split slots exist only with bf16 operands (the encoder graphs, which pass
// split scratch); fmha_launch plans a split for bf16 launches only.
template <int HDP> int launch_hdp(FmhaParams &p, bool bf16, int grid, cudaStream_t stream) {
    if (p.split_s > 1)
        return bf16 ? launch_typed<HDP, true, true>(p, grid, stream) : -2;
    return bf16 ? launch_typed<HDP, true, false>(p, grid, stream)
                : launch_typed<HDP, false, false>(p, grid, stream);
}

int fmha_sm_count() {
    static int sms = 0;
    if (!sms) {
        int dev = 0, n = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        sms = n;
    }
    return sms;
}

// Key split of the last round.  N items of up to t_max KV tiles on G CTAs:
// `full` (0 or 1) whole rounds, then `tail` items.  Each tail item is cut into
// s = min(G / tail, t_max, 8) parts; the split pays when the parts save at
// least kSplitMinTiles KV tiles of the last round: a part costs an item
// transition, and the combine pass (about 4 us on B200) reads its rows once
// more, against about 1.3 us per KV tile of 256 x 128 scores saved.  With a
// block window, a part wholly past a row's window leaves that row's max at
// -inf and its sum at 0, which the combine weights by 0.
constexpr int kSplitMinTiles = 6;
constexpr int kSplitHdrBytes = 16384; // int4 per split item: up to 1024 items

struct SplitPlan {
    int s = 1, first = 0, tail = 0, items = 0;
};

SplitPlan split_plan(long long n_items, int t_max, int skip_padded_q) {
    SplitPlan pl;
    const int G = fmha_sm_count();
    if (kSplit || skip_padded_q || n_items <= 0 || t_max <= 1 || G > 1024)
        return pl;
    const long long full = n_items / G, tail = n_items - full * G;
    // After more than one whole round the CTAs' finishing times already
    // spread by about what a split of the last round would save.
    if (tail == 0 || full > 1)
        return pl;
    int s = static_cast<int>(G / tail);
    s = s < t_max ? s : t_max;
    s = s < kSplitMaxParts ? s : kSplitMaxParts;
    if (s < 2 || t_max - (t_max + s - 1) / s < kSplitMinTiles)
        return pl;
    pl.s = s;
    pl.first = static_cast<int>(full * G);
    pl.tail = static_cast<int>(tail);
    pl.items = pl.first + pl.tail * s;
    return pl;
}

size_t split_bytes(int hdp) {
    const size_t G = static_cast<size_t>(fmha_sm_count());
    return kSplitHdrBytes + G * 256 * 4 * 2 + G * 256 * static_cast<size_t>(hdp) * 4;
}

size_t fmha_split_workspace(int batch, int heads, int L, int head_dim, int valid, int block,
                            int skip_padded_q) {
    const int hdp = padded_head_dim(head_dim);
    if (hdp < 0 || batch <= 0 || heads <= 0 || L <= 0)
        return 0;
    const int v = valid > 0 && valid < L ? valid : L;
    const long long n = static_cast<long long>(batch) * heads * ((L + 255) / 256);
    (void)block; // rows of a part past their block window come out as empty parts
    const SplitPlan pl = split_plan(n, (v + 127) / 128, skip_padded_q);
    return pl.s > 1 ? split_bytes(hdp) : 0;
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
            (rc = make_map(&p.tk1, a.k_ptr, a.bf16, a.k, w1, 128)))
            return rc;
    }
    // Row-sum column: V column `d` (first column past the data) holds 1.0 when
    // the PV output has room for it and the data ends on a 16-byte boundary.
    const int hdpo = head_out_cols(hdp);
    const int dv = a.v.d;
    p.ones_col = (hdpo > 64 && dv >= 64 && dv % 8 == 0 && dv < hdpo) ? dv : -1;
    // V's second chunk: TMA loads only the data columns [64, dv), 16-byte
    // granular; the rest of the 64-column atom keeps its zeros (and the ones).
    p.v1_width = dv > 64 ? ((dv - 64 + 7) / 8) * 8 : 0;
    if (p.v1_width > 64)
        p.v1_width = 64;
    // 128-byte swizzle whatever the box width: chunk 1 is a 64-column SW128 atom.
    if (p.v1_width > 0 && (rc = make_map(&p.tv1, a.v_ptr, a.bf16, a.v, p.v1_width, 128, 128)))
        return rc;
    // TMA output: 2-byte outputs whose layout TMA can address (same 16-byte
    // rules as the inputs); the tile geometry is the Q tile's.
    {
        TensorView ov;
        ov.d = a.out_d > 0 ? a.out_d : a.q.d;
        ov.tokens = a.q.tokens;
        ov.heads = a.q.heads;
        ov.batch = a.q.batch;
        ov.s_token = a.o_st;
        ov.s_head = a.o_sh;
        ov.s_batch = a.o_sb > 0 ? a.o_sb : a.o_st * a.q.tokens;
        p.o_tma = 0;
        if (a.out_dtype != kOutF32 && tma_view_ok(a.out, ov) && ov.d % 8 == 0 && ov.d <= hdp) {
            const bool obf = a.out_dtype == kOutBF16;
            if (make_map(&p.to0, a.out, obf, ov, w0, 128) == 0 &&
                (w1 == 0 || make_map(&p.to1, a.out, obf, ov, w1, 128) == 0))
                p.o_tma = (obf == a.bf16) ? 1 : 0; // staging packs with the operand type
        }
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
    // A window at least as long as the sequence limits nothing: no window
    // (which allows the sorted item order and the key split).
    p.block = a.block >= a.q.tokens ? 0 : a.block;
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
    p.sorted = (a.lengths != nullptr && p.block == 0 && a.q.batch > 1 && a.q.batch <= kSortMaxBatch) ? 1 : 0;
    // Persistent grid: one CTA per SM, each looping over (batch, head, 256-row) items.
    const int sms = fmha_sm_count();
    const long long items = static_cast<long long>(p.batch) * p.heads * ((p.L + 255) / 256);
    int grid_x = static_cast<int>(items < sms ? items : sms);
    // Key split of a partial last round (the whole batch when it has fewer
    // items than SMs); the lengths bound each item's tiles by L.
    if (a.split_ws && a.bf16) {
        const int v = a.lengths ? p.L : (p.valid > 0 && p.valid < p.L ? p.valid : p.L);
        const SplitPlan pl = split_plan(items, (v + 127) / 128, p.skip_padded_q);
        if (pl.s > 1 && a.split_ws_bytes >= split_bytes(hdp) &&
            reinterpret_cast<uintptr_t>(a.split_ws) % 256 == 0) {
            const size_t G = static_cast<size_t>(sms);
            char *w = static_cast<char *>(a.split_ws);
            p.split_s = pl.s;
            p.split_first = pl.first;
            p.split_tail = pl.tail;
            p.split_items = pl.items;
            p.split_hdr = reinterpret_cast<int4 *>(w);
            p.split_m = reinterpret_cast<float *>(w + kSplitHdrBytes);
            p.split_l = p.split_m + G * 256;
            p.split_o = p.split_l + G * 256;
            grid_x = sms;
        }
    }
    int rc2 = -2;
    switch (hdp) {
    case 16:
        rc2 = launch_hdp<16>(p, a.bf16, grid_x, stream);
        break;
    case 32:
        rc2 = launch_hdp<32>(p, a.bf16, grid_x, stream);
        break;
    case 64:
        rc2 = launch_hdp<64>(p, a.bf16, grid_x, stream);
        break;
    case 80:
        rc2 = launch_hdp<80>(p, a.bf16, grid_x, stream);
        break;
    case 96:
        rc2 = launch_hdp<96>(p, a.bf16, grid_x, stream);
        break;
    case 128:
        rc2 = launch_hdp<128>(p, a.bf16, grid_x, stream);
        break;
    }
    if (rc2 != 0 || p.split_s <= 1)
        return rc2;
    FmhaCombineParams c{};
    c.hdr = p.split_hdr;
    c.m = p.split_m;
    c.l = p.split_l;
    c.o = p.split_o;
    c.out = p.out;
    c.o_sb = p.o_sb;
    c.o_sh = p.o_sh;
    c.o_st = p.o_st;
    c.L = p.L;
    c.hd = p.hd;
    c.hdp = hdp;
    c.tail = p.split_tail;
    c.s = p.split_s;
    c.out_dtype = p.out_dtype;
    c.out_vec = p.out_vec;
    c.err = p.err;
    const dim3 cgrid(static_cast<unsigned>((256 * (hdp / 8) + 255) / 256), static_cast<unsigned>(p.split_tail));
    if (p.split_s <= 4)
        fmha_split_combine<4><<<cgrid, 256, 0, stream>>>(c);
    else
        fmha_split_combine<kSplitMaxParts><<<cgrid, 256, 0, stream>>>(c);
    return static_cast<int>(cudaGetLastError());
}

} // namespace omni_b200
