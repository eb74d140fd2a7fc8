// fmha.h -- host-side interface of the sm_100a attention kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace omni_b200 {

enum : int { kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2 };

// A (d, token, head, batch) view of 2-byte elements; strides in elements.
struct TensorView {
    int d = 0, tokens = 0, heads = 1, batch = 1;
    long long s_token = 0, s_head = 0, s_batch = 0;
};

// Kernel parameters (passed as a __grid_constant__ argument).
struct FmhaParams {
    CUtensorMap tq0, tq1, tk0, tk1, tv0, tv1; // chunk 0 / chunk 1 tile maps
    CUtensorMap to0, to1;                     // output tile maps (when o_tma)
    void *out;
    long long o_sb, o_sh, o_st; // output strides in elements (batch, head, token)
    const int *lengths;         // [batch] valid key counts, or nullptr
    int batch, heads, L, hd;
    int valid; // valid key count when lengths == nullptr
    int block; // block-causal window (0: none)
    int skip_padded_q;
    int out_dtype;
    int out_vec;
    int ones_col; // >= 0: V column holding 1.0 so that O[:, ones_col] = row sum of P
    int o_tma;    // 1: the output is staged in shared memory and written by TMA
    int v1_width; // columns of V's second chunk loaded by TMA (0: none)
    int sorted;   // 1: items of long sequences first, dealt to the CTAs in snake order
    // Split keys: the `split_tail` items of the last, partial
    // round are cut into `split_s` ranges of KV tiles, one CTA each; part v of
    // slot split_first + v writes its unnormalised O rows, row max and row sum
    // to split_o / split_m / split_l and fmha_split_combine merges them.
    int split_s;     // parts per split item (0 or 1: no split)
    int split_first; // first split slot (full rounds x grid)
    int split_tail;  // items that are split
    int split_items; // slots: split_first + split_tail * split_s
    int4 *split_hdr; // [split_tail] (batch, head, first query row, skip)
    float *split_m, *split_l, *split_o; // [part][256], [part][256], [part][256][HDP]
    float scale_log2;
    int *err;
};

// Parameters of the fp32 split-precision kernel (fmha_f32_sm100.cu): tensor
// maps of K and V over fp32 (d, token, head, batch) views with 32-column
// boxes; Q is read row by row (one query row per thread).
struct FmhaF32Params {
    CUtensorMap tk, tv;
    const float *q;
    long long q_sb, q_sh, q_st; // Q strides in elements (batch, head, token)
    int q_d;                    // Q columns present (zero beyond)
    int q_vec;                  // 16-byte loads allowed
    void *out;
    long long o_sb, o_sh, o_st; // output strides in elements (batch, head, token)
    const int *lengths;         // [batch] valid key counts, or nullptr
    int batch, heads, L, hd;
    int valid;
    int block;
    int skip_padded_q;
    int out_dtype;
    int out_vec;
    float scale_log2;
    int *err;
};

struct FmhaArgs {
    const void *q_ptr = nullptr, *k_ptr = nullptr, *v_ptr = nullptr;
    TensorView q, k, v;
    bool bf16 = true; // operand type: bf16 (true) or fp16 (false)
    void *out = nullptr;
    int out_dtype = kOutBF16;
    long long o_sb = 0, o_sh = 0, o_st = 0;
    const int *lengths = nullptr;
    int valid = 0;
    int block = 0;
    int skip_padded_q = 0;
    double scale = 0; // 0: out_d^-1/2
    int out_d = 0;    // output columns per head (0: q.d); the operands may be zero-padded wider
    int *err = nullptr;
    // Scratch for the key split of a partial last round (fmha_split_workspace
    // bytes, 256-byte aligned), or nullptr: no split.
    void *split_ws = nullptr;
    size_t split_ws_bytes = 0;
};

// Returns 0 on success, a CUDA error code, or a negative/1000+ code for an
// unsupported shape / tensor-map failure.
int fmha_launch(const FmhaArgs &args, cudaStream_t stream);

// Bytes of split scratch that fmha_launch uses for `batch` sequences of L
// tokens (keys limited to at most `valid`), `heads` heads of head_dim (16-bit
// operands), or 0 when it would not split (padded-query skip, or a last round
// that is full or too short to gain).
size_t fmha_split_workspace(int batch, int heads, int L, int head_dim, int valid, int block,
                            int skip_padded_q);

// Attention on row-major [batch*n, heads*hd] (fused: [batch*n, 3*heads*hd])
// rows: `batch` sequences of n tokens, keys of sequence b limited to
// lengths[b] (device int32, or nullptr: `valid` for all) and to the block
// window.  Same codes and error text as omni_b200_attention_rows.
size_t attention_rows_workspace(size_t rows, int heads, int head_dim, int dtype, int fused);
int attention_rows(const void *q, const void *k, const void *v, void *out, size_t n, int batch,
                   int heads, int head_dim, size_t block, size_t valid, const int *lengths,
                   int fused, int dtype, int out_dtype, void *workspace, size_t workspace_bytes,
                   cudaStream_t stream, void *split_ws = nullptr, size_t split_ws_bytes = 0);
// Split scratch for attention_rows on 16-bit rows (0 for fp32 or no split).
size_t attention_rows_split_workspace(size_t n, int batch, int heads, int head_dim, size_t block,
                                      size_t valid, int dtype);
bool tma_view_ok(const void *base, const TensorView &v);
int padded_head_dim(int hd);

// fp32 attention with split-precision (3 x tf32) tensor-core products.  The
// views in `args` count fp32 elements; q, k, v must satisfy
// tma_view_ok_f32 (16-byte aligned, strides multiples of 4 elements).  Head
// dims up to 128 (padded to 32, 64 or 128).  Same return codes as fmha_launch.
int fmha_f32_launch(const FmhaArgs &args, cudaStream_t stream);
int padded_head_dim_f32(int hd);
bool tma_view_ok_f32(const void *base, const TensorView &v);

} // namespace omni_b200
