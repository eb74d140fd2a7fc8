/*
 * omni_oracle.c -- CPU restatement of omni-tokenizer's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * omni-tokenizer_b200/csrc; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * library never links or calls it.
 *
 * Every function restates the scalar fp32 semantics of the reference CPU
 * backend (omni-tokenizer src/cpu.cpp) with the SAME reduction order, so that
 * its outputs are bit-identical to the reference's own CPU path.  That claim is
 * pinned by tests/test_oracle.py against oracle/_ref (the reference's cpu.cpp
 * compiled unchanged, see oracle/Makefile) and against the committed golden
 * fixtures in tests/golden/.
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fopenmp (no -march: the x86-64
 * baseline has no FMA instructions, so no expression is contracted, exactly as
 * in the reference's own build).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* omni-tokenizer src/internal.h:128-139 -- RNE fp32 -> bf16 with NaN quieting. */
float oracle_round_bf16(float f) {
    union {
        float f;
        uint32_t u;
    } v;
    v.f = f;
    if ((v.u & 0x7fffffffU) > 0x7f800000U)
        v.u |= 0x00400000U;
    else
        v.u += 0x7fffU + ((v.u >> 16) & 1U);
    v.u &= 0xffff0000U;
    return v.f;
}

static float rb(float x, int bf16) { return bf16 ? oracle_round_bf16(x) : x; }

/* omni-tokenizer src/internal.h:15-18 -- conservative gamma bound for the
 * expanded fp32 L2 distance. */
double oracle_fp32_distance_error_factor(size_t dimension) {
    const double e = ((double)dimension + 4) * 1.1920928955078125e-07; /* FLT_EPSILON */
    return e < 1 ? 2 * e / (1 - e) : INFINITY;
}

/*
 * omni-tokenizer src/cpu.cpp:122-172 (Cpu::attention).
 *
 * q is [n, cols] row-major with cols = d (unfused) or 3d (fused Q|K|V column
 * blocks); k and v are [n, d] and ignored when fused.  Output y is [n, d].
 * Head h uses columns [h*hd, (h+1)*hd).  Query row t sees keys
 * s < limit(t) = min(n, valid[, (t/block+1)*block when block > 0]).
 * Reduction order per (t, h): dot products over j in order, running max,
 * exp-and-sum over keys in order, then output[j] += (score/total) * v[j] in key
 * order.  bf16 outputs are rounded once at the end.
 */
void oracle_attention(const float *q, const float *k, const float *v, float *y, size_t n,
                      size_t cols, size_t heads, size_t block, size_t valid, int fused,
                      int bf16) {
    const size_t d = fused ? cols / 3 : cols, hd = d / heads;
    const float scale = 1 / sqrtf((float)hd);
    const float split_scale = (float)pow((double)hd, -.25);
    const long long tasks = (long long)(n * heads);
#pragma omp parallel
    {
        float *scores = (float *)malloc(sizeof(float) * (n ? n : 1));
#pragma omp for schedule(static)
        for (long long task = 0; task < tasks; ++task) {
            size_t t = (size_t)task / heads, h = (size_t)task % heads;
            size_t limit = n < valid ? n : valid;
            if (block) {
                size_t b = (t / block + 1) * block;
                if (b < limit)
                    limit = b;
            }
            float mx = -INFINITY;
            for (size_t s = 0; s < limit; ++s) {
                float z = 0;
                for (size_t j = 0; j < hd; ++j) {
                    float a = q[t * cols + h * hd + j];
                    float b = fused ? q[s * cols + d + h * hd + j] : k[s * d + h * hd + j];
                    z += fused ? (a * split_scale) * (b * split_scale) : (a * scale) * b;
                }
                scores[s] = z;
                mx = (mx < z) ? z : mx; /* std::max(mx, z): keeps mx on ties and NaN */
            }
            float total = 0;
            for (size_t s = 0; s < limit; ++s) {
                scores[s] = expf(scores[s] - mx);
                total += scores[s];
            }
            float *out = y + t * d + h * hd;
            for (size_t j = 0; j < hd; ++j)
                out[j] = 0.f;
            for (size_t s = 0; s < limit; ++s) {
                const float p = scores[s] / total;
                const float *value = fused ? q + s * cols + 2 * d + h * hd : v + s * d + h * hd;
                for (size_t j = 0; j < hd; ++j)
                    out[j] += p * value[j];
            }
            if (bf16)
                for (size_t j = 0; j < hd; ++j)
                    out[j] = oracle_round_bf16(out[j]);
        }
        free(scores);
    }
}

/*
 * Batched head-major form used by the op-level benchmarks:
 * q, k, v, y are [batch, heads, L, hd]; lengths (may be NULL) gives the valid
 * key count of each batch item (key-padding mask).  Each (batch, head) slice is
 * the reference attention above with heads=1, n=L, valid=lengths[b], so the
 * arithmetic is the reference's, in the same order.
 */
void oracle_attention_bhld(const float *q, const float *k, const float *v, float *y,
                           size_t batch, size_t heads, size_t L, size_t hd,
                           const int32_t *lengths, size_t block) {
    const float scale = 1 / sqrtf((float)hd);
    const long long tasks = (long long)(batch * heads * L);
#pragma omp parallel
    {
        float *scores = (float *)malloc(sizeof(float) * (L ? L : 1));
#pragma omp for schedule(static)
        for (long long task = 0; task < tasks; ++task) {
            size_t t = (size_t)task % L, bh = (size_t)task / L, b = bh / heads;
            size_t valid = lengths ? (size_t)lengths[b] : L;
            size_t limit = L < valid ? L : valid;
            if (block) {
                size_t c = (t / block + 1) * block;
                if (c < limit)
                    limit = c;
            }
            const float *qs = q + (bh * L + t) * hd, *ks = k + bh * L * hd, *vs = v + bh * L * hd;
            float mx = -INFINITY;
            for (size_t s = 0; s < limit; ++s) {
                float z = 0;
                for (size_t j = 0; j < hd; ++j)
                    z += (qs[j] * scale) * ks[s * hd + j];
                scores[s] = z;
                mx = (mx < z) ? z : mx;
            }
            float total = 0;
            for (size_t s = 0; s < limit; ++s) {
                scores[s] = expf(scores[s] - mx);
                total += scores[s];
            }
            float *out = y + (bh * L + t) * hd;
            for (size_t j = 0; j < hd; ++j)
                out[j] = 0.f;
            for (size_t s = 0; s < limit; ++s) {
                const float p = scores[s] / total;
                for (size_t j = 0; j < hd; ++j)
                    out[j] += p * vs[s * hd + j];
            }
        }
        free(scores);
    }
}

/* omni-tokenizer src/cpu.cpp:216-226 (Cpu::squares): per-row sum of
 * (bf16-rounded) squares in column order, rounded once more in bf16. */
void oracle_squares(const float *x, float *y, size_t rows, size_t cols, int bf16) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)rows; ++i) {
        float n = 0;
        for (size_t j = 0; j < cols; ++j)
            n += rb(x[i * cols + j] * x[i * cols + j], bf16);
        y[i] = rb(n, bf16);
    }
}

/*
 * omni-tokenizer src/cpu.cpp:227-287 (Cpu::quantize), with the dot products of
 * src/cpu.cpp:48-70 (Cpu::linear without CBLAS: sequential fp32 sum, rounded to
 * bf16 in the bf16 profile).
 *
 * bf16 profile: dist = r(r(|x|^2 + |c|^2) - r(2*dot)); the first code with
 * the strictly smallest dist wins (smallest id on ties).
 * fp32 profile: approximate dist = fma(-2, dot, |x|^2 + |c|^2) keeps a running
 * best; every code whose approximate dist lies within
 * gamma*(2|x|^2 + |c|^2 + |c_best|^2) of the running best is re-checked with a
 * direct fp64 sum of squared differences; the smallest direct distance wins,
 * smallest id on ties.  Codes are visited in tiles of 256, as in the reference,
 * because the running best used by the candidate filter depends on the tiling.
 *
 * Outputs: ids[rows]; best_out[rows] (optional) = the winning bf16/fp32 dist
 * (bf16 profile) or the winning direct fp64 distance (fp32 profile).
 */
void oracle_quantize(const float *x, size_t rows, size_t dim, const float *cb, size_t codes,
                     const float *cbnorm, int bf16, uint16_t *ids, double *best_out) {
    float *xn = (float *)malloc(sizeof(float) * (rows ? rows : 1));
    oracle_squares(x, xn, rows, dim, bf16);
    const double error_factor = oracle_fp32_distance_error_factor(dim);
    const size_t tile = 256;
#pragma omp parallel
    {
        float *dots = (float *)malloc(sizeof(float) * tile);
#pragma omp for schedule(static)
        for (long long ii = 0; ii < (long long)rows; ++ii) {
            const size_t i = (size_t)ii;
            float best = INFINITY;
            double precise_best = INFINITY;
            uint16_t id = 0, search_id = 0;
            for (size_t base = 0; base < codes; base += tile) {
                size_t n = codes - base < tile ? codes - base : tile;
                for (size_t j = 0; j < n; ++j) {
                    float s = 0;
                    for (size_t z = 0; z < dim; ++z)
                        s += x[i * dim + z] * cb[(base + j) * dim + z];
                    dots[j] = rb(s + 0, bf16);
                }
                for (size_t j = 0; j < n; ++j) {
                    float dot = dots[j], dist;
                    if (bf16) {
                        float sum = oracle_round_bf16(xn[i] + cbnorm[base + j]);
                        dist = oracle_round_bf16(sum - oracle_round_bf16(2 * dot));
                    } else
                        dist = fmaf(-2.f, dot, xn[i] + cbnorm[base + j]);
                    if (dist < best) {
                        best = dist;
                        if (bf16)
                            id = (uint16_t)(base + j);
                        else
                            search_id = (uint16_t)(base + j);
                    }
                }
                if (bf16)
                    continue;
                for (size_t j = 0; j < n; ++j) {
                    const size_t code = base + j;
                    const float distance = fmaf(-2.f, dots[j], xn[i] + cbnorm[code]);
                    const double tolerance =
                        error_factor * (2 * (double)xn[i] + cbnorm[code] + cbnorm[search_id]);
                    if ((double)distance > (double)best + tolerance)
                        continue;
                    double direct = 0;
                    for (size_t k = 0; k < dim; ++k) {
                        const double delta = (double)x[i * dim + k] - cb[code * dim + k];
                        direct += delta * delta;
                    }
                    if (direct < precise_best || (direct == precise_best && code < id)) {
                        precise_best = direct;
                        id = (uint16_t)code;
                    }
                }
            }
            ids[i] = id;
            if (best_out)
                best_out[i] = bf16 ? (double)best : precise_best;
        }
        free(dots);
    }
    free(xn);
}

/*
 * Top-2 distances per row in the reference's own distance metric (the
 * extension that the parity rule "codes identical except where the top-2 gap
 * is below 1e-3 relative" needs).  bf16 profile: the rounded bf16 dist of the
 * formula above; fp32 profile: the direct fp64 distance.  d1 is the minimum,
 * d2 the minimum over every other code (so d2 == d1 on exact ties).
 */
void oracle_quantize_top2(const float *x, size_t rows, size_t dim, const float *cb, size_t codes,
                          const float *cbnorm, int bf16, double *d1, double *d2) {
    float *xn = (float *)malloc(sizeof(float) * (rows ? rows : 1));
    oracle_squares(x, xn, rows, dim, bf16);
#pragma omp parallel for schedule(static)
    for (long long ii = 0; ii < (long long)rows; ++ii) {
        const size_t i = (size_t)ii;
        double a = INFINITY, b = INFINITY;
        for (size_t c = 0; c < codes; ++c) {
            double dist;
            if (bf16) {
                float s = 0;
                for (size_t z = 0; z < dim; ++z)
                    s += x[i * dim + z] * cb[c * dim + z];
                float dot = oracle_round_bf16(s);
                float sum = oracle_round_bf16(xn[i] + cbnorm[c]);
                dist = oracle_round_bf16(sum - oracle_round_bf16(2 * dot));
            } else {
                dist = 0;
                for (size_t k = 0; k < dim; ++k) {
                    const double delta = (double)x[i * dim + k] - cb[c * dim + k];
                    dist += delta * delta;
                }
            }
            if (dist < a) {
                b = a;
                a = dist;
            } else if (dist < b)
                b = dist;
        }
        d1[i] = a;
        d2[i] = b;
    }
    free(xn);
}

/* The deterministic generator of omni-tokenizer tests/native_cpu_attention.cpp:16-23
 * (and tests/native_cuda_attention.cpp:15-22): a 32-bit LCG mapped to [-1, 1). */
void oracle_lcg_values(float *out, size_t count, uint32_t seed) {
    for (size_t i = 0; i < count; ++i) {
        seed = 1664525U * seed + 1013904223U;
        out[i] = (float)((int32_t)(seed >> 8) - 8388608) / 8388608.f;
    }
}
