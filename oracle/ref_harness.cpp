// ref_harness.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A thin extern "C" wrapper around the reference's own CPU backend
// (omni-tokenizer src/cpu.cpp, compiled unchanged from where it lies in the
// reference checkout; see oracle/Makefile).  The resulting library
// oracle/_ref/libomni_ref_cpu.so is used (a) to pin the C restatement in
// oracle/omni_oracle.c bit-for-bit, (b) to generate tests/golden/ fixtures and
// (c) as the timed CPU baseline of bench.py (cpu_baseline.kind == "reference").
// Nothing in the product library links it.
#include "internal.h" // omni-tokenizer src/internal.h (Ops, Value)
#include <atomic>
#include <cstring>
#include <exception>

namespace {
std::unique_ptr<omni::Ops> &ops() {
    static std::unique_ptr<omni::Ops> instance = omni::make_cpu();
    return instance;
}
} // namespace

extern "C" {
// omni::Ops::attention (src/internal.h:81) on the reference CPU backend.
int ref_attention(const float *q, const float *k, const float *v, float *y, size_t n,
                  size_t cols, size_t heads, size_t block, size_t valid, int fused, int bf16) {
    try {
        auto &o = ops();
        const size_t d = fused ? cols / 3 : cols;
        auto qv = o->upload(q, n, cols, bf16 != 0);
        omni::Value kv, vv;
        if (!fused) {
            kv = o->upload(k, n, d, bf16 != 0);
            vv = o->upload(v, n, d, bf16 != 0);
        }
        auto out = o->download(
            o->attention(qv, fused ? nullptr : &kv, fused ? nullptr : &vv, heads, block, valid,
                         fused != 0));
        std::memcpy(y, out.data(), out.size() * sizeof(float));
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}

// omni::Ops::squares (src/internal.h:86).
int ref_squares(const float *x, float *y, size_t rows, size_t cols, int bf16) {
    try {
        auto &o = ops();
        auto out = o->download(o->squares(o->upload(x, rows, cols, bf16 != 0)));
        std::memcpy(y, out.data(), out.size() * sizeof(float));
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}

// omni::Ops::quantize (src/internal.h:87).  cbnorm is uploaded with the
// profile's rounding, exactly as omni::load does for codebook_norms.
int ref_quantize(const float *x, size_t rows, size_t dim, const float *cb, size_t codes,
                 const float *cbnorm, int bf16, uint16_t *ids) {
    try {
        auto &o = ops();
        auto xv = o->upload(x, rows, dim, bf16 != 0);
        auto cv = o->upload(cb, codes, dim, bf16 != 0);
        auto nv = o->upload(cbnorm, codes, 1, bf16 != 0);
        std::atomic<bool> cancel{false};
        auto out = o->quantize(xv, cv, nv, cancel);
        std::memcpy(ids, out.data(), out.size() * sizeof(uint16_t));
        return 0;
    } catch (const std::exception &) {
        return 1;
    }
}
}
