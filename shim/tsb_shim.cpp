// shim/tsb_shim.cpp - the reference's expert-layer C++ entry points defined over libtsb_moe.so's C ABI, so that
// TinyStrata's engines link against the B200 path with their call sites unchanged.  Compiled against the
// reference's own headers (include/strata/..., src/gemma4/mmq.hpp), which pin every signature; a maintainer adds it to
// the engine target in place of the reference's definitions (src/kernels/cuda/iq_kernels.cu, native_router.cu,
// src/gemma4/kernels.cu, src/gemma4/matvec.cu, src/gemma4/mmq.cu, src/prefill/moe_mmq.cu for the functions below).
//
// Error behaviour is the reference's: iq_kernels.cu prints and exits on a bad launch, native_router.cu and the MMQ
// wrappers throw std::runtime_error / std::invalid_argument; the C ABI's status is turned back into that.
#include "strata/kernels/iq_kernels.hpp"
#include "strata/kernels/native_router.hpp"
#include "strata/gemma4/kernels.hpp"
#include "strata/gemma4/matvec.hpp"
#include "strata/prefill/moe_mmq.hpp"
#include "gemma4/mmq.hpp"
#include "tsb_moe.h"

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

namespace {

void die(int rc, const char* what) {   // iq_kernels.cu:31-34: print and exit
    if (rc == TSB_OK) return;
    std::fprintf(stderr, "%s: %s\n", what, tsb_last_error());
    std::exit(1);
}
void raise(int rc, const char* what) {   // the MMQ wrappers and gemma4 kernels throw
    if (rc == TSB_OK) return;
    throw std::runtime_error(std::string(what) + ": " + tsb_last_error());
}
tsb_expert_layout to_c(const strata::kernels::NativeExpertLayout& L) {
    tsb_expert_layout c{};
    c.gu_type = L.gu_type;
    c.d_type = L.d_type;
    c.n_embd = L.n_embd;
    c.n_ff = L.n_ff;
    c.gu_row = L.gu_row;
    c.d_row = L.d_row;
    c.up_off = L.up_off;
    c.down_off = L.down_off;
    c.bytes = L.bytes;
    return c;
}

}  // namespace

// ------------------------------------------------------------------------------- include/strata/kernels/iq_kernels.hpp
namespace strata::kernels {

bool iq_supported(int ggml_type) noexcept { return tsb_type_supported(ggml_type) == 1; }

size_t iq_row_bytes(int ggml_type, int64_t n) noexcept {
    const int64_t b = tsb_row_bytes(ggml_type, n);
    return b > 0 ? (size_t) b : 0;
}

void quantize_q8_1_rows(const float* x, int64_t n_rows, int64_t n_cols, void* y, void* stream) {
    die(tsb_quantize_q8_1_rows(x, n_rows, n_cols, y, stream), "quantize_q8_1_rows");
}

NativeExpertLayout native_expert_layout(int gu_type, int d_type, int64_t n_embd, int64_t n_ff) {
    tsb_expert_layout c{};
    NativeExpertLayout L;
    if (tsb_native_expert_layout(gu_type, d_type, n_embd, n_ff, &c) != TSB_OK) return L;   // the reference: all zero
    L.gu_type = c.gu_type;
    L.d_type = c.d_type;
    L.n_embd = c.n_embd;
    L.n_ff = c.n_ff;
    L.gu_row = (size_t) c.gu_row;
    L.d_row = (size_t) c.d_row;
    L.up_off = (size_t) c.up_off;
    L.down_off = (size_t) c.down_off;
    L.bytes = (size_t) c.bytes;
    L.tail_off = 0;
    return L;
}

bool native_expert_supported(int gu_type, int d_type, int64_t n_embd, int64_t n_ff) noexcept {
    return tsb_native_expert_supported(gu_type, d_type, n_embd, n_ff) == 1;
}

size_t native_expert_scratch_bytes(int64_t cap_entries, int64_t n_ff) {
    return (size_t) tsb_native_expert_scratch_bytes(cap_entries, n_ff);
}

void native_expert_grouped(const NativeExpertLayout& L, const unsigned long long* grp_ptr, const int32_t* grp_start,
                           const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok, int64_t cap_groups,
                           int64_t cap_entries, const void* x_q8_1, void* scratch, float* out, void* stream,
                           int64_t grid_groups) {
    const tsb_expert_layout c = to_c(L);
    die(tsb_native_expert_grouped(&c, (const uint64_t*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok, cap_groups,
                                  cap_entries, x_q8_1, scratch, out, stream, grid_groups),
        "native_expert_grouped");
}

// ----------------------------------------------------------------------------- include/strata/kernels/native_router.hpp
bool native_router_topk_supported(int n_expert, int k) {
    return n_expert >= 32 && n_expert % 32 == 0 && n_expert <= 512 && k >= 1 && k <= 32 && k <= n_expert;
}

void native_router_topk(const float* logits, int32_t* ids, float* weights, int n_expert, int k, int n_tok,
                        void* stream) {
    if (tsb_native_router_topk(logits, ids, weights, n_expert, k, n_tok, n_expert, stream) != TSB_OK)
        throw std::invalid_argument(tsb_last_error());   // native_router.cu:103-110
}

// ------------------------------------------------------------------------------ include/strata/gemma4/matvec.hpp
// The cached-expert decode products: false (nothing launched) for a format without a kernel here, as the reference.
bool gemma_native_mmvq_slots(int ggml_type, const MmvqSlots& slots, int count, int n_in, int n_out, void* stream) {
    if (tsb_mmvq_supported(ggml_type) != 1) return false;
    tsb_mmvq_slots s{};
    for (int i = 0; i < count && i < kMmvqSlotsMax; ++i) {
        s.w[i] = slots.w[i];
        s.x[i] = slots.x[i];
        s.y[i] = slots.y[i];
    }
    const int rc = tsb_mmvq_run_slots(ggml_type, &s, count, n_in, n_out, stream);
    if (rc == TSB_ERR_UNSUPPORTED) return false;
    die(rc, "gemma_native_mmvq_slots");
    return true;
}

bool gemma_native_mmvq_ids_supported(int ggml_type) { return tsb_mmvq_supported(ggml_type) == 1; }

bool gemma_native_mmvq_ids(int ggml_type, const MmvqIds& ids, int count, int n_in, int n_out, void* stream) {
    if (tsb_mmvq_supported(ggml_type) != 1) return false;
    tsb_mmvq_ids m{};
    m.table = ids.table;
    m.ids = ids.ids;
    m.offset = ids.offset;
    m.x = ids.x;
    m.x_stride = ids.x_stride;
    m.x_every = ids.x_every;
    m.y = ids.y;
    m.y_stride = ids.y_stride;
    const int rc = tsb_mmvq_run_ids(ggml_type, &m, count, n_in, n_out, stream);
    if (rc == TSB_ERR_UNSUPPORTED) return false;
    die(rc, "gemma_native_mmvq_ids");
    return true;
}

}  // namespace strata::kernels

// ------------------------------------------------------------------------------- include/strata/gemma4/kernels.hpp
namespace strata::gemma4 {

void route_rows(const float* logits, int n_expert, int n_used, int rows, int gate, float in_scale, const float* bias,
                const float* escale, bool norm, float w_scale, int32_t* ids, float* w, void* stream) {
    raise(tsb_route_rows(logits, n_expert, n_used, rows, gate, in_scale, bias, escale, norm ? 1 : 0, w_scale, ids, w,
                         stream),
          "route_rows");
}

void moe_sum(const float* x, const float* w, float* acc, int n, int n_used, int rows, void* stream) {
    raise(tsb_moe_sum(x, w, acc, n, n_used, rows, stream), "moe_sum");
}

void add_scaled(const ScaledRows& rows, int count, int n, void* stream) {
    tsb_scaled_rows r{};
    for (int k = 0; k < count && k < 32; ++k) {
        r.x[k] = rows.x[k];
        r.acc[k] = rows.acc[k];
        r.w[k] = rows.w[k];
    }
    raise(tsb_add_scaled(&r, count, n, stream), "add_scaled");
}

// ----------------------------------------------------------------------------------------------- src/gemma4/mmq.hpp
Mmq::Mmq() = default;
Mmq::~Mmq() = default;

bool Mmq::fits(int ggml_type, int64_t w_rows, int64_t w_cols) {
    tsb_expert_layout c{};
    // the tensor-core product takes a matrix as the down rows of an expert of n_ff = w_cols, n_embd = w_rows
    return tsb_native_expert_layout(ggml_type, ggml_type, w_rows, w_cols, &c) == TSB_OK && w_rows % 64 == 0 &&
           w_rows >= 128 && w_cols % 64 == 0 && tsb_row_bytes(ggml_type, w_cols) > 0;
}

size_t Mmq::q8_bytes(int64_t rows, int64_t cols) { return (size_t) tsb_mmq_act_bytes(rows, cols); }

void Mmq::quantize(const float* x, const int32_t* ids, void* xq, int ggml_type, int64_t cols, int64_t ld, int64_t rows,
                   void* stream) {
    (void) ggml_type;   // one activation layout serves every weight type
    if (rows <= 0) return;
    raise(tsb_mmq_quantize(x, ld, ids, (int) rows, (int) cols, xq, stream), "mmq quantize");
}

void Mmq::mul(const void* w, int ggml_type, int64_t w_rows, int64_t w_cols, size_t stride, int n, const void* xq,
              const int32_t* bounds, const int32_t* ids, int64_t total_rows, int64_t max_rows, float* dst,
              int64_t ld_dst, void* stream) {
    if (n <= 0 || max_rows <= 0) return;
    raise(tsb_mmq_product(w, ggml_type, w_rows, w_cols, stride, n, xq, bounds, ids, total_rows, dst, ld_dst, stream),
          "mmq product");
}

}  // namespace strata::gemma4

// --------------------------------------------------------------------------- include/strata/prefill/moe_mmq.hpp
namespace strata::prefill::mmq {

bool built() { return true; }

bool supported(int ggml_type) {
    return ggml_type == 2 || ggml_type == 8 || ggml_type == 12 || ggml_type == 14 || ggml_type == 18 ||
           ggml_type == 21;   // Q4_0, Q8_0, Q4_K, Q6_K, IQ3_XXS, IQ3_S
}

bool fits(int ggml_type, int64_t w_rows) { return supported(ggml_type) && w_rows % 64 == 0 && w_rows >= 128; }

size_t q8_bytes(int64_t rows, int64_t cols) { return (size_t) tsb_mmq_act_bytes(rows, cols); }

void quantize(const float* x, const int32_t* ids, void* xq, int ggml_type, int64_t cols, int64_t ld, int64_t rows,
              void* stream, float* yscale) {
    (void) ggml_type;
    if (yscale) throw std::runtime_error("mmq quantize: NVFP4 activations are not built");
    if (rows <= 0) return;
    raise(tsb_mmq_quantize(x, ld, ids, (int) rows, (int) cols, xq, stream), "mmq quantize");
}

Context::Context() = default;
Context::~Context() = default;

void Context::run(const Product& p, void* stream) {
    if (p.y_scale) throw std::runtime_error("mmq: NVFP4 activations are not built");
    if (p.n <= 0 || p.max_rows <= 0) return;
    raise(tsb_mmq_product(p.w, p.type, p.w_rows, p.w_cols, p.expert_bytes, p.n, p.xq, p.bounds, p.ids, p.total_rows,
                          p.dst, p.ld_dst, stream),
          "mmq product");
}

}  // namespace strata::prefill::mmq
