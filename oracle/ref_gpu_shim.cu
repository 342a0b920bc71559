// oracle/ref_gpu_shim.cu - TEST INFRASTRUCTURE: a C face on TinyStrata's own decode CUDA kernels, compiled from the
// reference sources in place for sm_100a (oracle/Makefile `ref-gpu`) into oracle/_ref/libtsb_ref_gpu.so.  The GPU
// parity tests run these beside the product kernels on the same device buffers; nothing here is product code.
//
// Wrapped reference entry points (TinyStrata tree):
//   native_router_topk ........ include/strata/kernels/native_router.hpp:5-6 (native_router.cu:98-111)
//   quantize_q8_1_rows ........ include/strata/kernels/iq_kernels.hpp:24
//   iq_mmvq ................... include/strata/kernels/iq_kernels.hpp:27
//   native_expert_layout ...... include/strata/kernels/iq_kernels.hpp:53
//   native_expert_grouped ..... include/strata/kernels/iq_kernels.hpp:75-78
//   k_moe_out_small ........... src/qwen35/q36_kernels.cuh:252-290 (header-only kernel, instantiated here)
//   route_rows, moe_sum, add_scaled ... include/strata/gemma4/kernels.hpp:43-56 (src/gemma4/kernels.cu)
#include "strata/gemma4/kernels.hpp"
#include "strata/kernels/iq_kernels.hpp"
#include "strata/kernels/native_router.hpp"
#include "q36_kernels.cuh"

#include <cuda_runtime.h>
#include <exception>

namespace sk = strata::kernels;

extern "C" {

int ref_route_rows(const float* logits, int n_expert, int n_used, int rows, int gate, float in_scale, const float* bias,
                   const float* escale, int norm, float w_scale, int32_t* ids, float* w, void* stream) {
    try {
        strata::gemma4::route_rows(logits, n_expert, n_used, rows, gate, in_scale, bias, escale, norm != 0, w_scale,
                                   ids, w, stream);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

void ref_moe_sum(const float* x, const float* w, float* acc, int n, int n_used, int rows, void* stream) {
    strata::gemma4::moe_sum(x, w, acc, n, n_used, rows, stream);
}

int ref_add_scaled(const float* const* x, float* const* acc, const float* w, int count, int n, void* stream) {
    strata::gemma4::ScaledRows r{};
    for (int k = 0; k < count && k < 32; ++k) {
        r.x[k] = x[k];
        r.acc[k] = acc[k];
        r.w[k] = w[k];
    }
    try {
        strata::gemma4::add_scaled(r, count, n, stream);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

int ref_native_router_topk(const float* logits, int32_t* ids, float* w, int n_expert, int k, int n_tok, void* stream) {
    try {
        sk::native_router_topk(logits, ids, w, n_expert, k, n_tok, stream);
    } catch (const std::exception&) {
        return -1;
    }
    return 0;
}

void ref_quantize_q8_1_rows(const float* x, int64_t n_rows, int64_t n_cols, void* y, void* stream) {
    sk::quantize_q8_1_rows(x, n_rows, n_cols, y, stream);
}

void ref_iq_mmvq(int type, const void* w, const void* x_q8_1, float* y, int n_in, int n_out, int ncols, void* stream) {
    sk::iq_mmvq(type, w, x_q8_1, y, n_in, n_out, ncols, stream);
}

size_t ref_native_expert_bytes(int gu_type, int d_type, int64_t n_embd, int64_t n_ff) {
    return sk::native_expert_layout(gu_type, d_type, n_embd, n_ff).bytes;
}

size_t ref_native_expert_scratch_bytes(int64_t cap_entries, int64_t n_ff) {
    return sk::native_expert_scratch_bytes(cap_entries, n_ff);
}

void ref_native_expert_grouped(int gu_type, int d_type, int64_t n_embd, int64_t n_ff,
                               const unsigned long long* grp_ptr, const int32_t* grp_start, const int32_t* n_groups,
                               const int32_t* ent_dst, const int32_t* ent_tok, int64_t cap_groups, int64_t cap_entries,
                               const void* x_q8_1, void* scratch, float* out, void* stream) {
    const sk::NativeExpertLayout L = sk::native_expert_layout(gu_type, d_type, n_embd, n_ff);
    sk::native_expert_grouped(L, grp_ptr, grp_start, n_groups, ent_dst, ent_tok, cap_groups, cap_entries, x_q8_1,
                              scratch, out, stream, 0);
}

// x += sum_k w_k part_k + sigmoid(sgate) shared; h = rms(x) * wn; hq = q8_1(h).  One block per token (T <= 8).
void ref_moe_out_small(float* x, const float* parts, const int32_t* prow, const float* wts, int K, const float* shared,
                       const float* sgate, int sg_stride, const float* wn, float* h, int n, float eps, void* hq,
                       int n_tok, void* stream) {
    q36k::k_moe_out_small<<<n_tok, 1024, 0, (cudaStream_t) stream>>>(x, parts, prow, wts, K, shared, sgate, sg_stride, wn,
                                                                     h, n, eps, (q36k::QB*) hq);
}

int ref_last_cuda_error() { return (int) cudaGetLastError(); }

}  // extern "C"
