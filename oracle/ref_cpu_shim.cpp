// oracle/ref_cpu_shim.cpp - TEST INFRASTRUCTURE: a C face on TinyStrata's own CPU expert kernels, compiled from the
// reference sources in place (oracle/Makefile) into oracle/_ref/libtsb_ref_cpu.so.  Used to pin the oracle's
// codebook decode against the reference's compiled arithmetic and as the timed CPU baseline.  Nothing here is
// product code.
//
// Wrapped reference functions (TinyStrata tree):
//   q8k_quant_avx2 ............ src/kernels/cpu/iq_avx2.cpp:393 (ggml's quantize_row_q8_K, byte-identical)
//   iq512_gu_rows / iq512_rows  src/kernels/cpu/iq_avx512.cpp:245-262 (AVX-512 multi-token IQ rows, Q8_K acts)
//   iq256_gu_rows / iq256_rows  src/kernels/cpu/iq_avx2.cpp:527-535 (the AVX2 copy, same integer sums)
//   kq256_gu_rows / kq256_rows  src/kernels/cpu/kq_avx2.cpp (Q4_K gate/up, Q8_0 down, bit-exact vs ggml AVX2)
//   cpu_avx512_ok / cpu_avx2_ok src/kernels/cpu/cpu_features.cpp
#include "strata/kernels/cpu/cpu_features.hpp"
#include "strata/kernels/cpu/iq_avx2.hpp"
#include "strata/kernels/cpu/iq_avx512.hpp"
#include "strata/kernels/cpu/kq_avx2.hpp"

#include <cstddef>
#include <cstdint>
#include <algorithm>

namespace cpu = strata::kernels::cpu;

// iq_avx512.hpp / iq_avx2.hpp declare these; the reference defines them in native_expert.cpp (which needs ggml-cpu,
// absent here).  The same answers: the formats each kernel file implements.
namespace strata::kernels::cpu {
bool iq512_supported(int t) noexcept { return t == 16 || t == 17 || t == 18 || t == 21 || t == 22; }
bool iq256_supported(int t) noexcept { return t == 16 || t == 17 || t == 18 || t == 21 || t == 22 || t == 23; }
bool kq256_supported(int t) noexcept { return t == 12 || t == 7 || t == 8; }
}  // namespace strata::kernels::cpu

extern "C" {

int ref_cpu_isa() { return cpu::cpu_avx512_ok() ? 512 : cpu::cpu_avx2_ok() ? 256 : 0; }

void ref_q8k_quant(const float* x, void* y, int64_t n) { cpu::q8k_quant_avx2(x, y, n); }

// ff[t][r] = silu(gate_r . a[t]) * (up_r . a[t]) for rows [r0, r1)
int ref_gu_rows(int type, const uint8_t* blob, size_t gu_row, size_t up_off, int n, const void* const* act, int nt,
                float* const* ff, int r0, int r1) {
    if (type == 12) { cpu::kq256_gu_rows(type, blob, gu_row, up_off, n, act, nt, ff, r0, r1); return 0; }
    if (cpu::cpu_avx512_ok() && cpu::iq512_supported(type)) {
        cpu::iq512_gu_rows(type, blob, gu_row, up_off, n, act, nt, ff, r0, r1);
        return 0;
    }
    if (cpu::cpu_avx2_ok() && cpu::iq256_supported(type)) {
        cpu::iq256_gu_rows(type, blob, gu_row, up_off, n, act, nt, ff, r0, r1);
        return 0;
    }
    return -1;
}

// out[t][r] = w_r . a[t] for rows [r0, r1)
int ref_rows(int type, const uint8_t* w, size_t row_bytes, int n, const void* const* act, int nt, float* const* out,
             int r0, int r1) {
    if (type == 12 || type == 8 || type == 7) { cpu::kq256_rows(type, w, row_bytes, n, act, nt, out, r0, r1); return 0; }
    if (cpu::cpu_avx512_ok() && cpu::iq512_supported(type)) {
        cpu::iq512_rows(type, w, row_bytes, n, act, nt, out, r0, r1);
        return 0;
    }
    if (cpu::cpu_avx2_ok() && cpu::iq256_supported(type)) {
        cpu::iq256_rows(type, w, row_bytes, n, act, nt, out, r0, r1);
        return 0;
    }
    return -1;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------------
// The timed CPU baseline: TinyStrata's CPU expert path for decode tokens (call stack E, q36_engine.cu:3088 ->
// ExpertPool::run_split_multi_native, src/kernels/cpu/pool.cpp:773-817), driven by a fixed pool of worker threads in
// the pool's phases: Q8_K of the token, gate/up + SwiGLU rows split over the workers, Q8_K of each expert's hidden
// vector, down rows split over the workers, then the weighted sum.  The row kernels are the reference's own.
#include <atomic>
#include <barrier>
#include <chrono>
#include <functional>
#include <thread>
#include <vector>
#include <cstring>

namespace {
constexpr size_t kQ8K = 292;   // block_q8_K: float d, 256 int8, 16 int16 sums
}

extern "C" double ref_cpu_moe_decode(int gu_type, int d_type, const uint8_t* blobs, size_t blob_bytes, int n_embd,
                                     int n_ff, size_t gu_row, size_t d_row, const int32_t* ids, const float* w, int K,
                                     const float* x, int n_tok, float* out, int n_threads) {
    const size_t up_off = gu_row * (size_t) n_ff, down_off = 2 * up_off;
    std::vector<uint8_t> xq((size_t) n_embd / 256 * kQ8K);
    std::vector<float> ff((size_t) K * n_ff);
    std::vector<uint8_t> hq((size_t) K * (n_ff / 256) * kQ8K);
    std::vector<float> parts((size_t) K * n_embd);
    std::barrier sync(n_threads);
    std::atomic<int> tok{0};
    auto worker = [&](int tid) {
        for (int t = 0; t < n_tok; ++t) {
            const int32_t* id = ids + (size_t) t * K;
            if (tid == 0) cpu::q8k_quant_avx2(x + (size_t) t * n_embd, xq.data(), n_embd);
            sync.arrive_and_wait();
            {   // gate/up rows: (expert, row) pairs split evenly
                const long total = (long) K * n_ff, lo = total * tid / n_threads, hi = total * (tid + 1) / n_threads;
                for (long i = lo; i < hi;) {
                    const int k = (int) (i / n_ff), r0 = (int) (i % n_ff);
                    const int r1 = (int) std::min<long>(n_ff, r0 + (hi - i));
                    const void* act = xq.data();
                    float* f = ff.data() + (size_t) k * n_ff;
                    ref_gu_rows(gu_type, blobs + (size_t) id[k] * blob_bytes, gu_row, up_off, n_embd, &act, 1, &f, r0, r1);
                    i += r1 - r0;
                }
            }
            sync.arrive_and_wait();
            for (int k = tid; k < K; k += n_threads)
                cpu::q8k_quant_avx2(ff.data() + (size_t) k * n_ff, hq.data() + (size_t) k * (n_ff / 256) * kQ8K, n_ff);
            sync.arrive_and_wait();
            {   // down rows
                const long total = (long) K * n_embd, lo = total * tid / n_threads, hi = total * (tid + 1) / n_threads;
                for (long i = lo; i < hi;) {
                    const int k = (int) (i / n_embd), r0 = (int) (i % n_embd);
                    const int r1 = (int) std::min<long>(n_embd, r0 + (hi - i));
                    const void* act = hq.data() + (size_t) k * (n_ff / 256) * kQ8K;
                    float* o = parts.data() + (size_t) k * n_embd;
                    ref_rows(d_type, blobs + (size_t) id[k] * blob_bytes + down_off, d_row, n_ff, &act, 1, &o, r0, r1);
                    i += r1 - r0;
                }
            }
            sync.arrive_and_wait();
            {   // weighted sum in pick order
                const int lo = n_embd * tid / n_threads, hi = n_embd * (tid + 1) / n_threads;
                const float* wt = w + (size_t) t * K;
                for (int i = lo; i < hi; ++i) {
                    float acc = wt[0] * parts[i];
                    for (int k = 1; k < K; ++k) acc += wt[k] * parts[(size_t) k * n_embd + i];
                    out[(size_t) t * n_embd + i] = acc;
                }
            }
            sync.arrive_and_wait();
        }
    };
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> th;
    for (int i = 1; i < n_threads; ++i) th.emplace_back(worker, i);
    worker(0);
    for (auto& t : th) t.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}
