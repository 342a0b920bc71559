// shim/shim_check.cpp - host-side check of the shim through the reference's own headers (tests/test_shim.py): the
// layout, format and MMQ queries a TinyStrata engine makes before it launches anything, printed as JSON lines, and
// the router's argument error as the reference raises it.  Needs no GPU.
#include "strata/kernels/iq_kernels.hpp"
#include "strata/kernels/native_router.hpp"
#include "strata/gemma4/matvec.hpp"
#include "strata/prefill/moe_mmq.hpp"
#include "gemma4/mmq.hpp"

#include <cstdio>
#include <stdexcept>

int main() {
    using namespace strata::kernels;
    const int cases[][4] = {{18, 18, 2048, 512}, {18, 21, 2048, 512}, {2, 2, 2816, 704}, {12, 14, 2048, 1792},
                            {8, 8, 2048, 512}, {2, 2, 2816, 2112}};
    for (const auto& c : cases) {
        const NativeExpertLayout L = native_expert_layout(c[0], c[1], c[2], c[3]);
        std::printf("{\"kind\": \"layout\", \"gu\": %d, \"d\": %d, \"n_embd\": %d, \"n_ff\": %d, \"gu_row\": %zu, "
                    "\"d_row\": %zu, \"up_off\": %zu, \"down_off\": %zu, \"bytes\": %zu, \"supported\": %d}\n",
                    c[0], c[1], c[2], c[3], L.gu_row, L.d_row, L.up_off, L.down_off, L.bytes,
                    (int) native_expert_supported(c[0], c[1], c[2], c[3]));
    }
    for (int t : {2, 8, 12, 14, 18, 21, 1})
        std::printf("{\"kind\": \"type\", \"t\": %d, \"iq_supported\": %d, \"row_bytes_2048\": %zu, "
                    "\"mmq_supported\": %d}\n",
                    t, (int) iq_supported(t), iq_row_bytes(t, 2048), (int) strata::prefill::mmq::supported(t));
    std::printf("{\"kind\": \"mmq\", \"q8_bytes\": %zu, \"gemma_q8_bytes\": %zu, \"fits\": %d, \"gemma_fits\": %d, "
                "\"scratch\": %zu, \"router_256_8\": %d, \"router_33_8\": %d}\n",
                strata::prefill::mmq::q8_bytes(300, 2048), strata::gemma4::Mmq::q8_bytes(300, 2816),
                (int) strata::prefill::mmq::fits(18, 1024), (int) strata::gemma4::Mmq::fits(2, 1408, 2816),
                native_expert_scratch_bytes(64, 512), (int) native_router_topk_supported(256, 8),
                (int) native_router_topk_supported(33, 8));
    bool threw = false;
    try {
        native_router_topk(nullptr, nullptr, nullptr, 33, 8, 1, nullptr);   // refused before any launch
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    std::printf("{\"kind\": \"router_error\", \"threw\": %d}\n", (int) threw);
    strata::kernels::MmvqSlots slots{};   // a format without a kernel here: false, nothing launched (no GPU needed)
    std::printf("{\"kind\": \"mmvq\", \"ids_q4_0\": %d, \"ids_iq3_xxs\": %d, \"ids_q5_0\": %d, \"slots_q5_0\": %d}\n",
                (int) strata::kernels::gemma_native_mmvq_ids_supported(2),
                (int) strata::kernels::gemma_native_mmvq_ids_supported(18),
                (int) strata::kernels::gemma_native_mmvq_ids_supported(6),
                (int) strata::kernels::gemma_native_mmvq_slots(6, slots, 1, 2048, 64, nullptr));
    return 0;
}
