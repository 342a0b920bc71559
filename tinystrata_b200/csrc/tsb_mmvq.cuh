// tsb_mmvq.cuh - many small quantised matrix-vector products in one launch: up to 32 matrices of one format and shape,
// each times its own q8_1 activation column (the Gemma 4 / LFM2 engines' cached-expert decode step,
// include/strata/gemma4/matvec.hpp:143-171, gemma_native_mmvq_slots / gemma_native_mmvq_ids).
//
// One CTA column per matrix (blockIdx.y), eight warps a CTA, a warp per output row at a time: the activation's calls
// are loaded into registers once per warp, then each row is the row dot of the grouped expert kernels (the calls
// k = lane + 32 j, the per-lane sums, the xor tree: the reference's row_dot order, iq_kernels.cu:715-735), so a value
// equals the reference's iq_mmvq for the same row and column.  With ids, the matrices, the columns and the outputs are
// found on the device (a decode step's routed experts, nothing of the host).
#pragma once

#include "tsb_kernels.cuh"

namespace tsb {

constexpr int kMvMax = 32;   // matrices per launch (kMmvqSlotsMax)

struct MvArgs {
    const void* w[kMvMax];
    const void* x[kMvMax];
    float* y[kMvMax];
    // ids mode: matrix j = table[ids[j]] + offset, column x + (j / x_every) x_stride bytes, output y + j y_stride floats
    const void* const* table;
    const int32_t* ids;
    uint64_t offset;
    const uint8_t* xb;
    uint64_t x_stride;
    int x_every;
    float* yb;
    uint64_t y_stride;
    int by_ids;
    int n_in, n_out;
    uint32_t row_bytes;
};

template <int TY, int J>
__global__ void __launch_bounds__(256) k_mmvq(MvArgs a) {
    extern __shared__ __align__(128) uint8_t mv_tab[];
    build_tables<TY>(mv_tab);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const IqTab tab = make_tab(mv_tab, lane);
    const int j = blockIdx.y;
    const uint8_t* W;
    const BlockQ8_1* x;
    float* y;
    if (a.by_ids) {
        W = (const uint8_t*) a.table[__ldg(a.ids + j)] + a.offset;
        x = (const BlockQ8_1*) (a.xb + (uint64_t) (j / a.x_every) * a.x_stride);
        y = a.yb + (uint64_t) j * a.y_stride;
    } else {
        W = (const uint8_t*) a.w[j];
        x = (const BlockQ8_1*) a.x[j];
        y = a.y[j];
    }
    const int C = a.n_in / Fmt<TY>::qk * Fmt<TY>::cpb;
    typename Fmt<TY>::Act act[1][J];
    auto src = [&](int blk) { return qb_from_global(x + blk); };
#pragma unroll
    for (int jj = 0; jj < J; ++jj) {
        const int k = lane + 32 * jj;
        if (k < C) act[0][jj] = Fmt<TY>::act(src, k);
    }
    for (int r = blockIdx.x * 8 + warp; r < a.n_out; r += gridDim.x * 8) {
        float s[1];
        row_dot<TY, J, 1>(W + (size_t) r * a.row_bytes, C, lane, act, 1, tab, s);
        if (lane == 0) y[r] = s[0];
    }
}

}  // namespace tsb
