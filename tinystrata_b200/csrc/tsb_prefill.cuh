// tsb_prefill.cuh - the prefill (many-token) expert path's building blocks: the dispatch of routed entries into
// expert-contiguous rows (the reference's permutation, src/qwen35/q36_engine.cu:486-510), and the tcgen05 / TMEM
// helpers the tensor-core grouped products (tsb_mmq.cuh) issue.
#pragma once

#include "tsb_kernels.cuh"

#include <cuda_fp16.h>

namespace tsb {

// ------------------------------------------------------------------------------------------------ PTX helpers
// Shared-memory matrix descriptor of a K-major operand tile with the 128-byte swizzle: 8-row groups 1 KB apart.
__device__ __forceinline__ uint64_t pf_sdesc(uint32_t addr) {
    return (uint64_t) ((addr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) (1024 >> 4) << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}
// The mbarrier arrives once every tcgen05.mma this thread issued before it has completed.
__device__ __forceinline__ void pf_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// byte offset of the 16-byte chunk c (values 8c..8c+7) of row r inside a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t) ((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}


// ------------------------------------------------------------------------------------------------ dispatch
// bounds[e] = number of entries routed to experts < e (bounds[E] = the entries placed); one CTA.
__global__ void __launch_bounds__(1024) k_dispatch_count(const int32_t* __restrict__ ids, int n_ent, int E,
                                                         int32_t* __restrict__ bounds, int32_t* __restrict__ rinv) {
    __shared__ int32_t cnt[1024];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_ent; i += blockDim.x) {
        const int id = ids[i];
        if (id >= 0 && id < E) atomicAdd(&cnt[id], 1);
        rinv[i] = -1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int e = 0; e < E; ++e) {
            const int c = cnt[e];
            bounds[e] = s;
            s += c;
        }
        bounds[E] = s;
    }
}
// One CTA per expert: its entries in entry order (a stable sort by expert) -> rows bounds[e]...; row_ent[row] = entry,
// row_tok[row] = entry / K, rinv[entry] = row.  Each of the 32 warps owns a contiguous segment of the entries and scans
// it twice with coalesced loads: once to count the expert's entries (ballots), then, after an exclusive scan of the 32
// warp counts, to write them in order (a lane's rank is the popcount of the lanes below it in its ballot).
__global__ void __launch_bounds__(1024) k_dispatch_scatter(const int32_t* __restrict__ ids, int n_ent, int K,
                                                           const int32_t* __restrict__ bounds,
                                                           int32_t* __restrict__ row_ent, int32_t* __restrict__ row_tok,
                                                           int32_t* __restrict__ rinv) {
    __shared__ int32_t wbase[33];
    const int e = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seg = (n_ent + 32 * 32 - 1) / (32 * 32) * 32;   // entries a warp owns (a multiple of 32)
    const int lo = warp * seg, hi = min(lo + seg, n_ent);
    int cnt = 0;
    for (int i0 = lo; i0 < hi; i0 += 32) {
        const int i = i0 + lane;
        cnt += __popc(__ballot_sync(0xffffffffu, i < hi && __ldg(ids + i) == e));
    }
    if (lane == 0) wbase[warp + 1] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        wbase[0] = bounds[e];
        for (int w = 0; w < 32; ++w) wbase[w + 1] += wbase[w];
    }
    __syncthreads();
    int base = wbase[warp];
    const unsigned below = (1u << lane) - 1u;
    for (int i0 = lo; i0 < hi && base < wbase[warp + 1]; i0 += 32) {
        const int i = i0 + lane;
        const bool f = i < hi && __ldg(ids + i) == e;
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (f) {
            const int row = base + __popc(m & below);
            row_ent[row] = i;
            row_tok[row] = i / K;
            rinv[i] = row;
        }
        base += __popc(m);
    }
}

}  // namespace tsb
