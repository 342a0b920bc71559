// tsb_prefill_k.cuh - byte access into GGUF weight rows for the tensor-core products' producers (tsb_mmq.cuh): rows of
// 2-byte aligned blocks read as aligned words, fp16 scale fields, single bytes of a word array.
#pragma once

#include "tsb_prefill.cuh"

namespace tsb {

// ------------------------------------------------------------------------------------------------ byte access
// NW little-endian words from a 2-byte aligned address: aligned loads and funnel shifts.  Reads no aligned word past
// the one holding the last byte asked for.
template <int NW>
__device__ __forceinline__ void ldw(const uint8_t* p, uint32_t (&o)[NW]) {
    const uint32_t* a = (const uint32_t*) ((uintptr_t) p & ~(uintptr_t) 3);
    const uint32_t sh = ((uint32_t) (uintptr_t) p & 3u) * 8u;
    uint32_t w[NW + 1];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = __ldg(a + i);
    w[NW] = sh ? __ldg(a + NW) : 0u;
#pragma unroll
    for (int i = 0; i < NW; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}
__device__ __forceinline__ uint32_t ldh(const uint8_t* p) { return __ldg((const unsigned short*) p); }   // 2-aligned
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short) (bits & 0xFFFFu))); }
__device__ __forceinline__ uint32_t byte_of(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xFFu; }

}  // namespace tsb
