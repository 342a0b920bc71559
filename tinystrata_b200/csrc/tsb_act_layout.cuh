// tsb_act_layout.cuh - the activations' tensor-core layout (tsb_mmq_act_bytes): int8 codes [rows][K], then fp32 d
// [rows][ldS] and d * sum(codes) [rows][ldS], ldS = K / 32 rounded up to 4 (16-byte rows for the scale tiles' TMA),
// each part on 256 bytes.  Shared by every translation unit that writes or reads such a buffer.
#pragma once
#include <cstdint>

namespace tsb {

struct MmqView {
    int8_t* codes;
    float* d;
    float* s;
    int ldS;
};
static inline int mmq_lds(int64_t K) { return (int) ((K / 32 + 3) / 4 * 4); }
static inline uint64_t al256(uint64_t v) { return (v + 255) & ~255ull; }
static inline MmqView mmq_view(const void* base, int64_t rows, int64_t K) {
    MmqView v;
    v.ldS = mmq_lds(K);
    uint8_t* b = (uint8_t*) base;
    v.codes = (int8_t*) b;
    v.d = (float*) (b + al256((uint64_t) rows * K));
    v.s = (float*) (b + al256((uint64_t) rows * K) + al256((uint64_t) rows * v.ldS * 4));
    return v;
}
static inline uint64_t mmq_act_bytes(int64_t rows, int64_t K) {
    return al256((uint64_t) rows * K) + 2 * al256((uint64_t) rows * mmq_lds(K) * 4);
}

}  // namespace tsb
