// tsb_device.cuh - device building blocks of the B200 MoE expert path: the arithmetic the reference's fast-math kernels
// use, the q8_1 activation block, per-warp bulk-copy pipelines (cp.async.bulk + mbarrier) and the lane-banked i-quant
// codebook tables in shared memory.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace tsb {

enum : int { T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_IQ3_XXS = 18, T_IQ3_S = 21 };

// ---------------------------------------------------------------------------------------------------------- arithmetic
// The reference compiles its router, quantiser and expert kernels with --use_fast_math (CMakeLists.txt:204-207); these
// are the instructions that flag selects for `a / b`, `1.0f / a` and expf (q36_kernels.cuh:63-80 spells out the same).
__device__ __forceinline__ float fdiv_fm(float a, float b) {
    float r;
    asm("div.approx.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float frcp_fm(float a) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}
__device__ __forceinline__ float fexp_fm(float a) { return __expf(a); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------------------------------------- q8_1
// 32 values: fp16 scale d = amax / 127 and fp16 sum of the raw values, then 32 int8 codes (ggml block_q8_1, 36 bytes).
struct __align__(4) BlockQ8_1 {
    half2 ds;
    int8_t qs[32];
};
static_assert(sizeof(BlockQ8_1) == 36, "q8_1 block");

__device__ __forceinline__ float q8_finite(float v) { return fabsf(v) > 65504.0f ? copysignf(65504.0f, v) : v; }

// One lane's value v of a block whose 32 values are the warp's lanes (the reference's q8_1_store,
// iq_kernels.cu:1469-1480 with q8_1_finite.hpp): returns the code; the lane also receives d and the block sum.
__device__ __forceinline__ int8_t q8_1_warp(float v, float& d_out, float& sum_out) {
    float amax = fabsf(v), sum = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    const float d = q8_finite(fdiv_fm(amax, 127.0f));
    int8_t q = 0;
    if (amax != 0.0f) {
        const float r = roundf(fdiv_fm(v, d));
        q = (int8_t) (r > 127.0f ? 127.0f : r < -127.0f ? -127.0f : r);
    }
    d_out = d;
    sum_out = sum;
    return q;
}

// The same block computed by ONE lane from the 32 values in registers: the xor butterfly's balanced tree for the sum
// (every lane of the warp version ends with this tree) and the same instructions, so the same bits.
struct Q8Block {
    int q[8];   // 32 codes, 4 per word, value j in byte j % 4 of word j / 4
    float d;    // the float scale (before its fp16 rounding), what the codes were divided by
    half2 ds;   // what the block stores
};
__device__ __forceinline__ Q8Block q8_1_lane(const float (&x)[32]) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float p[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = x[i] + x[i + 16];
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = p[i] + p[i + 8];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = p[i] + p[i + 4];
#pragma unroll
    for (int i = 0; i < 2; ++i) p[i] = p[i] + p[i + 2];
    const float sum = p[0] + p[1];
    Q8Block b;
    b.d = q8_finite(fdiv_fm(amax, 127.0f));
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int8_t c = 0;
            if (amax != 0.0f) {
                const float r = roundf(fdiv_fm(x[4 * w + j], b.d));
                c = (int8_t) (r > 127.0f ? 127.0f : r < -127.0f ? -127.0f : r);
            }
            word |= (uint32_t) (uint8_t) c << (8 * j);
        }
        b.q[w] = (int) word;
    }
    b.ds = make_half2(__float2half(q8_finite(b.d)), __float2half(q8_finite(sum)));
    return b;
}

// ---------------------------------------------------------------------------------------------------------- PTX
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Global -> shared bulk copy (the non-tensor TMA): 16-byte aligned addresses, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 16 bytes global -> shared through L2 (cp.async.cg: the load/store unit, not the bulk-copy engine, so a warp issues 32
// of them per instruction), and an arrive on an mbarrier once every cp.async this thread issued before has landed
// (.noinc: the barrier's expected count includes the arriving threads).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Tagged exchange words between the CTAs of one launch: a float and the tag of the step that wrote it in one 8-byte
// word (low half the value bits, high half the tag), stored and loaded as single 64-bit accesses at gpu scope.  A
// reader polls the words it needs until every tag is the one it expects: the data is its own completion flag, one
// L2 round trip once the writer has stored it and no grid-wide barrier.
__device__ __forceinline__ void st_tag(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = (uint64_t) __float_as_uint(v) | ((uint64_t) tag << 32);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_tag(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Two consecutive words (16-byte aligned): two 64-bit accesses, each single-copy atomic.
__device__ __forceinline__ void ld_tag2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ float tag_val(uint64_t w) { return __uint_as_float((uint32_t) w); }
__device__ __forceinline__ bool tag_is(uint64_t w, uint32_t tag) { return (uint32_t) (w >> 32) == tag; }

// Non-blocking probe of a phase (test_wait returns at once; try_wait may suspend the thread for a while).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Device error word: a bounded wait that gives up records its site here and the kernel returns; the host reads it with
// tsb_device_error().  Nothing in these kernels waits without a bound.
__device__ __forceinline__ void report_error(unsigned* err, unsigned code) {
    if (err) atomicCAS(err, 0u, code);
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// The bound of every wait, per device: 2 s unless tsb_set_wait_limit_ns changed it (a bulk copy from valid memory
// completes in microseconds).  One copy per translation unit; the host setter writes each.
static __device__ unsigned long long g_wait_ns = 2000000000ull;
__device__ __forceinline__ uint64_t wait_limit_ns() { return g_wait_ns; }

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err, unsigned site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer(), lim = wait_limit_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer() - t0 > lim) {
            report_error(err, site);
            return false;
        }
    }
}

// The same with test_wait polls (never suspended): for a wait on the critical path whose phase usually completes within
// a few hundred cycles, where try_wait's suspension can oversleep the completion.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, unsigned* err, unsigned site) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer(), lim = wait_limit_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 1023u) == 0 && globaltimer() - t0 > lim) {
            report_error(err, site);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------- tables
// The IQ3_XXS grid and the sign masks of a 7-bit sign index, lane-banked in 64 KB of shared memory so that 32 lanes
// reading 32 different entries never share a bank:
//   grid word of index i for lane l ..... byte offset i * 256 + 4 l        (banks l)
//   sign masks of index s for lane l .... byte offset s * 256 + 128 + 8 (l & 15): {m0, m1}, byte j of m0 (m1) = 0xFF
//                                         where sign bit j (j + 4) of ksigns[s] is set
// The grid address is one byte_perm of the code word (byte 1 = the code, byte 0 = 4 l).
constexpr int kIqTabBytes = 256 * 256;

struct IqTab {
    const uint8_t* base;   // shared memory
    uint32_t lane4;        // 4 * lane
    uint32_t lane_s;       // 128 + 8 * (lane & 15)
};

}  // namespace tsb
