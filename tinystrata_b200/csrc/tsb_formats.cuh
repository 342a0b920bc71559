// tsb_formats.cuh - the GGUF weight formats against q8_1 activations, one "call" (a fixed slice of a block) at a time.
//
// A call's integer sum and its float value are the reference's (src/kernels/cuda/iq_kernels.cu: IQ3_XXS 188-211,
// IQ3_S 213-236, Q4_K 314-386, Q4_0 457-474, Q6_K 523-553, Q8_0 555-566; call layout Fmt<TY> 600-680).  Each format
// splits the call into `decode` (everything that depends only on the weight: signed codes, integer scales, the fp16
// block scale) and `apply` (the activation side), so a decoded call is applied to several tokens.  Weights are read
// from shared memory (staged by bulk copies), activations live in registers.
#pragma once

#include "tsb_device.cuh"

namespace tsb {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// 0xFF in byte j where bit j of the nibble n is set (n < 16): the bits land on the bytes' top bits, then replicated
__device__ __forceinline__ uint32_t spread4(uint32_t n) { return prmt(n * 0x10204080u, 0u, 0xBA98u); }
// a 32-bit word at a 2-byte aligned shared-memory address
__device__ __forceinline__ uint32_t lw2(const uint8_t* p) {
    const uint32_t lo = *(const uint16_t*) p, hi = *(const uint16_t*) (p + 2);
    return lo | (hi << 16);
}
__device__ __forceinline__ float lh(const uint8_t* p) { return __half2float(*(const __half*) p); }
__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// A q8_1 block as a call sees it: 8 code words and the float of its fp16 scale.
struct QB {
    int q[8];
    float d;
};
__device__ __forceinline__ QB qb_from_global(const BlockQ8_1* b) {
    QB r;
    const int* w = (const int*) b->qs;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = __ldg(w + i);
    r.d = __low2float(b->ds);
    return r;
}
__device__ __forceinline__ QB qb_from_f32(const float* x32) {
    float v[32];
    const float4* p = (const float4*) x32;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = p[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    const Q8Block b = q8_1_lane(v);
    QB r;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = b.q[i];
    r.d = __low2float(b.ds);
    return r;
}

// The same from memory other CTAs of the running kernel write (L1 bypassed).
__device__ __forceinline__ QB qb_from_f32_cg(const float* x32) {
    float v[32];
    const float4* p = (const float4*) x32;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = __ldcg(p + i);
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    const Q8Block b = q8_1_lane(v);
    QB r;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = b.q[i];
    r.d = __low2float(b.ds);
    return r;
}

template <int TY> struct Fmt;

// ------------------------------------------------------------------------------------------------ IQ3_XXS (type 18)
// 98-byte block of 256: fp16 d | 64 grid codes | 8 words (4 x 7-bit sign index, 4-bit scale).  Call c (0..7) is
// values 32c..32c+31: codes 8c..8c+7, word c; one q8_1 block.
template <> struct Fmt<T_IQ3_XXS> {
    static constexpr int qk = 256, bb = 98, cpb = 8;
    struct Act { int u[8]; float d; };
    struct W { int v[8]; int ls; float dw; };
    template <class Src> __device__ static Act act(const Src& src, int call) {
        const QB b = src(call);   // q8_1 block index = call (8 calls per 256-value block, one q8_1 block each)
        Act a;
#pragma unroll
        for (int i = 0; i < 8; ++i) a.u[i] = b.q[i];
        a.d = b.d;
        return a;
    }
    __device__ static W decode(const uint8_t* row, int call, const IqTab& t) {
        const uint8_t* wb = row + (call >> 3) * bb;
        const int c = call & 7;
        const uint32_t q0 = lw2(wb + 2 + 8 * c), q1 = lw2(wb + 6 + 8 * c), aux = lw2(wb + 66 + 4 * c);
        W w;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qw = l < 2 ? q0 : q1;
            const uint32_t j0 = (2 * l) & 3, j1 = (2 * l + 1) & 3;
            const uint32_t g0 = *(const uint32_t*) (t.base + prmt(qw, t.lane4, 0x5504u | (j0 << 4)));
            const uint32_t g1 = *(const uint32_t*) (t.base + prmt(qw, t.lane4, 0x5504u | (j1 << 4)));
            const uint32_t s7 = (aux >> (7 * l)) & 127u;
            const uint2 m = *(const uint2*) (t.base + ((s7 << 8) | t.lane_s));
            w.v[2 * l] = (int) ((g0 ^ m.x) + (m.x & 0x01010101u));
            w.v[2 * l + 1] = (int) ((g1 ^ m.y) + (m.y & 0x01010101u));
        }
        w.ls = (int) (aux >> 28);
        w.dw = lh(wb);
        return w;
    }
    __device__ static int sumi(const W& w, const Act& a) {
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) s = dp4a(w.v[j], a.u[j], s);
        return (w.ls * s + s / 2) / 2;
    }
    __device__ static float apply(const W& w, const Act& a) {
        const float d = w.dw * a.d;
        return d * (float) sumi(w, a);
    }
};

// ------------------------------------------------------------------------------------------------ IQ3_S (type 21)
// 110-byte block: fp16 d | 64 codes | 8 high bits bytes | 32 sign bytes | 4 scale bytes (two 4-bit scales).
template <> struct Fmt<T_IQ3_S> {
    static constexpr int qk = 256, bb = 110, cpb = 8;
    using Act = Fmt<T_IQ3_XXS>::Act;
    struct W { int v[8]; int mul; float dw; };
    template <class Src> __device__ static Act act(const Src& src, int call) { return Fmt<T_IQ3_XXS>::act(src, call); }
    // grid3s: the 512-word IQ3_S grid in shared memory (plain layout)
    __device__ static W decode(const uint8_t* row, int call, const uint32_t* grid3s) {
        const uint8_t* wb = row + (call >> 3) * bb;
        const int c = call & 7;
        const uint32_t q0 = lw2(wb + 2 + 8 * c), q1 = lw2(wb + 6 + 8 * c);
        const uint32_t qh = wb[66 + c];
        const uint32_t sg = lw2(wb + 74 + 4 * c);
        W w;
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qw = l < 2 ? q0 : q1;
            const int j0 = 2 * l, j1 = 2 * l + 1;
            const uint32_t i0 = ((qw >> (8 * (j0 & 3))) & 0xFFu) | (((qh >> j0) & 1u) << 8);
            const uint32_t i1 = ((qw >> (8 * (j1 & 3))) & 0xFFu) | (((qh >> j1) & 1u) << 8);
            const uint32_t s8 = (sg >> (8 * l)) & 0xFFu;
            const uint32_t m0 = spread4(s8 & 15u), m1 = spread4(s8 >> 4);
            w.v[j0] = (int) ((grid3s[i0] ^ m0) + (m0 & 0x01010101u));
            w.v[j1] = (int) ((grid3s[i1] ^ m1) + (m1 & 0x01010101u));
        }
        w.mul = 1 + 2 * ((wb[106 + c / 2] >> (4 * (c & 1))) & 15);
        w.dw = lh(wb);
        return w;
    }
    __device__ static int sumi(const W& w, const Act& a) {
        int s = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) s = dp4a(w.v[j], a.u[j], s);
        return s * w.mul;
    }
    __device__ static float apply(const W& w, const Act& a) {
        const float d = w.dw * a.d;
        return d * (float) sumi(w, a);
    }
};

// ------------------------------------------------------------------------------------------------ Q8_0 (type 8)
// 34-byte block of 32: fp16 d | 32 int8.  Call c (0..3): ints 2c, 2c+1 (values 8c..8c+7).
template <> struct Fmt<T_Q8_0> {
    static constexpr int qk = 32, bb = 34, cpb = 4;
    struct Act { int u[2]; float d; };
    struct W { int v[2]; float dw; };
    template <class Src> __device__ static Act act(const Src& src, int call) {
        const QB b = src(call >> 2);
        const int i = 2 * (call & 3);
        Act a;
        a.u[0] = b.q[i];
        a.u[1] = b.q[i + 1];
        a.d = b.d;
        return a;
    }
    __device__ static W decode(const uint8_t* row, int call, const IqTab&) {
        const uint8_t* wb = row + (call >> 2) * bb;
        const int i = 2 * (call & 3);
        W w;
        w.v[0] = (int) lw2(wb + 2 + 4 * i);
        w.v[1] = (int) lw2(wb + 6 + 4 * i);
        w.dw = lh(wb);
        return w;
    }
    __device__ static int sumi(const W& w, const Act& a) { return dp4a(w.v[1], a.u[1], dp4a(w.v[0], a.u[0], 0)); }
    __device__ static float apply(const W& w, const Act& a) { return w.dw * a.d * (float) sumi(w, a); }
};

// ------------------------------------------------------------------------------------------------ Q4_0 (type 2)
// 18-byte block of 32: fp16 d | 16 bytes (value j low nibble of byte j, value 16+j high nibble).  Call c (0..1): bytes
// 8c..8c+7 -> values 8c..8c+7 and 16+8c..; the codes centred (q - 8) as the reference does (iq_kernels.cu:457-462).
__device__ __forceinline__ int q4_0_centred(uint32_t v) {
    const uint32_t b = v ^ 0x08080808u;
    return (int) (b | ((b & 0x08080808u) * 0x1Eu));
}
template <> struct Fmt<T_Q4_0> {
    static constexpr int qk = 32, bb = 18, cpb = 2;
    struct Act { int u[4]; float d; };
    struct W { int v[4]; float dw; };
    template <class Src> __device__ static Act act(const Src& src, int call) {
        const QB b = src(call >> 1);
        const int i = 2 * (call & 1);
        Act a;
        a.u[0] = b.q[i];
        a.u[1] = b.q[i + 4];
        a.u[2] = b.q[i + 1];
        a.u[3] = b.q[i + 5];
        a.d = b.d;
        return a;
    }
    __device__ static W decode(const uint8_t* row, int call, const IqTab&) {
        const uint8_t* wb = row + (call >> 1) * bb;
        const int i = 2 * (call & 1);
        const uint32_t v0 = lw2(wb + 2 + 4 * i), v1 = lw2(wb + 6 + 4 * i);
        W w;
        w.v[0] = q4_0_centred(v0 & 0x0F0F0F0Fu);
        w.v[1] = q4_0_centred((v0 >> 4) & 0x0F0F0F0Fu);
        w.v[2] = q4_0_centred(v1 & 0x0F0F0F0Fu);
        w.v[3] = q4_0_centred((v1 >> 4) & 0x0F0F0F0Fu);
        w.dw = lh(wb);
        return w;
    }
    __device__ static int sumi(const W& w, const Act& a) {
        int s = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) s = dp4a(w.v[j], a.u[j], s);
        return s;
    }
    __device__ static float apply(const W& w, const Act& a) { return w.dw * a.d * (float) sumi(w, a); }
};

// ------------------------------------------------------------------------------------------------ Q4_K (type 12)
// 144-byte block of 256: fp16 d, fp16 dmin | 12 bytes of 6-bit scales and mins | 128 bytes of nibbles.  Call c
// (0..15): sub-blocks 2(c/4) (low nibbles) and 2(c/4)+1 (high), 8 values each at int c%4 and c%4+4.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& d, int& m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
template <> struct Fmt<T_Q4_K> {
    static constexpr int qk = 256, bb = 144, cpb = 16;
    struct Act { int u[4]; float d[2]; };
    struct W { int v0, v1; int sc[2], m[2]; float d, dmin; };
    template <class Src> __device__ static Act act(const Src& src, int call) {
        const int b = call >> 4, c = call & 15, off = 2 * (c >> 2), p = c & 3;
        Act a;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const QB q = src(b * 8 + off + i);
            a.u[2 * i] = q.q[p];
            a.u[2 * i + 1] = q.q[p + 4];
            a.d[i] = q.d;
        }
        return a;
    }
    __device__ static W decode(const uint8_t* row, int call, const IqTab&) {
        const uint8_t* wb = row + (call >> 4) * bb;
        const int c = call & 15, off = 2 * (c >> 2), p = c & 3;
        const uint8_t* q4 = wb + 16 + 16 * off + 4 * p;
        W w;
        w.v0 = (int) lw2(q4);
        w.v1 = (int) lw2(q4 + 16);
#pragma unroll
        for (int i = 0; i < 2; ++i) scale_min_k4(off + i, wb + 4, w.sc[i], w.m[i]);
        w.d = lh(wb);
        w.dmin = lh(wb + 2);
        return w;
    }
    // the raw integer dots of the call (before the 6-bit scales), summed: the per-call integer the tests pin
    __device__ static int sumi(const W& w, const Act& a) {
        int s = 0;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int v0i = (w.v0 >> (4 * i)) & 0x0F0F0F0F, v1i = (w.v1 >> (4 * i)) & 0x0F0F0F0F;
            s += dp4a(v1i, a.u[2 * i + 1], dp4a(v0i, a.u[2 * i], 0));
        }
        return s;
    }
    __device__ static float apply(const W& w, const Act& a) {
        float sumf_d = 0.0f, sumf_m = 0.0f;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int v0i = (w.v0 >> (4 * i)) & 0x0F0F0F0F, v1i = (w.v1 >> (4 * i)) & 0x0F0F0F0F;
            const int dot1 = dp4a(v1i, a.u[2 * i + 1], dp4a(v0i, a.u[2 * i], 0));
            const int dot2 = dp4a(0x01010101, a.u[2 * i + 1], dp4a(0x01010101, a.u[2 * i], 0));
            sumf_d += a.d[i] * (float) (dot1 * w.sc[i]);
            sumf_m += a.d[i] * (float) (dot2 * w.m[i]);
        }
        return w.d * sumf_d - w.dmin * sumf_m;
    }
};

// ------------------------------------------------------------------------------------------------ Q6_K (type 14)
// 210-byte block of 256: 128 bytes low nibbles | 64 bytes high 2-bit pairs | 16 int8 scales | fp16 d.  Call c (0..31).
template <> struct Fmt<T_Q6_K> {
    static constexpr int qk = 256, bb = 210, cpb = 32;
    struct Act { int u[2]; float d[2]; };
    struct W { int vl, vh; int sc[2]; float d; };
    template <class Src> __device__ static Act act(const Src& src, int call) {
        const int b = call >> 5, iqs = call & 31, off = 4 * (iqs / 16) + (iqs % 16) / 8;
        Act a;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const QB q = src(b * 8 + off + 2 * i);
            a.u[i] = q.q[iqs % 8];
            a.d[i] = q.d;
        }
        return a;
    }
    __device__ static W decode(const uint8_t* row, int call, const IqTab&) {
        const uint8_t* wb = row + (call >> 5) * bb;
        const int iqs = call & 31;
        const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
        const int vh_shift = 2 * ((iqs % 16) / 8);
        W w;
        w.vl = (int) lw2(wb + 4 * iqs);
        w.vh = (int) (lw2(wb + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift);
        w.sc[0] = (int8_t) wb[192 + scale_offset];
        w.sc[1] = (int8_t) wb[192 + scale_offset + 4];
        w.d = lh(wb + 208);
        return w;
    }
    __device__ static int code(const W& w, int i) {
        const int vil = (w.vl >> (4 * i)) & 0x0F0F0F0F;
        const int vih = ((w.vh >> (4 * i)) << 4) & 0x30303030;
        return (int) __vsub4((unsigned) (vil | vih), 0x20202020u);
    }
    __device__ static int sumi(const W& w, const Act& a) { return dp4a(code(w, 0), a.u[0], 0) + dp4a(code(w, 1), a.u[1], 0); }
    __device__ static float apply(const W& w, const Act& a) {
        float sumf = 0.0f;
#pragma unroll
        for (int i = 0; i < 2; ++i) sumf += a.d[i] * (float) (dp4a(code(w, i), a.u[i], 0) * w.sc[i]);
        return w.d * sumf;
    }
};


// ------------------------------------------------------------------------------------------------ IQ3_XXS, absolute
// The fused decode kernel keeps the lane-banked tables at shared-window address 0x10000, so one byte_perm of a code
// word with (0x10000 | 4 lane) is the full address of a grid entry and the sign-mask address is a shift and a
// three-input op; `ld.shared` takes them as they are.
constexpr uint32_t kAbsTab = 0x10000u;
struct AbsTab {
    uint32_t lane_g;   // kAbsTab | 4 lane
    uint32_t lane_s;   // kAbsTab | 128 | 8 (lane & 15)
};
__device__ __forceinline__ AbsTab make_abs_tab(int lane) {
    return {kAbsTab | (4u * (uint32_t) lane), kAbsTab | 128u | (8u * (uint32_t) (lane & 15))};
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
// the sign-mask address of 7-bit field l of aux: ((aux >> 7 l) & 127) << 8 | lane_s
template <int L> __device__ __forceinline__ uint32_t sign_addr(uint32_t aux, uint32_t lane_s) {
    constexpr int sh = 7 * L - 8;
    const uint32_t t = sh >= 0 ? (aux >> sh) : (aux << -sh);
    return (t & 0x7F00u) | lane_s;
}
// One IQ3_XXS call, decoded with the signs still separate: gx = grid ^ mask, m = mask (0xFF bytes where negative).
// sum(sign * grid * u) = dp4a(gx, u) - dp4a(m, u): (g ^ 0xFF) is -g - 1 as a signed byte and m is -1.
struct Iq3x {
    uint32_t gx[8], m[8];
    int ls;
    float dw;
};
__device__ __forceinline__ Iq3x iq3x_decode(const uint8_t* row, int call, const AbsTab& t) {
    const uint8_t* wb = row + (call >> 3) * 98;
    const int c = call & 7;
    const uint32_t q0 = lw2(wb + 2 + 8 * c), q1 = lw2(wb + 6 + 8 * c), aux = lw2(wb + 66 + 4 * c);
    Iq3x w;
    const uint2 m0 = lds_u64(sign_addr<0>(aux, t.lane_s)), m1 = lds_u64(sign_addr<1>(aux, t.lane_s));
    const uint2 m2 = lds_u64(sign_addr<2>(aux, t.lane_s)), m3 = lds_u64(sign_addr<3>(aux, t.lane_s));
    w.m[0] = m0.x; w.m[1] = m0.y; w.m[2] = m1.x; w.m[3] = m1.y;
    w.m[4] = m2.x; w.m[5] = m2.y; w.m[6] = m3.x; w.m[7] = m3.y;
    w.gx[0] = lds_u32(prmt(q0, t.lane_g, 0x7604u)) ^ w.m[0];
    w.gx[1] = lds_u32(prmt(q0, t.lane_g, 0x7614u)) ^ w.m[1];
    w.gx[2] = lds_u32(prmt(q0, t.lane_g, 0x7624u)) ^ w.m[2];
    w.gx[3] = lds_u32(prmt(q0, t.lane_g, 0x7634u)) ^ w.m[3];
    w.gx[4] = lds_u32(prmt(q1, t.lane_g, 0x7604u)) ^ w.m[4];
    w.gx[5] = lds_u32(prmt(q1, t.lane_g, 0x7614u)) ^ w.m[5];
    w.gx[6] = lds_u32(prmt(q1, t.lane_g, 0x7624u)) ^ w.m[6];
    w.gx[7] = lds_u32(prmt(q1, t.lane_g, 0x7634u)) ^ w.m[7];
    w.ls = (int) (aux >> 28);
    w.dw = lh(wb);
    return w;
}
__device__ __forceinline__ int iq3x_sumi(const Iq3x& w, const int (&u)[8]) {
    int a = 0, b = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        a = dp4a((int) w.gx[j], u[j], a);
        b = dp4a((int) w.m[j], u[j], b);
    }
    const int s = a - b;
    return (w.ls * s + s / 2) / 2;
}
__device__ __forceinline__ float iq3x_apply(const Iq3x& w, const Fmt<T_IQ3_XXS>::Act& a) {
    const float d = w.dw * a.d;
    return d * (float) iq3x_sumi(w, a.u);
}
// materialised signed codes (several tokens per decoded call)
__device__ __forceinline__ Fmt<T_IQ3_XXS>::W iq3x_signed(const Iq3x& x) {
    Fmt<T_IQ3_XXS>::W w;
#pragma unroll
    for (int j = 0; j < 8; ++j) w.v[j] = (int) (x.gx[j] + (x.m[j] & 0x01010101u));
    w.ls = x.ls;
    w.dw = x.dw;
    return w;
}


// The same decode with the block's alignment known at compile time (rows staged 4-byte aligned): a block at an even
// position of its row starts at 0 mod 4, an odd one at 2 mod 4 (98-byte blocks).  Aligned 32-bit loads and byte_perm
// replace the 16-bit loads.
template <bool ODD>
__device__ __forceinline__ Iq3x iq3x_decode_blk(const uint8_t* wb, int c, const AbsTab& t) {
    uint32_t q0, q1, aux;
    if constexpr (ODD) {
        q0 = *(const uint32_t*) (wb + 2 + 8 * c);
        q1 = *(const uint32_t*) (wb + 6 + 8 * c);
        aux = *(const uint32_t*) (wb + 66 + 4 * c);
    } else {
        const uint32_t* w = (const uint32_t*) (wb + 8 * c);
        const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
        q0 = prmt(w0, w1, 0x5432u);
        q1 = prmt(w1, w2, 0x5432u);
        const uint32_t* a = (const uint32_t*) (wb + 64 + 4 * c);
        aux = prmt(a[0], a[1], 0x5432u);
    }
    Iq3x w;
    const uint2 m0 = lds_u64(sign_addr<0>(aux, t.lane_s)), m1 = lds_u64(sign_addr<1>(aux, t.lane_s));
    const uint2 m2 = lds_u64(sign_addr<2>(aux, t.lane_s)), m3 = lds_u64(sign_addr<3>(aux, t.lane_s));
    w.m[0] = m0.x; w.m[1] = m0.y; w.m[2] = m1.x; w.m[3] = m1.y;
    w.m[4] = m2.x; w.m[5] = m2.y; w.m[6] = m3.x; w.m[7] = m3.y;
    w.gx[0] = lds_u32(prmt(q0, t.lane_g, 0x7604u)) ^ w.m[0];
    w.gx[1] = lds_u32(prmt(q0, t.lane_g, 0x7614u)) ^ w.m[1];
    w.gx[2] = lds_u32(prmt(q0, t.lane_g, 0x7624u)) ^ w.m[2];
    w.gx[3] = lds_u32(prmt(q0, t.lane_g, 0x7634u)) ^ w.m[3];
    w.gx[4] = lds_u32(prmt(q1, t.lane_g, 0x7604u)) ^ w.m[4];
    w.gx[5] = lds_u32(prmt(q1, t.lane_g, 0x7614u)) ^ w.m[5];
    w.gx[6] = lds_u32(prmt(q1, t.lane_g, 0x7624u)) ^ w.m[6];
    w.gx[7] = lds_u32(prmt(q1, t.lane_g, 0x7634u)) ^ w.m[7];
    w.ls = (int) (aux >> 28);
    w.dw = lh(wb);
    return w;
}

// Dispatch helper so every decode has one signature: IQ3_S reads its plain 512-word grid at t.base + kIqTabBytes.
template <int TY> __device__ __forceinline__ typename Fmt<TY>::W decode_call(const uint8_t* row, int call, const IqTab& t) {
    if constexpr (TY == T_IQ3_S) return Fmt<TY>::decode(row, call, (const uint32_t*) (t.base + kIqTabBytes));
    else return Fmt<TY>::decode(row, call, t);
}

}  // namespace tsb
