/*
 * oracle/tsb_oracle.c - CPU restatement of TinyStrata's MoE expert-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, smoke() and bench.py's cpu_baseline leg
 * compare the CUDA path against; no product code links or calls it.
 *
 * Every function restates one piece of the reference (paths relative to the TinyStrata tree):
 *   q8_1 quantiser ............ src/kernels/cuda/iq_kernels.cu:1469-1480, include/strata/kernels/q8_1_finite.hpp:17-31
 *   IQ3_XXS x q8_1 ............ src/kernels/cuda/iq_kernels.cu:188-211 (Split<18> 858-887)
 *   IQ3_S x q8_1 .............. src/kernels/cuda/iq_kernels.cu:213-236 (Split<21> 889-918)
 *   Q4_K x q8_1 ............... src/kernels/cuda/iq_kernels.cu:314-386 (k_scale_min 343-353, min term on the int8 codes)
 *   Q4_0 x q8_1 (centred) ..... src/kernels/cuda/iq_kernels.cu:457-474
 *   Q6_K x q8_1 ............... src/kernels/cuda/iq_kernels.cu:523-553
 *   Q8_0 x q8_1 ............... src/kernels/cuda/iq_kernels.cu:555-566
 *   call layout (ipb, step) ... src/kernels/cuda/iq_kernels.cu:600-680 (Fmt<TY>), row_dot 695-705
 *   softmax top-k router ...... src/kernels/cuda/native_router.cu:44-95
 *   Gemma/LFM router .......... src/gemma4/kernels.cu:289-356, src/gemma4/gemma4.cpp:650-668, src/lfm2/lfm2moe.cpp:413-435
 *   decode grouping ........... src/qwen35/q36_engine.cu:396-422 (k_group)
 *   prefill permutation ....... src/qwen35/q36_engine.cu:486-510 (stable (expert, entry) order, see or_dispatch)
 *   SwiGLU / GELU-tanh / clamp  src/kernels/cuda/iq_kernels.cu:1508-1512, src/gemma4/kernels.cu:251-263
 *   combine ................... src/qwen35/q36_engine.cu:307-332 (k_moe_out), src/gemma4/kernels.cu:358-366 (moe_sum)
 *
 * Integer work (codebook decode, per-call integer sums, routing ids, permutations) is exact.  Float results follow
 * the reference's per-call expressions in float; sums over calls and over experts are carried in double (the fp64
 * accumulation the tolerance checks are quoted against).  Divisions and exponentials are IEEE/libm here; the GPU
 * kernels use the fast-math instructions the reference was compiled with, so a q8_1 code may differ by one step
 * where x/d lies within a few ulp of a rounding boundary (the tests allow exactly that).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../tinystrata_b200/csrc/codebooks.inc"

static const uint32_t k_iq3xxs_grid[256] = TSB_IQ3XXS_GRID;
static const uint32_t k_iq3s_grid[512] = TSB_IQ3S_GRID;
static const uint8_t k_ksigns[128] = TSB_KSIGNS;

/* ggml type ids (ggml.h) */
enum { T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_IQ3_XXS = 18, T_IQ3_S = 21 };

/* ------------------------------------------------------------------------------------------------ fp16 */
float or_half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t) (h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) bits = s;
        else { /* subnormal: m * 2^-24 */
            float f = (float) m * 5.9604644775390625e-8f;
            memcpy(&bits, &f, 4);
            bits |= s;
        }
    } else if (e == 31) bits = s | 0x7f800000u | (m << 13);
    else bits = s | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* round-to-nearest-even float -> fp16 (the conversion __float2half performs) */
uint16_t or_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) { /* below the smallest normal half: a multiple of 2^-24, ties to even */
        const double v = fabs((double) f) / 5.9604644775390625e-8;
        return (uint16_t) (sign | (uint32_t) nearbyint(v));
    }
    /* normal: round mantissa from 23 to 10 bits, ties to even */
    uint32_t e = (ax >> 23) - 112, m = ax & 0x7fffffu;
    uint32_t hm = m >> 13, rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (hm & 1))) {
        ++hm;
        if (hm == 1024) { hm = 0; ++e; }
    }
    if (e >= 31) return (uint16_t) (sign | 0x7c00u);
    return (uint16_t) (sign | (e << 10) | hm);
}

static inline float h2f_at(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return or_half_to_float(h);
}
static inline uint32_t u32_at(const uint8_t* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
static inline int8_t sbyte(uint32_t w, int i) { return (int8_t) ((w >> (8 * i)) & 0xff); }

/* ------------------------------------------------------------------------------------------------ q8_1 */
/* A q8_1 block: fp16 d, fp16 sum, 32 int8 codes (36 bytes). */
#define Q8_1_BYTES 36

/* The warp's xor-butterfly sum (offsets 16, 8, 4, 2, 1): every lane ends with the same balanced-tree sum. */
static float tree_sum32(const float* v) {
    float p[32];
    memcpy(p, v, sizeof p);
    for (int o = 16; o > 0; o >>= 1)
        for (int i = 0; i < o; ++i) p[i] = p[i] + p[i + o];
    return p[0];
}

static inline float q8_1_finite(float v) { return fabsf(v) > 65504.0f ? copysignf(65504.0f, v) : v; }

/* One 32-value block, iq_kernels.cu:1469-1480 with q8_1_finite.hpp:17-31 (IEEE division here). */
void or_q8_1_block(const float* x, uint8_t* blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float sum = tree_sum32(x);
    const float d = q8_1_finite(amax / 127.0f);
    int8_t* q = (int8_t*) (blk + 4);
    for (int i = 0; i < 32; ++i) {
        if (amax == 0.0f) { q[i] = 0; continue; }
        const float r = roundf(x[i] / d);
        q[i] = (int8_t) (r > 127.0f ? 127.0f : r < -127.0f ? -127.0f : r);
    }
    const uint16_t hd = or_float_to_half(q8_1_finite(d)), hs = or_float_to_half(q8_1_finite(sum));
    memcpy(blk, &hd, 2);
    memcpy(blk + 2, &hs, 2);
}

/* n_rows rows of n_cols (a multiple of 32) -> n_rows * n_cols/32 blocks, iq_kernels.hpp:24 quantize_q8_1_rows. */
void or_quantize_q8_1_rows(const float* x, int64_t n_rows, int64_t n_cols, uint8_t* y) {
    const int64_t nb = n_cols / 32;
    for (int64_t r = 0; r < n_rows; ++r)
        for (int64_t b = 0; b < nb; ++b) or_q8_1_block(x + r * n_cols + b * 32, y + (r * nb + b) * Q8_1_BYTES);
}

/* ------------------------------------------------------------------------------------------------ formats */
int or_block_values(int type) {
    switch (type) {
        case T_Q4_0: case T_Q8_0: return 32;
        case T_Q4_K: case T_Q6_K: case T_IQ3_XXS: case T_IQ3_S: return 256;
        default: return 0;
    }
}
int or_block_bytes(int type) {
    switch (type) {
        case T_Q4_0: return 18;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        case T_IQ3_XXS: return 98;
        case T_IQ3_S: return 110;
        default: return 0;
    }
}
int64_t or_row_bytes(int type, int64_t n) {
    const int qk = or_block_values(type);
    return qk ? (n / qk) * or_block_bytes(type) : 0;
}
/* dot calls per block and the iqs step between them (Fmt<TY>, iq_kernels.cu:600-680) */
int or_calls_per_block(int type) {
    switch (type) {
        case T_Q4_0: return 2;   /* QI4_0 / VDR_Q4_0 = 4 / 2 */
        case T_Q8_0: return 4;   /* QI8_0 / VDR_Q8_0 = 8 / 2 */
        case T_Q4_K: return 16;  /* QI4_K / VDR_Q4_K = 32 / 2 */
        case T_Q6_K: return 32;  /* QI6_K / VDR_Q6_K = 32 / 1 */
        case T_IQ3_XXS: case T_IQ3_S: return 8;
        default: return 0;
    }
}
static int call_step(int type) { return type == T_Q6_K ? 1 : 2; }

static inline int dp4a(uint32_t a, uint32_t b, int c) {
    for (int i = 0; i < 4; ++i) c += (int) sbyte(a, i) * (int) sbyte(b, i);
    return c;
}
/* signed grid word: byte j negated where sign bit j is set */
static inline uint32_t apply_signs4(uint32_t g, uint32_t s4) {
    uint32_t r = 0;
    for (int j = 0; j < 4; ++j) {
        int v = (int) ((g >> (8 * j)) & 0xff);
        if ((s4 >> j) & 1) v = -v;
        r |= ((uint32_t) (uint8_t) (int8_t) v) << (8 * j);
    }
    return r;
}

typedef struct {
    int32_t sumi;   /* the call's integer sum after the format's integer scale step (IQ3_*) or the raw sum */
    float value;    /* the call's float result, the reference's expression */
} call_t;

/* K-quant 6-bit scale/min of sub-block j (0..7): ggml's get_scale_min_k4 */
static void scale_min_k4(int j, const uint8_t* q, int* d, int* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* One dot call: weight block `wb` (call index c within the block), activation q8_1 blocks `xb` (the weight block's
 * first q8_1 block).  Also reports the raw (unscaled) int8 dots of the call through `raw`, up to 4 of them. */
static call_t dot_call(int type, const uint8_t* wb, const uint8_t* xb, int c) {
    call_t r = {0, 0.0f};
    const int iqs = call_step(type) * c;
    switch (type) {
        case T_IQ3_XXS: {
            const uint8_t* qs = wb + 2;
            const uint32_t aux32 = u32_at(qs + 64 + 4 * (iqs / 2));
            const uint8_t* xq = xb + (iqs / 2) * Q8_1_BYTES;
            int sumi = 0;
            for (int l = 0; l < 4; ++l) { /* 8 values per 7-bit sign field */
                const uint8_t s8 = k_ksigns[(aux32 >> (7 * l)) & 127];
                const uint32_t g0 = k_iq3xxs_grid[qs[4 * iqs + 2 * l + 0]];
                const uint32_t g1 = k_iq3xxs_grid[qs[4 * iqs + 2 * l + 1]];
                sumi = dp4a(apply_signs4(g0, s8 & 15), u32_at(xq + 4 + 8 * l), sumi);
                sumi = dp4a(apply_signs4(g1, s8 >> 4), u32_at(xq + 4 + 8 * l + 4), sumi);
            }
            const int ls = (int) (aux32 >> 28);
            sumi = (ls * sumi + sumi / 2) / 2;
            const float d = h2f_at(wb) * h2f_at(xq);
            r.sumi = sumi;
            r.value = d * (float) sumi;
            break;
        }
        case T_IQ3_S: {
            const uint8_t* qs = wb + 2;
            const uint8_t qh = wb[66 + iqs / 2];
            const uint8_t* signs = wb + 74 + 4 * (iqs / 2);
            const uint8_t* xq = xb + (iqs / 2) * Q8_1_BYTES;
            int sumi = 0;
            for (int l = 0; l < 4; ++l) {
                const uint8_t s8 = signs[l];
                const int j0 = 2 * l, j1 = 2 * l + 1;
                const uint32_t g0 = k_iq3s_grid[qs[4 * iqs + j0] | (((qh >> j0) & 1) << 8)];
                const uint32_t g1 = k_iq3s_grid[qs[4 * iqs + j1] | (((qh >> j1) & 1) << 8)];
                sumi = dp4a(apply_signs4(g0, s8 & 15), u32_at(xq + 4 + 8 * l), sumi);
                sumi = dp4a(apply_signs4(g1, s8 >> 4), u32_at(xq + 4 + 8 * l + 4), sumi);
            }
            const uint8_t sc = wb[106 + iqs / 4];
            sumi *= 1 + 2 * ((sc >> ((iqs << 1) & 4)) & 0x0F);
            const float d = h2f_at(wb) * h2f_at(xq);
            r.sumi = sumi;
            r.value = d * (float) sumi;
            break;
        }
        case T_Q4_0: {
            const uint8_t* qs = wb + 2;
            int sumi = 0;
            for (int i = 0; i < 2; ++i) {
                const uint32_t v = u32_at(qs + 4 * (iqs + i));
                uint32_t lo = 0, hi = 0;
                for (int j = 0; j < 4; ++j) {
                    const int b = (v >> (8 * j)) & 0xff;
                    lo |= (uint32_t) (uint8_t) (int8_t) ((b & 15) - 8) << (8 * j);
                    hi |= (uint32_t) (uint8_t) (int8_t) ((b >> 4) - 8) << (8 * j);
                }
                sumi = dp4a(lo, u32_at(xb + 4 + 4 * (iqs + i)), sumi);
                sumi = dp4a(hi, u32_at(xb + 4 + 4 * (iqs + i + 4)), sumi);
            }
            r.sumi = sumi;
            r.value = h2f_at(wb) * h2f_at(xb) * (float) sumi;
            break;
        }
        case T_Q8_0: {
            int sumi = 0;
            for (int i = 0; i < 2; ++i) sumi = dp4a(u32_at(wb + 2 + 4 * (iqs + i)), u32_at(xb + 4 + 4 * (iqs + i)), sumi);
            r.sumi = sumi;
            r.value = h2f_at(wb) * h2f_at(xb) * (float) sumi;
            break;
        }
        case T_Q4_K: {
            /* block: d, dmin (fp16), scales[12], qs[128]; call iqs covers 8 values of sub-blocks 2j and 2j+1 */
            const int bq8_offset = 2 * ((iqs / 2) / 4);
            const uint8_t* q4 = wb + 16 + 16 * bq8_offset + 4 * ((iqs / 2) % 4);
            const uint32_t v0 = u32_at(q4), v1 = u32_at(q4 + 16);
            float sumf_d = 0.0f, sumf_m = 0.0f;
            int32_t raw = 0;
            for (int i = 0; i < 2; ++i) {
                int sc, m;
                scale_min_k4(bq8_offset + i, wb + 4, &sc, &m);
                const uint8_t* x = xb + (bq8_offset + i) * Q8_1_BYTES;
                const uint32_t u0 = u32_at(x + 4 + 4 * ((iqs / 2) % 4)), u1 = u32_at(x + 4 + 4 * ((iqs / 2) % 4) + 16);
                const uint32_t v0i = (v0 >> (4 * i)) & 0x0F0F0F0Fu, v1i = (v1 >> (4 * i)) & 0x0F0F0F0Fu;
                const int dot1 = dp4a(v1i, u1, dp4a(v0i, u0, 0));
                const int dot2 = dp4a(0x01010101u, u1, dp4a(0x01010101u, u0, 0));
                const float d8 = h2f_at(x);
                sumf_d += d8 * (float) (dot1 * sc);
                sumf_m += d8 * (float) (dot2 * m);
                raw += dot1;
            }
            r.sumi = raw;
            r.value = h2f_at(wb) * sumf_d - h2f_at(wb + 2) * sumf_m;
            break;
        }
        case T_Q6_K: {
            /* block: ql[128], qh[64], scales[16] int8, d fp16 */
            const int bq8_offset = 4 * (iqs / 16) + (iqs % 16) / 8;
            const int scale_offset = 8 * (iqs / 16) + (iqs % 16) / 4;
            const int vh_shift = 2 * ((iqs % 16) / 8);
            const uint32_t vl = u32_at(wb + 4 * iqs);
            const uint32_t vh = u32_at(wb + 128 + 4 * (8 * (iqs / 16) + iqs % 8)) >> vh_shift;
            float sumf = 0.0f;
            int32_t raw = 0;
            for (int i = 0; i < 2; ++i) {
                const int sc = (int8_t) wb[192 + scale_offset + 4 * i];
                const uint32_t vil = (vl >> (4 * i)) & 0x0F0F0F0Fu;
                const uint32_t vih = ((vh >> (4 * i)) << 4) & 0x30303030u;
                uint32_t vi = 0;
                for (int j = 0; j < 4; ++j) {
                    const int b = (int) (((vil | vih) >> (8 * j)) & 0xff) - 32;
                    vi |= (uint32_t) (uint8_t) (int8_t) b << (8 * j);
                }
                const uint8_t* x = xb + (bq8_offset + 2 * i) * Q8_1_BYTES;
                const int dot = dp4a(vi, u32_at(x + 4 + 4 * (iqs % 8)), 0);
                sumf += h2f_at(x) * (float) (dot * sc);
                raw += dot;
            }
            r.sumi = raw;
            r.value = h2f_at(wb + 208) * sumf;
            break;
        }
        default: break;
    }
    return r;
}

/* The number of dot calls of a row of n values. */
int64_t or_row_calls(int type, int64_t n) {
    const int qk = or_block_values(type);
    return qk ? (n / qk) * or_calls_per_block(type) : 0;
}

/* Per-call integer sums and float values of one row against one q8_1 activation of n values (call k = block k/ipb,
 * part k%ipb: the order row_dot walks them, iq_kernels.cu:695-705). */
void or_row_dot_calls(int type, const uint8_t* row, const uint8_t* xq, int64_t n, int32_t* sumi, float* val) {
    const int qk = or_block_values(type), bb = or_block_bytes(type), ipb = or_calls_per_block(type);
    const int64_t nb = n / qk;
    for (int64_t b = 0; b < nb; ++b)
        for (int c = 0; c < ipb; ++c) {
            const call_t r = dot_call(type, row + b * bb, xq + b * (qk / 32) * Q8_1_BYTES, c);
            if (sumi) sumi[b * ipb + c] = r.sumi;
            if (val) val[b * ipb + c] = r.value;
        }
}

/* The row's dot: the calls' float values summed in double. */
double or_row_dot(int type, const uint8_t* row, const uint8_t* xq, int64_t n) {
    const int qk = or_block_values(type), bb = or_block_bytes(type), ipb = or_calls_per_block(type);
    const int64_t nb = n / qk;
    double s = 0.0;
    for (int64_t b = 0; b < nb; ++b)
        for (int c = 0; c < ipb; ++c) s += (double) dot_call(type, row + b * bb, xq + b * (qk / 32) * Q8_1_BYTES, c).value;
    return s;
}

/* y[r] = W[r] . x for rows [0, n_out) of a matrix of n_in values per row, float results of or_row_dot. */
void or_mat_vec(int type, const uint8_t* w, const uint8_t* xq, int64_t n_in, int64_t n_out, float* y) {
    const int64_t rb = or_row_bytes(type, n_in);
    for (int64_t r = 0; r < n_out; ++r) y[r] = (float) or_row_dot(type, w + r * rb, xq, n_in);
}

/* Dequantised weights (the value each code means), for cross-checks against independent decoders. */
void or_dequant_row(int type, const uint8_t* row, int64_t n, float* out) {
    const int qk = or_block_values(type), bb = or_block_bytes(type);
    for (int64_t b = 0; b < n / qk; ++b) {
        const uint8_t* w = row + b * bb;
        float* y = out + b * qk;
        switch (type) {
            case T_IQ3_XXS: {
                const float d = h2f_at(w);
                for (int s = 0; s < 8; ++s) { /* 32-value sub-block s */
                    const uint32_t aux = u32_at(w + 2 + 64 + 4 * s);
                    const float db = d * (0.5f + (float) (aux >> 28)) * 0.5f;
                    for (int l = 0; l < 4; ++l) {
                        const uint8_t s8 = k_ksigns[(aux >> (7 * l)) & 127];
                        for (int h = 0; h < 2; ++h) {
                            const uint32_t g = k_iq3xxs_grid[w[2 + 8 * s + 2 * l + h]];
                            for (int j = 0; j < 4; ++j) {
                                const float v = (float) ((g >> (8 * j)) & 0xff);
                                y[32 * s + 8 * l + 4 * h + j] = db * v * (((s8 >> (4 * h + j)) & 1) ? -1.0f : 1.0f);
                            }
                        }
                    }
                }
                break;
            }
            case T_IQ3_S: {
                const float d = h2f_at(w);
                for (int s = 0; s < 8; ++s) {
                    const int sc = (w[106 + s / 2] >> (4 * (s & 1))) & 15;
                    const float db = d * (float) (1 + 2 * sc);
                    const uint8_t qh = w[66 + s];
                    for (int l = 0; l < 4; ++l) {
                        const uint8_t s8 = w[74 + 4 * s + l];
                        for (int h = 0; h < 2; ++h) {
                            const int j8 = 2 * l + h;
                            const uint32_t g = k_iq3s_grid[w[2 + 8 * s + j8] | (((qh >> j8) & 1) << 8)];
                            for (int j = 0; j < 4; ++j) {
                                const float v = (float) ((g >> (8 * j)) & 0xff);
                                y[32 * s + 8 * l + 4 * h + j] = db * v * (((s8 >> (4 * h + j)) & 1) ? -1.0f : 1.0f);
                            }
                        }
                    }
                }
                break;
            }
            case T_Q4_0: {
                const float d = h2f_at(w);
                for (int j = 0; j < 16; ++j) {
                    y[j] = (float) ((w[2 + j] & 15) - 8) * d;
                    y[j + 16] = (float) ((w[2 + j] >> 4) - 8) * d;
                }
                break;
            }
            case T_Q8_0: {
                const float d = h2f_at(w);
                for (int j = 0; j < 32; ++j) y[j] = (float) (int8_t) w[2 + j] * d;
                break;
            }
            case T_Q4_K: {
                const float d = h2f_at(w), dmin = h2f_at(w + 2);
                const uint8_t* q = w + 16;
                for (int j = 0; j < 4; ++j) { /* 64 values: sub-blocks 2j (low nibbles) and 2j+1 (high) */
                    int sc, m;
                    scale_min_k4(2 * j, w + 4, &sc, &m);
                    const float d1 = d * (float) sc, m1 = dmin * (float) m;
                    scale_min_k4(2 * j + 1, w + 4, &sc, &m);
                    const float d2 = d * (float) sc, m2 = dmin * (float) m;
                    for (int l = 0; l < 32; ++l) y[64 * j + l] = d1 * (float) (q[32 * j + l] & 15) - m1;
                    for (int l = 0; l < 32; ++l) y[64 * j + 32 + l] = d2 * (float) (q[32 * j + l] >> 4) - m2;
                }
                break;
            }
            case T_Q6_K: {
                const float d = h2f_at(w + 208);
                const uint8_t* ql = w;
                const uint8_t* qh = w + 128;
                const int8_t* sc = (const int8_t*) (w + 192);
                for (int half = 0; half < 2; ++half) {
                    for (int l = 0; l < 32; ++l) {
                        const int is = l / 16;
                        const int q1 = (int) ((ql[64 * half + l] & 0xF) | (((qh[32 * half + l] >> 0) & 3) << 4)) - 32;
                        const int q2 = (int) ((ql[64 * half + l + 32] & 0xF) | (((qh[32 * half + l] >> 2) & 3) << 4)) - 32;
                        const int q3 = (int) ((ql[64 * half + l] >> 4) | (((qh[32 * half + l] >> 4) & 3) << 4)) - 32;
                        const int q4 = (int) ((ql[64 * half + l + 32] >> 4) | (((qh[32 * half + l] >> 6) & 3) << 4)) - 32;
                        y[128 * half + l + 0] = d * (float) sc[8 * half + is + 0] * (float) q1;
                        y[128 * half + l + 32] = d * (float) sc[8 * half + is + 2] * (float) q2;
                        y[128 * half + l + 64] = d * (float) sc[8 * half + is + 4] * (float) q3;
                        y[128 * half + l + 96] = d * (float) sc[8 * half + is + 6] * (float) q4;
                    }
                }
                break;
            }
            default: break;
        }
    }
}

/* The integer weight codes each block dot multiplies the q8_1 codes by, per value of a row of n values: Q4_0 nibble - 8
 * (q4_0_centred), Q8_0 the int8 code, Q4_K the nibble (its min is a separate term), Q6_K the 6-bit code - 32, IQ3_XXS /
 * IQ3_S the grid byte with its sign applied (the dp4a operands of iq_kernels.cu:188-236, 314-386, 457-474, 523-566).
 * The layouts are the ones or_dequant_row decodes; a tensor-core block sum is the plain integer dot of these codes with
 * the activation codes over the block's values. */
void or_weight_codes(int type, const uint8_t* row, int64_t n, int8_t* out) {
    const int qk = or_block_values(type), bb = or_block_bytes(type);
    for (int64_t b = 0; b < n / qk; ++b) {
        const uint8_t* w = row + b * bb;
        int8_t* y = out + b * qk;
        switch (type) {
            case T_IQ3_XXS:
                for (int s = 0; s < 8; ++s) {
                    const uint32_t aux = u32_at(w + 2 + 64 + 4 * s);
                    for (int l = 0; l < 4; ++l) {
                        const uint8_t s8 = k_ksigns[(aux >> (7 * l)) & 127];
                        for (int h = 0; h < 2; ++h) {
                            const uint32_t g = k_iq3xxs_grid[w[2 + 8 * s + 2 * l + h]];
                            for (int j = 0; j < 4; ++j) {
                                const int v = (int) ((g >> (8 * j)) & 0xff);
                                y[32 * s + 8 * l + 4 * h + j] = (int8_t) (((s8 >> (4 * h + j)) & 1) ? -v : v);
                            }
                        }
                    }
                }
                break;
            case T_IQ3_S:
                for (int s = 0; s < 8; ++s) {
                    const uint8_t qh = w[66 + s];
                    for (int l = 0; l < 4; ++l) {
                        const uint8_t s8 = w[74 + 4 * s + l];
                        for (int h = 0; h < 2; ++h) {
                            const int j8 = 2 * l + h;
                            const uint32_t g = k_iq3s_grid[w[2 + 8 * s + j8] | (((qh >> j8) & 1) << 8)];
                            for (int j = 0; j < 4; ++j) {
                                const int v = (int) ((g >> (8 * j)) & 0xff);
                                y[32 * s + 8 * l + 4 * h + j] = (int8_t) (((s8 >> (4 * h + j)) & 1) ? -v : v);
                            }
                        }
                    }
                }
                break;
            case T_Q4_0:
                for (int j = 0; j < 16; ++j) {
                    y[j] = (int8_t) ((w[2 + j] & 15) - 8);
                    y[j + 16] = (int8_t) ((w[2 + j] >> 4) - 8);
                }
                break;
            case T_Q8_0:
                for (int j = 0; j < 32; ++j) y[j] = (int8_t) w[2 + j];
                break;
            case T_Q4_K:
                for (int j = 0; j < 4; ++j)
                    for (int l = 0; l < 32; ++l) {
                        y[64 * j + l] = (int8_t) (w[16 + 32 * j + l] & 15);
                        y[64 * j + 32 + l] = (int8_t) (w[16 + 32 * j + l] >> 4);
                    }
                break;
            case T_Q6_K: {
                const uint8_t* ql = w;
                const uint8_t* qh = w + 128;
                for (int half = 0; half < 2; ++half)
                    for (int l = 0; l < 32; ++l) {
                        y[128 * half + l + 0] = (int8_t) ((int) ((ql[64 * half + l] & 0xF) | (((qh[32 * half + l] >> 0) & 3) << 4)) - 32);
                        y[128 * half + l + 32] = (int8_t) ((int) ((ql[64 * half + l + 32] & 0xF) | (((qh[32 * half + l] >> 2) & 3) << 4)) - 32);
                        y[128 * half + l + 64] = (int8_t) ((int) ((ql[64 * half + l] >> 4) | (((qh[32 * half + l] >> 4) & 3) << 4)) - 32);
                        y[128 * half + l + 96] = (int8_t) ((int) ((ql[64 * half + l + 32] >> 4) | (((qh[32 * half + l] >> 6) & 3) << 4)) - 32);
                    }
                break;
            }
            default: break;
        }
    }
}

/* ------------------------------------------------------------------------------------------------ routers */
/* Qwen: softmax over n_expert logits (max-shifted), NaN -> -FLT_MAX, k argmax picks (lowest id on ties),
 * w = p / max(sum of picked p, 6.103515625e-5).  native_router.cu:44-95.  Returns the number of tokens whose
 * k-th and (k+1)-th probabilities are within `tie_ulps` float ulps (ids there depend on the exp rounding). */
static float ulp_gap(float a, float b) {
    int32_t ia, ib;
    memcpy(&ia, &a, 4);
    memcpy(&ib, &b, 4);
    if (ia < 0) ia = (int32_t) 0x80000000 - ia;
    if (ib < 0) ib = (int32_t) 0x80000000 - ib;
    return fabsf((float) ia - (float) ib);
}

int or_router_softmax_topk(const float* logits, int n_tok, int n_expert, int ld, int k, int32_t* ids, float* w,
                           float tie_ulps) {
    float* p = (float*) malloc(sizeof(float) * (size_t) n_expert);
    int near_ties = 0;
    for (int t = 0; t < n_tok; ++t) {
        const float* lg = logits + (size_t) t * ld;
        float mx = -INFINITY;
        for (int e = 0; e < n_expert; ++e) mx = fmaxf(mx, lg[e]);
        double sum = 0.0;
        for (int e = 0; e < n_expert; ++e) { p[e] = expf(lg[e] - mx); sum += p[e]; }
        const float rec = (float) (1.0 / sum);
        for (int e = 0; e < n_expert; ++e) {
            p[e] *= rec;
            if (isnan(p[e])) p[e] = -3.402823466e38f;
        }
        float picked = 0.0f;
        float sel[64];
        for (int r = 0; r < k; ++r) {
            int best = 0;
            for (int e = 1; e < n_expert; ++e)
                if (p[e] > p[best]) best = e;
            ids[(size_t) t * k + r] = best;
            sel[r] = p[best];
            picked += p[best];
            p[best] = -INFINITY;
        }
        /* near-tie check between the last pick and the best unpicked, and between consecutive picks */
        float nxt = -INFINITY;
        for (int e = 0; e < n_expert; ++e) nxt = fmaxf(nxt, p[e]);
        if (ulp_gap(sel[k - 1], nxt) <= tie_ulps) ++near_ties;
        else
            for (int r = 1; r < k; ++r)
                if (ulp_gap(sel[r - 1], sel[r]) <= tie_ulps) { ++near_ties; break; }
        const float denom = fmaxf(picked, 6.103515625e-5f);
        for (int r = 0; r < k; ++r) w[(size_t) t * k + r] = sel[r] / denom;
    }
    free(p);
    return near_ties;
}

/* Gemma/LFM route_rows (gemma4/kernels.cu:289-356): gate 0 = softmax(logit * in_scale), gate 1 = sigmoid;
 * the pick is the largest p + bias (lowest id on ties); w = p (the bare gate) [/ max(sum, 6.1e-5) when norm]
 * [* escale[id]] [* w_scale when nonzero]. */
void or_route_rows(const float* logits, int n_expert, int n_used, int rows, int gate, float in_scale, const float* bias,
                   const float* escale, int norm, float w_scale, int32_t* ids, float* w) {
    float* p = (float*) malloc(sizeof(float) * (size_t) n_expert * 2);
    float* pick = p + n_expert;
    for (int t = 0; t < rows; ++t) {
        const float* lg = logits + (size_t) t * n_expert;
        if (gate == 0) {
            float mx = -INFINITY;
            for (int e = 0; e < n_expert; ++e) mx = fmaxf(mx, lg[e] * in_scale);
            double sum = 0.0;
            for (int e = 0; e < n_expert; ++e) { p[e] = expf(lg[e] * in_scale - mx); sum += p[e]; }
            const float inv = (float) (1.0 / sum);
            for (int e = 0; e < n_expert; ++e) p[e] *= inv;
        } else {
            for (int e = 0; e < n_expert; ++e) p[e] = 1.0f / (1.0f + expf(-(lg[e] * in_scale)));
        }
        for (int e = 0; e < n_expert; ++e) pick[e] = p[e] + (bias ? bias[e] : 0.0f);
        float sum = 0.0f;
        for (int j = 0; j < n_used; ++j) {
            int best = 0;
            for (int e = 1; e < n_expert; ++e)
                if (pick[e] > pick[best]) best = e;
            pick[best] = -INFINITY;
            ids[(size_t) t * n_used + j] = best;
            w[(size_t) t * n_used + j] = p[best];
            sum += p[best];
        }
        for (int j = 0; j < n_used; ++j) {
            float v = w[(size_t) t * n_used + j];
            if (norm) v /= fmaxf(sum, 6.103515625e-5f);
            if (escale) v *= escale[ids[(size_t) t * n_used + j]];
            if (w_scale != 0.0f) v *= w_scale;
            w[(size_t) t * n_used + j] = v;
        }
    }
    free(p);
}

/* ------------------------------------------------------------------------------------------------ grouping */
/* Decode grouping, q36_engine.cu:396-422: one group per expert used (ascending id), its entries in entry order;
 * entry e = t * K + k.  grp_expert[g] is the expert id (the reference stores its blob address).  Returns n_groups. */
int or_group(const int32_t* ids, int n_ent, int K, int n_expert, int32_t* grp_expert, int32_t* grp_start,
             int32_t* ent_dst, int32_t* ent_tok) {
    int* cnt = (int*) calloc((size_t) n_expert, sizeof(int));
    int* off = (int*) calloc((size_t) n_expert, sizeof(int));
    for (int e = 0; e < n_ent; ++e) cnt[ids[e]]++;
    int g = 0, pos = 0;
    for (int x = 0; x < n_expert; ++x) {
        off[x] = pos;
        if (cnt[x] == 0) continue;
        grp_expert[g] = x;
        grp_start[g] = pos;
        pos += cnt[x];
        ++g;
    }
    grp_start[g] = pos;
    for (int e = 0; e < n_ent; ++e) {
        const int p = off[ids[e]]++;
        ent_dst[p] = e;
        ent_tok[p] = e / K;
    }
    free(cnt);
    free(off);
    return g;
}

/* Prefill permutation, q36_engine.cu:486-510 (count, exclusive scan, scatter, inverse), in the stable
 * (expert, entry) order: bounds[x]..bounds[x+1] are expert x's sorted rows, dst[r] the entry, src[r] its token,
 * inv[e] the sorted row of entry e.  Returns the largest expert's row count. */
int or_dispatch(const int32_t* ids, int n_ent, int K, int n_expert, int32_t* bounds, int32_t* dst, int32_t* src,
                int32_t* inv) {
    int* cur = (int*) calloc((size_t) n_expert + 1, sizeof(int));
    for (int e = 0; e < n_ent; ++e) cur[ids[e]]++;
    int pos = 0, mx = 0;
    for (int x = 0; x < n_expert; ++x) {
        bounds[x] = pos;
        const int c = cur[x];
        cur[x] = pos;
        pos += c;
        if (c > mx) mx = c;
    }
    bounds[n_expert] = pos;
    for (int e = 0; e < n_ent; ++e) {
        const int r = cur[ids[e]]++;
        dst[r] = e;
        src[r] = e / K;
        inv[e] = r;
    }
    free(cur);
    return mx;
}

/* ------------------------------------------------------------------------------------------------ activations */
enum { ACT_SWIGLU = 0, ACT_GELU_TANH = 1, ACT_SWIGLU_CLAMP = 2 };

static float act_apply(int act, float g, float u, float limit) {
    switch (act) {
        case ACT_GELU_TANH: {
            const float c = 0.5f * g * (1.0f + tanhf(0.79788456080286535587989211986876f * g * (1.0f + 0.044715f * g * g)));
            return c * u;
        }
        case ACT_SWIGLU_CLAMP: {
            const float gc = fminf(g, limit);
            const float uc = fminf(fmaxf(u, -limit), limit);
            return gc / (1.0f + expf(-gc)) * uc;
        }
        default: return (g / (1.0f + expf(-g))) * u;
    }
}

/* ------------------------------------------------------------------------------------------------ the layer */
/* One expert's gated FFN for one token: hq (q8_1 of the token's activation, n_embd values) -> out (n_embd).
 * gate rows at blob, up rows at blob + up_off, down rows at blob + down_off (NativeExpertLayout, iq_kernels.cu:2120).
 * The hidden h = act(gate, up) is quantised to q8_1 (iq_kernels.cu:1496-1516) before the down product. */
void or_expert_ffn(int gu_type, int d_type, const uint8_t* blob, int64_t n_embd, int64_t n_ff, int act, float limit,
                   const uint8_t* xq, float* out, float* h_out) {
    const int64_t gu_row = or_row_bytes(gu_type, n_embd), d_row = or_row_bytes(d_type, n_ff);
    const int64_t up_off = n_ff * gu_row, down_off = 2 * up_off;
    float* h = (float*) malloc(sizeof(float) * (size_t) n_ff);
    uint8_t* hq = (uint8_t*) malloc((size_t) (n_ff / 32) * Q8_1_BYTES);
    for (int64_t r = 0; r < n_ff; ++r) {
        const float g = (float) or_row_dot(gu_type, blob + r * gu_row, xq, n_embd);
        const float u = (float) or_row_dot(gu_type, blob + up_off + r * gu_row, xq, n_embd);
        h[r] = act_apply(act, g, u, limit);
    }
    if (h_out) memcpy(h_out, h, sizeof(float) * (size_t) n_ff);
    or_quantize_q8_1_rows(h, 1, n_ff, hq);
    for (int64_t i = 0; i < n_embd; ++i) out[i] = (float) or_row_dot(d_type, blob + down_off + i * d_row, hq, n_ff);
    free(h);
    free(hq);
}

/* Combine one token (k_moe_out, q36_engine.cu:307-332): acc = w0 p0; acc = fma(w_k, p_k, acc) in pick order;
 * acc += gs * shared (gs = sigmoid(sgate), or 1 with no gate); out = x + acc.  Carried in double here. */
void or_combine_token(const float* x, const float* const* parts, const float* wts, int K, const float* shared,
                      float gs, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        double acc = (double) wts[0] * parts[0][i];
        for (int k = 1; k < K; ++k) acc += (double) wts[k] * parts[k][i];
        if (shared) acc += (double) gs * shared[i];
        out[i] = (float) ((double) (x ? x[i] : 0.0f) + acc);
    }
}

/* RMS norm and q8_1 of the next layer's input (k_moe_out_small epilogue, q36_kernels.cuh:252-290). */
void or_rms_q8_1(const float* x, const float* wn, int64_t n, float eps, float* h, uint8_t* hq) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double) x[i] * x[i];
    const float r = (float) (1.0 / sqrt(s / (double) n + (double) eps));
    for (int64_t i = 0; i < n; ++i) h[i] = x[i] * r * (wn ? wn[i] : 1.0f);
    if (hq) or_quantize_q8_1_rows(h, 1, n, hq);
}
