// tsb_mmq.cuh - the prefill (many-token) grouped expert products as int8 contractions on the 5th-generation tensor
// cores: tcgen05.mma.kind::i8 with TMA-staged activation tiles and int32 block sums in tensor memory.
//
// Reference: the prompt path runs llama.cpp's MMQ over rows sorted by expert (src/prefill/moe_mmq.cu:334-384,
// moe_mmq.hpp:58-81; src/gemma4/mmq.cu:74-110): per 32-value block an exact integer dot of the q8_1 activation codes
// with the weight's integer codes, then the block's scales in fp32, summed block after block.  Here:
//   * the activations live in the "mmq" layout (the role of the reference's block_q8_1_mmq): int8 codes [rows][K] and
//     fp32 block scales [rows][ldS] (d, and d * sum of codes for Q4_K's min term), written by tsb_mmq_quantize (fp32
//     rows, optionally gathered by a row map: the expert-sorted order) or by the gate/up epilogue (the hidden vectors);
//     TMA loads 128-row x 128-value code tiles with the 128-byte swizzle the MMA descriptors read, and the scale tiles;
//   * producer warps decode each weight row's GGUF blocks into the int8 codes the block dot multiplies (Q4_0 nibble - 8,
//     Q8_0 codes, Q4_K nibbles, Q6_K codes - 32, IQ3 signed grid bytes) in the same swizzled layout, and stage the
//     per-(row, block) scale terms;
//   * one thread issues one tcgen05.mma.kind::i8 M128 N128 K32 per 32-value block (Q6_K: two, one per 16-value half,
//     the other half's weight codes zero) into one of four int32 block-sum buffers in tensor memory;
//   * eight epilogue warps (two per tensor-memory lane quarter, 64 columns each) read a block's sums, add the word
//     0x4B400000 to each (an integer add: the float bits of 1.5 * 2^23 + S for the block sum S, |S| < 2^22, so no
//     conversion instruction; fma(fb, d_x, -d_x * 1.5 * 2^23) is d_x * S rounded once, d_x * 1.5 * 2^23 being exact)
//     and add d_w (d_x S) into fp32 register accumulators block after block with packed FMAs -- the reference's
//     per-block scaling, two FMAs per output per block;
//   * gate/up tiles interleave the matrices in 32-row groups (B rows 0-31 gate, 32-63 up of the same hidden values,
//     64-95 gate, 96-127 up of the next 32), so a thread's 64 columns are the gate and up sums of one q8_1 block of
//     hidden values: the activation, the q8_1 quantisation (the reference's arithmetic) and the store of the hidden
//     vector in the mmq layout happen in the epilogue; down tiles store fp32 rows.
// The exact per-block integer sums are the contract (the block dots of the reference, bit for bit); the fp32 scaling
// and sum follow the reference's per-block order (within fp32 rounding of its MMQ, whose source is not available here).
#pragma once

#include "tsb_prefill_k.cuh"

#include <cuda.h>

namespace tsb {

constexpr int kMqBM = 128, kMqBN = 128, kMqBK = 128, kMqBlk = kMqBK / 32;   // 4 blocks of 32 values per ring stage
// 11 warps: at most three share an SM sub-partition, so a thread may hold 168 registers (16 K registers a
// sub-partition; 13 warps would put four on one and cap every thread at 128, which spills the epilogue's 64
// accumulators and 64 block sums).  Producers: two warps, a thread stages two weight rows.
constexpr int kMqProd = 2, kMqMma = 2, kMqEpi0 = 3, kMqEpi = 8, kMqWarps = 11;
constexpr int kMqThreads = kMqWarps * 32;
constexpr int kMqBufs = 4;                                   // tensor-memory block-sum buffers of 128 columns
constexpr uint32_t kMqTile = 128 * 128;                      // an int8 operand tile: 16 KB
constexpr uint32_t kMqXScale = 128 * kMqBlk * 4;             // a [128 rows][4 blocks] fp32 scale tile (2 KB)
constexpr uint32_t kMqWTerm = kMqBlk * 128 * 4;              // a [4 blocks][128 columns] fp32 weight term (2 KB)
constexpr uint32_t kMqMagic = 0x4B400000u;                   // float bits of 1.5 * 2^23
constexpr float kMqMagicF = 12582912.0f;
constexpr int kMqMaxGroups = 512;
// The MMA thread signals block sums two units at a time (a tile always holds an even number of units: K is a
// multiple of 64), halving the epilogue's barrier waits (3-4 % faster gate/up and down).
constexpr bool kMqPairHandoff = true;
constexpr uint32_t kMqSmemBudget = 220 * 1024;
// instruction descriptor: D s32, A s8, B s8, both K-major, N = 128, M = 128
constexpr uint32_t kMqIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (kMqBN >> 3) << 17) |
                              ((uint32_t) (kMqBM >> 4) << 24);

// Per weight format: the weight block (values, bytes), tensor-core sums per 32-value block, fp32 weight terms per
// (column, block), whether the min term (activation d * sum of codes) is used, and the codebook table words.
template <int WT> struct MqFmt;
template <> struct MqFmt<T_Q4_0> { static constexpr int kQK = 32, kBytes = 18, kSplit = 1, kTerms = 1; static constexpr bool kSx = false; static constexpr int kTab = 0; };
template <> struct MqFmt<T_Q8_0> { static constexpr int kQK = 32, kBytes = 34, kSplit = 1, kTerms = 1; static constexpr bool kSx = false; static constexpr int kTab = 0; };
template <> struct MqFmt<T_Q4_K> { static constexpr int kQK = 256, kBytes = 144, kSplit = 1, kTerms = 2; static constexpr bool kSx = true; static constexpr int kTab = 0; };
template <> struct MqFmt<T_Q6_K> { static constexpr int kQK = 256, kBytes = 210, kSplit = 2, kTerms = 2; static constexpr bool kSx = false; static constexpr int kTab = 0; };
template <> struct MqFmt<T_IQ3_XXS> { static constexpr int kQK = 256, kBytes = 98, kSplit = 1, kTerms = 2; static constexpr bool kSx = false; static constexpr int kTab = 256; };
template <> struct MqFmt<T_IQ3_S> { static constexpr int kQK = 256, kBytes = 110, kSplit = 1, kTerms = 1; static constexpr bool kSx = false; static constexpr int kTab = 512; };

template <int WT>
struct MqLayout {   // one ring stage: A | B (x split) | d_x | (s_x) | weight terms
    static constexpr uint32_t kA = 0, kB = kMqTile, kDx = kB + MqFmt<WT>::kSplit * kMqTile;
    static constexpr uint32_t kSx = kDx + kMqXScale;
    static constexpr uint32_t kW = kSx + (MqFmt<WT>::kSx ? kMqXScale : 0u);
    static constexpr uint32_t kStage = (kW + MqFmt<WT>::kTerms * kMqWTerm + 1023u) & ~1023u;
    static constexpr uint32_t kTabBytes = MqFmt<WT>::kTab * 4u;
    static constexpr int kStages = (int) ((kMqSmemBudget - 1024u - kTabBytes) / kStage) > 6 ? 6
                                 : (int) ((kMqSmemBudget - 1024u - kTabBytes) / kStage);
    static constexpr uint32_t kSmem = kStages * kStage + kTabBytes + 1024u;
    static constexpr uint32_t kTxBytes = kMqTile + kMqXScale * (MqFmt<WT>::kSx ? 2u : 1u);
};

enum : int { MQ_GU = 0, MQ_DOWN = 1 };

struct MqParams {
    // groups: group g owns rows [bounds[g], bounds[g+1]) of the activations and the weight matrix of blob g
    const int32_t* bounds;     // [n_groups + 1] on the device (null: one group of n_rows rows)
    int n_groups, n_rows;
    const uint8_t* blobs;
    uint64_t blob_stride;
    uint64_t w_off;            // byte offset of the matrix in the blob (gate rows; down rows)
    uint64_t up_off;           // gate/up: offset of the up rows from the gate rows
    uint32_t w_row;            // bytes per weight row
    int K;                     // contraction length (a multiple of 32; of 256 for the super-block formats)
    int N;                     // output columns (gate/up: n_ff hidden values; down: n_embd)
    // gate/up output: the hidden vectors in the mmq layout, [n_rows][N] codes and [n_rows][ldh] scales
    int8_t* hc;
    float* hd;
    float* hs;
    int ldh;
    float* D;                  // down output: fp32 rows of ld_d floats, row drow[r] (r when drow is null)
    const int32_t* drow;
    long long ld_d;
    int act;
    float limit;
    unsigned* err;
    int32_t* dbg;              // optional: the block sums of this launch's first tile [K / 32][split][128][128]
};

// ------------------------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ void mq_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n"
                 ::"r"(tmem), "l"(da), "l"(db), "r"(kMqIdesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"((uint64_t) map), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t) map) : "memory");
}
__device__ __forceinline__ void tmem_ld32u(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                   "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(addr));
}
// Two columns at once: a += w * (fma(f, dx, ndxm)) with the packed fp32 pipe instructions (the same IEEE roundings as
// two scalar fma pairs, half the instructions).  The intrinsic, not inline assembly: the compiler schedules it.
__device__ __forceinline__ void mq_fma2(float& a0, float& a1, float w0, float w1, uint32_t f0, uint32_t f1, float dx,
                                        float ndxm) {
    const float2 t = __ffma2_rn(make_float2(__uint_as_float(f0), __uint_as_float(f1)), make_float2(dx, dx),
                                make_float2(ndxm, ndxm));
    const float2 r = __ffma2_rn(make_float2(w0, w1), t, make_float2(a0, a1));
    a0 = r.x;
    a1 = r.y;
}
// Four weight terms from shared memory, in program order with the FMAs that use them (volatile: the compiler may not
// hoist all sixteen of a block's loads ahead of its FMAs, which would need 64 more registers than a thread has).
__device__ __forceinline__ float4 lds4(const float4* p) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(smem_u32(p)));
    return v;
}
// a += w * t for two columns, t given (packed).
__device__ __forceinline__ void mq_fma2t(float& a0, float& a1, float w0, float w1, float t0, float t1) {
    const float2 r = __ffma2_rn(make_float2(w0, w1), make_float2(t0, t1), make_float2(a0, a1));
    a0 = r.x;
    a1 = r.y;
}

// Four int8 values b - 8 from four nibbles b (one per byte): (b + 0x78) ^ 0x80 per byte, with no carry between bytes.
__device__ __forceinline__ uint32_t centre4(uint32_t nib) { return ((nib & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u; }
// Byte masks (0xFF where bit k of the 4-bit s is set, byte k) and a grid word with those signs applied: for a byte g
// in 1..127 and mask m in {0, 0xFF}, (g ^ m) + (m & 1) is g or -g with no carry out of the byte.
__device__ __forceinline__ uint32_t sign_mask4(uint32_t s) { return ((s * 0x00204081u) & 0x01010101u) * 0xFFu; }
__device__ __forceinline__ uint32_t apply_sign4(uint32_t g, uint32_t s) {
    const uint32_t m = sign_mask4(s & 15u);
    return (g ^ m) + (m & 0x01010101u);
}

// ------------------------------------------------------------------------------------------------ weight staging
// The raw bytes one producer thread loads for one ring stage (128 values of one weight row), a stage ahead of their
// conversion: 4-byte words from the row's 4-byte (Q4_0), 8-byte (Q8_0) or 16-byte (K-quants) aligned stage start, or
// a 2-byte aligned start read with funnel shifts (Q6_K, IQ3: rows of 210 / 98 / 110-byte blocks).
template <int WT> struct MqRaw;
template <> struct MqRaw<T_Q4_0> { uint32_t w[18]; };   // 4 blocks x 18 bytes
template <> struct MqRaw<T_Q8_0> { uint32_t w[34]; };   // 4 blocks x 34 bytes
template <> struct MqRaw<T_Q4_K> { uint32_t h[4]; uint32_t q[16]; };   // header (d, dmin, scales) + 64 qs bytes
template <> struct MqRaw<T_Q6_K> { uint32_t ql[16]; uint32_t qh[8]; uint32_t sc[2]; uint32_t d; };
template <> struct MqRaw<T_IQ3_XXS> { uint32_t qs[8]; uint32_t aux[4]; uint32_t d; };
template <> struct MqRaw<T_IQ3_S> { uint32_t qs[8]; uint32_t qh; uint32_t sg[4]; uint32_t sc; uint32_t d; };

// Stage ks of a row: values [128 ks, 128 ks + nbs * 32) (nbs < 4 only at the end of the row).
template <int WT>
__device__ __forceinline__ void mq_load(MqRaw<WT>& R, const uint8_t* wrow, int ks, int nbs) {
    if (!wrow) return;
    if constexpr (WT == T_Q4_0 || WT == T_Q8_0) {
        constexpr int BB = MqFmt<WT>::kBytes;   // 18 or 34 bytes a block; the stage starts at 4 BB ks (8-aligned)
        const uint8_t* src = wrow + (size_t) ks * 4 * BB;
        const int nw = (BB * nbs + 3) / 4;      // words of the nbs blocks present
        if (((uintptr_t) src & 7u) == 0) {
#pragma unroll
            for (int i = 0; i < BB / 2; ++i) {
                if (2 * i + 1 < nw) {
                    const uint2 v = __ldg((const uint2*) src + i);
                    R.w[2 * i] = v.x;
                    R.w[2 * i + 1] = v.y;
                } else if (2 * i < nw) {   // an odd last word: nothing past the row's last block is read
                    R.w[2 * i] = __ldg((const uint32_t*) src + 2 * i);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < BB; ++i)
                if (i < nw) R.w[i] = __ldg((const uint32_t*) src + i);
        }
    } else if constexpr (WT == T_Q4_K) {
        const uint8_t* b = wrow + (size_t) (ks >> 1) * 144;
        const uint4 h = __ldg((const uint4*) b);
        R.h[0] = h.x; R.h[1] = h.y; R.h[2] = h.z; R.h[3] = h.w;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg((const uint4*) (b + 16 + 64 * (ks & 1)) + i);
            R.q[4 * i] = v.x; R.q[4 * i + 1] = v.y; R.q[4 * i + 2] = v.z; R.q[4 * i + 3] = v.w;
        }
    } else if constexpr (WT == T_Q6_K) {
        const uint8_t* b = wrow + (size_t) (ks >> 1) * 210;
        const int n = ks & 1;
        ldw<16>(b + 64 * n, R.ql);
        ldw<8>(b + 128 + 32 * n, R.qh);
        ldw<2>(b + 192 + 8 * n, R.sc);
        R.d = ldh(b + 208);
    } else if constexpr (WT == T_IQ3_XXS) {
        const uint8_t* b = wrow + (size_t) (ks >> 1) * 98;
        const int n = ks & 1;
        ldw<8>(b + 2 + 32 * n, R.qs);
        ldw<4>(b + 66 + 16 * n, R.aux);
        R.d = ldh(b);
    } else {   // T_IQ3_S
        const uint8_t* b = wrow + (size_t) (ks >> 1) * 110;
        const int n = ks & 1;
        ldw<8>(b + 2 + 32 * n, R.qs);
        uint32_t t[1];
        ldw<1>(b + 66 + 4 * n, t);
        R.qh = t[0];
        ldw<4>(b + 74 + 16 * n, R.sg);
        R.sc = ldh(b + 106 + 2 * n);
        R.d = ldh(b);
    }
}

// Bytes i .. i + 3 of a word array, any i (funnel shift across the two words).
__device__ __forceinline__ uint32_t word_at(const uint32_t* w, int i) {
    const int q = i >> 2, sh = (i & 3) * 8;
    return sh ? __funnelshift_r(w[q], w[q + 1], sh) : w[q];
}

// Stage the int8 codes of block b (values 32 b .. 32 b + 31 of the stage) into chunks 2b, 2b + 1 of tile row r (Q6_K:
// tile 0 the first 16 values with the rest zero, tile 1 the second 16), and the block's weight terms.
template <int WT>
__device__ __forceinline__ void mq_stage(const MqRaw<WT>& R, int b, uint8_t* tile, int r, float* wt, const uint32_t* tab) {
    if constexpr (WT == T_Q4_0) {
        const int o = 18 * b;   // d at o, nibbles at o + 2
        uint32_t q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = word_at(R.w, o + 2 + 4 * i);
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(centre4(q[0]), centre4(q[1]), centre4(q[2]), centre4(q[3]));
        *(uint4*) (tile + sw128(r, 2 * b + 1)) =
            make_uint4(centre4(q[0] >> 4), centre4(q[1] >> 4), centre4(q[2] >> 4), centre4(q[3] >> 4));
        wt[b * 128 + r] = h2f(word_at(R.w, o));
    } else if constexpr (WT == T_Q8_0) {
        const int o = 34 * b;
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = word_at(R.w, o + 2 + 4 * i);
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(q[0], q[1], q[2], q[3]);
        *(uint4*) (tile + sw128(r, 2 * b + 1)) = make_uint4(q[4], q[5], q[6], q[7]);
        wt[b * 128 + r] = h2f(word_at(R.w, o));
    } else if constexpr (WT == T_Q4_K) {
        // sub-block j = 4 (ks & 1) + b: the low (b even) or high (b odd) nibbles of qs bytes 32 (b / 2) .. + 32 of the stage
        const uint32_t* q = R.q + 8 * (b >> 1);
        const int sh = 4 * (b & 1);
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (q[i] >> sh) & 0x0F0F0F0Fu;
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(v[0], v[1], v[2], v[3]);
        *(uint4*) (tile + sw128(r, 2 * b + 1)) = make_uint4(v[4], v[5], v[6], v[7]);
        // (the sub-block index and scale words are set by the caller's stage half: see mq_stage_q4k_terms)
    } else if constexpr (WT == T_Q6_K) {
        // block b of the half: values l = 0..31 take ql[l + 32 (b & 1)] (low nibble for b < 2, high for b >= 2) and
        // qh[l] bits 2b, 2b + 1 (ggml's q1..q4 order); code - 32
        const uint32_t* ql = R.ql + 8 * (b & 1);
        const int lsh = 4 * (b >> 1), hsh = 2 * b;
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t lo = (ql[i] >> lsh) & 0x0F0F0F0Fu;
            const uint32_t hi = ((R.qh[i] >> hsh) & 0x03030303u) << 4;
            v[i] = ((lo | hi) + 0x60606060u) ^ 0x80808080u;   // (c + 0x60) ^ 0x80 = c - 32 per byte, c < 64
        }
        uint8_t* t1 = tile + kMqTile;
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(v[0], v[1], v[2], v[3]);   // values 0..15: tile 0
        *(uint4*) (tile + sw128(r, 2 * b + 1)) = make_uint4(0u, 0u, 0u, 0u);
        *(uint4*) (t1 + sw128(r, 2 * b)) = make_uint4(0u, 0u, 0u, 0u);
        *(uint4*) (t1 + sw128(r, 2 * b + 1)) = make_uint4(v[4], v[5], v[6], v[7]);   // values 16..31: tile 1
        const float d = h2f(R.d);
        const uint32_t scw = R.sc[b >> 1] >> (16 * (b & 1));   // sc[2b], sc[2b + 1] of the half
        wt[b * 128 + r] = d * (float) (int8_t) (scw & 0xFFu);
        wt[kMqBlk * 128 + b * 128 + r] = d * (float) (int8_t) ((scw >> 8) & 0xFFu);
    } else if constexpr (WT == T_IQ3_XXS) {
        const uint32_t aux = R.aux[b];
        uint32_t v[8];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t sidx = (aux >> (7 * l)) & 127u;
            const uint32_t sgn = sidx | ((uint32_t) (__popc(sidx) & 1) << 7);   // the even-parity sign byte
            const uint32_t qw = R.qs[2 * b + (l >> 1)] >> (16 * (l & 1));
            v[2 * l] = apply_sign4(tab[qw & 0xFFu], sgn);
            v[2 * l + 1] = apply_sign4(tab[(qw >> 8) & 0xFFu], sgn >> 4);
        }
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(v[0], v[1], v[2], v[3]);
        *(uint4*) (tile + sw128(r, 2 * b + 1)) = make_uint4(v[4], v[5], v[6], v[7]);
        wt[b * 128 + r] = h2f(R.d);
        wt[kMqBlk * 128 + b * 128 + r] = __int_as_float((int) (aux >> 28));   // ls, as an integer
    } else {   // T_IQ3_S
        const uint32_t qh = (R.qh >> (8 * b)) & 0xFFu;
        uint32_t v[8];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t qw = R.qs[2 * b + (l >> 1)] >> (16 * (l & 1));
            const uint32_t i0 = (qw & 0xFFu) | (((qh >> (2 * l)) & 1u) << 8);
            const uint32_t i1 = ((qw >> 8) & 0xFFu) | (((qh >> (2 * l + 1)) & 1u) << 8);
            const uint32_t s8 = (R.sg[b] >> (8 * l)) & 0xFFu;
            v[2 * l] = apply_sign4(tab[i0], s8);
            v[2 * l + 1] = apply_sign4(tab[i1], s8 >> 4);
        }
        *(uint4*) (tile + sw128(r, 2 * b)) = make_uint4(v[0], v[1], v[2], v[3]);
        *(uint4*) (tile + sw128(r, 2 * b + 1)) = make_uint4(v[4], v[5], v[6], v[7]);
        const uint32_t sc = (R.sc >> (4 * b)) & 0xFu;
        wt[b * 128 + r] = h2f(R.d) * (float) (1 + 2 * (int) sc);
    }
}
// Q4_K's terms of block b of stage ks: d * sc_j and dmin * m_j of sub-block j = 4 (ks & 1) + b (scale_min_k4).
__device__ __forceinline__ void mq_q4k_terms(const MqRaw<T_Q4_K>& R, int ks, int b, int r, float* wt) {
    const int j = 4 * (ks & 1) + b;
    const uint32_t sc12[3] = {R.h[1], R.h[2], R.h[3]};
    int sc, m;
    if (j < 4) {
        sc = (int) byte_of(sc12, j) & 63;
        m = (int) byte_of(sc12, j + 4) & 63;
    } else {
        sc = (int) ((byte_of(sc12, j + 4) & 0xFu) | ((byte_of(sc12, j - 4) >> 6) << 4));
        m = (int) ((byte_of(sc12, j + 4) >> 4) | ((byte_of(sc12, j) >> 6) << 4));
    }
    wt[b * 128 + r] = h2f(R.h[0]) * (float) sc;
    wt[kMqBlk * 128 + b * 128 + r] = -(h2f(R.h[0] >> 16) * (float) m);
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int MODE, int WT>
__global__ void __launch_bounds__(kMqThreads, 1)
    k_mmq(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dx,
          const __grid_constant__ CUtensorMap tm_sx, MqParams p) {
    using F = MqFmt<WT>;
    using LY = MqLayout<WT>;
    constexpr int NST = LY::kStages, SPLIT = F::kSplit;
    extern __shared__ __align__(1024) uint8_t mq_raw[];
    uint8_t* smem = (uint8_t*) (((uintptr_t) mq_raw + 1023) & ~(uintptr_t) 1023);
    uint32_t* tab = (uint32_t*) (smem + NST * LY::kStage);
    __shared__ uint64_t full[NST], empty[NST], t_full[kMqBufs], t_empty[kMqBufs];
    __shared__ uint32_t tbase;
    __shared__ volatile int abort_flag;
    __shared__ int32_t gstart[kMqMaxGroups + 1];   // row starts
    __shared__ int32_t gtile[kMqMaxGroups + 1];    // prefix of 128-row tiles
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.n_groups;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], kMqProd + 1);         // the producer warps, and the TMA's expect-tx arrive
            mbar_init(&empty[s], 1 + kMqEpi);         // the MMAs' commit and every epilogue warp (scales read)
        }
        for (int b = 0; b < kMqBufs; ++b) {
            mbar_init(&t_full[b], 1);
            mbar_init(&t_empty[b], kMqEpi);
        }
        abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_dx);
        if (F::kSx) tma_prefetch_desc(&tm_sx);
    }
    if (threadIdx.x == 32) {
        int t = 0;
        for (int g = 0; g <= G; ++g) {
            const int s = p.bounds ? __ldg(p.bounds + g) : (g == 0 ? 0 : p.n_rows);
            gstart[g] = s;
            gtile[g] = t;
            if (g < G) {
                const int e = p.bounds ? __ldg(p.bounds + g + 1) : p.n_rows;
                t += (max(e - s, 0) + kMqBM - 1) / kMqBM;
            }
        }
    }
    if constexpr (F::kTab > 0) {
        for (int i = threadIdx.x; i < F::kTab; i += blockDim.x)
            tab[i] = WT == T_IQ3_XXS ? g_iq3xxs_grid[i] : g_iq3s_grid[i];
    }
    if (warp == kMqMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tbase;
    const int q = warp & 3;                              // an epilogue warp's tensor-memory lane quarter (warp % 4)
    const int half = (warp - kMqEpi0) >> 2;              // ... and its 64 columns (warps 3-6: 0..63, 7-10: 64..127)
    const uint32_t lane_base = tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (64 * half);

    const int n_mt = gtile[G];
    const int per_tile = MODE == MQ_GU ? 64 : kMqBN;   // hidden values (gate/up) or output columns per tile
    const int n_nt = (p.N + per_tile - 1) / per_tile;
    const int n_tiles = n_mt * n_nt;
    const int nb = p.K / 32;                            // 32-value blocks of K
    const int nks = (nb + kMqBlk - 1) / kMqBlk;         // ring stages per tile
    auto tile_of = [&](int t, int& g, int& row0, int& row1, int& n0) {
        const int mt = t / n_nt, nt = t % n_nt;
        int lo = 0, hi = G - 1;
        while (lo < hi) {   // last group with gtile[g] <= mt (empty groups share their successor's start)
            const int mid = (lo + hi + 1) >> 1;
            if (gtile[mid] <= mt) lo = mid; else hi = mid - 1;
        }
        g = lo;
        row0 = gstart[g] + (mt - gtile[g]) * kMqBM;
        row1 = min(row0 + kMqBM, gstart[g + 1]);
        n0 = nt * per_tile;
    };

    if (warp < kMqProd) {
        // ------------------------------------------------------------------------ producers
        // thread r: weight rows r and r + 64 of every stage (their raw bytes loaded a stage ahead, except Q8_0's, whose
        // two 136-byte stages would not fit the registers); thread 0 also issues the stage's activation and scale TMA
        // loads as soon as the stage is free
        constexpr bool kAhead = WT != T_Q8_0;
        const int r = threadIdx.x;
        uint32_t it = 0;
        MqRaw<WT> R0[2], R1[2];
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            int g, row0, row1, n0;
            tile_of(tile, g, row0, row1, n0);
            const uint8_t* wrow[2] = {nullptr, nullptr};
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int br = r + 64 * k;   // the B row
                const uint8_t* base = p.blobs + (size_t) g * p.blob_stride + p.w_off;
                if (MODE == MQ_GU) {   // 32-row groups: gate, up, gate, up
                    const int j = n0 + (br >> 6) * 32 + (br & 31);
                    if (j < p.N) wrow[k] = base + ((br & 32) ? p.up_off : 0) + (size_t) j * p.w_row;
                } else {
                    const int j = n0 + br;
                    if (j < p.N) wrow[k] = base + (size_t) j * p.w_row;
                }
            }
            auto load = [&](MqRaw<WT> (&R)[2], int ks) {
                const int nbs = min(kMqBlk, nb - ks * kMqBlk);
                mq_load<WT>(R[0], wrow[0], ks, nbs);
                mq_load<WT>(R[1], wrow[1], ks, nbs);
            };
            auto stage = [&](const MqRaw<WT> (&cur)[2], int ks) -> bool {
                const int s = (int) (it % NST);
                if (it >= (uint32_t) NST) {
                    const uint32_t par = ((it / NST) - 1) & 1u;
                    const uint64_t t0 = globaltimer(), lim = wait_limit_ns();
                    while (!mbar_try_wait(&empty[s], par))
                        if (abort_flag || globaltimer() - t0 > lim) {
                            report_error(p.err, 0x601u);
                            abort_flag = 1;
                            return false;
                        }
                }
                uint8_t* st = smem + s * LY::kStage;
                if (r == 0) {
                    mbar_expect_tx(&full[s], LY::kTxBytes);
                    tma_load_2d(smem_u32(st + LY::kA), &tm_x, ks * kMqBK, row0, &full[s]);
                    tma_load_2d(smem_u32(st + LY::kDx), &tm_dx, ks * kMqBlk, row0, &full[s]);
                    if (F::kSx) tma_load_2d(smem_u32(st + LY::kSx), &tm_sx, ks * kMqBlk, row0, &full[s]);
                }
                const int nbs = min(kMqBlk, nb - ks * kMqBlk);
                float* wt = (float*) (st + LY::kW);
                uint8_t* tb = st + LY::kB;
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int br = r + 64 * k;
                    if (wrow[k]) {
#pragma unroll
                        for (int b = 0; b < kMqBlk; ++b)
                            if (b < nbs) {
                                mq_stage<WT>(cur[k], b, tb, br, wt, tab);
                                if constexpr (WT == T_Q4_K) mq_q4k_terms(cur[k], ks, b, br, wt);
                            }
                    } else {
#pragma unroll
                        for (int b = 0; b < kMqBlk; ++b)
                            if (b < nbs) {
#pragma unroll
                                for (int h = 0; h < SPLIT; ++h) {
                                    *(uint4*) (tb + h * kMqTile + sw128(br, 2 * b)) = make_uint4(0u, 0u, 0u, 0u);
                                    *(uint4*) (tb + h * kMqTile + sw128(br, 2 * b + 1)) = make_uint4(0u, 0u, 0u, 0u);
                                }
#pragma unroll
                                for (int t = 0; t < F::kTerms; ++t) wt[t * kMqBlk * 128 + b * 128 + br] = 0.0f;
                            }
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                ++it;
                return true;
            };
            if constexpr (kAhead) {
                load(R0, 0);
                for (int ks = 0; ks < nks && ok; ks += 2) {
                    if (ks + 1 < nks) load(R1, ks + 1);
                    ok = stage(R0, ks);
                    if (ok && ks + 1 < nks) {
                        if (ks + 2 < nks) load(R0, ks + 2);
                        ok = stage(R1, ks + 1);
                    }
                }
            } else {
                for (int ks = 0; ks < nks && ok; ++ks) {
                    load(R0, ks);
                    ok = stage(R0, ks);
                }
            }
        }
        // every TMA load this CTA issued has landed before the CTA may exit (bounded; they complete in microseconds)
        if (r == 0)
            for (uint32_t j = it > (uint32_t) NST ? it - NST : 0; j < it; ++j)
                mbar_wait_bounded(&full[j % NST], (j / NST) & 1u, p.err, 0x606u);
    } else if (warp == kMqMma) {
        // ------------------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t it = 0, u = 0;   // ring stage counter, MMA unit counter (blocks x split, across tiles)
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok && !abort_flag; tile += gridDim.x) {
                for (int ks = 0; ks < nks && ok; ++ks, ++it) {
                    const int s = (int) (it % NST);
                    if (!mbar_wait_bounded(&full[s], (it / NST) & 1u, p.err, 0x603u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int nbs = min(kMqBlk, nb - ks * kMqBlk);
                    const uint32_t a0 = smem_u32(smem + s * LY::kStage + LY::kA);
                    const uint32_t b0 = smem_u32(smem + s * LY::kStage + LY::kB);
                    for (int b = 0; b < nbs && ok; ++b) {
#pragma unroll
                        for (int h = 0; h < SPLIT; ++h, ++u) {
                            const int buf = (int) (u % kMqBufs);
                            if (u >= (uint32_t) kMqBufs &&
                                !mbar_wait_bounded(&t_empty[buf], ((u / kMqBufs) - 1) & 1u, p.err, 0x602u)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            mq_mma(tmem + (uint32_t) buf * 128, pf_sdesc(a0 + 32 * b), pf_sdesc(b0 + h * kMqTile + 32 * b), 0u);
                            if (!kMqPairHandoff || (u & 1u)) pf_commit(&t_full[buf]);
                        }
                    }
                    pf_commit(&empty[s]);   // the stage's operands are free once these MMAs complete
                }
            }
            if (!ok) abort_flag = 1;
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------------ epilogue (warps 5-12)
        uint32_t it = 0, u = 0;
        bool ok = true;
        const bool dbg_tile = p.dbg != nullptr && blockIdx.x == 0;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            int g, row0, row1, n0;
            tile_of(tile, g, row0, row1, n0);
            const int rl = q * 32 + lane;   // the tile row this thread owns
            const int row = row0 + rl;
            float acc[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
            for (int ks = 0; ks < nks && ok; ++ks, ++it) {
                const int s = (int) (it % NST);
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (it / NST) & 1u, p.err, 0x605u));
                if (!ok) break;
                const uint8_t* st = smem + s * LY::kStage;
                const float4 dx4 = *(const float4*) (st + LY::kDx + 16 * rl);
                float4 sx4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (F::kSx) sx4 = *(const float4*) (st + LY::kSx + 16 * rl);
                const float* wt = (const float*) (st + LY::kW);
                const int nbs = min(kMqBlk, nb - ks * kMqBlk);
                for (int b = 0; b < nbs; ++b) {
                    const float dx = b == 0 ? dx4.x : b == 1 ? dx4.y : b == 2 ? dx4.z : dx4.w;
                    const float ndxm = -dx * kMqMagicF;   // exact: 1.5 * 2^23 has two significant bits
                    const int buf0 = (int) (u % kMqBufs);
                    if (kMqPairHandoff) {
                        // units u, u + 1 (one block, or a Q6_K block's two halves) hand over together: the MMA
                        // commits after the odd one, whose completion implies the even one's
                        if ((u & 1u) == 0) {
                            const uint32_t w = u | 1u;
                            ok = __all_sync(0xffffffffu, mbar_wait_bounded(&t_full[w % kMqBufs], (w / kMqBufs) & 1u,
                                                                           p.err, 0x604u));
                            if (!ok) break;
                            tc_fence_after();
                        }
                    } else {
                        bool got = true;
                        for (int h = 0; h < SPLIT && got; ++h)
                            got = mbar_wait_bounded(&t_full[(buf0 + h) % kMqBufs], ((u + h) / kMqBufs) & 1u, p.err,
                                                    0x604u);
                        ok = __all_sync(0xffffffffu, got);
                        if (!ok) break;
                        tc_fence_after();
                    }
                    const float4* w4 = (const float4*) (wt + b * 128 + 64 * half);
                    if constexpr (SPLIT == 1) {
                        uint32_t f0[32], f1[32];
                        tmem_ld32u(lane_base + buf0 * 128, f0);
                        tmem_ld32u(lane_base + buf0 * 128 + 32, f1);
                        tmem_wait_ld();
                        auto fb = [&](int j) { return j < 32 ? f0[j] : f1[j - 32]; };
                        if (dbg_tile && tile == (int) blockIdx.x) {
                            int32_t* d = p.dbg + ((size_t) (ks * kMqBlk + b) * 128 + rl) * 128 + 64 * half;
#pragma unroll
                            for (int j = 0; j < 64; ++j) d[j] = (int32_t) fb(j);
                        }
                        if constexpr (WT == T_IQ3_XXS) {
                            // the reference's integer step (ls S + S / 2) / 2 (C division), then d_x times it
                            const float4* l4 = (const float4*) (wt + kMqBlk * 128 + b * 128 + 64 * half);
#pragma unroll
                            for (int j4 = 0; j4 < 16; ++j4) {
                                const float4 w = lds4(w4 + j4), lsf = lds4(l4 + j4);
                                const int ls[4] = {__float_as_int(lsf.x), __float_as_int(lsf.y), __float_as_int(lsf.z),
                                                   __float_as_int(lsf.w)};
                                uint32_t vb[4];
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int S = (int) fb(4 * j4 + k);
                                    vb[k] = (uint32_t) ((ls[k] * S + S / 2) / 2) + kMqMagic;
                                }
                                mq_fma2(acc[4 * j4], acc[4 * j4 + 1], w.x, w.y, vb[0], vb[1], dx, ndxm);
                                mq_fma2(acc[4 * j4 + 2], acc[4 * j4 + 3], w.z, w.w, vb[2], vb[3], dx, ndxm);
                            }
                        } else {
#pragma unroll
                            for (int j4 = 0; j4 < 16; ++j4) {
                                const float4 w = lds4(w4 + j4);
                                mq_fma2(acc[4 * j4], acc[4 * j4 + 1], w.x, w.y, fb(4 * j4) + kMqMagic,
                                        fb(4 * j4 + 1) + kMqMagic, dx, ndxm);
                                mq_fma2(acc[4 * j4 + 2], acc[4 * j4 + 3], w.z, w.w, fb(4 * j4 + 2) + kMqMagic,
                                        fb(4 * j4 + 3) + kMqMagic, dx, ndxm);
                            }
                            if constexpr (F::kSx) {   // Q4_K's min term: - (dmin m) (d_x sum q_x)
                                const float sx = b == 0 ? sx4.x : b == 1 ? sx4.y : b == 2 ? sx4.z : sx4.w;
                                const float4* m4 = (const float4*) (wt + kMqBlk * 128 + b * 128 + 64 * half);
#pragma unroll
                                for (int j4 = 0; j4 < 16; ++j4) {
                                    const float4 m = lds4(m4 + j4);
                                    mq_fma2t(acc[4 * j4], acc[4 * j4 + 1], m.x, m.y, sx, sx);
                                    mq_fma2t(acc[4 * j4 + 2], acc[4 * j4 + 3], m.z, m.w, sx, sx);
                                }
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&t_empty[buf0]);
                    } else {   // Q6_K: two sums per block (16-value halves), 32 columns at a time
                        const float4* v4 = (const float4*) (wt + kMqBlk * 128 + b * 128 + 64 * half);
                        const int buf1 = (buf0 + 1) % kMqBufs;
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            uint32_t fa[32], fc[32];
                            tmem_ld32u(lane_base + buf0 * 128 + 32 * c, fa);
                            tmem_ld32u(lane_base + buf1 * 128 + 32 * c, fc);
                            tmem_wait_ld();
                            if (dbg_tile && tile == (int) blockIdx.x) {
                                int32_t* d = p.dbg + ((size_t) (ks * kMqBlk + b) * 2 * 128 + rl) * 128 + 64 * half + 32 * c;
#pragma unroll
                                for (int j = 0; j < 32; ++j) {
                                    d[j] = (int32_t) fa[j];
                                    d[128 * 128 + j] = (int32_t) fc[j];
                                }
                            }
#pragma unroll
                            for (int j4 = 0; j4 < 8; ++j4) {
                                const float4 wa = lds4(w4 + 8 * c + j4), wb = lds4(v4 + 8 * c + j4);
                                float* a = acc + 32 * c + 4 * j4;
                                mq_fma2(a[0], a[1], wa.x, wa.y, fa[4 * j4] + kMqMagic, fa[4 * j4 + 1] + kMqMagic, dx,
                                        ndxm);
                                mq_fma2(a[2], a[3], wa.z, wa.w, fa[4 * j4 + 2] + kMqMagic, fa[4 * j4 + 3] + kMqMagic,
                                        dx, ndxm);
                                mq_fma2(a[0], a[1], wb.x, wb.y, fc[4 * j4] + kMqMagic, fc[4 * j4 + 1] + kMqMagic, dx,
                                        ndxm);
                                mq_fma2(a[2], a[3], wb.z, wb.w, fc[4 * j4 + 2] + kMqMagic, fc[4 * j4 + 3] + kMqMagic,
                                        dx, ndxm);
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&t_empty[buf0]);
                            mbar_arrive(&t_empty[buf1]);
                        }
                    }
                    u += SPLIT;
                }
                if (!ok) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);   // the stage's scales are read
            }
            if (!ok) {
                abort_flag = 1;
                break;
            }
            // the tile's sums: gate/up -> activation -> q8_1 (mmq layout); down -> fp32
            if (MODE == MQ_GU) {
                const int hb = n0 / 32 + half;   // this thread's q8_1 block of hidden values
                if (row < row1 && 32 * hb < p.N) {
                    float h[32], amax = 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        h[j] = act_value(p.act, acc[j], acc[32 + j], p.limit);
                        amax = fmaxf(amax, fabsf(h[j]));
                    }
                    const float d = q8_finite(fdiv_fm(amax, 127.0f));
                    uint32_t words[8];
                    int csum = 0;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        uint32_t word = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            int c = 0;
                            if (amax != 0.0f) {
                                const float rq = roundf(fdiv_fm(h[4 * w + k], d));
                                c = (int) (rq > 127.0f ? 127.0f : rq < -127.0f ? -127.0f : rq);
                            }
                            csum += c;
                            word |= (uint32_t) (uint8_t) (int8_t) c << (8 * k);
                        }
                        words[w] = word;
                    }
                    uint4* o = (uint4*) (p.hc + (size_t) row * p.N + 32 * hb);
                    o[0] = make_uint4(words[0], words[1], words[2], words[3]);
                    o[1] = make_uint4(words[4], words[5], words[6], words[7]);
                    const float dh = __half2float(__float2half(d));
                    p.hd[(size_t) row * p.ldh + hb] = dh;
                    p.hs[(size_t) row * p.ldh + hb] = dh * (float) csum;
                }
            } else {
                const int col = n0 + 64 * half;
                if (row < row1 && col < p.N) {
                    const long long orow = p.drow ? (long long) __ldg(p.drow + row) : (long long) row;
                    float4* dst = (float4*) (p.D + (size_t) orow * p.ld_d + col);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        dst[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
                }
            }
        }
        if (!ok) abort_flag = 1;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMqMma) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// ------------------------------------------------------------------------------------------------ activations
// fp32 rows -> the mmq layout: row r of the output is source row src[r] (null: r) of x (row stride ld_x floats); one
// CTA per output row, eight lanes per 32-value block with four values each (16-byte loads, 4-byte code stores).  The
// reference's q8_1 quantiser (iq_kernels.cu:1469-1480): d = amax / 127 with the fast-math division, codes roundf(x / d)
// clamped to +-127 -- the same codes and fp16 scale whatever the lane layout; codes [rows][K], d [rows][ldS] (the
// fp16-rounded scale), s [rows][ldS] = d * sum of the codes.
__global__ void __launch_bounds__(256) k_mmq_quantize(const float* __restrict__ x, long long ld_x,
                                                      const int32_t* __restrict__ src, int n_rows, int K,
                                                      int8_t* __restrict__ codes, float* __restrict__ ds,
                                                      float* __restrict__ ss, int ldS) {
    const int r = blockIdx.x;
    const int sr = src ? __ldg(src + r) : r;
    const float4* xr = (const float4*) (x + (size_t) sr * ld_x);
    uint32_t* cr = (uint32_t*) (codes + (size_t) r * K);
    const int lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i - lane < K / 4; i += blockDim.x) {   // whole warps: 8 blocks of 32 values a pass
        const bool in = i < K / 4;
        const float4 v = in ? __ldg(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = q8_finite(fdiv_fm(amax, 127.0f));
        const float xs[4] = {v.x, v.y, v.z, v.w};
        uint32_t word = 0;
        int cs = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int c = 0;
            if (amax != 0.0f) {
                const float rq = roundf(fdiv_fm(xs[j], d));
                c = (int) (rq > 127.0f ? 127.0f : rq < -127.0f ? -127.0f : rq);
            }
            cs += c;
            word |= (uint32_t) (uint8_t) (int8_t) c << (8 * j);
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
        if (in) {
            cr[i] = word;
            if ((lane & 7) == 0) {
                const float dh = __half2float(__float2half(d));
                ds[(size_t) r * ldS + (i >> 3)] = dh;
                ss[(size_t) r * ldS + (i >> 3)] = dh * (float) cs;
            }
        }
    }
}
// q8_1 blocks -> the mmq layout (the same codes and scales), row r from source row src[r] (null: r).
__global__ void __launch_bounds__(256) k_mmq_from_q8_1(const BlockQ8_1* __restrict__ xq, const int32_t* __restrict__ src,
                                                       int n_rows, int K, int8_t* __restrict__ codes,
                                                       float* __restrict__ ds, float* __restrict__ ss, int ldS) {
    const int nb = K / 32;
    const long long wid = (long long) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (wid >= (long long) n_rows * nb) return;
    const int lane = threadIdx.x & 31;
    const int r = (int) (wid / nb), b = (int) (wid % nb);
    const int sr = src ? __ldg(src + r) : r;
    const BlockQ8_1* blk = xq + (size_t) sr * nb + b;
    const int8_t qv = blk->qs[lane];
    codes[(size_t) r * K + 32 * b + lane] = qv;
    int cs = qv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
    if (lane == 0) {
        const float dh = __low2float(blk->ds);
        ds[(size_t) r * ldS + b] = dh;
        ss[(size_t) r * ldS + b] = dh * (float) cs;
    }
}

}  // namespace tsb
