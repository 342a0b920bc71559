// tsb_prefill_k.cuh - the prefill grouped expert products for the K-quant, i-quant and Q8_0 weight formats (Q4_K,
// Q6_K, IQ3_XXS, IQ3_S; Q8_0 for the Qwen layer's dense shared expert) on tcgen05.  The kernel has the shape of the
// Q4_0 kernel (tsb_prefill.cuh: producers, one MMA thread, eight epilogue warps holding fp32 accumulators in
// registers); what changes is the weight side:
//   * the producers decode each weight row's 64 values of a ring stage into exact fp16 integers -- Q4_K codes 0..15,
//     Q6_K codes - 32, IQ3 grid bytes with their signs applied -- and stage the per-(row, 32-value block) scale terms
//     the reference applies after its integer dot (src/kernels/cuda/iq_kernels.cu:188-236, 314-386, 523-553);
//   * the tensor core forms the block's integer sum S = sum q_x q_w exactly (Q6_K: one sum per 16-value sub-block,
//     whose int8 scales differ), and the epilogue applies the format's integer step and scales:
//       Q4_K    acc += (d sc d_x) S - (dmin m) (d_x sum(q_x))        (the min term uses the activation code sum)
//       Q6_K    acc += (d d_x) (sc_a S_a + sc_b S_b)                  (an exact integer in fp32)
//       IQ3_XXS acc += (d d_x) ((ls S + S / 2) / 2)                   (C integer division, as the reference)
//       IQ3_S   acc += ((d (1 + 2 sc)) d_x) S
//       Q8_0    acc += (d d_x) S                                       (32-value blocks: int8 codes, one fp16 scale)
// The activation side (q8_1 codes, exact in fp16) and the gate/up and down epilogues are the Q4_0 kernel's.
#pragma once

#include "tsb_prefill.cuh"

namespace tsb {

constexpr int kPxStages = 5;
constexpr int kPxWTerms = 3, kPxXTerms = 2;   // per (row, block): weight scale terms; activation terms
constexpr uint32_t kPxStageScales = (uint32_t) (kPxWTerms + kPxXTerms) * 2 * kPfBN * 4;
constexpr uint32_t kPxStage = kPfTileA + kPfTileB + kPxStageScales;
constexpr uint32_t kPxTabBytes = (256 + 512) * 4;   // the IQ3_XXS and IQ3_S grids
constexpr uint32_t kPxSmem = kPxStages * kPxStage + kPxTabBytes + 1024;

template <int WT> struct PxFmt;   // per weight format: super-block bytes, sub-sums per 32-value block
template <> struct PxFmt<T_Q4_K> { static constexpr int kBytes = 144, kSplit = 1; };
template <> struct PxFmt<T_Q6_K> { static constexpr int kBytes = 210, kSplit = 2; };
template <> struct PxFmt<T_IQ3_XXS> { static constexpr int kBytes = 98, kSplit = 1; };
template <> struct PxFmt<T_IQ3_S> { static constexpr int kBytes = 110, kSplit = 1; };
template <> struct PxFmt<T_Q8_0> { static constexpr int kBytes = 34, kSplit = 1; };   // per 32 values

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

// Eight integers 0 <= v < 1024 -> four fp16 pairs: 1024 + v built from the exponent pattern, minus `bias` exactly.
__device__ __forceinline__ uint4 pack8_unsigned(const uint32_t (&v)[8], float bias) {
    const half2 b = __float2half2_rn(bias);
    uint32_t out[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t bits = 0x64006400u | v[2 * p] | (v[2 * p + 1] << 16);
        const half2 h = __hsub2(*(const half2*) &bits, b);
        out[p] = *(const uint32_t*) &h;
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}
// Grid bytes (two words of four values) with sign bits: bit k of sgn negates value k (an exact fp16 sign flip).
__device__ __forceinline__ uint4 pack8_signed(uint32_t g0, uint32_t g1, uint32_t sgn) {
    uint32_t v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[k] = (g0 >> (8 * k)) & 0xFFu;
        v[4 + k] = (g1 >> (8 * k)) & 0xFFu;
    }
    uint4 u = pack8_unsigned(v, 1024.0f);
    uint32_t s[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) s[p] = (((sgn >> (2 * p)) & 1u) << 15) | (((sgn >> (2 * p + 1)) & 1u) << 31);
    u.x ^= s[0];
    u.y ^= s[1];
    u.z ^= s[2];
    u.w ^= s[3];
    return u;
}

// ------------------------------------------------------------------------------------------------ weight staging
// Stage ks of a weight row (values 64 ks .. 64 ks + 63: super-block ks / 4, quarter ks % 4) into chunks 0..7 of
// tile row r, and the scale terms of its two 32-value blocks: wt[t * 2 * 128 + hb * 128 + r].
template <int WT>
__device__ __forceinline__ void px_stage_w(const uint8_t* wrow, int ks, uint8_t* tile, int r, float* wt,
                                           const uint32_t* gxxs, const uint32_t* gs) {
    const int sb = ks >> 2, s = ks & 3;
    const uint8_t* base = wrow + (size_t) sb * PxFmt<WT>::kBytes;
    if constexpr (WT == T_Q8_0) {
        // blocks 2 ks, 2 ks + 1: (d, 32 int8 codes) each, 68 bytes from a 2-byte aligned address
        uint32_t w[17];
        ldw<17>(wrow + (size_t) ks * 68, w);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
            const int o = 34 * hb;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = byte_of(w, o + 2 + 8 * c + k) ^ 0x80u;   // code + 128
                *(uint4*) (tile + sw128(r, 4 * hb + c)) = pack8_unsigned(v, 1152.0f);
            }
            wt[(0 * 2 + hb) * kPfBN + r] = h2f(byte_of(w, o) | (byte_of(w, o + 1) << 8));
        }
    } else if constexpr (WT == T_Q4_K) {
        // d, dmin, scales[12], qs[128]: the stage's sub-blocks 2s, 2s+1 are the low / high nibbles of qs[32s .. +32)
        const uint4 hdr = __ldg((const uint4*) base);
        const uint4 qa = __ldg((const uint4*) (base + 16 + 32 * s)), qb = __ldg((const uint4*) (base + 32 + 32 * s));
        const uint32_t sc12[3] = {hdr.y, hdr.z, hdr.w};
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
            const int j = 2 * s + hb;
            int sc, m;
            if (j < 4) {
                sc = (int) byte_of(sc12, j) & 63;
                m = (int) byte_of(sc12, j + 4) & 63;
            } else {
                sc = (int) ((byte_of(sc12, j + 4) & 0xFu) | ((byte_of(sc12, j - 4) >> 6) << 4));
                m = (int) ((byte_of(sc12, j + 4) >> 4) | ((byte_of(sc12, j) >> 6) << 4));
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = (byte_of(q, 8 * c + k) >> (4 * hb)) & 0xFu;
                *(uint4*) (tile + sw128(r, 4 * hb + c)) = pack8_unsigned(v, 1024.0f);
            }
            wt[(0 * 2 + hb) * kPfBN + r] = d * (float) sc;
            wt[(1 * 2 + hb) * kPfBN + r] = dmin * (float) m;
        }
    } else if constexpr (WT == T_Q6_K) {
        // ql[128], qh[64], scales[16] int8, d: quarter s is half n = s / 2 of the super-block; its first 32 values
        // take ql[64n + l] and qh[32n + l] bits 0-1 (s even) or the high nibble and bits 4-5 (s odd), its second 32
        // ql[64n + 32 + l] with bits 2-3 / 6-7; the 16-value sub-blocks' scales are scales[4s .. 4s + 3]
        const int n = s >> 1, odd = s & 1;
        uint32_t ql[16], qh[8], scw[1];
        ldw<16>(base + 64 * n, ql);
        ldw<8>(base + 128 + 32 * n, qh);
        ldw<1>(base + 192 + 4 * s, scw);
        const float d = h2f(ldh(base + 208));
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t v[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int l = 8 * c + k;
                    const uint32_t lo = (byte_of(ql, 32 * hb + l) >> (4 * odd)) & 0xFu;
                    const uint32_t hi = (byte_of(qh, l) >> (4 * odd + 2 * hb)) & 3u;
                    v[k] = lo | (hi << 4);
                }
                *(uint4*) (tile + sw128(r, 4 * hb + c)) = pack8_unsigned(v, 1056.0f);   // code - 32
            }
            wt[(0 * 2 + hb) * kPfBN + r] = d;
            wt[(1 * 2 + hb) * kPfBN + r] = (float) (int8_t) ((scw[0] >> (16 * hb)) & 0xFFu);
            wt[(2 * 2 + hb) * kPfBN + r] = (float) (int8_t) ((scw[0] >> (16 * hb + 8)) & 0xFFu);
        }
    } else if constexpr (WT == T_IQ3_XXS) {
        // d, qs[64] (8 grid indices per 32 values), 32 bytes of sign/scale words (one per 32 values)
        uint32_t qs[4], aux[2];
        ldw<4>(base + 2 + 16 * s, qs);
        ldw<2>(base + 66 + 8 * s, aux);
        const float d = h2f(ldh(base));
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t sidx = (aux[hb] >> (7 * l)) & 127u;
                const uint32_t sgn = sidx | ((uint32_t) (__popc(sidx) & 1) << 7);   // the even-parity sign byte
                const uint32_t g0 = gxxs[byte_of(qs, 8 * hb + 2 * l)], g1 = gxxs[byte_of(qs, 8 * hb + 2 * l + 1)];
                *(uint4*) (tile + sw128(r, 4 * hb + l)) = pack8_signed(g0, g1, sgn);
            }
            wt[(0 * 2 + hb) * kPfBN + r] = d;
            wt[(1 * 2 + hb) * kPfBN + r] = (float) (aux[hb] >> 28);
        }
    } else {   // T_IQ3_S
        // d, qs[64] (low 8 bits of 9-bit grid indices), qh[8] (their high bits), signs[32], scales[4] (nibbles)
        uint32_t qs[4], sg[2];
        ldw<4>(base + 2 + 16 * s, qs);
        ldw<2>(base + 74 + 8 * s, sg);
        const uint32_t qh2 = ldh(base + 66 + 2 * s);
        const uint32_t scb = (ldh(base + 106 + (s & ~1)) >> (8 * (s & 1))) & 0xFFu;
        const float d = h2f(ldh(base));
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
            const uint32_t qh = (qh2 >> (8 * hb)) & 0xFFu;
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t i0 = byte_of(qs, 8 * hb + 2 * l) | (((qh >> (2 * l)) & 1u) << 8);
                const uint32_t i1 = byte_of(qs, 8 * hb + 2 * l + 1) | (((qh >> (2 * l + 1)) & 1u) << 8);
                *(uint4*) (tile + sw128(r, 4 * hb + l)) = pack8_signed(gs[i0], gs[i1], byte_of(sg, 4 * hb + l));
            }
            wt[(0 * 2 + hb) * kPfBN + r] = d * (float) (1 + 2 * (int) ((scb >> (4 * hb)) & 0xFu));
        }
    }
}

// The epilogue's contribution of one block for one column: S (and S2 for Q6_K) the tensor core's integer sums,
// w0..w2 the column's weight terms, x0 = d_x, x1 = d_x * sum(q_x) (Q4_K).
template <int WT>
__device__ __forceinline__ float px_epi(float acc, float S, float S2, float w0, float w1, float w2, float x0, float x1) {
    if constexpr (WT == T_Q4_K) {
        return fmaf(-w1, x1, fmaf(w0 * x0, S, acc));
    } else if constexpr (WT == T_Q6_K) {
        return fmaf(w0 * x0, fmaf(w1, S, w2 * S2), acc);
    } else if constexpr (WT == T_IQ3_XXS) {
        const int si = __float2int_rn(S), ls = (int) w1;
        const int v = (ls * si + si / 2) / 2;
        return fmaf(w0 * x0, (float) v, acc);
    } else {
        return fmaf(w0 * x0, S, acc);
    }
}

__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(addr));
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int MODE, int WT, bool A16>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm_x(PfParams p) {
    constexpr int SPLIT = PxFmt<WT>::kSplit;
    constexpr int NBUF = SPLIT == 2 ? 2 : kPfSBuf;          // block-sum buffers of 128 * SPLIT TMEM columns
    extern __shared__ __align__(1024) uint8_t px_raw[];
    uint8_t* smem = (uint8_t*) (((uintptr_t) px_raw + 1023) & ~(uintptr_t) 1023);
    uint32_t* gxxs = (uint32_t*) (smem + kPxStages * kPxStage);
    uint32_t* gs = gxxs + 256;
    __shared__ uint64_t full[kPxStages], empty[kPxStages], s_full[kPfSBuf], s_empty[kPfSBuf];
    __shared__ uint32_t tbase;
    __shared__ volatile int abort_flag;
    __shared__ int32_t gstart[kPfMaxGroups + 1];
    __shared__ int32_t gtile[kPfMaxGroups + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.n_groups;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPxStages; ++s) {
            mbar_init(&full[s], kPfProducerWarps);
            mbar_init(&empty[s], 1 + kPfEpiWarps);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], kPfEpiWarps);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    if (threadIdx.x == 32) {
        int t = 0;
        for (int g = 0; g <= G; ++g) {
            const int s = p.bounds ? __ldg(p.bounds + g) : (g == 0 ? 0 : p.n_rows);
            gstart[g] = s;
            gtile[g] = t;
            if (g < G) {
                const int e = p.bounds ? __ldg(p.bounds + g + 1) : p.n_rows;
                t += (max(e - s, 0) + kPfBM - 1) / kPfBM;
            }
        }
    }
    if (WT == T_IQ3_XXS || WT == T_IQ3_S)
        for (int i = threadIdx.x; i < 256 + 512; i += blockDim.x) gxxs[i] = i < 256 ? g_iq3xxs_grid[i] : g_iq3s_grid[i - 256];
    if (warp == kPfMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tbase;
    const int n_mt = gtile[G];
    const int per_tile = MODE == PF_GU ? 64 : kPfBN;
    const int n_nt = (p.N + per_tile - 1) / per_tile;
    const int n_tiles = n_mt * n_nt;
    const int nb = p.K / 32;
    const int nks = p.K / kPfBK;
    auto tile_of = [&](int t, int& g, int& row0, int& row1, int& n0) {
        const int mt = t / n_nt, nt = t % n_nt;
        int lo = 0, hi = G - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (gtile[mid] <= mt) lo = mid; else hi = mid - 1;
        }
        g = lo;
        row0 = gstart[g] + (mt - gtile[g]) * kPfBM;
        row1 = min(row0 + kPfBM, gstart[g + 1]);
        n0 = nt * per_tile;
    };

    if (warp < kPfProducerWarps) {
        // ------------------------------------------------------------------------ producers
        // thread r: activation row r (its q8_1 windows loaded a stage ahead) and weight row r of every stage
        const int r = threadIdx.x;
        uint32_t it = 0;
        PfRaw R, R2;
        for (int tile = blockIdx.x; tile < n_tiles && !abort_flag; tile += gridDim.x) {
            int g, row0, row1, n0;
            tile_of(tile, g, row0, row1, n0);
            const BlockQ8_1* xrow = nullptr;
            if (row0 + r < row1) xrow = p.X + (size_t) (p.row_tok ? __ldg(p.row_tok + row0 + r) : row0 + r) * nb;
            const uint8_t* wrow = nullptr;
            {
                const uint8_t* base = p.blobs + (size_t) g * p.blob_stride + p.w_off;
                if (MODE == PF_GU) {
                    const int j = n0 + (r >> 6) * 32 + (r & 31);
                    if (j < p.N) wrow = base + ((r & 32) ? p.up_off : 0) + (size_t) j * p.w_row;
                } else {
                    const int j = n0 + r;
                    if (j < p.N) wrow = base + (size_t) j * p.w_row;
                }
            }
            // one ring stage; false: a wait gave up
            auto stage = [&](const PfRaw& cur, int ks) -> bool {
                const int s = (int) (it % kPxStages);
                if (it >= (uint32_t) kPxStages) {
                    const uint32_t par = ((it / kPxStages) - 1) & 1u;
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(&empty[s], par))
                        if (globaltimer() - t0 > wait_limit_ns() || abort_flag) {
                            report_error(p.err, 0x511u);
                            abort_flag = 1;
                            return false;
                        }
                }
                uint8_t* sa = smem + s * kPxStage;
                uint8_t* sb = sa + kPfTileA;
                float* wt = (float*) (sb + kPfTileB);                   // [kPxWTerms][2 blocks][128 rows]
                float* xt = wt + kPxWTerms * 2 * kPfBN;                // [kPxXTerms][2 blocks][128 rows]
#pragma unroll
                for (int hb = 0; hb < 2; ++hb) {
                    uint32_t ab[9];
                    if (!A16 || (ks & 1) == 0) pf_a_block<0>(cur, hb, ab); else pf_a_block<8>(cur, hb, ab);
                    if (xrow) {
                        stage_q8_codes(ab, sa, r, hb);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c) *(uint4*) (sa + sw128(r, 4 * hb + c)) = make_uint4(0, 0, 0, 0);
                    }
                    const float dx = h2f(ab[0]);
                    xt[hb * kPfBN + r] = dx;
                    if (WT == T_Q4_K) {   // the activation code sum of the block (the min term)
                        int sq = 0;
#pragma unroll
                        for (int k = 1; k < 9; ++k) sq = __dp4a((int) ab[k], 0x01010101, sq);
                        xt[(2 + hb) * kPfBN + r] = xrow ? dx * (float) sq : 0.0f;
                    }
                }
                if (wrow) {
                    px_stage_w<WT>(wrow, ks, sb, r, wt, gxxs, gs);
                } else {
#pragma unroll
                    for (int c = 0; c < 8; ++c) *(uint4*) (sb + sw128(r, c)) = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int t = 0; t < kPxWTerms * 2; ++t) wt[t * kPfBN + r] = 0.0f;
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                ++it;
                return true;
            };
            // two raw activation buffers in turn: stage ks converts from one while stage ks + 1's bytes load
            pf_load<A16, false>(R, xrow, nullptr, 0);
            bool ok = true;
            for (int ks = 0; ks < nks && ok; ks += 2) {
                if (ks + 1 < nks) pf_load<A16, false>(R2, xrow, nullptr, ks + 1);
                ok = stage(R, ks);
                if (ok && ks + 1 < nks) {
                    if (ks + 2 < nks) pf_load<A16, false>(R, xrow, nullptr, ks + 2);
                    ok = stage(R2, ks + 1);
                }
            }
            if (!ok) break;
        }
    } else if (warp == kPfMmaWarp) {
        // ------------------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t it = 0, gb = 0;
            for (int tile = blockIdx.x; tile < n_tiles && !abort_flag; tile += gridDim.x) {
                bool ok = true;
                for (int kb = 0; kb < nb; ++kb, ++gb) {
                    const int s = (int) (it % kPxStages);
                    if ((kb & 1) == 0 && !mbar_wait_bounded(&full[s], (it / kPxStages) & 1u, p.err, 0x513u)) {
                        ok = false;
                        break;
                    }
                    const int b = (int) (gb % NBUF);
                    if (gb >= (uint32_t) NBUF && !mbar_wait_bounded(&s_empty[b], ((gb / NBUF) - 1) & 1u, p.err, 0x512u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + s * kPxStage) + (uint32_t) (kb & 1) * 64;
                    const uint32_t b0 = a0 + kPfTileA;
                    const uint32_t d = tmem + (uint32_t) b * kPfBN * SPLIT;
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        if (SPLIT == 2)   // one sum per 16-value sub-block
                            pf_mma(d + (uint32_t) kk * kPfBN, pf_sdesc(a0 + kk * 32), pf_sdesc(b0 + kk * 32), 0u);
                        else
                            pf_mma(d, pf_sdesc(a0 + kk * 32), pf_sdesc(b0 + kk * 32), kk ? 1u : 0u);
                    }
                    pf_commit(&s_full[b]);
                    if (kb & 1) {
                        pf_commit(&empty[s]);
                        ++it;
                    }
                }
                if (!ok) {
                    abort_flag = 1;
                    break;
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int half = (warp - kPfEpiWarp0) >> 2;
        const uint32_t lane_base = tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (64 * half);
        uint32_t gb = 0;
        for (int tile = blockIdx.x; tile < n_tiles && !abort_flag; tile += gridDim.x) {
            int g, row0, row1, n0;
            tile_of(tile, g, row0, row1, n0);
            const int row = row0 + q * 32 + lane;
            float acc[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
            bool ok = true;
            for (int kb = 0; kb < nb; ++kb, ++gb) {
                const int b = (int) (gb % NBUF);
                const uint32_t it = gb >> 1;
                const int s = (int) (it % kPxStages);
                if (lane == 0) {
                    ok = mbar_wait_bounded(&s_full[b], (gb / NBUF) & 1u, p.err, 0x514u);
                    if (ok) ok = mbar_wait_bounded(&full[s], (it / kPxStages) & 1u, p.err, 0x515u);
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                __syncwarp();
                tc_fence_after();
                const uint32_t sbuf = lane_base + (uint32_t) b * kPfBN * SPLIT;
                const float* wt = (const float*) (smem + s * kPxStage + kPfTileA + kPfTileB) + (kb & 1) * kPfBN + 64 * half;
                const float* xt = wt - 64 * half + kPxWTerms * 2 * kPfBN + q * 32 + lane;
                const float x0 = xt[0];
                const float x1 = WT == T_Q4_K ? xt[2 * kPfBN] : 0.0f;   // term 1 of the block
#pragma unroll
                for (int hh = 0; hh < 4; ++hh) {   // 16 columns at a time
                    float sv[16], sv2[16];
                    tmem_ld16(sbuf + 16 * hh, sv);
                    if (SPLIT == 2) tmem_ld16(sbuf + kPfBN + 16 * hh, sv2);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int c = 16 * hh + j;
                        const float w0 = wt[c];
                        const float w1 = (WT == T_Q6_K || WT == T_Q4_K || WT == T_IQ3_XXS) ? wt[2 * kPfBN + c] : 0.0f;
                        const float w2 = WT == T_Q6_K ? wt[4 * kPfBN + c] : 0.0f;
                        acc[c] = px_epi<WT>(acc[c], sv[j], SPLIT == 2 ? sv2[j] : 0.0f, w0, w1, w2, x0, x1);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&s_empty[b]);
                    if (kb & 1) mbar_arrive(&empty[s]);
                }
            }
            if (!ok) {
                abort_flag = 1;
                break;
            }
            if (MODE == PF_GU) {
                const int blk = half;
                float h[32], amax = 0.0f, sum = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    h[j] = act_value(p.act, acc[j], acc[32 + j], p.limit);
                    amax = fmaxf(amax, fabsf(h[j]));
                    sum += h[j];
                }
                if (row < row1 && n0 + 32 * blk < p.N) {
                    const float d = q8_finite(fdiv_fm(amax, 127.0f));
                    uint32_t* o = (uint32_t*) (p.Hq + (size_t) row * (p.N / 32) + (n0 / 32) + blk);
                    const half2 ds = make_half2(__float2half(d), __float2half(q8_finite(sum)));
                    o[0] = *(const uint32_t*) &ds;
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
                            word |= (uint32_t) (uint8_t) (int8_t) c << (8 * k);
                        }
                        o[1 + w] = word;
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; c += 32) {
                    const int col = n0 + 64 * half + c;
                    if (row < row1 && col < p.N) {
                        float4* dst = (float4*) (p.D + (size_t) row * p.N + col);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            dst[j] = make_float4(acc[c + 4 * j], acc[c + 4 * j + 1], acc[c + 4 * j + 2], acc[c + 4 * j + 3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPfMmaWarp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

}  // namespace tsb
