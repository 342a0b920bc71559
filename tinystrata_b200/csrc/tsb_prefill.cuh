// tsb_prefill.cuh - the prefill (many-token) expert path: dispatch into expert-contiguous rows and the grouped expert
// products on the 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Reference: the prompt path runs llama.cpp's MMQ over rows sorted by expert (src/prefill/moe_mmq.cu:334-384,
// moe_mmq.hpp:58-81; permutation q36_engine.cu:486-510; SwiGLU moe_mmq.cu:123-131): per 32-value block an exact
// integer dot of the q8_1 activation codes with the weight codes, scaled by both blocks' scales and summed in fp32.
// The same arithmetic here, on tcgen05:
//   * per 32-value block the tensor core forms the integer S = sum_k q_x[k] (q_w[k] - 8) exactly (codes and centred
//     nibbles are exact in fp16, and every partial sum is an integer far below 2^24);
//   * the epilogue warps then add S * (d_w d_x) into fp32 accumulators held in registers, block after block, with
//     round-to-nearest FMAs, as the reference's scale-and-sum does.
// The hidden vector between the products is re-quantised to q8_1 as the reference's quantiser does, so it is the
// reference's but for values within fp32 rounding of a code boundary.
//
// Kernel shape (one CTA per SM, persistent over output tiles of 128 rows x 128 columns):
//   warps 0-3   producers: per ring stage (64 values of K) 128 activation rows (two q8_1 blocks each -> fp16 codes)
//               and 128 weight rows (two Q4_0 blocks -> fp16 centred nibbles, and their scales), in the tensor core's
//               K-major 128-byte-swizzled layout; a thread stages one activation row and one weight row, loading the
//               16-byte windows that cover the stage's bytes one stage ahead;
//   warp 4      tensor-memory allocation and the MMA issue (one thread): per 32-value block 2 x tcgen05.mma M128 N128
//               K16 into one of three block-sum buffers; tcgen05.commit hands the buffer to the epilogue;
//   warps 5-12  epilogue: two warps per TMEM lane quarter, a thread owns one output row and 64 columns of the tile;
//               per block, two tcgen05.ld of its 64 block sums and one FMA each with d_w d_x into 64 register
//               accumulators; at the end of the tile the activation and the q8_1 quantisation (gate/up) or the fp32
//               store (down).  A ring stage is free again once the MMAs read it and the epilogue read its scales.
// Gate/up tiles interleave the matrices in 32-row groups: B rows 0..31 are gate rows j0..j0+31, 32..63 the up rows of
// the same hidden values, 64..95 gate rows j0+32.., 96..127 their up rows, so a thread's 64 columns are the gate and up
// sums of one q8_1 block of 32 hidden values.
#pragma once

#include "tsb_kernels.cuh"

#include <cuda_fp16.h>

namespace tsb {

constexpr int kPfBM = 128, kPfBN = 128, kPfBK = 64, kPfStages = 6, kPfSBuf = 4;
constexpr int kPfProducerWarps = 4, kPfMmaWarp = 4, kPfEpiWarp0 = 5, kPfEpiWarps = 8, kPfWarps = 13;
constexpr int kPfThreads = kPfWarps * 32;
constexpr uint32_t kPfTileA = kPfBM * kPfBK * 2, kPfTileB = kPfBN * kPfBK * 2;   // 16 KB each
constexpr uint32_t kPfStageScales = 2 * 2 * kPfBN * 4;   // d_w [2 blocks][128 rows], then d_x [2 blocks][128 rows]
constexpr uint32_t kPfStage = kPfTileA + kPfTileB + kPfStageScales;             // A | B | scales
constexpr uint32_t kPfSmem = kPfStages * kPfStage + 1024;   // + slack (swizzled tiles sit on 1 KB)
constexpr int kPfMaxGroups = 512;
// instruction descriptor: D f32, A f16, B f16, both K-major, N = 128, M = 128
constexpr uint32_t kPfIdesc = (1u << 4) | ((uint32_t) (kPfBN >> 3) << 17) | ((uint32_t) (kPfBM >> 4) << 24);

enum : int { PF_GU = 0, PF_DOWN = 1 };

struct PfParams {
    // groups: group g owns output rows [bounds[g], bounds[g+1]) and the weight matrix of blob blobs + g * blob_stride
    const int32_t* bounds;     // [n_groups + 1] on the device (null: one group of n_rows rows)
    int n_groups;
    int n_rows;
    const uint8_t* blobs;
    uint64_t blob_stride;
    uint64_t w_off;            // byte offset of the matrix in the blob (gate rows; down rows)
    uint64_t up_off;           // gate/up: offset of the up rows from the gate rows
    uint32_t w_row;            // bytes per weight row
    int K;                     // contraction length (a multiple of 64)
    int N;                     // output columns (gate/up: n_ff hidden values; down: n_embd)
    const BlockQ8_1* X;        // activations: row r reads q8_1 row a_row(r) (K / 32 blocks)
    const int32_t* row_tok;    // a_row(r) = row_tok[r] (null -> r)
    BlockQ8_1* Hq;             // gate/up output: q8_1 of the hidden vectors [n_rows][N / 32]
    float* D;                  // down output: fp32 [n_rows][N]
    int act;
    float limit;
    unsigned* err;
};

// ------------------------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint64_t pf_sdesc(uint32_t addr) {   // K-major, 128-byte swizzle, 8-row groups 1 KB apart
    return (uint64_t) ((addr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) (1024 >> 4) << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}
__device__ __forceinline__ void pf_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t acc) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n"
                 ::"r"(tmem), "l"(da), "l"(db), "r"(kPfIdesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void pf_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                   "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                   "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(addr));
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tmem_st32(uint32_t addr, const float (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                 ::"r"(addr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                   "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                   "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
                   "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
                   "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
                   "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
                   "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
                   "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
                   "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
                   "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
                   "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
                 : "memory");
}
// Two columns of a block at once: a += (w dx) s lane by lane with the packed fp32 pipe instructions (mul.rn.f32x2,
// fma.rn.f32x2: the same IEEE roundings as two scalar mul / fma pairs, half the instructions).
__device__ __forceinline__ void fma2_scaled(float& a0, float& a1, float w0, float w1, float dx, float s0, float s1) {
    asm("{\n .reg .b64 w, d, s, a;\n mov.b64 w, {%2, %3};\n mov.b64 d, {%4, %4};\n mov.b64 s, {%5, %6};\n"
        " mov.b64 a, {%0, %1};\n mul.rn.f32x2 w, w, d;\n fma.rn.f32x2 a, w, s, a;\n mov.b64 {%0, %1}, a;\n}\n"
        : "+f"(a0), "+f"(a1)
        : "f"(w0), "f"(w1), "f"(dx), "f"(s0), "f"(s1));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// byte offset of the 16-byte chunk c (values 8c..8c+7) of row r inside a K-major 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t) ((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// ------------------------------------------------------------------------------------------------ operand staging
// The raw bytes of one ring stage for one producer thread (one activation row, one weight row), loaded a stage ahead
// of their conversion.  With 16-byte-aligned rows (A16 / W16) the loads are the 16-byte windows covering the stage:
// the two q8_1 blocks (72 bytes at 72 ks, five windows from byte 72 ks rounded down to 16) and the two Q4_0 blocks
// (36 bytes at 36 ks, three windows); otherwise the bytes themselves in 8- and 4-byte words.
struct PfRaw {
    uint32_t a[20];
    uint32_t w[12];
};
template <bool A16, bool W16>
__device__ __forceinline__ void pf_load(PfRaw& R, const BlockQ8_1* xrow, const uint8_t* wrow, int ks) {
    if (xrow) {
        const uint8_t* src = (const uint8_t*) xrow + 72 * ks;
        if (A16) {
            const uint4* v = (const uint4*) ((uintptr_t) src & ~(uintptr_t) 15);
#pragma unroll
            for (int k = 0; k < 5; ++k) {
                const uint4 t = __ldg(v + k);
                R.a[4 * k] = t.x; R.a[4 * k + 1] = t.y; R.a[4 * k + 2] = t.z; R.a[4 * k + 3] = t.w;
            }
        } else {
            const uint2* v = (const uint2*) src;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const uint2 t = __ldg(v + k);
                R.a[2 * k] = t.x; R.a[2 * k + 1] = t.y;
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < 20; ++k) R.a[k] = 0u;
    }
    if (wrow) {
        const uint8_t* src = wrow + 36 * ks;
        if (W16) {
            const uint4* v = (const uint4*) ((uintptr_t) src & ~(uintptr_t) 15);
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const uint4 t = __ldg(v + k);
                R.w[4 * k] = t.x; R.w[4 * k + 1] = t.y; R.w[4 * k + 2] = t.z; R.w[4 * k + 3] = t.w;
            }
        } else {
            const uint32_t* v = (const uint32_t*) src;
#pragma unroll
            for (int k = 0; k < 9; ++k) R.w[k] = __ldg(v + k);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 12; ++k) R.w[k] = 0u;
    }
}
// The q8_1 block hb of the stage as 9 words (scale word, 8 code words): word offset oa / 4 + 9 hb in the window.
template <int OA>
__device__ __forceinline__ void pf_a_block(const PfRaw& R, int hb, uint32_t (&b)[9]) {
#pragma unroll
    for (int k = 0; k < 9; ++k) b[k] = R.a[OA / 4 + 9 * hb + k];
}
// The Q4_0 block hb of the stage as (d word, 4 nibble words): block 0 at byte OB of the window (d, then 16 bytes at
// OB + 2: two-byte shifted words), block 1 at OB + 18 (d in the high half of word (OB + 16) / 4, nibbles aligned).
template <int OB>
__device__ __forceinline__ void pf_w_block(const PfRaw& R, int hb, uint32_t (&b)[5]) {
    if (hb == 0) {
        b[0] = R.w[OB / 4] & 0xFFFFu;
#pragma unroll
        for (int k = 0; k < 4; ++k) b[1 + k] = __byte_perm(R.w[OB / 4 + k], R.w[OB / 4 + k + 1], 0x5432);
    } else {
        b[0] = R.w[(OB + 16) / 4] >> 16;
#pragma unroll
        for (int k = 0; k < 4; ++k) b[1 + k] = R.w[(OB + 20) / 4 + k];
    }
}
// q8_1 codes -> fp16 (exact) into chunks 4h..4h+3 of row r: the byte c + 128 under the exponent of 1024 is the fp16
// 1024 + c + 128, and an exact subtraction of 1152 leaves c.
__device__ __forceinline__ void stage_q8_codes(const uint32_t (&blk)[9], uint8_t* tile, int r, int h) {
    const half2 bias = __float2half2_rn(1152.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {   // 8 codes: words 1 + 2c, 2 + 2c
        const uint32_t w0 = blk[1 + 2 * c] ^ 0x80808080u, w1 = blk[2 + 2 * c] ^ 0x80808080u;
        uint32_t out[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {   // codes 2p, 2p+1 of the chunk
            const uint32_t bits = __byte_perm(p < 2 ? w0 : w1, 0x64646464u, (p & 1) ? 0x4342u : 0x4140u);
            const half2 v = __hsub2(*(const half2*) &bits, bias);
            out[p] = *(const uint32_t*) &v;
        }
        *(uint4*) (tile + sw128(r, 4 * h + c)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}
// Q4_0 centred nibbles q - 8 -> fp16 (exact) into chunks 4h..4h+3 of row r.  Values 0..15 of a block are the low
// nibbles of bytes 0..15, values 16..31 the high nibbles.  Four nibbles at a time: one mask leaves them as bytes, two
// byte permutes put each under the fp16 exponent pattern 0x64 (1024 + q), one subtraction of 1032 per pair leaves q - 8.
__device__ __forceinline__ void stage_q4_0(const uint32_t (&blk)[5], uint8_t* tile, int r, int h) {
    const half2 bias = __float2half2_rn(1032.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {   // chunk c: values 8c..8c+7 (c < 2 low nibbles, c >= 2 high nibbles)
        uint32_t out[4];
#pragma unroll
        for (int k = 0; k < 2; ++k) {   // the chunk's source words: bytes 8 (c & 1) + 4k ..
            const uint32_t w = blk[1 + (c & 1) * 2 + k];
            const uint32_t b = (c >> 1 ? (w >> 4) : w) & 0x0F0F0F0Fu;
            const uint32_t p0 = __byte_perm(b, 0x64646464u, 0x5140), p1 = __byte_perm(b, 0x64646464u, 0x7362);
            const half2 v0 = __hsub2(*(const half2*) &p0, bias), v1 = __hsub2(*(const half2*) &p1, bias);
            out[2 * k] = *(const uint32_t*) &v0;
            out[2 * k + 1] = *(const uint32_t*) &v1;
        }
        *(uint4*) (tile + sw128(r, 4 * h + c)) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

// ------------------------------------------------------------------------------------------------ the kernel
template <int MODE, bool A16, bool W16>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(PfParams p) {
    extern __shared__ __align__(1024) uint8_t pf_raw[];
    uint8_t* smem = (uint8_t*) (((uintptr_t) pf_raw + 1023) & ~(uintptr_t) 1023);
    __shared__ uint64_t full[kPfStages], empty[kPfStages], s_full[kPfSBuf], s_empty[kPfSBuf];
    __shared__ uint32_t tbase;
    __shared__ volatile int abort_flag;
    __shared__ int32_t gstart[kPfMaxGroups + 1];   // row starts
    __shared__ int32_t gtile[kPfMaxGroups + 1];    // prefix of 128-row tiles
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.n_groups;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&full[s], kPfProducerWarps);
            mbar_init(&empty[s], 1 + kPfEpiWarps);   // the MMAs' commit and every epilogue warp (scales read)
        }
        for (int b = 0; b < kPfSBuf; ++b) {
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
    if (warp == kPfMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tbase;
    const int n_mt = gtile[G];
    const int per_tile = MODE == PF_GU ? 64 : kPfBN;   // hidden values (gate/up) or output columns per tile
    const int n_nt = (p.N + per_tile - 1) / per_tile;
    const int n_tiles = n_mt * n_nt;
    const int nb = p.K / 32;            // 32-value blocks of K
    const int nks = p.K / kPfBK;        // ring stages per tile
    auto tile_of = [&](int t, int& g, int& row0, int& row1, int& n0) {
        const int mt = t / n_nt, nt = t % n_nt;
        int lo = 0, hi = G - 1;
        while (lo < hi) {   // last group with gtile[g] <= mt (empty groups share their successor's start)
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
        // thread r: activation row r and weight row r of every stage; a stage's raw bytes are loaded while the
        // previous stage is converted
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
                if (MODE == PF_GU) {   // 32-row groups: gate, up, gate, up
                    const int j = n0 + (r >> 6) * 32 + (r & 31);
                    if (j < p.N) wrow = base + ((r & 32) ? p.up_off : 0) + (size_t) j * p.w_row;
                } else {
                    const int j = n0 + r;
                    if (j < p.N) wrow = base + (size_t) j * p.w_row;
                }
            }
            // one ring stage from its raw bytes; false: a wait gave up
            auto stage = [&](const PfRaw& cur, int ks) -> bool {
                const int s = (int) (it % kPfStages);
                if (it >= (uint32_t) kPfStages) {
                    const uint32_t par = ((it / kPfStages) - 1) & 1u;
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(&empty[s], par))
                        if (globaltimer() - t0 > wait_limit_ns() || abort_flag) {
                            report_error(p.err, 0x501u);
                            abort_flag = 1;
                            return false;
                        }
                }
                uint8_t* sa = smem + s * kPfStage;
                uint8_t* sb = sa + kPfTileA;
                float* sdw = (float*) (sb + kPfTileB);   // [2 blocks][128 rows]
                float* sdx = sdw + 2 * kPfBN;             // [2 blocks][128 rows]
#pragma unroll
                for (int hb = 0; hb < 2; ++hb) {
                    uint32_t ab[9], wb[5];
                    if (!A16 || (ks & 1) == 0) pf_a_block<0>(cur, hb, ab); else pf_a_block<8>(cur, hb, ab);
                    if (!W16) {
                        pf_w_block<0>(cur, hb, wb);
                    } else {
                        switch (ks & 3) {
                            case 0: pf_w_block<0>(cur, hb, wb); break;
                            case 1: pf_w_block<4>(cur, hb, wb); break;
                            case 2: pf_w_block<8>(cur, hb, wb); break;
                            default: pf_w_block<12>(cur, hb, wb); break;
                        }
                    }
                    if (xrow) {
                        stage_q8_codes(ab, sa, r, hb);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c) *(uint4*) (sa + sw128(r, 4 * hb + c)) = make_uint4(0, 0, 0, 0);
                    }
                    sdx[hb * kPfBN + r] = __half2float(__ushort_as_half((unsigned short) (ab[0] & 0xFFFFu)));
                    stage_q4_0(wb, sb, r, hb);
                    sdw[hb * kPfBN + r] = __half2float(__ushort_as_half((unsigned short) (wb[0] & 0xFFFFu)));
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                ++it;
                return true;
            };
            // two raw buffers in turn: stage ks converts from one while stage ks + 1's bytes load into the other
            pf_load<A16, W16>(R, xrow, wrow, 0);
            bool ok = true;
            for (int ks = 0; ks < nks && ok; ks += 2) {
                if (ks + 1 < nks) pf_load<A16, W16>(R2, xrow, wrow, ks + 1);
                ok = stage(R, ks);
                if (ok && ks + 1 < nks) {
                    if (ks + 2 < nks) pf_load<A16, W16>(R, xrow, wrow, ks + 2);
                    ok = stage(R2, ks + 1);
                }
            }
            if (!ok) break;
        }
    } else if (warp == kPfMmaWarp) {
        // ------------------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t it = 0, gb = 0;   // ring stage counter, block counter (both across tiles)
            for (int tile = blockIdx.x; tile < n_tiles && !abort_flag; tile += gridDim.x) {
                bool ok = true;
                for (int kb = 0; kb < nb; ++kb, ++gb) {
                    const int s = (int) (it % kPfStages);
                    if ((kb & 1) == 0 && !mbar_wait_bounded(&full[s], (it / kPfStages) & 1u, p.err, 0x503u)) {
                        ok = false;
                        break;
                    }
                    const int b = (int) (gb % kPfSBuf);
                    if (gb >= (uint32_t) kPfSBuf &&
                        !mbar_wait_bounded(&s_empty[b], ((gb / kPfSBuf) - 1) & 1u, p.err, 0x502u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + s * kPfStage) + (uint32_t) (kb & 1) * 64;
                    const uint32_t b0 = a0 + kPfTileA;
                    const uint32_t d = tmem + (uint32_t) b * kPfBN;
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) pf_mma(d, pf_sdesc(a0 + kk * 32), pf_sdesc(b0 + kk * 32), kk ? 1u : 0u);
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
        // ------------------------------------------------------------------------ epilogue (warps 3-10)
        const int q = warp & 3;                            // the TMEM lane quarter this warp may access
        const int half = (warp - kPfEpiWarp0) >> 2;        // columns 64 half ..
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
                const int b = (int) (gb % kPfSBuf);
                const uint32_t it = gb >> 1;   // the ring stage of this block (two blocks a stage)
                const int s = (int) (it % kPfStages);
                if (lane == 0) {
                    ok = mbar_wait_bounded(&s_full[b], (gb / kPfSBuf) & 1u, p.err, 0x504u);
                    // the stage's scales: its fill is complete (and cannot be refilled before this warp releases it)
                    if (ok) ok = mbar_wait_bounded(&full[s], (it / kPfStages) & 1u, p.err, 0x505u);
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                __syncwarp();
                tc_fence_after();
                const uint32_t sb = lane_base + (uint32_t) b * kPfBN;
                const float* scales = (const float*) (smem + s * kPfStage + kPfTileA + kPfTileB);
                const float4* dw4 = (const float4*) scales + (kb & 1) * (kPfBN / 4) + 16 * half;
                const float dx = scales[2 * kPfBN + (kb & 1) * kPfBN + q * 32 + lane];
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {   // 32 columns at a time
                    float sv[32];
                    tmem_ld32(sb + 32 * hh, sv);
                    tmem_wait_ld();
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 w0 = dw4[8 * hh + j4];
                        float* a = acc + 32 * hh + 4 * j4;
                        fma2_scaled(a[0], a[1], w0.x, w0.y, dx, sv[4 * j4 + 0], sv[4 * j4 + 1]);
                        fma2_scaled(a[2], a[3], w0.z, w0.w, dx, sv[4 * j4 + 2], sv[4 * j4 + 3]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&s_empty[b]);
                    if (kb & 1) mbar_arrive(&empty[s]);   // both blocks' scales of the stage read
                }
            }
            if (!ok) {
                abort_flag = 1;
                break;
            }
            // the tile's sums: gate/up -> activation -> q8_1; down -> fp32
            if (MODE == PF_GU) {
                // this thread's q8_1 block of hidden values: gate sums acc[j], up sums acc[32 + j]
                {
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
