// tsb_decode.cuh - the whole decode MoE block of every layer of a step in ONE persistent kernel.
//
// Per layer (the reference's call stack A, src/qwen35/q36_engine.cu:2821-2925, with k_moe_out_small's epilogue):
//   P0  every CTA: h = rms(x) (the 256-slot order of q36_kernels.cuh:252-290) and its q8_1 image in shared memory
//   P1  router logits (fp32 rows, the shared-gate row appended) and the shared expert's gate/up + SwiGLU
//   --- grid barrier
//   R   every CTA: softmax top-k of every token (native_router.cu:44-95) and the grouping (q36_engine.cu:396-422)
//   P2  routed experts' gate/up + SwiGLU (IQ3_XXS), the shared expert's down rows (Q8_0)
//   --- grid barrier
//   P3  routed down rows of this CTA's row chunks for every group, then the combine of those rows:
//       x += sum_k w_k part_k (fma in pick order) + sigmoid(gate) shared
//   --- grid barrier
//
// One CTA per SM (cooperative launch), 16 warps: warp 15 lane 0 is the producer, streaming every unit of work's weight
// bytes with cp.async.bulk into a ring of shared-memory slots (full / empty mbarriers per slot) as far ahead as the
// ring allows: the next phase's bytes (and the next layer's router and shared-expert rows) are in flight while this
// phase computes and while the grid barriers wait.  Warps 0-14 consume units in order, claiming them from a counter.
// Every wait is bounded (2 s of %globaltimer); a wait that gives up records its site in the error word and the kernel
// winds down.
#pragma once

#include "tsb_kernels.cuh"

#include <cfloat>

namespace tsb {

constexpr int kDecWarps = 16, kDecConsumers = 15, kDecThreads = kDecWarps * 32, kDecCThreads = kDecConsumers * 32;
constexpr int kSlots = 14;   // 14 x 4352 bytes below the tables (which sit at shared address 0x10000)
constexpr uint32_t kSlotBytes = 4352;
constexpr int kDecMaxT = 16, kDecMaxEnt = 128, kDecMaxRows = 16;   // rows of H per CTA in P3 (<= 4 chunks of 4)

struct DecLayer {
    const uint8_t* blobs;    // [E][blob_bytes]
    const float* router;     // [E + 1][H]: the expert rows, then the shared-gate row
    const uint8_t* sh_blob;  // the shared expert
};

struct DecParams {
    int n_layers, T, H, F, E, K, FS;
    uint32_t gu_row, d_row, sgu_row, sd_row;
    uint64_t up_off, down_off, blob_bytes, s_up_off, s_down_off;
    int R;                    // routed down rows per chunk (R * d_row % 16 == 0)
    int rt_per_unit, sd_per_unit, dn_per_unit;   // items packed per ring slot
    const DecLayer* layers;
    float* x;                 // [T][H] residual stream, in / out
    float* logits;            // [T][E + 1][2]: the two half-row partial dots
    float* hsh;               // [T][FS] shared hidden
    float* hbuf;              // [T * K][F] routed hidden, by entry
    float* sh_out;            // [T][H] shared expert output
    int32_t* ids_rec;         // [layers][T][K] or null
    float* w_rec;
    unsigned* bar;            // grid barrier counter (zero at launch)
    unsigned* err;
    unsigned long long* trace;   // optional phase stamps: [layer][kTraceEvents][CTA] of %globaltimer, or null
    float eps;
    uint32_t smem_base;       // the shared-window address the dynamic shared memory starts at (checked)
};
constexpr int kTraceEvents = 16;

struct DecShared {
    uint64_t full[kSlots], empty[kSlots], route;
    int claim;
    int abort;
    volatile int prod_seq, prod_state;   // the producer's progress (diagnostics of a wait that gives up)
    volatile int warp_unit[kDecConsumers];   // the ring sequence each consumer warp waits on or works on
    volatile int warp_state[kDecConsumers];  // 1 waiting, 2 computing, 3 released
    // The ring lap the producer has started on each slot.  A consumer may claim a unit a whole lap ahead of a slot's
    // previous unit; waiting on the full barrier's parity is only unambiguous once the producer has started that lap
    // (a barrier still in phase lap - 1 answers a wait on parity lap & 1 as complete: the preceding phase).
    volatile int slot_lap[kSlots];
    unsigned canary;
    int n_groups;
    float rms[kDecMaxT];
    float gs[kDecMaxT];
    int32_t ids[kDecMaxEnt];
    float w[kDecMaxEnt];
    int32_t grp_expert[kDecMaxEnt], grp_start[kDecMaxEnt + 1], ent_dst[kDecMaxEnt], ent_tok[kDecMaxEnt];
    float red[256];
};

// Offsets inside the dynamic shared memory (dynamic base at shared address b0 <= 0x10000 - kSlots * kSlotBytes):
//   [0, kSlots * kSlotBytes)              the ring
//   [0x10000 - b0, +64 KB)                the IQ3_XXS tables at shared address 0x10000
//   [0x20000 - b0, ...)                   DecShared, parts [kDecMaxEnt][kDecMaxRows], then the activation union:
//       P0..P2: xq codes [T][H], xq scales [T][H / 32], hshq codes [T][FS], hshq scales [T][FS / 32]
//       P3:     hq codes [T K][F], hq scales [T K][F / 32]
struct DecSmem {
    uint32_t tab, shared, parts, uni, xq_d, hs, hs_d, hq_d, total;
};
__host__ __device__ inline DecSmem dec_smem(uint32_t b0, int T, int H, int F, int FS, int K) {
    auto al = [](uint32_t v, uint32_t a) { return (v + a - 1) / a * a; };
    DecSmem m;
    m.tab = 0x10000u - b0;
    m.shared = 0x20000u - b0;
    m.parts = al(m.shared + (uint32_t) sizeof(DecShared), 16);
    m.uni = al(m.parts + (uint32_t) (kDecMaxEnt * kDecMaxRows * 4), 128);
    m.xq_d = m.uni + (uint32_t) (T * H);
    m.hs = al(m.xq_d + (uint32_t) (T * (H / 32) * 4), 16);
    m.hs_d = m.hs + (uint32_t) (T * FS);
    const uint32_t end1 = m.hs_d + (uint32_t) (T * (FS / 32) * 4);
    m.hq_d = m.uni + (uint32_t) (T * K * F);
    const uint32_t end2 = m.hq_d + (uint32_t) (T * K * (F / 32) * 4);
    m.total = end1 > end2 ? end1 : end2;
    return m;
}

// -------------------------------------------------------------------------------------------------- small helpers
// A wait that gave up: the first one records its site and four words of context after the error word.
__device__ __forceinline__ void report_detail(unsigned* err, unsigned site, unsigned a, unsigned b, unsigned c,
                                              unsigned d) {
    if (err && atomicCAS(err, 0u, site) == 0u) {
        err[1] = a;
        err[2] = b;
        err[3] = c;
        err[4] = d;
        __threadfence();
    }
}
// Phase stamps (consumers: 0 layer start, 1 P0, 2 P1, 3 barrier, 4 routing, 5 P2, 6 barrier, 7 P3 + combine,
// 8 barrier; producer: 9 P1 issued, 10 routing seen, 11 P2 issued, 12 P3 issued).
__device__ __forceinline__ void stamp(const DecParams& p, int l, int ev) {
    if (p.trace) p.trace[((size_t) l * kTraceEvents + ev) * gridDim.x + blockIdx.x] = globaltimer();
    if (ev < 9) ((volatile unsigned*) p.err)[128 + blockIdx.x] = ((unsigned) l << 8) | (unsigned) ev;
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Consumers: all 480 threads.  Thread 0 publishes this CTA's arrival and waits for the others (acquire), bounded.
__device__ bool grid_barrier(const DecParams& p, DecShared& S, unsigned& target, unsigned site) {
    named_sync(1, kDecCThreads);
    target += gridDim.x;
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(p.bar, 1u);
        const uint64_t t0 = globaltimer();
        unsigned v;
        while ((v = ld_acquire(p.bar)) < target) {
            if (globaltimer() - t0 > kWaitNs || S.abort) {
                report_error(p.err, site);
                if (p.err && atomicCAS(p.err + 99, 0u, 1u) == 0u) {
                    p.err[100] = site;
                    p.err[101] = v;
                    p.err[102] = target;
                    p.err[103] = (unsigned) S.prod_state;
                    p.err[104] = blockIdx.x;
                }
                S.abort = 1;
                break;
            }
        }
    }
    named_sync(1, kDecCThreads);
    return !S.abort;
}

// -------------------------------------------------------------------------------------------------- unit lists
// P1: 2 (E + 1) router half rows, then FS shared gate/up pairs.  P2: routed gate/up pairs packed rt_per_unit to a
// slot, then shared down rows packed sd_per_unit.  P3: this CTA's (chunk, group) tasks packed dn_per_unit.
struct Range {
    int lo, hi;
};
__device__ __forceinline__ Range split(int n, int parts, int i) { return {(int) ((long long) n * i / parts), (int) ((long long) n * (i + 1) / parts)}; }

__device__ __forceinline__ int p1_units(const DecParams& p) { return 2 * (p.E + 1) + p.FS; }
__device__ __forceinline__ int p2_rt_units(const DecParams& p, int ng) { return (ng * p.F + p.rt_per_unit - 1) / p.rt_per_unit; }
__device__ __forceinline__ int p2_units(const DecParams& p, int ng) { return p2_rt_units(p, ng) + p.H / p.sd_per_unit; }
__device__ __forceinline__ Range my_chunks(const DecParams& p) { return split(p.H / p.R, gridDim.x, blockIdx.x); }
__device__ __forceinline__ int p3_units(const DecParams& p, int ng) {
    const Range c = my_chunks(p);
    return ((c.hi - c.lo) * ng + p.dn_per_unit - 1) / p.dn_per_unit;
}

// -------------------------------------------------------------------------------------------------- producer
struct BulkCopy {
    const void* src;
    uint32_t dst;     // offset in the slot
    uint32_t bytes;
};

struct Producer {
    uint32_t seq = 0;   // ring sequence number of the next unit (identical in every lane of the producer warp)
    uint8_t* ring;
    DecShared* S;
    const DecParams* p;

    __device__ uint8_t* slot_ptr(uint32_t slot) const { return ring + (size_t) slot * kSlotBytes; }
    // Is the slot of sequence number s free (its previous lap released by the consumers)?  wait: bounded wait.
    __device__ bool slot_free(uint32_t s, bool wait) {
        if (s < (uint32_t) kSlots) return true;
        const uint32_t slot = s % kSlots, par = ((s / kSlots) - 1) & 1u;
        if (!wait) return mbar_test_wait(&S->empty[slot], par);
        if (mbar_try_wait(&S->empty[slot], par)) return true;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&S->empty[slot], par)) {
            if (globaltimer() - t0 > kWaitNs || S->abort) {
                report_detail(p->err, 0x310u, s, (unsigned) S->prod_state, (unsigned) S->claim, blockIdx.x);
                S->abort = 1;
                return false;
            }
        }
        return true;
    }
    // Units [lo, hi) of a phase.  copies(u): bulk copies of unit u (<= 32 over a batch); bytes(u): their total;
    // copy(u, c): copy c of unit u (source, offset in the slot, bytes).  Lane 0 takes the next slot (waiting) and the
    // free ones after it; lane j starts unit j of the batch (publishes its lap, arms its barrier); then every lane
    // issues its copy in ONE converged instruction (a cp.async.bulk issued under divergence goes out lane by lane,
    // each holding the warp for a fraction of a memory latency).
    template <class NC, class NB, class CP>
    __device__ bool produce(int lo, int hi, NC copies, NB bytes, CP copy) {
        const int lane = threadIdx.x & 31;
        for (int u = lo; u < hi;) {
            int nb = 0;
            if (lane == 0 && slot_free(seq, true)) {
                int ncp = copies(u);
                nb = 1;
                while (u + nb < hi && nb < kSlots && ncp + copies(u + nb) <= 32 && slot_free(seq + nb, false))
                    ncp += copies(u + nb++);
            }
            nb = __shfl_sync(0xffffffffu, nb, 0);
            if (nb == 0) return false;
            if (lane < nb) {
                const uint32_t s = seq + lane, slot = s % kSlots;
                S->slot_lap[slot] = (int) (s / kSlots);
                mbar_expect_tx(&S->full[slot], bytes(u + lane));
            }
            __syncwarp();
            int mj = -1, mc = 0, base = 0;
            for (int j = 0; j < nb; ++j) {
                const int n = copies(u + j);
                if (lane >= base && lane < base + n) {
                    mj = j;
                    mc = lane - base;
                }
                base += n;
            }
            const BulkCopy cp = copy(u + max(mj, 0), mc);
            const uint32_t slot = (seq + (uint32_t) max(mj, 0)) % kSlots;
            if (mj >= 0) bulk_g2s(slot_ptr(slot) + cp.dst, cp.src, cp.bytes, &S->full[slot]);
            __syncwarp();
            seq += (uint32_t) nb;
            u += nb;
            if (lane == 0) S->prod_seq = (int) seq;
        }
        return true;
    }
};

// -------------------------------------------------------------------------------------------------- activations
// This CTA's q8_1 image of h for the step's tokens: codes [T][H] and fp16-rounded scales [T][H / 32].
struct XqView {
    const int8_t* codes;
    const float* d;
    int H;   // values per row
    __device__ QB block(int t, int b) const {
        QB r;
        const int4* c = (const int4*) (codes + (size_t) t * H + 32 * b);
        const int4 a0 = c[0], a1 = c[1];
        r.q[0] = a0.x; r.q[1] = a0.y; r.q[2] = a0.z; r.q[3] = a0.w;
        r.q[4] = a1.x; r.q[5] = a1.y; r.q[6] = a1.z; r.q[7] = a1.w;
        r.d = d[t * (H / 32) + b];
        return r;
    }
};

// Rows of fp32 (written by other CTAs of this launch) into a q8_1 image in shared memory: one warp per 32-value block,
// the reference's quantiser (the same bits as q8_1_lane / the standalone kernel).
__device__ __forceinline__ void quantize_rows_to_smem(const float* src, int rows, int n, int8_t* codes, float* dsc,
                                                      int warp, int lane, int nwarps) {
    const int nb = n / 32;
    for (int b = warp; b < rows * nb; b += nwarps) {
        const int r = b / nb, k = b % nb;
        const float v = __ldcg(src + (size_t) r * n + 32 * k + lane);
        float d, sum;
        const int8_t q = q8_1_warp(v, d, sum);
        codes[(size_t) r * n + 32 * k + lane] = q;
        if (lane == 0) dsc[b] = __half2float(__float2half(q8_finite(d)));
    }
}

// A contiguous fp32 array (rows of 32-value blocks; written by other CTAs of this launch, or in shared memory) into
// q8_1 codes and fp16-rounded scales in shared memory: 8 lanes per block, 4 values each (float4), B loads in flight
// per lane before any arithmetic.  The block scale is amax / 127 with the reference's division and the codes
// round(x / d): the same codes and scale as the reference's quantiser, whatever the lane layout (the fp16 sum it also
// stores is not formed: no format here reads it).
template <bool FROM_SMEM, int B = FROM_SMEM ? 1 : 2>
__device__ __forceinline__ void quantize_blocks(const float* src, int n, int8_t* codes, float* dsc, int warp, int lane,
                                                int nwarps) {
    const int n4 = n / 4;
    const int stride = nwarps * 32;
    for (int base = warp * 32 + lane; base - lane < n4; base += B * stride) {
        float4 v[B];
#pragma unroll
        for (int it = 0; it < B; ++it) {
            const int i = base + it * stride;
            if (i < n4) v[it] = FROM_SMEM ? ((const float4*) src)[i] : __ldcg((const float4*) src + i);
        }
#pragma unroll
        for (int it = 0; it < B; ++it) {
            const int i = base + it * stride;
            if (i - lane >= n4) break;   // warp-uniform: whole warps of float4s
            float amax = fmaxf(fmaxf(fabsf(v[it].x), fabsf(v[it].y)), fmaxf(fabsf(v[it].z), fabsf(v[it].w)));
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float d = q8_finite(fdiv_fm(amax, 127.0f));
            uint32_t word = 0;
            const float xs[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int8_t c = 0;
                if (amax != 0.0f) {
                    const float r = roundf(fdiv_fm(xs[j], d));
                    c = (int8_t) (r > 127.0f ? 127.0f : r < -127.0f ? -127.0f : r);
                }
                word |= (uint32_t) (uint8_t) c << (8 * j);
            }
            ((uint32_t*) codes)[i] = word;
            if ((lane & 7) == 0) dsc[i >> 3] = __half2float(__float2half(d));
        }
    }
}

// IQ3_XXS gate/up row of 8 blocks (H = 2048) against one activation, with the block parity uniform per step: lane
// l = 8 q + c decodes call c of block 2 q (step 0, 4-byte aligned) and of block 2 q + 1 (step 1, 2 mod 4); a[j] is the
// q8_1 block of that call (iq3_par_call).  The sum has the bits of the reference's row order -- lane L adds call L's
// product and then call L + 32's (multiply-add), an xor tree over 32 lanes -- rebuilt by exchanges: lanes 16..31 hold
// the calls 32..63, take the products of calls 0..31 from lane l ^ 16 and form the 32 lane sums two per lane (blocks
// even / odd), whose xor-16 level is a xor-8 exchange here and whose xor-8 level an add in the lane.  Every lane
// returns the sum (lanes 0..15 a value of no use).
__device__ __forceinline__ float iq3_row_par(const uint8_t* row, int lane, const Fmt<T_IQ3_XXS>::Act (&a)[2],
                                             const AbsTab& t) {
    const int c = lane & 7, q = lane >> 3;
    const Iq3x xe = iq3x_decode_blk<false>(row + 196 * q, c, t);
    const float de = __fmul_rn(xe.dw, a[0].d), fe = (float) iq3x_sumi(xe, a[0].u);
    const Iq3x xo = iq3x_decode_blk<true>(row + 196 * q + 98, c, t);
    const float dd = __fmul_rn(xo.dw, a[1].d), fo = (float) iq3x_sumi(xo, a[1].u);
    const float pe = __shfl_xor_sync(0xffffffffu, __fmul_rn(de, fe), 16);
    const float po = __shfl_xor_sync(0xffffffffu, __fmul_rn(dd, fo), 16);
    float se = __fmaf_rn(de, fe, pe), so = __fmaf_rn(dd, fo, po);
    se = __fadd_rn(se, __shfl_xor_sync(0xffffffffu, se, 8));
    so = __fadd_rn(so, __shfl_xor_sync(0xffffffffu, so, 8));
    float s = __fadd_rn(se, so);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    return s;
}
__device__ __forceinline__ int iq3_par_call(int lane, int j) { return 16 * (lane >> 3) + 8 * j + (lane & 7); }

// IQ3_XXS row against nc <= 2 activations (dual-dp4a signs for one, materialised signs for two), calls lane + 32 j.
template <int J>
__device__ __forceinline__ void iq3_row(const uint8_t* row, int C, int lane, const Fmt<T_IQ3_XXS>::Act (&a)[2][J],
                                        int nc, const AbsTab& t, float (&s)[2]) {
    s[0] = s[1] = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int k = lane + 32 * j;
        if (k < C) {
            const Iq3x x = iq3x_decode(row, k, t);
            if (nc == 1) {
                s[0] += iq3x_apply(x, a[0][j]);
            } else {
                const Fmt<T_IQ3_XXS>::W w = iq3x_signed(x);
                s[0] += Fmt<T_IQ3_XXS>::apply(w, a[0][j]);
                s[1] += Fmt<T_IQ3_XXS>::apply(w, a[1][j]);
            }
        }
    }
    s[0] = warp_sum(s[0]);
    if (nc > 1) s[1] = warp_sum(s[1]);
}

// -------------------------------------------------------------------------------------------------- the kernel
template <int V>   // V = E / 32 router values per lane
__global__ void __launch_bounds__(kDecThreads, 1) k_decode_layers(DecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const DecSmem M = dec_smem(p.smem_base, p.T, p.H, p.F, p.FS, p.K);
    uint8_t* ring = smem;
    uint8_t* tab = smem + M.tab;
    DecShared& S = *(DecShared*) (smem + M.shared);
    float* parts = (float*) (smem + M.parts);
    int8_t* xq_codes = (int8_t*) (smem + M.uni);
    float* xq_d = (float*) (smem + M.xq_d);
    int8_t* hs_codes = (int8_t*) (smem + M.hs);
    float* hs_d = (float*) (smem + M.hs_d);
    int8_t* hq_codes = (int8_t*) (smem + M.uni);   // P3 reuses the union
    float* hq_d = (float*) (smem + M.hq_d);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (smem_u32(smem) != p.smem_base) {   // the layout assumes the base the host computed it for
        if (threadIdx.x == 0) report_error(p.err, 0x300u);
        return;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(&S.route, 1);
        S.claim = 0;
        S.abort = 0;
        S.prod_seq = 0;
        S.prod_state = 0;
        S.canary = 0xC0FFEE01u;
        for (int q = 0; q < kSlots; ++q) S.slot_lap[q] = -1;
        if (blockIdx.x == 0 && p.err) {   // the layout as the device sees it
            p.err[110] = smem_u32(smem);
            p.err[111] = smem_u32(tab);
            p.err[112] = smem_u32(&S);
            p.err[113] = smem_u32(parts);
            p.err[114] = smem_u32(xq_codes);
            p.err[115] = M.total;
        }
        fence_mbar_init();
    }
    __syncthreads();

    // ============================================================================================ producer
    // The whole warp: lane 0 takes free ring slots in order, then the lanes issue the batch's bulk copies side by side
    // (one thread's cp.async.bulk issues serialise at a memory latency's fraction each; 32 lanes overlap them).
    if (warp == kDecWarps - 1) {
        Producer pr;
        pr.ring = ring;
        pr.S = &S;
        pr.p = &p;
        for (int l = 0; l < p.n_layers && !S.abort; ++l) {
            const DecLayer L = p.layers[l];
            if (lane == 0) S.prod_state = (l << 4) | 1;
            // P1: router half rows (one copy), shared gate/up row pairs (two)
            const Range r1 = split(p1_units(p), gridDim.x, blockIdx.x);
            const int nrh = 2 * (p.E + 1);
            auto p1_copies = [&](int u) { return u < nrh ? 1 : 2; };
            auto p1_bytes = [&](int u) { return u < nrh ? (uint32_t) (p.H / 2 * 4) : 2 * p.sgu_row; };
            auto p1_copy = [&](int u, int c) -> BulkCopy {
                if (u < nrh) {
                    const int o = u >> 1, half = u & 1;
                    return {L.router + (size_t) o * p.H + half * (p.H / 2), 0u, (uint32_t) (p.H / 2 * 4)};
                }
                const size_t off = (size_t) (u - nrh) * p.sgu_row + (c ? p.s_up_off : 0);
                return {L.sh_blob + off, c * p.sgu_row, p.sgu_row};
            };
            if (!pr.produce(r1.lo, r1.hi, p1_copies, p1_bytes, p1_copy)) break;
            if (lane == 0) stamp(p, l, 9);
            if (lane == 0) S.prod_state = (l << 4) | 2;
            {   // this layer's routing (lane 0 waits; the warp barrier orders the routing tables for the other lanes)
                int ok = 1;
                if (lane == 0) {
                    const uint64_t t0 = globaltimer();
                    while (!mbar_try_wait(&S.route, (uint32_t) (l & 1))) {
                        if (globaltimer() - t0 > kWaitNs || S.abort) {
                            report_error(p.err, 0x320u);
                            S.abort = 1;
                            break;
                        }
                    }
                    ok = !S.abort;
                }
                __syncwarp();
                if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            }
            const int ng = S.n_groups;
            if (lane == 0) stamp(p, l, 10);
            if (lane == 0) S.prod_state = (l << 4) | 3 | (ng << 16);
            // P2: routed gate/up rows (rt_per_unit consecutive rows of one expert: the gate block, then the up block),
            // then shared down rows (sd_per_unit consecutive rows, one copy)
            const int n2 = p2_units(p, ng), nrt = p2_rt_units(p, ng);
            const Range r2 = split(n2, gridDim.x, blockIdx.x);
            auto p2_copies = [&](int u) { return u < nrt ? 2 : 1; };
            auto p2_bytes = [&](int u) {
                return u < nrt ? (uint32_t) (min(p.rt_per_unit, ng * p.F - u * p.rt_per_unit) * 2 * p.gu_row)
                               : (uint32_t) p.sd_per_unit * p.sd_row;
            };
            auto p2_copy = [&](int u, int c) -> BulkCopy {
                if (u < nrt) {
                    const int i0 = u * p.rt_per_unit, n = min(p.rt_per_unit, ng * p.F - i0);
                    const int g = i0 / p.F, r = i0 % p.F;
                    const uint8_t* b = L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + (size_t) r * p.gu_row;
                    return {b + (c ? p.up_off : 0), (uint32_t) (c * n) * p.gu_row, (uint32_t) n * p.gu_row};
                }
                const int r0 = (u - nrt) * p.sd_per_unit;
                return {L.sh_blob + p.s_down_off + (size_t) r0 * p.sd_row, 0u, (uint32_t) p.sd_per_unit * p.sd_row};
            };
            if (!pr.produce(r2.lo, r2.hi, p2_copies, p2_bytes, p2_copy)) break;
            if (lane == 0) stamp(p, l, 11);
            if (lane == 0) S.prod_state = (l << 4) | 4 | (ng << 16);
            // P3: this CTA's down rows of each group, task i = (group i / nch, chunk i % nch): a unit's tasks of one
            // group are consecutive rows, one copy per group it touches
            const Range ch = my_chunks(p);
            const int nch = ch.hi - ch.lo, ntask = nch * ng;
            const uint32_t cb = (uint32_t) p.R * p.d_row;
            auto p3_copies = [&](int u) {
                const int i0 = u * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                return (i1 - 1) / nch - i0 / nch + 1;
            };
            auto p3_bytes = [&](int u) {
                const int i0 = u * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                return (uint32_t) (i1 - i0) * cb;
            };
            auto p3_copy = [&](int u, int c) -> BulkCopy {
                const int i0 = u * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                const int g = i0 / nch + c;
                const int a0 = max(i0, g * nch), a1 = min(i1, (g + 1) * nch);
                const uint8_t* b = L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + p.down_off +
                                   (size_t) (ch.lo + a0 - g * nch) * cb;
                return {b, (uint32_t) (a0 - i0) * cb, (uint32_t) (a1 - a0) * cb};
            };
            if (!pr.produce(0, p3_units(p, ng), p3_copies, p3_bytes, p3_copy)) break;
            if (lane == 0) stamp(p, l, 12);
        }
        // wind down: every copy issued is complete before the CTA may exit (bounded)
        if (lane == 0)
            for (uint32_t s = pr.seq > kSlots ? pr.seq - kSlots : 0; s < pr.seq; ++s) {
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(&S.full[s % kSlots], (s / kSlots) & 1u))
                    if (globaltimer() - t0 > kWaitNs) break;
            }
        return;
    }

    // ============================================================================================ consumers
    fill_tables<T_IQ3_XXS>(tab, kDecCThreads);   // consumers only, so a named barrier (not __syncthreads)
    named_sync(1, kDecCThreads);
    if (threadIdx.x == 0 && S.canary != 0xC0FFEE01u) {
        report_error(p.err, 0x3F0u);
        if (p.err) p.err[116] = S.canary;
    }
    const IqTab itab = make_tab(tab, lane);
    const AbsTab atab = make_abs_tab(lane);
    uint32_t seq = 0;               // the ring sequence number of the next unit, identical in every consumer
    int claim_base = 0;
    unsigned target = 0;
    const int T = p.T, H = p.H, F = p.F, E = p.E, K = p.K;
    const XqView xv{xq_codes, xq_d, H};
    const XqView hsv{hs_codes, hs_d, p.FS};
    const XqView hqv{hq_codes, hq_d, F};

    auto claim = [&](int n, int& k) -> bool {   // this warp's next unit of the phase, or false
        int v = 0;
        if (lane == 0) v = atomicAdd(&S.claim, 1);
        v = __shfl_sync(0xffffffffu, v, 0);
        k = v - claim_base;
        return k < n;
    };
    int cur_layer = 0, cur_phase = 0;
    auto wait_full = [&](uint32_t s) -> bool {
        const uint32_t slot = s % kSlots, par = (s / kSlots) & 1u;
        if (lane == 0) {
            S.warp_unit[warp] = (int) s;
            S.warp_state[warp] = 1;
        }
        const uint64_t t0 = globaltimer();
        bool failed = false;
        while (S.slot_lap[slot] < (int) (s / kSlots)) {   // the producer has not started this lap on the slot yet
            if (globaltimer() - t0 > kWaitNs) {
                failed = true;
                break;
            }
        }
        bool done = failed || mbar_try_wait(&S.full[slot], par);
        while (!done) {   // every lane observes the phase itself (the bulk copy's bytes are then visible to it)
            done = mbar_try_wait(&S.full[slot], par);
            if (!done && globaltimer() - t0 > kWaitNs) {
                failed = true;
                break;
            }
        }
        if (__all_sync(0xffffffffu, !failed)) {   // one verdict for the whole warp
            if (lane == 0) S.warp_state[warp] = 2;
            return true;
        }
        {
            {
                report_error(p.err, 0x330u | ((unsigned) cur_phase << 12));
                if (p.err && atomicCAS(p.err + 61, 0u, 1u) == 0u) {
                    p.err[1] = s | ((unsigned) cur_layer << 24);
                    p.err[2] = (unsigned) S.prod_seq;
                    p.err[3] = (unsigned) S.prod_state;
                    p.err[4] = (unsigned) claim_base | (blockIdx.x << 20);
                    p.err[5] = (unsigned) S.claim;
                    for (int w = 0; w < kDecConsumers; ++w)
                        p.err[6 + w] = (unsigned) S.warp_unit[w] | ((unsigned) S.warp_state[w] << 16);
                    for (int q = 0; q < kSlots; ++q) {   // raw mbarrier words of every slot
                        const unsigned long long f = *(volatile unsigned long long*) &S.full[q];
                        const unsigned long long e = *(volatile unsigned long long*) &S.empty[q];
                        p.err[24 + 4 * q] = (unsigned) f;
                        p.err[25 + 4 * q] = (unsigned) (f >> 32);
                        p.err[26 + 4 * q] = (unsigned) e;
                        p.err[27 + 4 * q] = (unsigned) (e >> 32);
                    }
                    __threadfence();
                }
                S.abort = 1;
                return false;
            }
        }
        return true;
    };
    auto release = [&](uint32_t s) {
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&S.empty[s % kSlots]);
            S.warp_state[warp] = 3;
        }
    };
    auto end_phase = [&](int n) {   // every consumer warp overshoots its claims once
        claim_base += n + kDecConsumers;
        seq += (uint32_t) n;
    };

    const int Cs = H / 32 * 4;           // Q8_0 calls per shared gate/up row
    const int Csd = p.FS / 32 * 4;       // Q8_0 calls per shared down row

    for (int l = 0; l < p.n_layers; ++l) {
        if (threadIdx.x == 0) stamp(p, l, 0);
        // ---------------------------------------------------------------- P0: rms and q8_1 of every token
        // The reference's order (k_moe_out_small): 256 slots s = sum over i = s mod 256 of x_i^2 in order, then the
        // halving tree; thread i < 32 forms the tree's 32-slot level from 8 slots, shuffles finish it.
        float* xs = parts;   // the token's row in shared memory (the parts buffer is free until P3)
        for (int t = 0; t < T; ++t) {
            const float* xr = p.x + (size_t) t * H;
            for (int i = threadIdx.x; i < H / 4; i += kDecCThreads) ((float4*) xs)[i] = __ldcg((const float4*) xr + i);
            named_sync(1, kDecCThreads);
            if (threadIdx.x < 256) {
                float s = 0.0f;
                for (int i = threadIdx.x; i < H; i += 256) s += xs[i] * xs[i];
                S.red[threadIdx.x] = s;
            }
            named_sync(1, kDecCThreads);
            if (warp == 0) {
                const float* r = S.red;
                const int i = lane;
                float a = ((r[i] + r[i + 128]) + (r[i + 64] + r[i + 192])) +
                          ((r[i + 32] + r[i + 160]) + (r[i + 96] + r[i + 224]));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) a += __shfl_down_sync(0xffffffffu, a, o);
                if (lane == 0) S.rms[t] = rsqrtf(fdiv_fm(a, (float) H) + p.eps);
            }
            named_sync(1, kDecCThreads);
            const float r = S.rms[t];
            for (int i = threadIdx.x; i < H; i += kDecCThreads) xs[i] = __fmul_rn(xs[i], r);   // h = x r (wn = 1)
            named_sync(1, kDecCThreads);
            quantize_blocks<true>(xs, H, xq_codes + (size_t) t * H, xq_d + t * (H / 32), warp, lane, kDecConsumers);
            if (t + 1 < T) named_sync(1, kDecCThreads);
        }
        named_sync(1, kDecCThreads);
        if (threadIdx.x == 0) stamp(p, l, 1);
        cur_layer = l;
        cur_phase = 1;

        // ---------------------------------------------------------------- P1: router rows, shared gate/up
        {
            const int n1 = p1_units(p);
            const Range r1 = split(n1, gridDim.x, blockIdx.x);
            const int mine = r1.hi - r1.lo;
            int k;
            while (claim(mine, k)) {
                const uint32_t s = seq + (uint32_t) k;
                if (!wait_full(s)) break;
                const uint8_t* buf = ring + (size_t) (s % kSlots) * kSlotBytes;
                const int u = r1.lo + k;
                if (u < 2 * (E + 1)) {
                    const int o = u >> 1, half = u & 1;
                    const float4* wr = (const float4*) buf;
                    for (int t = 0; t < T; ++t) {
                        const float* xr = p.x + (size_t) t * H + half * (H / 2);
                        const float r = S.rms[t];
                        float acc = 0.0f;
                        if (T == 1) {   // h of the only token is in shared memory
                            const float4* hs4 = (const float4*) (xs + half * (H / 2));
#pragma unroll 4
                            for (int i = lane; i < H / 8; i += 32) {
                                const float4 w = wr[i], hv = hs4[i];
                                acc += w.x * hv.x + w.y * hv.y + w.z * hv.z + w.w * hv.w;
                            }
                        } else {
#pragma unroll 4
                            for (int i = lane; i < H / 8; i += 32) {
                                const float4 w = wr[i];
                                const float4 xv4 = __ldcg((const float4*) xr + i);
                                acc += w.x * __fmul_rn(xv4.x, r) + w.y * __fmul_rn(xv4.y, r) + w.z * __fmul_rn(xv4.z, r) +
                                       w.w * __fmul_rn(xv4.w, r);
                            }
                        }
                        acc = warp_sum(acc);
                        if (lane == 0) p.logits[((size_t) t * (E + 1) + o) * 2 + half] = acc;
                    }
                } else {
                    const int r = u - 2 * (E + 1);
                    const uint8_t* gate = buf;
                    const uint8_t* up = buf + p.sgu_row;
                    for (int t = 0; t < T; ++t) {
                        // row_dot's order (lane + 32 j, j ascending, then the xor tree), one activation at a time
                        auto src = [&](int blk) { return xv.block(t, blk); };
                        float sg = 0.0f, su = 0.0f;
#pragma unroll 2
                        for (int k = lane; k < Cs; k += 32) {
                            const typename Fmt<T_Q8_0>::Act a = Fmt<T_Q8_0>::act(src, k);
                            sg += Fmt<T_Q8_0>::apply(decode_call<T_Q8_0>(gate, k, itab), a);
                            su += Fmt<T_Q8_0>::apply(decode_call<T_Q8_0>(up, k, itab), a);
                        }
                        sg = warp_sum(sg);
                        su = warp_sum(su);
                        if (lane == 0) p.hsh[(size_t) t * p.FS + r] = act_value(ACT_SWIGLU, sg, su, INFINITY);
                    }
                }
                release(s);
            }
            end_phase(mine);
        }
        if (threadIdx.x == 0) stamp(p, l, 2);
        if (!grid_barrier(p, S, target, 0x340u)) break;
        if (threadIdx.x == 0) stamp(p, l, 3);

        // ---------------------------------------------------------------- R: routing, grouping; shared hidden -> q8_1
        for (int t = warp; t < T; t += kDecConsumers) {
            const float* lg = p.logits + (size_t) t * (E + 1) * 2;
            float values[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const float2 pp = __ldcg((const float2*) lg + lane + i * 32);
                values[i] = pp.x + pp.y;
            }
            float maximum = -INFINITY;
#pragma unroll
            for (int i = 0; i < V; ++i) maximum = fmaxf(maximum, values[i]);
            maximum = warp_max(maximum);
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < V; ++i) {
                values[i] = fexp_fm(values[i] - maximum);
                sum += values[i];
            }
            const float reciprocal = frcp_fm(warp_sum(sum));
#pragma unroll
            for (int i = 0; i < V; ++i) {
                values[i] *= reciprocal;
                if (__isnanf(values[i])) values[i] = -FLT_MAX;
            }
            float selected = 0.0f, selected_sum = 0.0f;
            for (int rank = 0; rank < K; ++rank) {
                float best = values[0];
                int expert = lane;
#pragma unroll
                for (int i = 1; i < V; ++i)
                    if (values[i] > best) {
                        best = values[i];
                        expert = lane + i * 32;
                    }
#pragma unroll
                for (int m = 16; m; m >>= 1) {
                    const float ob = __shfl_xor_sync(0xffffffffu, best, m);
                    const int oi = __shfl_xor_sync(0xffffffffu, expert, m);
                    if (ob > best || (ob == best && oi < expert)) {
                        best = ob;
                        expert = oi;
                    }
                }
                if ((expert & 31) == lane) {
#pragma unroll
                    for (int i = 0; i < V; ++i)
                        if (i == expert / 32) values[i] = -INFINITY;
                    S.ids[t * K + rank] = expert;
                    selected_sum += best;
                }
                if (rank == lane) selected = best;
            }
            selected_sum = fmaxf(warp_sum(selected_sum), 6.103515625e-5f);
            const float inv = frcp_fm(selected_sum);
            if (lane < K) S.w[t * K + lane] = selected * inv;
            if (lane == 0) {
                const float2 pg = __ldcg((const float2*) lg + E);
                S.gs[t] = frcp_fm(1.0f + fexp_fm(-(pg.x + pg.y)));
            }
        }
        // the shared expert's hidden vectors into q8_1, by the warps that route no token
        if (T < kDecConsumers && warp >= T)
            quantize_blocks<false>(p.hsh, T * p.FS, hs_codes, hs_d, warp - T, lane, kDecConsumers - T);
        else if (T >= kDecConsumers)
            quantize_blocks<false>(p.hsh, T * p.FS, hs_codes, hs_d, warp, lane, kDecConsumers);
        named_sync(1, kDecCThreads);
        {
            const int n_ent = T * K;
            const int e = threadIdx.x;
            int id = 0, rank = 0;
            if (e < n_ent) {
                id = S.ids[e];
                for (int e2 = 0; e2 < n_ent; ++e2) {
                    const int id2 = S.ids[e2];
                    rank += (id2 < id || (id2 == id && e2 < e)) ? 1 : 0;
                }
                S.ent_dst[rank] = e;
                S.ent_tok[rank] = e / K;
                if (blockIdx.x == 0 && p.ids_rec) {
                    p.ids_rec[(size_t) l * n_ent + e] = id;
                    p.w_rec[(size_t) l * n_ent + e] = S.w[e];
                }
            }
            named_sync(1, kDecCThreads);
            if (e < n_ent) {   // group g starts at the sorted position of the first entry of its expert
                const int pos = rank;
                const int prev_id = pos > 0 ? S.ids[S.ent_dst[pos - 1]] : -1;
                if (prev_id != id) {
                    int g = 0;
                    for (int q = 1; q <= pos; ++q) g += S.ids[S.ent_dst[q - 1]] != S.ids[S.ent_dst[q]] ? 1 : 0;
                    S.grp_expert[g] = id;
                    S.grp_start[g] = pos;
                }
            }
            if (e == 0) {
                int G = n_ent > 0 ? 1 : 0;
                for (int q = 1; q < n_ent; ++q) G += S.ids[S.ent_dst[q - 1]] != S.ids[S.ent_dst[q]] ? 1 : 0;
                S.grp_start[G] = n_ent;
                S.n_groups = G;
            }
            named_sync(1, kDecCThreads);
            if (threadIdx.x == 0) mbar_arrive(&S.route);   // the producer may stream this layer's P2 and P3
        }
        const int ng = S.n_groups;
        if (threadIdx.x == 0) stamp(p, l, 4);

        // ---------------------------------------------------------------- P2: routed gate/up, shared down
        cur_phase = 2;
        {
            const int n2 = p2_units(p, ng), nrt = p2_rt_units(p, ng);
            const Range r2 = split(n2, gridDim.x, blockIdx.x);
            const int mine = r2.hi - r2.lo;
            int k;
            while (claim(mine, k)) {
                const uint32_t s = seq + (uint32_t) k;
                if (!wait_full(s)) break;
                const uint8_t* buf = ring + (size_t) (s % kSlots) * kSlotBytes;
                const int u = r2.lo + k;
                if (u < nrt) {
                    const int i0 = u * p.rt_per_unit, i1 = min(i0 + p.rt_per_unit, ng * F);
                    for (int i = i0; i < i1; ++i) {   // the unit's gate rows, then its up rows
                        const int g = i / F, r = i % F;
                        const uint8_t* gate = buf + (size_t) (i - i0) * p.gu_row;
                        const uint8_t* up = gate + (size_t) (i1 - i0) * p.gu_row;
                        const int e0 = S.grp_start[g], e1 = S.grp_start[g + 1];
                        for (int eb = e0; eb < e1; ++eb) {   // decode groups rarely hold more than one entry
                            const int tok = S.ent_tok[eb];
                            auto src = [&](int blk) { return xv.block(tok, blk); };
                            Fmt<T_IQ3_XXS>::Act a[2];
#pragma unroll
                            for (int j = 0; j < 2; ++j) a[j] = Fmt<T_IQ3_XXS>::act(src, iq3_par_call(lane, j));
                            const float sg = iq3_row_par(gate, lane, a, atab);
                            const float su = iq3_row_par(up, lane, a, atab);
                            if (lane == 16) p.hbuf[(size_t) S.ent_dst[eb] * F + r] = act_value(ACT_SWIGLU, sg, su, INFINITY);
                        }
                    }
                } else {
                    const int r0 = (u - nrt) * p.sd_per_unit;
                    for (int t0 = 0; t0 < T; t0 += 2) {
                        const int nc = min(2, T - t0);
                        typename Fmt<T_Q8_0>::Act a[2][2];
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            if (c >= nc) break;
                            auto src = [&](int blk) { return hsv.block(t0 + c, blk); };
#pragma unroll
                            for (int j = 0; j < 2; ++j)
                                if (lane + 32 * j < Csd) a[c][j] = Fmt<T_Q8_0>::act(src, lane + 32 * j);
                        }
                        for (int rr = 0; rr < p.sd_per_unit; ++rr) {
                            float sv[2];
                            row_dot<T_Q8_0, 2, 2>(buf + (size_t) rr * p.sd_row, Csd, lane, a, nc, itab, sv);
                            if (lane < nc) p.sh_out[(size_t) (t0 + lane) * H + r0 + rr] = lane == 0 ? sv[0] : sv[1];
                        }
                    }
                }
                release(s);
            }
            end_phase(mine);
        }
        if (threadIdx.x == 0) stamp(p, l, 5);
        if (!grid_barrier(p, S, target, 0x350u)) break;
        if (threadIdx.x == 0) stamp(p, l, 6);

        // ---------------------------------------------------------------- P3: routed down rows, combine
        cur_phase = 3;
        {
            quantize_blocks<false>(p.hbuf, T * K * F, hq_codes, hq_d, warp, lane, kDecConsumers);
            named_sync(1, kDecCThreads);
            const Range ch = my_chunks(p);
            const int nch = ch.hi - ch.lo, ntask = nch * ng;
            const int mine = p3_units(p, ng);
            int k;
            while (claim(mine, k)) {
                const uint32_t s = seq + (uint32_t) k;
                if (!wait_full(s)) break;
                const uint8_t* buf = ring + (size_t) (s % kSlots) * kSlotBytes;
                const int i0 = k * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                for (int i = i0; i < i1; ++i) {
                    const int cl = i % nch, g = i / nch;   // chunk index within this CTA, group (group-major tasks)
                    const uint8_t* rows = buf + (size_t) (i - i0) * p.R * p.d_row;
                    const int e0 = S.grp_start[g], e1 = S.grp_start[g + 1];
                    for (int eb = e0; eb < e1; ++eb) {
                        const int ent = S.ent_dst[eb];
                        auto src = [&](int blk) { return hqv.block(ent, blk); };
                        const Fmt<T_IQ3_XXS>::Act a0 = Fmt<T_IQ3_XXS>::act(src, lane & 7);
                        const Fmt<T_IQ3_XXS>::Act a1 = Fmt<T_IQ3_XXS>::act(src, 8 + (lane & 7));
                        // 4 rows of 2 blocks (F = 512): block 0 of row r at 196 r (0 mod 4), block 1 at 196 r + 98.  The
                        // reference's row sum is an xor tree over 16 lanes of one call each: its first level (calls c and
                        // c + 8) is the add in the lane here, the rest the same exchanges.
                        const uint8_t* rw = rows + (size_t) (lane >> 3) * p.d_row;
                        const Iq3x x0 = iq3x_decode_blk<false>(rw, lane & 7, atab);
                        const float v0 = __fmul_rn(__fmul_rn(x0.dw, a0.d), (float) iq3x_sumi(x0, a0.u));
                        const Iq3x x1 = iq3x_decode_blk<true>(rw + 98, lane & 7, atab);
                        float v = __fadd_rn(v0, __fmul_rn(__fmul_rn(x1.dw, a1.d), (float) iq3x_sumi(x1, a1.u)));
#pragma unroll
                        for (int o = 4; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                        if ((lane & 7) == 0) parts[ent * kDecMaxRows + cl * p.R + (lane >> 3)] = v;
                    }
                }
                release(s);
            }
            end_phase(mine);
            named_sync(1, kDecCThreads);
            // combine this CTA's rows for every token
            const int nrows = (ch.hi - ch.lo) * p.R;
            for (int i = threadIdx.x; i < T * nrows; i += kDecCThreads) {
                const int t = i / nrows, lr = i % nrows;
                const int row = ch.lo * p.R + lr;
                const float* wr = S.w + t * K;
                float acc = wr[0] * parts[(t * K) * kDecMaxRows + lr];
                for (int kk = 1; kk < K; ++kk) acc = fmaf(wr[kk], parts[(t * K + kk) * kDecMaxRows + lr], acc);
                acc += S.gs[t] * __ldcg(p.sh_out + (size_t) t * H + row);
                p.x[(size_t) t * H + row] = __ldcg(p.x + (size_t) t * H + row) + acc;
            }
        }
        if (threadIdx.x == 0) stamp(p, l, 7);
        if (!grid_barrier(p, S, target, 0x360u)) break;
        if (threadIdx.x == 0) stamp(p, l, 8);
    }
}

}  // namespace tsb
