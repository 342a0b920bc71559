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
constexpr int kSlots = 24;
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
};
constexpr int kTraceEvents = 16;

struct DecShared {
    uint64_t full[kSlots], empty[kSlots], route;
    int claim;
    int abort;
    int n_groups;
    float rms[kDecMaxT];
    float gs[kDecMaxT];
    int32_t ids[kDecMaxEnt];
    float w[kDecMaxEnt];
    int32_t grp_expert[kDecMaxEnt], grp_start[kDecMaxEnt + 1], ent_dst[kDecMaxEnt], ent_tok[kDecMaxEnt];
    float red[256];
};

// -------------------------------------------------------------------------------------------------- small helpers
// Phase stamps (consumers: 0 layer start, 1 P0, 2 P1, 3 barrier, 4 routing, 5 P2, 6 barrier, 7 P3 + combine,
// 8 barrier; producer: 9 P1 issued, 10 routing seen, 11 P2 issued, 12 P3 issued).
__device__ __forceinline__ void stamp(const DecParams& p, int l, int ev) {
    if (p.trace) p.trace[((size_t) l * kTraceEvents + ev) * gridDim.x + blockIdx.x] = globaltimer();
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Consumers: all 480 threads.  Thread 0 publishes this CTA's arrival and waits for the others (acquire), bounded.
__device__ bool grid_barrier(const DecParams& p, DecShared& S, unsigned& target, unsigned site) {
    named_sync(1, kDecCThreads);
    target += gridDim.x;
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(p.bar, 1u);
        const uint64_t t0 = globaltimer();
        while (ld_acquire(p.bar) < target) {
            if (globaltimer() - t0 > kWaitNs || S.abort) {
                report_error(p.err, site);
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
struct Producer {
    uint32_t seq = 0;
    uint8_t* ring;
    DecShared* S;
    const DecParams* p;

    __device__ bool acquire(uint32_t& slot) {
        slot = seq % kSlots;
        if (seq >= (uint32_t) kSlots) {
            const uint32_t par = ((seq / kSlots) - 1) & 1u;
            if (!mbar_try_wait(&S->empty[slot], par)) {
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(&S->empty[slot], par)) {
                    if (globaltimer() - t0 > kWaitNs || S->abort) {
                        report_error(p->err, 0x310u);
                        S->abort = 1;
                        return false;
                    }
                }
            }
        }
        return true;
    }
    __device__ uint8_t* slot_ptr(uint32_t slot) const { return ring + (size_t) slot * kSlotBytes; }
    __device__ void finish(uint32_t slot) { ++seq; (void) slot; }
};

// -------------------------------------------------------------------------------------------------- activations
// This CTA's q8_1 image of h for the step's tokens: codes [T][H] and fp16-rounded scales [T][H / 32].
struct XqView {
    const int8_t* codes;
    const float* d;
    int H;
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

// -------------------------------------------------------------------------------------------------- the kernel
template <int V>   // V = E / 32 router values per lane
__global__ void __launch_bounds__(kDecThreads, 1) k_decode_layers(DecParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* tab = smem;                                        // 64 KB lane-banked IQ3_XXS tables
    uint8_t* ring = smem + kIqTabBytes;                         // kSlots x kSlotBytes
    DecShared& S = *(DecShared*) (ring + (size_t) kSlots * kSlotBytes);
    // [T][H] codes, read with 16-byte loads: 128-byte aligned past the shared state
    int8_t* xq_codes = (int8_t*) (((uintptr_t) (&S + 1) + 127) & ~(uintptr_t) 127);
    float* xq_d = (float*) (xq_codes + (size_t) p.T * p.H);     // [T][H / 32]
    float* parts = xq_d + p.T * (p.H / 32);                     // [T * K][kDecMaxRows]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(&S.route, 1);
        S.claim = 0;
        S.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // ============================================================================================ producer
    if (warp == kDecWarps - 1) {
        if (lane != 0) return;
        Producer pr;
        pr.ring = ring;
        pr.S = &S;
        pr.p = &p;
        for (int l = 0; l < p.n_layers && !S.abort; ++l) {
            const DecLayer L = p.layers[l];
            // P1
            const Range r1 = split(p1_units(p), gridDim.x, blockIdx.x);
            for (int u = r1.lo; u < r1.hi; ++u) {
                uint32_t slot;
                if (!pr.acquire(slot)) break;
                uint8_t* dst = pr.slot_ptr(slot);
                if (u < 2 * (p.E + 1)) {
                    const int o = u >> 1, half = u & 1;
                    const uint32_t nb = (uint32_t) (p.H / 2 * 4);
                    mbar_expect_tx(&S.full[slot], nb);
                    bulk_g2s(dst, L.router + (size_t) o * p.H + half * (p.H / 2), nb, &S.full[slot]);
                } else {
                    const int r = u - 2 * (p.E + 1);
                    mbar_expect_tx(&S.full[slot], 2 * p.sgu_row);
                    bulk_g2s(dst, L.sh_blob + (size_t) r * p.sgu_row, p.sgu_row, &S.full[slot]);
                    bulk_g2s(dst + p.sgu_row, L.sh_blob + p.s_up_off + (size_t) r * p.sgu_row, p.sgu_row, &S.full[slot]);
                }
                pr.finish(slot);
            }
            stamp(p, l, 9);
            // wait for this layer's routing
            {
                const uint64_t t0 = globaltimer();
                while (!mbar_try_wait(&S.route, (uint32_t) (l & 1))) {
                    if (globaltimer() - t0 > kWaitNs || S.abort) {
                        report_error(p.err, 0x320u);
                        S.abort = 1;
                        break;
                    }
                }
                if (S.abort) break;
            }
            const int ng = S.n_groups;
            stamp(p, l, 10);
            // P2
            const int n2 = p2_units(p, ng), nrt = p2_rt_units(p, ng);
            const Range r2 = split(n2, gridDim.x, blockIdx.x);
            for (int u = r2.lo; u < r2.hi; ++u) {
                uint32_t slot;
                if (!pr.acquire(slot)) break;
                uint8_t* dst = pr.slot_ptr(slot);
                if (u < nrt) {
                    const int i0 = u * p.rt_per_unit, i1 = min(i0 + p.rt_per_unit, ng * p.F);
                    mbar_expect_tx(&S.full[slot], (uint32_t) (i1 - i0) * 2 * p.gu_row);
                    for (int i = i0; i < i1; ++i) {
                        const int g = i / p.F, r = i % p.F;
                        const uint8_t* b = L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + (size_t) r * p.gu_row;
                        bulk_g2s(dst, b, p.gu_row, &S.full[slot]);
                        bulk_g2s(dst + p.gu_row, b + p.up_off, p.gu_row, &S.full[slot]);
                        dst += 2 * p.gu_row;
                    }
                } else {
                    const int r0 = (u - nrt) * p.sd_per_unit;
                    const uint32_t nb = (uint32_t) p.sd_per_unit * p.sd_row;
                    mbar_expect_tx(&S.full[slot], nb);
                    bulk_g2s(dst, L.sh_blob + p.s_down_off + (size_t) r0 * p.sd_row, nb, &S.full[slot]);
                }
                pr.finish(slot);
            }
            stamp(p, l, 11);
            // P3
            const Range ch = my_chunks(p);
            const int ntask = (ch.hi - ch.lo) * ng;
            const int n3 = p3_units(p, ng);
            const uint32_t cb = (uint32_t) p.R * p.d_row;
            for (int u = 0; u < n3; ++u) {
                uint32_t slot;
                if (!pr.acquire(slot)) break;
                uint8_t* dst = pr.slot_ptr(slot);
                const int i0 = u * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                mbar_expect_tx(&S.full[slot], (uint32_t) (i1 - i0) * cb);
                for (int i = i0; i < i1; ++i) {
                    const int c = ch.lo + i / ng, g = i % ng;
                    const uint8_t* b = L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + p.down_off + (size_t) c * cb;
                    bulk_g2s(dst, b, cb, &S.full[slot]);
                    dst += cb;
                }
                pr.finish(slot);
            }
            stamp(p, l, 12);
        }
        // wind down: every copy issued is complete before the CTA may exit (bounded)
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
    const IqTab itab = make_tab(tab, lane);
    uint32_t seq = 0;               // the ring sequence number of the next unit, identical in every consumer
    int claim_base = 0;
    unsigned target = 0;
    const int T = p.T, H = p.H, F = p.F, E = p.E, K = p.K;
    const XqView xv{xq_codes, xq_d, H};

    auto claim = [&](int n, int& k) -> bool {   // this warp's next unit of the phase, or false
        int v = 0;
        if (lane == 0) v = atomicAdd(&S.claim, 1);
        v = __shfl_sync(0xffffffffu, v, 0);
        k = v - claim_base;
        return k < n;
    };
    auto wait_full = [&](uint32_t s) -> bool {
        const uint32_t slot = s % kSlots, par = (s / kSlots) & 1u;
        if (mbar_try_wait(&S.full[slot], par)) return true;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(&S.full[slot], par)) {
            if (globaltimer() - t0 > kWaitNs || S.abort) {
                report_error(p.err, 0x330u);
                S.abort = 1;
                return false;
            }
        }
        return true;
    };
    auto release = [&](uint32_t s) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s % kSlots]);
    };
    auto end_phase = [&](int n) {   // every consumer warp overshoots its claims once
        claim_base += n + kDecConsumers;
        seq += (uint32_t) n;
    };

    const int Cg = H / 256 * 8;          // IQ3_XXS calls per gate/up row (64 at H = 2048)
    const int Cs = H / 32 * 4;           // Q8_0 calls per shared gate/up row
    const int Csd = p.FS / 32 * 4;       // Q8_0 calls per shared down row
    const int Cd = F / 256 * 8;          // IQ3_XXS calls per routed down row (16 at F = 512)

    for (int l = 0; l < p.n_layers; ++l) {
        if (threadIdx.x == 0) stamp(p, l, 0);
        // ---------------------------------------------------------------- P0: rms and q8_1 of every token
        for (int t = 0; t < T; ++t) {
            const float* xr = p.x + (size_t) t * H;
            if (threadIdx.x < 256) {
                float s = 0.0f;
                for (int i = threadIdx.x; i < H; i += 256) {
                    const float v = __ldcg(xr + i);
                    s += v * v;
                }
                S.red[threadIdx.x] = s;
            }
            named_sync(1, kDecCThreads);
            for (int o = 128; o > 0; o >>= 1) {
                if ((int) threadIdx.x < o) S.red[threadIdx.x] += S.red[threadIdx.x + o];
                named_sync(1, kDecCThreads);
            }
            if (threadIdx.x == 0) S.rms[t] = rsqrtf(fdiv_fm(S.red[0], (float) H) + p.eps);
            named_sync(1, kDecCThreads);
            const float r = S.rms[t];
            for (int b = warp; b < H / 32; b += kDecConsumers) {
                const float hv = __fmul_rn(__ldcg(xr + 32 * b + lane), r);
                float d, sum;
                const int8_t q = q8_1_warp(hv, d, sum);
                xq_codes[(size_t) t * H + 32 * b + lane] = q;
                if (lane == 0) xq_d[t * (H / 32) + b] = __half2float(__float2half(q8_finite(d)));
            }
            named_sync(1, kDecCThreads);
        }

        if (threadIdx.x == 0) stamp(p, l, 1);
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
                        for (int i = lane; i < H / 8; i += 32) {
                            const float4 w = wr[i];
                            const float4 xv4 = __ldcg((const float4*) xr + i);
                            acc += w.x * __fmul_rn(xv4.x, r) + w.y * __fmul_rn(xv4.y, r) + w.z * __fmul_rn(xv4.z, r) +
                                   w.w * __fmul_rn(xv4.w, r);
                        }
                        acc = warp_sum(acc);
                        if (lane == 0) p.logits[((size_t) t * (E + 1) + o) * 2 + half] = acc;
                    }
                } else {
                    const int r = u - 2 * (E + 1);
                    const uint8_t* gate = buf;
                    const uint8_t* up = buf + p.sgu_row;
                    for (int t = 0; t < T; ++t) {
                        typename Fmt<T_Q8_0>::Act a[1][8];
                        auto src = [&](int blk) { return xv.block(t, blk); };
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (lane + 32 * j < Cs) a[0][j] = Fmt<T_Q8_0>::act(src, lane + 32 * j);
                        float sg[1], su[1];
                        row_dot<T_Q8_0, 8, 1>(gate, Cs, lane, a, 1, itab, sg);
                        row_dot<T_Q8_0, 8, 1>(up, Cs, lane, a, 1, itab, su);
                        if (lane == 0) p.hsh[(size_t) t * p.FS + r] = act_value(ACT_SWIGLU, sg[0], su[0], INFINITY);
                    }
                }
                release(s);
            }
            end_phase(mine);
        }
        if (threadIdx.x == 0) stamp(p, l, 2);
        if (!grid_barrier(p, S, target, 0x340u)) break;
        if (threadIdx.x == 0) stamp(p, l, 3);

        // ---------------------------------------------------------------- R: routing and grouping
        for (int t = warp; t < T; t += kDecConsumers) {   // 15 consumer warps: token 15 goes round again
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
            // group g starts at the sorted position of the first entry of its expert
            if (e < n_ent) {
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
                    for (int i = i0; i < i1; ++i) {
                        const int g = i / F, r = i % F;
                        const uint8_t* gate = buf + (size_t) (i - i0) * 2 * p.gu_row;
                        const uint8_t* up = gate + p.gu_row;
                        const int e0 = S.grp_start[g], e1 = S.grp_start[g + 1];
                        for (int eb = e0; eb < e1; eb += 2) {
                            const int nc = min(2, e1 - eb);
                            typename Fmt<T_IQ3_XXS>::Act a[2][2];
#pragma unroll
                            for (int c = 0; c < 2; ++c) {
                                if (c >= nc) break;
                                const int tok = S.ent_tok[eb + c];
                                auto src = [&](int blk) { return xv.block(tok, blk); };
#pragma unroll
                                for (int j = 0; j < 2; ++j)
                                    if (lane + 32 * j < Cg) a[c][j] = Fmt<T_IQ3_XXS>::act(src, lane + 32 * j);
                            }
                            float sg[2], su[2];
                            row_dot<T_IQ3_XXS, 2, 2>(gate, Cg, lane, a, nc, itab, sg);
                            row_dot<T_IQ3_XXS, 2, 2>(up, Cg, lane, a, nc, itab, su);
#pragma unroll
                            for (int c = 0; c < 2; ++c)
                                if (c < nc && lane == c)
                                    p.hbuf[(size_t) S.ent_dst[eb + c] * F + r] = act_value(ACT_SWIGLU, sg[c], su[c], INFINITY);
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
                            const float* hx = p.hsh + (size_t) (t0 + c) * p.FS;
                            auto src = [&](int blk) { return qb_from_f32_cg(hx + 32 * blk); };
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
        {
            const Range ch = my_chunks(p);
            const int ntask = (ch.hi - ch.lo) * ng;
            const int mine = p3_units(p, ng);
            const int P = 32 / Cd;   // rows per pass (Cd = 16 -> 2)
            int k;
            while (claim(mine, k)) {
                const uint32_t s = seq + (uint32_t) k;
                if (!wait_full(s)) break;
                const uint8_t* buf = ring + (size_t) (s % kSlots) * kSlotBytes;
                const int i0 = k * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
                for (int i = i0; i < i1; ++i) {
                    const int cl = i / ng, g = i % ng;   // chunk index within this CTA, group
                    const uint8_t* rows = buf + (size_t) (i - i0) * p.R * p.d_row;
                    const int e0 = S.grp_start[g], e1 = S.grp_start[g + 1];
                    for (int eb = e0; eb < e1; eb += 4) {
                        const int nc = min(4, e1 - eb);
                        typename Fmt<T_IQ3_XXS>::Act a[4][1];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            if (c >= nc) break;
                            const float* hx = p.hbuf + (size_t) S.ent_dst[eb + c] * F;
                            auto src = [&](int blk) { return qb_from_f32_cg(hx + 32 * blk); };
                            a[c][0] = Fmt<T_IQ3_XXS>::act(src, lane % Cd);
                        }
                        for (int rr = 0; rr < p.R; rr += P) {
                            float sv[4];
                            row_dot_packed<T_IQ3_XXS, 4>(rows + (size_t) rr * p.d_row, p.d_row, Cd, lane, a, nc, itab, sv);
                            const int rl = lane / Cd, cl2 = lane % Cd;
#pragma unroll
                            for (int c = 0; c < 4; ++c)
                                if (c < nc && cl2 == c)
                                    parts[S.ent_dst[eb + c] * kDecMaxRows + cl * p.R + rr + rl] = sv[c];
                        }
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
