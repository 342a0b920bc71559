// tsb_decode.cuh - the whole decode MoE block of every layer of a step in ONE persistent kernel.
//
// Per layer (the reference's call stack A, src/qwen35/q36_engine.cu:2821-2925, with k_moe_out_small's epilogue):
//   P0  every CTA: x (the previous layer's rows from every CTA), h = rms(x) (the 256-slot order of
//       q36_kernels.cuh:252-290) and its q8_1 image in shared memory
//   P1  router logits (fp32 rows, the shared-gate row appended) and the shared expert's gate/up + SwiGLU
//   R   every CTA: softmax top-k of every token (native_router.cu:44-95) once the logits of every CTA are in, the
//       grouping (q36_engine.cu:396-422), then the shared hidden vector into q8_1
//   P2  routed experts' gate/up + SwiGLU (IQ3_XXS), the shared expert's down rows (Q8_0)
//   P3  the routed hidden vectors of every CTA into q8_1, routed down rows of this CTA's row chunks for every group,
//       then the combine of those rows: x += sum_k w_k part_k (fma in pick order) + sigmoid(gate) shared
//
// No grid-wide barrier: every value one CTA hands to others (logits, hidden vectors, shared output, x) travels as a
// tagged 8-byte word (value, layer + 1) and the readers poll the words they need until the tags are the layer's, so a
// phase waits one L2 round trip for its slowest input instead of a barrier's arrive + release.  The dependencies order
// the reuse of every buffer: a CTA overwrites a word of layer l only after reading inputs that every CTA produced after
// it had read that word (P1 of l + 1 needs every CTA's x of l, which follows their P3 of l; P2 of l + 1 needs every
// CTA's shared hidden of l + 1, which follows their P0 of l + 1; P3 of l + 1 writes x after every CTA's P1 of l + 1).
//
// One CTA per SM (cooperative launch: every CTA resident), 12 warps (three per SM sub-partition: 168 registers a
// thread, no spills).  Every warp streams its own units of weight bytes: unit j of a phase goes to warp j mod 12, and
// lane 0 issues the unit's cp.async.bulk copies into one of the warp's two shared-memory slots, completing on that
// slot's mbarrier, two units ahead of the warp's compute.  The stream runs across phases -- the first routed-down
// rows are in flight while the last gate/up rows compute, the next layer's router and shared-expert rows while this
// layer's down rows compute -- and no warp waits for another to move its data (a single producer warp, tried first,
// was starved of issue slots by the compute warps sharing its sub-partition).  Every wait is bounded (2 s of
// %globaltimer); a wait that gives up records its site in the error word, the other CTAs see the word and the
// kernel winds down.
#pragma once

#include "tsb_kernels.cuh"

#include <cfloat>

namespace tsb {

constexpr int kDecWarps = 12, kDecConsumers = kDecWarps, kDecThreads = kDecWarps * 32, kDecCThreads = kDecThreads;
constexpr uint32_t kSlotBytes = 4352;   // the largest unit: a shared gate/up row pair, 8 shared down rows
constexpr int kLowWarps = 7;            // warps whose two slots sit below the tables (7 x 2 x 4352 bytes)
constexpr int kDecMaxT = 16, kDecMaxEnt = 128, kDecMaxRows = 16;   // rows of H per CTA in P3 (<= 4 chunks of 4)

struct DecLayer {
    const uint8_t* blobs;    // [E][blob_bytes]
    const float* router;     // [E + 1][H]: the expert rows, then the shared-gate row
    const uint8_t* sh_blob;  // the shared expert
    const float* prior;      // optional [T][E] added to the router logits before the softmax (null: none)
};

struct DecParams {
    int n_layers, T, H, F, E, K, FS;
    uint32_t gu_row, d_row, sgu_row, sd_row;
    uint64_t up_off, down_off, blob_bytes, s_up_off, s_down_off;
    int R;                    // routed down rows per chunk (R * d_row % 16 == 0)
    int rt_per_unit, sd_per_unit, dn_per_unit;   // items packed per unit (one slot)
    int nslot;                // slots per warp: 2 (prefetch a unit ahead), 1 when shared memory is short (large T)
    const DecLayer* layers;
    float* x;                 // [T][H] residual stream, in / out
    // tagged words (value, layer + 1), zero at launch
    uint64_t* logits;         // [T][E + 1][2]: the two half-row partial dots
    uint64_t* hsh;            // [T][FS] shared hidden
    uint64_t* hbuf;           // [T * K][F] routed hidden, by entry
    uint64_t* sh_out;         // [T][H] shared expert output
    uint64_t* xt;             // [T][H] the residual stream after each layer
    int32_t* ids_rec;         // [layers][T][K] or null
    float* w_rec;
    float* x_rec;             // [layers][T][H]: x after each layer, or null
    unsigned* err;
    unsigned long long* trace;   // optional phase stamps: [layer][kTraceEvents][CTA] of %globaltimer, or null
    int dbg_withhold;         // tests of the bounded waits: CTA dbg_withhold - 1 never publishes its layer-0 logits
    float eps;
    uint32_t smem_base;       // the shared-window address the dynamic shared memory starts at (checked)
};
constexpr int kTraceEvents = 16;

struct DecShared {
    uint64_t bar[kDecWarps][2];   // per warp and slot: the bulk copies of the unit in the slot have landed
    volatile int abort;
    unsigned canary;
    int n_groups;
    float rms[kDecMaxT];
    float gs[kDecMaxT];
    int32_t ids[kDecMaxEnt];
    float w[kDecMaxEnt];
    int32_t grp_expert[kDecMaxEnt], grp_start[kDecMaxEnt + 1], ent_dst[kDecMaxEnt], ent_tok[kDecMaxEnt];
    float red[256];
    float xown[kDecMaxT][kDecMaxRows];   // this CTA's rows of x (it is their only writer)
};

// Offsets inside the dynamic shared memory (dynamic base at shared address b0 <= 0x10000 - 14 * kSlotBytes):
//   [0, 14 * kSlotBytes)                  warps 0..6's two slots each (nslot 2), or every warp's one slot (nslot 1)
//   [0x10000 - b0, +64 KB)                the IQ3_XXS tables at shared address 0x10000
//   [0x20000 - b0, ...)                   DecShared, parts [kDecMaxEnt][kDecMaxRows], then the activation union:
//       P0..P2: xq codes [T][H], xq scales [T][H / 32], hshq codes [T][FS], hshq scales [T][FS / 32]
//       P3:     hq codes [T K][F], hq scales [T K][F / 32]
//   then (nslot 2) warps 7..11's two slots each
struct DecSmem {
    uint32_t tab, shared, parts, uni, xq_d, hs, hs_d, hq_d, slots_hi, total;
};
__host__ __device__ inline DecSmem dec_smem(uint32_t b0, int T, int H, int F, int FS, int K, int nslot) {
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
    m.slots_hi = al(end1 > end2 ? end1 : end2, 128);
    m.total = m.slots_hi + (nslot == 2 ? (uint32_t) (kDecWarps - kLowWarps) * 2 * kSlotBytes : 0u);
    return m;
}
// The shared-memory offset of slot s of warp w.
__device__ __forceinline__ uint32_t slot_offset(const DecSmem& m, int nslot, int w, int s) {
    if (nslot == 1) return (uint32_t) w * kSlotBytes;
    return w < kLowWarps ? (uint32_t) (2 * w + s) * kSlotBytes : m.slots_hi + (uint32_t) (2 * (w - kLowWarps) + s) * kSlotBytes;
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
// Phase stamps of thread 0: 0 layer start, 1 P0, 2 P1, 3 routed, 4 shared hidden quantised, 5 P2, 6 routed hidden
// quantised, 7 P3 + combine, 8 layer end.
__device__ __forceinline__ void stamp(const DecParams& p, int l, int ev) {
    if (p.trace) p.trace[((size_t) l * kTraceEvents + ev) * gridDim.x + blockIdx.x] = globaltimer();
    if (ev < 9) ((volatile unsigned*) p.err)[128 + blockIdx.x] = ((unsigned) l << 8) | (unsigned) ev;
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// A named barrier that also ORs one flag over its threads: every thread gets the same verdict, whatever another thread
// writes to the flag's source after the barrier -- the warps leave the layer loop together.
__device__ __forceinline__ bool named_sync_or(int id, int n, int flag) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(flag), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One pass of a poll found a word not yet written: poll again (no sleep: __nanosleep measured here oversleeps by
// microseconds, and a pass is an L2 round trip already), or give up after the bound or when another CTA has recorded
// an error (then this CTA winds down too).  Returns true when the caller must stop waiting.
__device__ __forceinline__ bool poll_give_up(const DecParams& p, DecShared& S, uint64_t t0, unsigned site) {
    if (S.abort || *(volatile unsigned*) p.err != 0u || globaltimer() - t0 > wait_limit_ns()) {
        report_error(p.err, site);
        S.abort = 1;
        return true;
    }
    return false;
}

// n tagged words (n even, 16-byte aligned) into floats in shared memory once all carry `tag`; threads tid of nth,
// up to 8 words of a thread in flight per pass.  false: gave up (S.abort set).
__device__ bool poll_copy(const DecParams& p, DecShared& S, const uint64_t* src, int n, uint32_t tag, float* dst,
                          int tid, int nth, unsigned site) {
    const int np = n / 2;
    for (int base = tid; base < np; base += 4 * nth) {
        const uint64_t t0 = globaltimer();
        for (;;) {
            uint64_t w[8];
            bool ok = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = base + j * nth;
                if (i < np) {
                    ld_tag2(src + 2 * i, w[2 * j], w[2 * j + 1]);
                    ok &= tag_is(w[2 * j], tag) & tag_is(w[2 * j + 1], tag);
                }
            }
            if (ok) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int i = base + j * nth;
                    if (i < np) {
                        dst[2 * i] = tag_val(w[2 * j]);
                        dst[2 * i + 1] = tag_val(w[2 * j + 1]);
                    }
                }
                break;
            }
            if (poll_give_up(p, S, t0, site)) return false;
        }
    }
    return true;
}

// -------------------------------------------------------------------------------------------------- unit lists
// P1: 2 (E + 1) router half rows, then FS shared gate/up pairs.  P2: routed gate/up pairs packed rt_per_unit to a
// slot, then shared down rows packed sd_per_unit.  P3: this CTA's (chunk, group) tasks packed dn_per_unit.
struct Range {
    int lo, hi;
};
// 32-bit products (n * parts < 2^32 for every split here: at most 2^16 units over the SMs).
__device__ __forceinline__ Range split(int n, int parts, int i) {
    return {(int) ((uint32_t) n * (uint32_t) i / (uint32_t) parts), (int) ((uint32_t) n * (uint32_t) (i + 1) / (uint32_t) parts)};
}

__device__ __forceinline__ int p1_units(const DecParams& p) { return 2 * (p.E + 1) + p.FS; }
__device__ __forceinline__ int p2_rt_units(const DecParams& p, int ng) { return (ng * p.F + p.rt_per_unit - 1) / p.rt_per_unit; }
__device__ __forceinline__ int p2_units(const DecParams& p, int ng) { return p2_rt_units(p, ng) + p.H / p.sd_per_unit; }
__device__ __forceinline__ Range my_chunks(const DecParams& p) { return split(p.H / p.R, gridDim.x, blockIdx.x); }
// Units [0, n) are dealt to the warps round robin: how many warp w gets.
__device__ __forceinline__ int per_warp(int n, int w) { return n > w ? (n - w + kDecWarps - 1) / kDecWarps : 0; }
__device__ __forceinline__ int p3_units(const DecParams& p, int ng) {
    const Range c = my_chunks(p);
    return ((c.hi - c.lo) * ng + p.dn_per_unit - 1) / p.dn_per_unit;
}

// -------------------------------------------------------------------------------------------------- unit copies
struct BulkCopy {
    const void* src;
    uint32_t dst;     // offset in the slot
    uint32_t bytes;
};
// P1 unit u: a router half row (one copy) or a shared gate/up row pair (two).
__device__ __forceinline__ int p1_copies(const DecParams& p, const DecLayer& L, int u, BulkCopy (&c)[2]) {
    const int nrh = 2 * (p.E + 1);
    if (u < nrh) {
        const int o = u >> 1, half = u & 1;
        c[0] = {L.router + (size_t) o * p.H + half * (p.H / 2), 0u, (uint32_t) (p.H / 2 * 4)};
        return 1;
    }
    const size_t off = (size_t) (u - nrh) * p.sgu_row;
    c[0] = {L.sh_blob + off, 0u, p.sgu_row};
    c[1] = {L.sh_blob + off + p.s_up_off, p.sgu_row, p.sgu_row};
    return 2;
}
// P2 unit u: rt_per_unit routed gate rows then the same up rows (two copies, one expert), or sd_per_unit shared down rows.
__device__ __forceinline__ int p2_copies(const DecParams& p, const DecLayer& L, const DecShared& S, int ng, int u,
                                         BulkCopy (&c)[2]) {
    const int nrt = p2_rt_units(p, ng);
    if (u < nrt) {
        const int i0 = u * p.rt_per_unit, n = min(p.rt_per_unit, ng * p.F - i0);
        const int g = i0 / p.F, r = i0 % p.F;
        const uint8_t* b = L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + (size_t) r * p.gu_row;
        c[0] = {b, 0u, (uint32_t) n * p.gu_row};
        c[1] = {b + p.up_off, (uint32_t) n * p.gu_row, (uint32_t) n * p.gu_row};
        return 2;
    }
    const int r0 = (u - nrt) * p.sd_per_unit;
    c[0] = {L.sh_blob + p.s_down_off + (size_t) r0 * p.sd_row, 0u, (uint32_t) p.sd_per_unit * p.sd_row};
    return 1;
}
// P3 unit k: this CTA's tasks [k dn, (k + 1) dn) (task i = chunk i % nch of group i / nch): one copy per group touched.
__device__ __forceinline__ int p3_copies(const DecParams& p, const DecLayer& L, const DecShared& S, int ng, Range ch,
                                         int k, BulkCopy (&c)[2]) {
    const int nch = ch.hi - ch.lo, ntask = nch * ng;
    const uint32_t cb = (uint32_t) p.R * p.d_row;
    const int i0 = k * p.dn_per_unit, i1 = min(i0 + p.dn_per_unit, ntask);
    int n = 0;
    for (int g = i0 / nch; g <= (i1 - 1) / nch && n < 2; ++g) {
        const int a0 = max(i0, g * nch), a1 = min(i1, (g + 1) * nch);
        c[n++] = {L.blobs + (size_t) S.grp_expert[g] * p.blob_bytes + p.down_off + (size_t) (ch.lo + a0 - g * nch) * cb,
                  (uint32_t) (a0 - i0) * cb, (uint32_t) (a1 - a0) * cb};
    }
    return n;
}

// One warp's stream of units through its slots: issue (lane 0: expect the unit's bytes on the slot's barrier, then
// its bulk copies), wait (every lane observes the slot's phase), release.  Units are consumed in the order issued.
struct WarpStream {
    uint32_t slot[2];   // shared addresses
    uint64_t* bar;      // the warp's two barriers
    uint32_t issued = 0, consumed = 0;
    int nslot;
    __device__ bool can_issue() const { return issued - consumed < (uint32_t) nslot; }
    __device__ void issue(const BulkCopy (&c)[2], int n, int lane) {
        const uint32_t k = issued % (uint32_t) nslot;
        if (lane == 0) {
            uint32_t bytes = 0;
            for (int i = 0; i < n; ++i) bytes += c[i].bytes;
            mbar_expect_tx(&bar[k], bytes);
            for (int i = 0; i < n; ++i)
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                 slot[k] + c[i].dst),
                             "l"(c[i].src), "r"(c[i].bytes), "r"(smem_u32(&bar[k]))
                             : "memory");
        }
        ++issued;
    }
    // The next unit's bytes (generic pointer into the dynamic shared memory at smem_ptr / smem_base), or null when the
    // wait gave up.
    __device__ const uint8_t* wait(uint8_t* smem_ptr, uint32_t smem_base) {
        const uint32_t k = consumed % (uint32_t) nslot, par = (consumed / (uint32_t) nslot) & 1u;
        bool done = mbar_try_wait(&bar[k], par);
        const uint64_t t0 = done ? 0 : globaltimer();
        while (!done) {
            done = mbar_try_wait(&bar[k], par);
            if (!done && globaltimer() - t0 > wait_limit_ns()) break;
        }
        if (!__all_sync(0xffffffffu, done)) return nullptr;
        return smem_ptr + (slot[k] - smem_base);
    }
    // The warp has read the slot: order those reads before the next bulk copy into it (async proxy).
    __device__ void release() {
        fence_proxy_async();
        __syncwarp();
        ++consumed;
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

// quantize_blocks over tagged words written by other CTAs of this launch: each pass loads a lane's 2 x 4 words and
// polls until their tags are `tag` (the lanes of a block rejoin before its shuffles).  false: gave up (S.abort set).
__device__ bool quantize_tagged(const DecParams& p, DecShared& S, const uint64_t* src, int n, uint32_t tag,
                                int8_t* codes, float* dsc, int warp, int lane, int nwarps, unsigned site) {
    const int n4 = n / 4;
    const int stride = nwarps * 32;
    bool good = true;
    for (int base = warp * 32 + lane; base - lane < n4; base += 2 * stride) {
        float4 v[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
        const uint64_t t0 = globaltimer();
        while (good) {
            uint64_t w[8];
            bool ok = true;
#pragma unroll
            for (int it = 0; it < 2; ++it) {
                const int i = base + it * stride;
                if (i < n4) {
                    ld_tag2(src + 4 * i, w[4 * it], w[4 * it + 1]);
                    ld_tag2(src + 4 * i + 2, w[4 * it + 2], w[4 * it + 3]);
                    ok &= tag_is(w[4 * it], tag) & tag_is(w[4 * it + 1], tag) & tag_is(w[4 * it + 2], tag) &
                          tag_is(w[4 * it + 3], tag);
                }
            }
            if (ok) {
#pragma unroll
                for (int it = 0; it < 2; ++it)
                    v[it] = make_float4(tag_val(w[4 * it]), tag_val(w[4 * it + 1]), tag_val(w[4 * it + 2]),
                                        tag_val(w[4 * it + 3]));
                break;
            }
            if (poll_give_up(p, S, t0, site)) good = false;
        }
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int i = base + it * stride;
            if (i - lane >= n4) break;   // warp-uniform: whole warps of 4-value groups
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
            if (i < n4) {
                ((uint32_t*) codes)[i] = word;
                if ((lane & 7) == 0) dsc[i >> 3] = __half2float(__float2half(d));
            }
        }
    }
    return good;
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
    DecShared& S = *(DecShared*) (smem + (0x20000u - p.smem_base));
    const DecSmem M = dec_smem(p.smem_base, p.T, p.H, p.F, p.FS, p.K, p.nslot);
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
        for (int w = 0; w < kDecWarps; ++w) {
            mbar_init(&S.bar[w][0], 1);
            mbar_init(&S.bar[w][1], 1);
        }
        S.abort = 0;
        S.canary = 0xC0FFEE01u;
        if (blockIdx.x == 0 && p.err) {   // the layout as the device sees it
            p.err[110] = smem_u32(smem);
            p.err[111] = M.tab;
            p.err[112] = smem_u32(&S);
            p.err[113] = M.parts;
            p.err[114] = M.uni;
            p.err[115] = M.total;
        }
        fence_mbar_init();
    }
    fill_tables<T_IQ3_XXS>(smem + (0x10000u - p.smem_base), kDecThreads);
    __syncthreads();
    if (threadIdx.x == 0 && S.canary != 0xC0FFEE01u) {
        report_error(p.err, 0x3F0u);
        if (p.err) p.err[116] = S.canary;
    }
    const IqTab itab = make_tab(smem + M.tab, lane);
    const AbsTab atab = make_abs_tab(lane);
    const int T = p.T, H = p.H, F = p.F, E = p.E, K = p.K;
    const XqView xv{xq_codes, xq_d, H};
    const XqView hsv{hs_codes, hs_d, p.FS};
    const XqView hqv{hq_codes, hq_d, F};
    const int Cs = H / 32 * 4;           // Q8_0 calls per shared gate/up row
    const int Csd = p.FS / 32 * 4;       // Q8_0 calls per shared down row

    WarpStream st;
    st.nslot = p.nslot;
    st.bar = S.bar[warp];
    st.slot[0] = p.smem_base + slot_offset(M, p.nslot, warp, 0);
    st.slot[1] = p.smem_base + slot_offset(M, p.nslot, warp, 1);
    auto fail = [&](unsigned site, int l) {   // a wait gave up
        report_detail(p.err, site, (unsigned) warp | ((unsigned) l << 8), st.issued, st.consumed, blockIdx.x);
        S.abort = 1;
    };

    // P1 units: the same ones every layer, dealt to the CTAs round robin (unit u to CTA u % grid: the router half rows
    // and the T-times heavier shared gate/up pairs mix on every CTA); this warp's j-th is p1_unit(j)
    const int n1 = p1_units(p);
    const int n1c = (int) blockIdx.x < n1 ? (n1 - (int) blockIdx.x + (int) gridDim.x - 1) / (int) gridDim.x : 0;
    const int n1w = per_warp(n1c, warp);
    auto p1_unit = [&](int j) { return (int) blockIdx.x + (int) gridDim.x * (warp + j * kDecWarps); };
    int pre1 = 0;   // P1 units of the coming layer already issued
    {
        const DecLayer L0 = p.layers[0];
        while (pre1 < n1w && st.can_issue()) {
            BulkCopy c[2];
            const int n = p1_copies(p, L0, p1_unit(pre1), c);
            st.issue(c, n, lane);
            ++pre1;
        }
    }

    for (int l = 0; l < p.n_layers; ++l) {
        if (threadIdx.x == 0) stamp(p, l, 0);
        const DecLayer L = p.layers[l];
        const uint32_t tag = (uint32_t) l + 1u;   // what this layer writes
        // ---------------------------------------------------------------- P0: rms and q8_1 of every token
        // The reference's order (k_moe_out_small): 256 slots s = sum over i = s mod 256 of x_i^2 in order, then the
        // halving tree; thread i < 32 forms the tree's 32-slot level from 8 slots, shuffles finish it.
        float* xs = parts;   // the token's row in shared memory (the parts buffer is free until P3)
        const Range own = my_chunks(p);
        const int nown = (own.hi - own.lo) * p.R, own0 = own.lo * p.R;
        for (int t = 0; t < T; ++t) {
            if (l == 0) {   // the caller's x
                const float* xr = p.x + (size_t) t * H;
                for (int i = threadIdx.x; i < H / 4; i += kDecCThreads) ((float4*) xs)[i] = __ldcg((const float4*) xr + i);
            } else {        // every CTA's rows of the previous layer
                poll_copy(p, S, p.xt + (size_t) t * H, H, tag - 1u, xs, threadIdx.x, kDecCThreads, 0x340u);
            }
            named_sync(1, kDecCThreads);
            if (threadIdx.x < nown) S.xown[t][threadIdx.x] = xs[own0 + threadIdx.x];
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
        if (named_sync_or(1, kDecCThreads, S.abort)) break;
        if (threadIdx.x == 0) stamp(p, l, 1);

        // ---------------------------------------------------------------- P1: router rows, shared gate/up
        {
            const float* xs = parts;   // h of the token (T = 1), left by P0
            int next1 = pre1;
            for (int j = 0; j < n1w; ++j) {
                const uint8_t* buf = st.wait(smem, p.smem_base);
                if (!buf) {
                    fail(0x331u, l);
                    break;
                }
                const int u = p1_unit(j);
                if (u < 2 * (E + 1)) {
                    const int o = u >> 1, half = u & 1;
                    const float4* wr = (const float4*) buf;
                    for (int t = 0; t < T; ++t) {
                        const float* xr = p.x + (size_t) t * H + half * (H / 2);
                        const uint64_t* xw = p.xt + (size_t) t * H + half * (H / 2);
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
                                float4 xv4;
                                if (l == 0) {
                                    xv4 = __ldcg((const float4*) xr + i);
                                } else {   // the words P0 polled: their tags are this layer's input already
                                    uint64_t a, b, c, d;
                                    ld_tag2(xw + 4 * i, a, b);
                                    ld_tag2(xw + 4 * i + 2, c, d);
                                    xv4 = make_float4(tag_val(a), tag_val(b), tag_val(c), tag_val(d));
                                }
                                acc += w.x * __fmul_rn(xv4.x, r) + w.y * __fmul_rn(xv4.y, r) + w.z * __fmul_rn(xv4.z, r) +
                                       w.w * __fmul_rn(xv4.w, r);
                            }
                        }
                        acc = warp_sum(acc);
                        const bool withheld = l == 0 && p.dbg_withhold == (int) blockIdx.x + 1;
                        if (lane == 0 && !withheld) st_tag(p.logits + ((size_t) t * (E + 1) + o) * 2 + half, acc, tag);
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
                        if (lane == 0) st_tag(p.hsh + (size_t) t * p.FS + r, act_value(ACT_SWIGLU, sg, su, INFINITY), tag);
                    }
                }
                st.release();
                if (next1 < n1w) {
                    BulkCopy c[2];
                    const int n = p1_copies(p, L, p1_unit(next1), c);
                    st.issue(c, n, lane);
                    ++next1;
                }
            }
        }
        if (threadIdx.x == 0) stamp(p, l, 2);

        // ---------------------------------------------------------------- R: routing, grouping; shared hidden -> q8_1
        // Warps [0, gw) route (once every CTA's logits of the token are in) and group while the other warps wait.
        const int gw = T <= 4 ? 4 : kDecConsumers;
        if (warp < gw) {
            for (int t = warp; t < T; t += gw) {
                const uint64_t* lg = p.logits + (size_t) t * (E + 1) * 2;
                float values[V];
                float gate_logit = 0.0f;
                const uint64_t t0 = globaltimer();
                for (;;) {
                    bool ok = true;
#pragma unroll
                    for (int i = 0; i < V; ++i) {
                        uint64_t a, b;
                        ld_tag2(lg + 2 * (lane + i * 32), a, b);
                        values[i] = tag_val(a) + tag_val(b);
                        ok &= tag_is(a, tag) & tag_is(b, tag);
                    }
                    if (L.prior) {
#pragma unroll
                        for (int i = 0; i < V; ++i) values[i] += __ldg(L.prior + (size_t) t * E + lane + i * 32);
                    }
                    if (lane == 0) {
                        uint64_t a, b;
                        ld_tag2(lg + 2 * E, a, b);
                        gate_logit = tag_val(a) + tag_val(b);
                        ok &= tag_is(a, tag) & tag_is(b, tag);
                    }
                    if (ok || poll_give_up(p, S, t0, 0x345u)) break;
                }
                if (threadIdx.x == 0) stamp(p, l, 9);
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
                // Top-k as the reference's argmax rounds (largest value, then lowest expert id), on order-preserving
                // integer keys: a lane's best key, one warp max reduction, then one min reduction over the ids that hold it.
                uint32_t key[V];
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    const uint32_t b = __float_as_uint(values[i]);
                    key[i] = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
                }
                float selected = 0.0f, selected_sum = 0.0f;
                uint32_t taken = 0;   // this lane's keys already picked: 0, below every value (the reference's -inf)
                for (int rank = 0; rank < K; ++rank) {
                    uint32_t kb = (taken & 1u) ? 0u : key[0];
                    int ib = 0;
#pragma unroll
                    for (int i = 1; i < V; ++i) {
                        const uint32_t ki = (taken >> i & 1u) ? 0u : key[i];
                        if (ki > kb) {
                            kb = ki;
                            ib = i;
                        }
                    }
                    const uint32_t kmax = __reduce_max_sync(0xffffffffu, kb);
                    const int expert = (int) __reduce_min_sync(0xffffffffu, kb == kmax ? (uint32_t) (lane + 32 * ib) : 0xffffffffu);
                    const float best = __uint_as_float((kmax & 0x80000000u) ? (kmax & 0x7fffffffu) : ~kmax);
                    if ((expert & 31) == lane) {
                        taken |= 1u << (expert / 32);
                        S.ids[t * K + rank] = expert;
                        selected_sum += best;
                    }
                    if (rank == lane) selected = best;
                }
                selected_sum = fmaxf(warp_sum(selected_sum), 6.103515625e-5f);
                const float inv = frcp_fm(selected_sum);
                if (lane < K) S.w[t * K + lane] = selected * inv;
                if (lane == 0) S.gs[t] = frcp_fm(1.0f + fexp_fm(-gate_logit));
            }
            if (threadIdx.x == 0) stamp(p, l, 10);
            named_sync(2, gw * 32);
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
            named_sync(2, gw * 32);
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
            named_sync(2, gw * 32);
            if (threadIdx.x == 0) stamp(p, l, 3);
        }
        if (named_sync_or(1, kDecCThreads, S.abort)) break;
        const int ng = S.n_groups;

        // This warp's units after the routing, in stream order: its P2 units, its P3 units, the next layer's P1 units.
        // P2 units are dealt to the CTAs round robin (unit u to CTA u % grid): the shared down units, which sit after
        // the routed ones and cost T times a routed unit, spread over every CTA instead of landing on the last few
        const int n2 = p2_units(p, ng), nrt = p2_rt_units(p, ng);
        const int n2c = (int) blockIdx.x < n2 ? (n2 - (int) blockIdx.x + (int) gridDim.x - 1) / (int) gridDim.x : 0;
        const int n2w = per_warp(n2c, warp);
        auto p2_unit = [&](int j) { return (int) blockIdx.x + (int) gridDim.x * (warp + j * kDecWarps); };
        const Range ch = my_chunks(p);
        const int nch = ch.hi - ch.lo, ntask = nch * ng;
        const int n3w = per_warp(p3_units(p, ng), warp);
        const bool more = l + 1 < p.n_layers;
        const DecLayer Ln = more ? p.layers[l + 1] : L;
        const int npost = n2w + n3w + (more ? n1w : 0);
        int post = 0;
        auto issue_post = [&]() {
            BulkCopy c[2];
            int n;
            if (post < n2w)
                n = p2_copies(p, L, S, ng, p2_unit(post), c);
            else if (post < n2w + n3w)
                n = p3_copies(p, L, S, ng, ch, warp + (post - n2w) * kDecWarps, c);
            else
                n = p1_copies(p, Ln, p1_unit(post - n2w - n3w), c);
            st.issue(c, n, lane);
            ++post;
        };
        while (post < npost && st.can_issue()) issue_post();
        // the shared hidden vector into q8_1 (every CTA's P1) while this warp's first P2 rows land
        quantize_tagged(p, S, p.hsh, T * p.FS, tag, hs_codes, hs_d, warp, lane, kDecConsumers, 0x348u);
        if (named_sync_or(1, kDecCThreads, S.abort)) break;
        if (threadIdx.x == 0) stamp(p, l, 4);

        // ---------------------------------------------------------------- P2: routed gate/up, shared down
        for (int j = 0; j < n2w; ++j) {
            const uint8_t* buf = st.wait(smem, p.smem_base);
            if (!buf) {
                fail(0x332u, l);
                break;
            }
            const int u = p2_unit(j);
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
                        if (lane == 16)
                            st_tag(p.hbuf + (size_t) S.ent_dst[eb] * F + r, act_value(ACT_SWIGLU, sg, su, INFINITY), tag);
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
                        if (lane < nc) st_tag(p.sh_out + (size_t) (t0 + lane) * H + r0 + rr, lane == 0 ? sv[0] : sv[1], tag);
                    }
                }
            }
            st.release();
            if (post < npost) issue_post();
        }
        if (threadIdx.x == 0) stamp(p, l, 5);

        // ---------------------------------------------------------------- P3: routed down rows, combine
        {
            named_sync(1, kDecCThreads);   // P2's activations (the union P3's codes overwrite) are no longer read
            quantize_tagged(p, S, p.hbuf, T * K * F, tag, hq_codes, hq_d, warp, lane, kDecConsumers, 0x350u);
            if (named_sync_or(1, kDecCThreads, S.abort)) break;
            if (threadIdx.x == 0) stamp(p, l, 6);
            for (int j = 0; j < n3w; ++j) {
                const uint8_t* buf = st.wait(smem, p.smem_base);
                if (!buf) {
                    fail(0x333u, l);
                    break;
                }
                const int k = warp + j * kDecWarps;
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
                st.release();
                if (post < npost) issue_post();
            }
            named_sync(1, kDecCThreads);
            // combine this CTA's rows for every token
            const int nrows = (ch.hi - ch.lo) * p.R;
            for (int i = threadIdx.x; i < T * nrows; i += kDecCThreads) {
                const int t = i / nrows, lr = i % nrows;
                const int row = ch.lo * p.R + lr;
                const float* wr = S.w + t * K;
                float acc = wr[0] * parts[(t * K) * kDecMaxRows + lr];
                for (int kk = 1; kk < K; ++kk) acc = fmaf(wr[kk], parts[(t * K + kk) * kDecMaxRows + lr], acc);
                const uint64_t* so = p.sh_out + (size_t) t * H + row;
                uint64_t w = ld_tag(so);
                const uint64_t t0 = globaltimer();
                while (!tag_is(w, tag) && !poll_give_up(p, S, t0, 0x360u)) w = ld_tag(so);
                acc += S.gs[t] * tag_val(w);
                const float xn = S.xown[t][lr] + acc;
                p.x[(size_t) t * H + row] = xn;
                if (p.x_rec) p.x_rec[((size_t) l * T + t) * H + row] = xn;
                st_tag(p.xt + (size_t) t * H + row, xn, tag);
            }
        }
        pre1 = post > n2w + n3w ? post - n2w - n3w : 0;
        if (threadIdx.x == 0) stamp(p, l, 7);
        if (named_sync_or(1, kDecCThreads, S.abort)) break;   // (the next layer's P0 reuses the parts buffer)
        if (threadIdx.x == 0) stamp(p, l, 8);
    }
    // wind down: every copy this warp issued has landed before the CTA may exit (bounded)
    while (st.consumed < st.issued) {
        if (!st.wait(smem, p.smem_base)) break;
        st.release();
    }
}

}  // namespace tsb
