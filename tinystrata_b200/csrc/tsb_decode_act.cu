// tsb_decode_act.cu - the Gemma 4 / LFM2 decode MoE layer in one cooperative launch.
//
// The reference runs the decode MoE block of these engines as a chain of launches (src/gemma4/engine.cpp:2436-2457:
// route_rows, the experts' gate/up gemma_native_mmvq_ids, geglu_rows / swiglu_clamp_rows, the hidden rows' q8_1,
// the down gemma_native_mmvq_ids, moe_sum; the dense shared MLP beside it).  Here one persistent CTA per SM runs the
// whole block in three phases, separated by grid barriers (bounded waits):
//   A  the router logits (the fp32 GEMV, one warp per expert row) and the shared MLP's gate/up rows -> its hidden
//      vectors;
//   B  every CTA routes every token itself (the route_kernel arithmetic) and groups the entries by expert (k_group's
//      order); the routed experts' gate/up rows -> hidden vectors;
//   C  the hidden vectors (routed and shared) are quantised to q8_1 once over the grid (a third barrier) and copied
//      into every CTA's shared memory; a warp takes rows of the down matrices of every used expert and sums its picks'
//      weighted rows in pick order (moe_sum) straight into the output, or rows of the shared MLP's down matrix.
// Weight rows are read in place from HBM by the warps (no staging): each lane's calls of a row are independent loads.
// Every value is computed by the same device code as the layer-by-layer kernels (row_dot's per-lane order and xor
// tree, act_value, the q8_1 quantiser, route_row_warp, the router GEMV's expression, moe_sum's order), so the outputs
// equal theirs bit for bit.
#include "tsb_kernels.cuh"
#include "../../include/tsb_moe.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace tsb {

void set_last_error(const char* msg);   // tsb_moe.cu: the text tsb_last_error returns
unsigned* device_error_word();          // tsb_moe.cu: the current device's error word (tsb_device_error)

namespace {

constexpr int kAWarps = 8;
constexpr int kAThreads = kAWarps * 32;
constexpr int kAJ = 8;           // calls per lane: rows of up to 256 calls
constexpr int kAJQ4K = 4;        // Q4_K gate/up rows: up to 128 calls (n_embd <= 2048), fewer registers
constexpr int kASR = 2;          // shared down rows per unit
constexpr int kAMaxT = 16;
constexpr int kAMaxEnt = 128;
constexpr int kAMaxE = 512;

int afail(int code, const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    set_last_error(b);
    return code;
}

struct ActParams {
    int T, H, F, E, K, FS;
    const float* router;          // [E][H] fp32
    const float* h;               // [T][H] the router's input
    const BlockQ8_1* hq;          // [T][H / 32] the experts' input
    int gate, norm;
    float in_scale, w_scale, limit;
    const float* bias;
    const float* escale;
    const uint8_t* blobs;
    unsigned long long stride, gu_row, up_off, d_row, down_off;
    const uint8_t* sh;            // null: no shared MLP
    unsigned long long sgu_row, s_up_off, sd_row, s_down_off;
    int act, sh_act, accumulate;
    float* out;                   // [T][H]: (out +) sum_k w_k down_k
    float* sh_out;                // [T][H]: the shared MLP's output
    int32_t* ids;                 // [T][K] (optional)
    float* w;                     // [T][K] (optional)
    float* logits;                // workspace [T][E]
    float* hid;                   // workspace [T * K][F]
    float* shid;                  // workspace [T][FS]
    BlockQ8_1* hqh;               // workspace: q8_1 of the routed hidden rows, then of the shared MLP's
    unsigned* bar;                // workspace: arrival count, generation (zero before the launch)
    unsigned* err;
    unsigned long long blob_bytes, sh_bytes;
    uint32_t sb;                  // bytes of a staging buffer
    int nst;                      // staging buffers per warp (2 .. 4)
    int ar, br;                   // routed down rows per unit (2, 4, 8); routed gate/up rows per unit (1, 2)
};

// Shared memory: the q8_1 hidden rows of phase C (the routed ones, then the shared MLP's), the routing tables, the down
// units' per-warp partial values, nst staging buffers of sb bytes per warp.
struct ActSmem {
    uint32_t q8, ids, w, gexp, gstart, gent, cnt, off, ng, part, stage, total;
};
__host__ __device__ inline ActSmem act_smem(int T, int F, int FS, int K, uint32_t sb, int nst, int ar) {
    auto al = [](uint32_t v) { return (v + 15u) & ~15u; };
    ActSmem m;
    const uint32_t qb = (uint32_t) (T * K * (F / 32) + T * (FS / 32)) * (uint32_t) sizeof(BlockQ8_1);
    uint32_t o = 0;
    m.q8 = o;     o = al(o + qb);
    m.ids = o;    o = al(o + kAMaxEnt * 4);
    m.w = o;      o = al(o + kAMaxEnt * 4);
    m.gexp = o;   o = al(o + kAMaxEnt * 4);
    m.gstart = o; o = al(o + (kAMaxEnt + 1) * 4);
    m.gent = o;   o = al(o + kAMaxEnt * 4);
    m.cnt = o;    o = al(o + kAMaxE * 4);
    m.off = o;    o = al(o + kAMaxE * 4);
    m.ng = o;     o = al(o + 16);
    m.part = o;   o = al(o + kAWarps * kAMaxEnt * ar * 4);
    m.stage = o;  o = al(o + kAWarps * nst * sb);
    m.total = o;
    return m;
}

// A word other CTAs of the launch release (acquire load at gpu scope).
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bring [p, p + n) into L2 (bulk prefetch, 32 KB a request) with the range widened to 16-byte boundaries inside
// [lo, hi): the weights of units a warp computes later, requested while it computes earlier ones.
__device__ __forceinline__ void prefetch_l2(const uint8_t* p, unsigned long long n, const uint8_t* lo, const uint8_t* hi) {
    uintptr_t a = (uintptr_t) p & ~(uintptr_t) 15, b = ((uintptr_t) (p + n) + 15) & ~(uintptr_t) 15;
    if (a < (uintptr_t) lo) a = (uintptr_t) lo;
    if (b > (uintptr_t) hi) b = (uintptr_t) hi;
    for (; a < b; a += 32768) {
        const uint32_t m = (uint32_t) min((uintptr_t) 32768, b - a);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(m) : "memory");
    }
}

// Grid barrier for a cooperative launch: arrival count and generation word.  A wait past the bound records `site` in
// the error word and goes on (the outputs are then invalid, the kernel still ends).
__device__ void grid_barrier(unsigned* bar, unsigned* err, unsigned site) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned g = ld_acquire_u32(bar + 1);
        __threadfence();
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const uint64_t t0 = globaltimer(), lim = wait_limit_ns();
            for (uint32_t i = 1; ld_acquire_u32(bar + 1) == g; ++i)
                if ((i & 255u) == 0 && globaltimer() - t0 > lim) {
                    report_error(err, site);
                    break;
                }
        }
        __threadfence();
    }
    __syncthreads();
}

__device__ __forceinline__ QB qb_from_smem(const BlockQ8_1* b) {
    QB r;
    const int* w = (const int*) b->qs;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = w[i];
    r.d = __low2float(b->ds);
    return r;
}
template <int PER>
__device__ __forceinline__ void route_token(const ActParams& p, int t, int lane, int32_t* ids_s, float* w_s) {
    const float* lg = p.logits + (size_t) t * p.E;
    route_row_warp<PER>([&](int e) { return __ldcg(lg + e); }, p.E, p.K, p.gate, p.in_scale, p.bias, p.escale, p.norm,
                        p.w_scale, lane, ids_s + t * p.K, w_s + t * p.K);
}

// Phase stamps (globaltimer) of every CTA when a trace buffer is set: [CTA][8] = start, phase A done, barrier 1
// passed, routed and grouped, phase B done, barrier 2 passed, hidden rows quantised (over the grid, barrier 3) and in
// shared memory, end.
__device__ unsigned long long* g_act_trace = nullptr;
__device__ __forceinline__ void act_stamp(int ev) {
    unsigned long long* t = g_act_trace;
    if (t && threadIdx.x == 0) t[blockIdx.x * 8 + ev] = globaltimer();
}

// Per-warp staging: an item's weight bytes copied global -> shared by the warp's lanes (cp.async, 16 bytes each, one
// commit group per item) into one of nst stages, so that nst - 1 items are in flight while one computes.  A range is
// widened to 16-byte boundaries inside its blob; the row pointer is the stage plus the skew.
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// at most nst - 1 groups still pending (the oldest item has landed)
__device__ __forceinline__ void cp_wait_ring(int nst) {
    if (nst >= 4) asm volatile("cp.async.wait_group 3;" ::: "memory");
    else if (nst == 3) asm volatile("cp.async.wait_group 2;" ::: "memory");
    else asm volatile("cp.async.wait_group 1;" ::: "memory");
}
__device__ __forceinline__ uint32_t stage_range(uint8_t* st, const uint8_t* p, unsigned long long n, int lane) {
    const uintptr_t a = (uintptr_t) p & ~(uintptr_t) 15, b = ((uintptr_t) (p + n) + 15) & ~(uintptr_t) 15;
    const uint32_t dst = smem_u32(st);
    for (uintptr_t o = (uintptr_t) lane * 16; a + o < b; o += 512) cp_async16(dst + (uint32_t) o, (const void*) (a + o));
    return (uint32_t) ((uintptr_t) p - a);
}
// Items 0 .. n - 1 of a warp: issue(i, stage) stages item i, compute(i, stage) consumes it.
template <class Issue, class Compute>
__device__ __forceinline__ void staged_items(int n, int nst, const Issue& issue, const Compute& compute) {
    for (int k = 0; k < nst - 1; ++k) {
        if (k < n) issue(k, k);
        cp_commit();
    }
    int si = 0, sn = nst - 1;   // stages of item i and of item i + nst - 1
    for (int i = 0; i < n; ++i) {
        if (i + nst - 1 < n) issue(i + nst - 1, sn);
        cp_commit();
        cp_wait_ring(nst);
        __syncwarp();
        compute(i, si);
        __syncwarp();
        si = si + 1 == nst ? 0 : si + 1;
        sn = sn + 1 == nst ? 0 : sn + 1;
    }
    cp_wait_all();
    __syncwarp();
}
// Warp w's share of `chunks` 32 KB L2 prefetch chunks of a list of regions (every warp of the grid takes chunk
// w, w + W, ...): the weights of a phase requested at once while the warps compute in order.
__device__ __forceinline__ void prefetch_share(const uint8_t* base, unsigned long long bytes, long long& c0, long long gw,
                                               long long W) {
    const long long n = (long long) ((bytes + 32767) / 32768);
    long long c = c0 > gw ? ((c0 - gw + W - 1) / W) * W + gw : gw;   // first chunk index >= c0 of this warp
    for (; c < c0 + n; c += W) {
        const unsigned long long o = (unsigned long long) (c - c0) * 32768;
        prefetch_l2(base + o, min(32768ull, bytes - o), base, base + bytes);
    }
    c0 += n;
}
template <int GU, int D, int JG, int NC>
__global__ void __launch_bounds__(kAThreads, 1) k_decode_act(ActParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const ActSmem M = act_smem(p.T, p.F, p.FS, p.K, p.sb, p.nst, p.ar);
    BlockQ8_1* q8 = (BlockQ8_1*) (smem + M.q8);
    int32_t* ids_s = (int32_t*) (smem + M.ids);
    float* w_s = (float*) (smem + M.w);
    int* gexp = (int*) (smem + M.gexp);
    int* gstart = (int*) (smem + M.gstart);
    int* gent = (int*) (smem + M.gent);
    int* cnt = (int*) (smem + M.cnt);
    int* off = (int*) (smem + M.off);
    int* ngp = (int*) (smem + M.ng);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int AR = p.ar, BR = p.br;
    float* part = (float*) (smem + M.part) + (size_t) warp * kAMaxEnt * AR;
    uint8_t* stg0 = smem + M.stage + (size_t) warp * p.nst * p.sb;
    auto stg = [&](int s) { return stg0 + (size_t) s * p.sb; };
    const long long W = (long long) gridDim.x * kAWarps, gw = (long long) blockIdx.x * kAWarps + warp;
    const IqTab tab = make_tab(nullptr, lane);
    const int T = p.T, H = p.H, F = p.F, K = p.K, nst = p.nst;
    const int Cg = H / Fmt<GU>::qk * Fmt<GU>::cpb;      // calls per gate/up row (routed and shared)
    const int Cd = F / Fmt<D>::qk * Fmt<D>::cpb;        // calls per routed down row
    const int Csd = p.FS / Fmt<D>::qk * Fmt<D>::cpb;    // calls per shared down row
    const int xb = H / 32;
    act_stamp(0);

    typename Fmt<GU>::Act ag[NC][JG];
    typename Fmt<D>::Act ad[NC][kAJ];
    auto load_in = [&](int t0, int nc) {   // the tokens' input rows (global, written before the launch)
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            if (c >= nc) break;
            const BlockQ8_1* x = p.hq + (size_t) (t0 + c) * xb;
            auto src = [&](int blk) { return qb_from_global(x + blk); };
#pragma unroll
            for (int j = 0; j < JG; ++j) {
                const int k = lane + 32 * j;
                if (k < Cg) ag[c][j] = Fmt<GU>::act(src, k);
            }
        }
    };
    // nr gate rows from r, then the same up rows, of a blob (16-byte aligned rows) into stage s
    auto stage_gu = [&](int s, const uint8_t* blob, int r, int nr, unsigned long long up_off) {
        stage_range(stg(s), blob + (size_t) r * p.gu_row, (unsigned long long) nr * p.gu_row, lane);
        stage_range(stg(s) + (size_t) nr * p.gu_row, blob + up_off + (size_t) r * p.gu_row,
                    (unsigned long long) nr * p.gu_row, lane);
    };

    // everything known before routing into L2: the router, the shared MLP
    if (lane == 0) {
        long long c0 = 0;
        prefetch_share((const uint8_t*) p.router, (unsigned long long) p.E * H * 4, c0, gw, W);
        if (p.sh) prefetch_share(p.sh, p.sh_bytes, c0, gw, W);
    }

    // ---------------------------------------------------------------- A: router logits, shared gate/up
    // phase A deals its units by pw = warp * grid + CTA, so that the router rows land on different CTAs
    const long long pw = (long long) warp * gridDim.x + blockIdx.x;
    for (long long u = pw; u < p.E; u += W) {   // router row u (fp32, direct loads): k_router_logits' expression and order
        const int o = (int) u;
        const float4* wr = (const float4*) (p.router + (size_t) o * H);
        float acc[kAMaxT];
#pragma unroll
        for (int t = 0; t < kAMaxT; ++t) acc[t] = 0.0f;
#pragma unroll 4
        for (int i = lane; i < H / 4; i += 32) {
            const float4 w = __ldg(wr + i);
#pragma unroll
            for (int t = 0; t < kAMaxT; ++t)
                if (t < T) {
                    const float4 x = __ldg((const float4*) (p.h + (size_t) t * H) + i);
                    acc[t] += w.x * x.x + w.y * x.y + w.z * x.z + w.w * x.w;
                }
        }
#pragma unroll
        for (int t = 0; t < kAMaxT; ++t)
            if (t < T) {
                const float v = warp_sum(acc[t]);
                if (lane == 0) p.logits[(size_t) t * p.E + o] = v;
            }
    }
    if (p.sh) {   // shared gate/up rows: warp w takes rows w, w + W, ... after the router rows of the same sequence
        const int first = (int) (pw < p.E ? pw + ((p.E - pw + W - 1) / W) * W : pw);
        const int nA = p.E + p.FS, Wi = (int) W;
        const int n = first < nA ? (nA - first + Wi - 1) / Wi : 0;
        if (T <= NC) load_in(0, T);
        staged_items(
            n, nst, [&](int i, int s) { stage_gu(s, p.sh, first + i * Wi - p.E, 1, p.s_up_off); },
            [&](int i, int s) {
                const int r = first + i * Wi - p.E;
                const uint8_t* gate = stg(s);
                const uint8_t* up = gate + p.gu_row;
                for (int t0 = 0; t0 < T; t0 += NC) {
                    const int nc = min(NC, T - t0);
                    if (T > NC) load_in(t0, nc);
                    float sg[NC], su[NC];
                    row_dot<GU, JG, NC>(gate, Cg, lane, ag, nc, tab, sg);
                    row_dot<GU, JG, NC>(up, Cg, lane, ag, nc, tab, su);
#pragma unroll
                    for (int c = 0; c < NC; ++c)
                        if (c < nc && lane == c)
                            p.shid[(size_t) (t0 + c) * p.FS + r] = act_value(p.sh_act, sg[c], su[c], p.limit);
                }
            });
    }
    __syncthreads();
    act_stamp(1);
    grid_barrier(p.bar, p.err, 0x610u);
    act_stamp(2);

    // ---------------------------------------------------------------- B: routing, grouping, routed gate/up
    for (int t = warp; t < T; t += kAWarps) {
        switch (p.E / 32) {
            case 1: route_token<1>(p, t, lane, ids_s, w_s); break;
            case 2: route_token<2>(p, t, lane, ids_s, w_s); break;
            case 4: route_token<4>(p, t, lane, ids_s, w_s); break;
            case 8: route_token<8>(p, t, lane, ids_s, w_s); break;
            default: route_token<16>(p, t, lane, ids_s, w_s); break;
        }
    }
    for (int x = threadIdx.x; x < p.E; x += blockDim.x) cnt[x] = 0;
    __syncthreads();
    const int n_ent = T * K;
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x)
        if (ids_s[e] >= 0 && ids_s[e] < p.E) atomicAdd(&cnt[ids_s[e]], 1);
    __syncthreads();
    if (warp == 0) {   // k_group's order: groups of ascending expert id (lane l scans experts l * per ...)
        const int per = (p.E + 31) / 32, x0 = lane * per;
        int rows = 0, used = 0;
        for (int x = x0; x < min(x0 + per, p.E); ++x) rows += cnt[x], used += cnt[x] > 0;
        int rb = rows, ub = used;   // inclusive scans over the lanes
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, rb, o), b = __shfl_up_sync(0xffffffffu, ub, o);
            if (lane >= o) rb += a, ub += b;
        }
        int pos = rb - rows, g = ub - used;
        for (int x = x0; x < min(x0 + per, p.E); ++x) {
            off[x] = pos;
            if (cnt[x]) {
                gexp[g] = x;
                gstart[g] = pos;
                ++g;
            }
            pos += cnt[x];
        }
        if (lane == 31) {
            gstart[ub] = rb;
            *ngp = ub;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {   // entries of an expert in entry order
        const int id = ids_s[e];
        if (id < 0 || id >= p.E) continue;
        int before = 0;
        for (int e2 = 0; e2 < e; ++e2) before += ids_s[e2] == id;
        gent[off[id] + before] = e;
    }
    if (blockIdx.x == 0 && threadIdx.x < n_ent) {
        if (p.ids) p.ids[threadIdx.x] = ids_s[threadIdx.x];
        if (p.w) p.w[threadIdx.x] = w_s[threadIdx.x];
    }
    __syncthreads();
    const int ng = *ngp;
    act_stamp(3);
    if (lane == 0) {   // the used experts' blobs into L2, shared by every warp of the grid
        long long c0 = 0;
        for (int g = 0; g < ng; ++g) prefetch_share(p.blobs + (size_t) gexp[g] * p.stride, p.blob_bytes, c0, gw, W);
    }
    {
        // units: (group, BR rows) of the routed gate/up.  A warp takes a contiguous range, so its activations stay in
        // registers across the units of one group.
        const int upg = F / BR;   // units per group
        const long long nB = (long long) ng * upg;
        const int lo = (int) (nB * gw / W), hi = (int) (nB * (gw + 1) / W);
        const int g0 = lo / upg, b0 = lo - g0 * upg;   // the first unit's group and row block; later ones by increments
        int cur = -1;   // the (group, first entry) whose activations are in registers
        staged_items(
            hi - lo, nst,
            [&](int i, int s) {
                const int bb = b0 + i, g = g0 + bb / upg;
                stage_gu(s, p.blobs + (size_t) gexp[g] * p.stride, (bb - (g - g0) * upg) * BR, BR, p.up_off);
            },
            [&](int i, int s) {
                const int bb = b0 + i, g = g0 + bb / upg, r0 = (bb - (g - g0) * upg) * BR;
                for (int eb = gstart[g]; eb < gstart[g + 1]; eb += NC) {
                    const int nc = min(NC, gstart[g + 1] - eb);
                    const int key = g * kAMaxEnt + eb;
                    if (key != cur) {
#pragma unroll
                        for (int c = 0; c < NC; ++c) {
                            if (c >= nc) break;
                            const BlockQ8_1* x = p.hq + (size_t) (gent[eb + c] / K) * xb;
                            auto src = [&](int blk) { return qb_from_global(x + blk); };
#pragma unroll
                            for (int j = 0; j < JG; ++j) {
                                const int k = lane + 32 * j;
                                if (k < Cg) ag[c][j] = Fmt<GU>::act(src, k);
                            }
                        }
                        cur = key;
                    }
                    for (int rr = 0; rr < BR; ++rr) {
                        const uint8_t* gate = stg(s) + (size_t) rr * p.gu_row;
                        const uint8_t* up = stg(s) + (size_t) (BR + rr) * p.gu_row;
                        float sg[NC], su[NC];
                        row_dot<GU, JG, NC>(gate, Cg, lane, ag, nc, tab, sg);
                        row_dot<GU, JG, NC>(up, Cg, lane, ag, nc, tab, su);
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            if (c < nc && lane == c)
                                p.hid[(size_t) gent[eb + c] * F + r0 + rr] = act_value(p.act, sg[c], su[c], p.limit);
                    }
                }
            });
    }
    __syncthreads();
    act_stamp(4);
    grid_barrier(p.bar, p.err, 0x611u);
    act_stamp(5);

    // ---------------------------------------------------------------- C: routed down rows + pick-order sum; shared down
    BlockQ8_1* q8s = q8 + (size_t) n_ent * (F / 32);   // the shared hidden rows after the routed ones
    {
        // every hidden row's q8_1 once over the grid (a warp per block: q8_1_warp, the same bits as the layer-by-layer
        // kernels' q8_1_lane), then into every CTA's shared memory
        const int nbr = n_ent * (F / 32), nbt = nbr + (p.sh ? T * (p.FS / 32) : 0);
        for (long long b = gw; b < nbt; b += W) {
            const float* src = b < nbr ? p.hid + (size_t) (b / (F / 32)) * F + 32 * (b % (F / 32))
                                       : p.shid + (size_t) ((b - nbr) / (p.FS / 32)) * p.FS + 32 * ((b - nbr) % (p.FS / 32));
            float d, sum;
            const int8_t q = q8_1_warp(__ldcg(src + lane), d, sum);
            p.hqh[b].qs[lane] = q;
            if (lane == 0) p.hqh[b].ds = make_half2(__float2half(q8_finite(d)), __float2half(q8_finite(sum)));
        }
        __syncthreads();
        grid_barrier(p.bar, p.err, 0x612u);
        const uint32_t bytes = ((uint32_t) nbt * (uint32_t) sizeof(BlockQ8_1) + 15u) & ~15u;
        const uint32_t dst = smem_u32(q8);
        for (uint32_t o = threadIdx.x * 16u; o < bytes; o += blockDim.x * 16u)
            cp_async16(dst + o, (const uint8_t*) p.hqh + o);
        cp_commit();
        cp_wait_all();
        __syncthreads();
    }
    act_stamp(6);
    {
        // routed units u < nR: AR rows of every used expert's down matrix, one item per group (gi items), summed per
        // token in pick order at the unit's last item; shared units: kASR rows of the shared MLP's down matrix (one
        // item).  Warps split the items evenly; a unit belongs to the warp whose share holds its first item.
        const int nR = H / AR, nS = p.sh ? H / kASR : 0;
        const int gi = max(ng, 1);
        const long long total = (long long) nR * gi + nS;
        const int cw0 = (int) (total * gw / W), cw1 = (int) (total * (gw + 1) / W);
        const int ru0 = min(nR, (cw0 + gi - 1) / gi), ru1 = min(nR, (cw1 + gi - 1) / gi);
        const int su0 = min(nS, max(0, cw0 - nR * gi)), su1 = min(nS, max(0, cw1 - nR * gi));
        const int nri = (ru1 - ru0) * gi;
        uint32_t skew[4] = {0, 0, 0, 0};
        int cur = -1;   // shared-down token chunk whose activations are in registers
        staged_items(
            nri + (su1 - su0), nst,
            [&](int i, int s) {
                if (i < nri) {
                    const int u = ru0 + i / gi, g = i - (u - ru0) * gi;
                    if (g >= ng) return;
                    const uint8_t* rows = p.blobs + (size_t) gexp[g] * p.stride + p.down_off + (size_t) u * AR * p.d_row;
                    skew[s] = stage_range(stg(s), rows, (unsigned long long) AR * p.d_row, lane);
                } else {
                    const int u = su0 + (i - nri);
                    const uint8_t* rows = p.sh + p.s_down_off + (size_t) u * kASR * p.sd_row;
                    skew[s] = stage_range(stg(s), rows, (unsigned long long) kASR * p.sd_row, lane);
                }
            },
            [&](int i, int s) {
                const uint8_t* rows = stg(s) + skew[s];
                if (i < nri) {
                    const int u = ru0 + i / gi, g = i - (u - ru0) * gi, i0 = u * AR;
                    if (g == 0) {
                        for (int q = lane; q < n_ent * AR; q += 32) part[q] = 0.0f;   // entries without a group: 0
                        __syncwarp();
                    }
                    if (g < ng) {
                        for (int eb = gstart[g]; eb < gstart[g + 1]; eb += NC) {
                            const int nc = min(NC, gstart[g + 1] - eb);
#pragma unroll
                            for (int c = 0; c < NC; ++c) {
                                if (c >= nc) break;
                                const BlockQ8_1* x = q8 + (size_t) gent[eb + c] * (F / 32);
                                auto src = [&](int blk) { return qb_from_smem(x + blk); };
#pragma unroll
                                for (int j = 0; j < kAJ; ++j) {
                                    const int k = lane + 32 * j;
                                    if (k < Cd) ad[c][j] = Fmt<D>::act(src, k);
                                }
                            }
#pragma unroll
                            for (int rr = 0; rr < AR; ++rr) {
                                float sv[NC];
                                row_dot<D, kAJ, NC>(rows + (size_t) rr * p.d_row, Cd, lane, ad, nc, tab, sv);
#pragma unroll
                                for (int c = 0; c < NC; ++c)
                                    if (c < nc && lane == c) part[gent[eb + c] * AR + rr] = sv[c];
                            }
                        }
                    }
                    cur = -1;
                    if (g == gi - 1) {
                        __syncwarp();
                        for (int q = lane; q < T * AR; q += 32) {   // moe_sum's expression and order
                            const int t = q / AR, rr = q % AR;
                            float sum = 0.0f;
                            for (int k = 0; k < K; ++k) sum += w_s[t * K + k] * part[(t * K + k) * AR + rr];
                            float* o = p.out + (size_t) t * H + i0 + rr;
                            *o = p.accumulate ? *o + sum : sum;
                        }
                    }
                } else {
                    const int i0 = (su0 + (i - nri)) * kASR;
                    for (int t0 = 0; t0 < T; t0 += NC) {
                        const int nc = min(NC, T - t0);
                        if (cur != t0) {
#pragma unroll
                            for (int c = 0; c < NC; ++c) {
                                if (c >= nc) break;
                                const BlockQ8_1* x = q8s + (size_t) (t0 + c) * (p.FS / 32);
                                auto src = [&](int blk) { return qb_from_smem(x + blk); };
#pragma unroll
                                for (int j = 0; j < kAJ; ++j) {
                                    const int k = lane + 32 * j;
                                    if (k < Csd) ad[c][j] = Fmt<D>::act(src, k);
                                }
                            }
                            cur = t0;
                        }
#pragma unroll
                        for (int rr = 0; rr < kASR; ++rr) {
                            float sv[NC];
                            row_dot<D, kAJ, NC>(rows + (size_t) rr * p.sd_row, Csd, lane, ad, nc, tab, sv);
#pragma unroll
                            for (int c = 0; c < NC; ++c)
                                if (c < nc && lane == c) p.sh_out[(size_t) (t0 + c) * H + i0 + rr] = sv[c];
                        }
                    }
                }
            });
    }
    __syncthreads();
    act_stamp(7);
}

// The shared-memory opt-in and the one-CTA-per-SM check, once per (device, kernel, size).
struct ActAttr {
    size_t smem[4] = {0, 0, 0, 0};
};
ActAttr g_act_attr[64];
std::mutex g_act_mu;

template <int GU, int D, int JG, int NC>
int launch_act(const ActParams& p, size_t smem, int sms, int dev, int which, cudaStream_t s) {
    auto kern = k_decode_act<GU, D, JG, NC>;
    {
        std::lock_guard<std::mutex> lk(g_act_mu);
        ActAttr& A = g_act_attr[dev & 63];
        if (A.smem[which] < smem) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess)
                return afail(TSB_ERR_CUDA, "decode_act: shared memory attribute: %s",
                             cudaGetErrorString(cudaGetLastError()));
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAThreads, smem) != cudaSuccess ||
                per_sm < 1) {
                cudaGetLastError();
                return afail(TSB_ERR_UNSUPPORTED, "decode_act: no room for a CTA per SM (%zu bytes of shared memory)",
                             smem);
            }
            A.smem[which] = smem;
        }
    }
    ActParams q = p;
    void* args[] = {&q};
    if (cudaLaunchCooperativeKernel((const void*) kern, dim3((unsigned) sms), dim3(kAThreads), args, smem, s) !=
        cudaSuccess)
        return afail(TSB_ERR_CUDA, "decode_act: launch: %s", cudaGetErrorString(cudaGetLastError()));
    return TSB_OK;
}

struct ActWs {
    size_t logits, hid, shid, hqh, bar, total;
};
ActWs act_ws(const tsb_decode_act_desc* d) {
    auto al = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    ActWs w;
    size_t o = 0;
    w.logits = o; o += al((size_t) d->n_tok * d->n_expert * 4);
    w.hid = o;    o += al((size_t) d->n_tok * d->n_used * d->n_ff * 4);
    w.shid = o;   o += al((size_t) d->n_tok * (d->sh_n_ff > 0 ? d->sh_n_ff : 1) * 4);
    w.hqh = o;    o += al(((size_t) d->n_tok * d->n_used * (d->n_ff / 32) +
                           (size_t) d->n_tok * (d->sh_n_ff > 0 ? d->sh_n_ff / 32 : 0)) * sizeof(BlockQ8_1));
    w.bar = o;    o += 256;
    w.total = o;
    return w;
}

int qk_t(int t) { return t == T_Q4_0 || t == T_Q8_0 ? 32 : 256; }
int cpb_t(int t) {
    switch (t) {
        case T_Q4_0: return 2;
        case T_Q8_0: return 4;
        case T_Q4_K: return 16;
        case T_Q6_K: return 32;
        default: return 8;
    }
}
int bb_t(int t) {
    switch (t) {
        case T_Q4_0: return 18;
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        case T_IQ3_XXS: return 98;
        case T_IQ3_S: return 110;
        default: return 0;
    }
}

}  // namespace

// The phase-stamp buffer of this translation unit's kernel (null: off).
int decode_act_set_trace(unsigned long long* buf) {
    return cudaMemcpyToSymbol(g_act_trace, &buf, sizeof buf) == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

// This translation unit's copy of the wait bound (tsb_set_wait_limit_ns sets every copy on the current device).
int decode_act_set_wait_limit(unsigned long long ns) {
    return cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof ns) == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

}  // namespace tsb

using namespace tsb;

extern "C" {

int tsb_moe_decode_act_set_trace(unsigned long long* buf) {
    if (decode_act_set_trace(buf) != TSB_OK)
        return afail(TSB_ERR_CUDA, "decode_act: trace: %s", cudaGetErrorString(cudaGetLastError()));
    return TSB_OK;
}

uint64_t tsb_moe_decode_act_workspace_bytes(const tsb_decode_act_desc* d) {
    if (!d || d->struct_size != sizeof(tsb_decode_act_desc)) return 0;
    return act_ws(d).total;
}

int tsb_moe_decode_act(const tsb_decode_act_desc* d, const float* router, const float* bias, const float* escale,
                       const float* h, const void* hq, const void* blobs, uint64_t blob_stride, const void* sh_blob,
                       float* out, int accumulate, float* sh_out, int32_t* ids, float* w, void* workspace,
                       uint64_t ws_bytes, void* stream) {
    if (!d || d->struct_size != sizeof(tsb_decode_act_desc)) return afail(TSB_ERR_ARG, "decode_act: descriptor size");
    const int T = d->n_tok, H = d->n_embd, F = d->n_ff, E = d->n_expert, K = d->n_used, FS = d->sh_n_ff;
    const int GU = d->gu_type, D = d->d_type;
    const bool q40 = GU == T_Q4_0 && D == T_Q4_0, kq = GU == T_Q4_K && D == T_Q6_K;
    if (!q40 && !kq)
        return afail(TSB_ERR_UNSUPPORTED, "decode_act: Q4_0 / Q4_0 or Q4_K / Q6_K experts (gate-up / down) only");
    if (T < 1 || T > kAMaxT || K < 1 || K > 32 || T * K > kAMaxEnt || E < 32 || E % 32 || E > kAMaxE || K > E)
        return afail(TSB_ERR_UNSUPPORTED, "decode_act: 1..16 tokens, T*K <= 128, experts a multiple of 32 up to 512");
    if (d->gate != 0 && d->gate != 1) return afail(TSB_ERR_ARG, "decode_act: gate 0 (softmax) or 1 (sigmoid)");
    if (d->act < 0 || d->act > 2 || (FS > 0 && (d->sh_act < 0 || d->sh_act > 2)))
        return afail(TSB_ERR_ARG, "decode_act: activation 0, 1 or 2");
    if (H % 4 || H % qk_t(GU) || F % 32 || F % qk_t(D) || FS < 0 || (FS > 0 && (FS % 32 || FS % qk_t(D))))
        return afail(TSB_ERR_UNSUPPORTED, "decode_act: sizes not in whole blocks");
    const int Cg = H / qk_t(GU) * cpb_t(GU), Cd = F / qk_t(D) * cpb_t(D), Csd = FS / qk_t(D) * cpb_t(D);
    const int jg = q40 ? kAJ : kAJQ4K;
    if (Cg > 32 * jg || Cd > 32 * kAJ || Csd > 32 * kAJ || H % 2 || H % kASR)
        return afail(TSB_ERR_UNSUPPORTED, "decode_act: rows longer than %d (gate/up) or %d (down) calls", 32 * jg,
                     32 * kAJ);
    if (!router || !h || !hq || !blobs || !out || !workspace || (FS > 0 && (!sh_blob || !sh_out)))
        return afail(TSB_ERR_ARG, "decode_act: null argument");
    if ((uintptr_t) router % 16 || (uintptr_t) h % 16 || (uintptr_t) hq % 4 || (uintptr_t) workspace % 256 ||
        (uintptr_t) blobs % 2 || blob_stride % 2 || (sh_blob && (uintptr_t) sh_blob % 2))
        return afail(TSB_ERR_ALIGN, "decode_act: alignment (router / h 16 bytes, q8_1 4, workspace 256, blobs 2)");
    const ActWs wl = act_ws(d);
    if (ws_bytes < wl.total)
        return afail(TSB_ERR_WORKSPACE, "decode_act: workspace %llu < %llu bytes", (unsigned long long) ws_bytes,
                     (unsigned long long) wl.total);
    int dev = 0, sms = 0, coop = 0, max_smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (!coop) return afail(TSB_ERR_UNSUPPORTED, "decode_act: device without cooperative launch");
    const uint64_t gu_row = (uint64_t) H / qk_t(GU) * bb_t(GU), d_row = (uint64_t) F / qk_t(D) * bb_t(D);
    const uint64_t sd_row = FS > 0 ? (uint64_t) FS / qk_t(D) * bb_t(D) : 0;

    const uint64_t blob_bytes = 2 * (uint64_t) F * gu_row + (uint64_t) H * d_row;
    const uint64_t sh_bytes = FS > 0 ? 2 * (uint64_t) FS * gu_row + (uint64_t) H * sd_row : 0;
    // rows are staged in 16-byte pieces: blob bases, the stride, gate/up rows and the blobs' ends on 16 bytes
    if ((uintptr_t) blobs % 16 || blob_stride % 16 || gu_row % 16 || blob_bytes % 16 ||
        (FS > 0 && ((uintptr_t) sh_blob % 16 || sh_bytes % 16)))
        return afail(TSB_ERR_ALIGN, "decode_act: blobs, stride, gate/up rows and blob sizes must be 16-byte multiples");
    // rows per unit (gate/up, down) and staging depth: one gate/up row pair and two down rows per unit, four buffers
    // deep, measured fastest wherever a step uses few experts; from 32 entries (about 30 distinct experts) units of two
    // gate/up row pairs and 8 down rows of each expert, so that a warp's share comes in fewer, larger pieces.  The
    // first choice whose staging fits beside the hidden rows two deep at least, as deep as fits up to four.
    static const int kFew[1][2] = {{1, 2}};
    static const int kMany[4][2] = {{2, 8}, {2, 4}, {1, 4}, {1, 2}};
    const int (*choice)[2] = T * K >= 32 ? kMany : kFew;
    const int n_choice = T * K >= 32 ? 4 : 1;
    int br = 0, ar = 0, nst = 0;
    uint64_t sb = 0;
    for (int i = 0; i < n_choice && !nst; ++i) {
        const int* c = choice[i];
        if (F % c[0] || H % c[1]) continue;
        const uint64_t b =
            (std::max({(uint64_t) 2 * c[0] * gu_row, c[1] * d_row + 32, kASR * sd_row + 32}) + 15) / 16 * 16;
        const uint32_t base = act_smem(T, F, FS > 0 ? FS : 0, K, (uint32_t) b, 0, c[1]).total;
        const int n = max_smem > (int) base ? std::min<int>(4, (int) ((max_smem - base) / (kAWarps * b))) : 0;
        if (n >= 2) br = c[0], ar = c[1], nst = n, sb = b;
    }
    if (!nst) return afail(TSB_ERR_UNSUPPORTED, "decode_act: the staging buffers do not fit in %d bytes", max_smem);
    const ActSmem M = act_smem(T, F, FS > 0 ? FS : 0, K, (uint32_t) sb, nst, ar);
    ActParams p{};
    p.T = T; p.H = H; p.F = F; p.E = E; p.K = K; p.FS = FS > 0 ? FS : 0;
    p.router = router; p.h = h; p.hq = (const BlockQ8_1*) hq;
    p.gate = d->gate; p.norm = d->norm; p.in_scale = d->in_scale; p.w_scale = d->w_scale; p.limit = d->limit;
    p.bias = bias; p.escale = escale;
    p.blobs = (const uint8_t*) blobs; p.stride = blob_stride;
    p.gu_row = gu_row; p.up_off = (uint64_t) F * gu_row; p.d_row = d_row; p.down_off = 2 * p.up_off;
    if (FS > 0) {
        p.sh = (const uint8_t*) sh_blob;
        p.sgu_row = gu_row;
        p.s_up_off = (uint64_t) FS * gu_row;
        p.sd_row = sd_row;
        p.s_down_off = 2 * p.s_up_off;
    }
    p.blob_bytes = blob_bytes;
    p.sh_bytes = sh_bytes;
    p.sb = (uint32_t) sb;
    p.nst = nst;
    p.ar = ar;
    p.br = br;
    p.act = d->act; p.sh_act = d->sh_act; p.accumulate = accumulate;
    p.out = out; p.sh_out = sh_out; p.ids = ids; p.w = w;
    uint8_t* ws = (uint8_t*) workspace;
    p.logits = (float*) (ws + wl.logits);
    p.hid = (float*) (ws + wl.hid);
    p.shid = (float*) (ws + wl.shid);
    p.hqh = (BlockQ8_1*) (ws + wl.hqh);
    p.bar = (unsigned*) (ws + wl.bar);
    p.err = device_error_word();
    if (!p.err) return afail(TSB_ERR_CUDA, "decode_act: device error word");
    cudaStream_t s = (cudaStream_t) stream;
    if (cudaMemsetAsync(p.bar, 0, 8, s) != cudaSuccess)
        return afail(TSB_ERR_CUDA, "decode_act: barrier reset: %s", cudaGetErrorString(cudaGetLastError()));
    // one token column per row pass at T = 1 (the decode step of one sequence: half the code in the hot loops),
    // two otherwise
    if (T == 1)
        return q40 ? launch_act<T_Q4_0, T_Q4_0, kAJ, 1>(p, M.total, sms, dev, 0, s)
                   : launch_act<T_Q4_K, T_Q6_K, kAJQ4K, 1>(p, M.total, sms, dev, 1, s);
    return q40 ? launch_act<T_Q4_0, T_Q4_0, kAJ, 2>(p, M.total, sms, dev, 2, s)
               : launch_act<T_Q4_K, T_Q6_K, kAJQ4K, 2>(p, M.total, sms, dev, 3, s);
}

}  // extern "C"
