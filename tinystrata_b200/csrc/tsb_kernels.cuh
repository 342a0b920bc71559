// tsb_kernels.cuh - the grouped expert GEMV kernels (decode) and their shared-memory machinery.
//
// Layout in HBM (the reference's, so the engines' buffers work unchanged): expert blob [gate rows | up rows | down rows]
// of raw GGUF blocks (NativeExpertLayout, iq_kernels.hpp:45-53); q8_1 activations of 36-byte blocks; groups as
// k_group writes them (grp_ptr = blob address, grp_start, n_groups on the device, ent_dst, ent_tok).
//
// Execution model: persistent CTAs (one or two per SM), each warp an independent pipeline over a contiguous range of
// (group, row) tasks.  Lane 0 streams the task's weight rows into a per-warp ring of shared-memory stages with
// cp.async.bulk (completion on one mbarrier per stage), the warp decodes them from shared memory while the next stages
// are in flight.  A lane always handles the same calls (k = lane + 32 j) of every row, so the activations of those calls
// sit in registers for the warp's whole range; the IQ3_XXS codebook and sign masks are lane-banked in shared memory.
#pragma once

#include "tsb_formats.cuh"

namespace tsb {

#include "codebooks.inc"
__device__ const uint32_t g_iq3xxs_grid[256] = TSB_IQ3XXS_GRID;
__device__ const uint32_t g_iq3s_grid[512] = TSB_IQ3S_GRID;
__device__ const uint8_t g_ksigns[128] = TSB_KSIGNS;

template <int TY> __host__ __device__ constexpr int table_bytes() {
    return TY == T_IQ3_XXS ? kIqTabBytes : TY == T_IQ3_S ? kIqTabBytes + 2048 : 0;
}

// Fill the lane-banked IQ3_XXS grid and sign masks (and the plain IQ3_S grid when asked) with threads
// [0, nthreads); the caller synchronises them afterwards.
template <int TY>
__device__ void fill_tables(uint8_t* tab, int nthreads) {
    if constexpr (TY == T_IQ3_XXS) {
        // grid: 256 indices x 32 lanes; sign masks: 128 indices x 16 lane slots x 8 bytes
        for (int i = threadIdx.x; i < 256 * 8; i += nthreads) {
            const int idx = i >> 3, q = i & 7;
            const uint32_t g = g_iq3xxs_grid[idx];
            *(uint4*) (tab + idx * 256 + q * 16) = make_uint4(g, g, g, g);
        }
        for (int i = threadIdx.x; i < 128 * 8; i += nthreads) {
            const int s = i >> 3, q = i & 7;
            const uint32_t ks = g_ksigns[s];
            const uint32_t m0 = spread4(ks & 15u), m1 = spread4(ks >> 4);
            *(uint4*) (tab + s * 256 + 128 + q * 16) = make_uint4(m0, m1, m0, m1);
        }
    } else if constexpr (TY == T_IQ3_S) {
        uint32_t* g3 = (uint32_t*) (tab + kIqTabBytes);
        for (int i = threadIdx.x; i < 512; i += nthreads) g3[i] = g_iq3s_grid[i];
    }
}
// Whole CTA, then __syncthreads.
template <int TY>
__device__ void build_tables(uint8_t* tab) {
    fill_tables<TY>(tab, blockDim.x);
    __syncthreads();
}

__device__ __forceinline__ IqTab make_tab(const uint8_t* tab, int lane) {
    IqTab t;
    t.base = tab;
    t.lane4 = 4u * (uint32_t) lane;
    t.lane_s = 128u + 8u * (uint32_t) (lane & 15);
    return t;
}

// ------------------------------------------------------------------------------------------------ per-warp pipeline
struct WarpRing {
    uint8_t* buf;
    uint64_t* bar;
    uint32_t stage_bytes;
    uint32_t parity;   // bit s: the parity the next wait on stage s expects

    __device__ void init(uint8_t* b, uint64_t* br, uint32_t sb, int nst, int lane) {
        buf = b;
        bar = br;
        stage_bytes = sb;
        parity = 0;
        if (lane == 0)
            for (int s = 0; s < nst; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
        __syncwarp();
    }
    __device__ uint8_t* stage(int s) const { return buf + (size_t) s * stage_bytes; }
    // lane 0: copy `n` pieces (src_i, bytes_i) back to back into stage s
    __device__ void issue2(int s, const void* a, uint32_t na, const void* b, uint32_t nb, int lane) {
        if (lane == 0) {
            mbar_expect_tx(&bar[s], na + nb);
            bulk_g2s(stage(s), a, na, &bar[s]);
            if (nb) bulk_g2s(stage(s) + na, b, nb, &bar[s]);
        }
    }
    __device__ bool wait(int s, unsigned* err, unsigned site) {
        const bool ok = mbar_wait_bounded(&bar[s], (parity >> s) & 1u, err, site);
        parity ^= 1u << s;
        return ok;
    }
};

struct GroupArgs {
    const unsigned long long* grp_ptr;
    const int32_t* grp_start;
    const int32_t* n_groups;
    const int32_t* ent_dst;
    const int32_t* ent_tok;
    int cap_groups, cap_entries;   // the caller's capacities: device counts beyond them are clamped (and reported)
    // The group count as read on the device, at most cap_groups; a larger count is recorded at `site` in err.
    __device__ int groups(unsigned* err, unsigned site) const {
        const int ng = *n_groups;
        if (ng > cap_groups && threadIdx.x == 0 && blockIdx.x == 0) report_error(err, site);
        return ng < 0 ? 0 : (ng > cap_groups ? cap_groups : ng);
    }
    // Entries [e0, e1) of group g, inside [0, cap_entries).
    __device__ void entries(int g, int& e0, int& e1) const {
        e0 = max(grp_start[g], 0);
        e1 = min(grp_start[g + 1], cap_entries);
    }
};

enum : int { ACT_SWIGLU = 0, ACT_GELU_TANH = 1, ACT_SWIGLU_CLAMP = 2 };

// The hidden value of one row: the reference's expressions (SwiGLU iq_kernels.cu:1508-1512 with the fast-math
// division, GELU-tanh gemma4/kernels.cu:261-263, clamped SwiGLU gemma4/kernels.cu:251-258).
__device__ __forceinline__ float act_value(int act, float g, float u, float limit) {
    if (act == ACT_GELU_TANH) {
        const float c = 0.5f * g * (1.0f + tanhf(0.79788456080286535587989211986876f * g * (1.0f + 0.044715f * g * g)));
        return c * u;
    }
    if (act == ACT_SWIGLU_CLAMP) {
        const float gc = fminf(g, limit);
        const float uc = fminf(fmaxf(u, -limit), limit);
        return gc / (1.0f + expf(-gc)) * uc;
    }
    return __fmul_rn(fdiv_fm(g, 1.0f + __expf(-g)), u);
}

// ------------------------------------------------------------------------------------------------ Gemma / LFM routing
// One token's routing by one warp (route_kernel, gemma4/kernels.cu:289-356; built without fast-math, as that file):
// gate 0 softmax of logit * in_scale, gate 1 sigmoid; pick on p + bias (lowest id on ties); w = p [/ max(sum, floor)]
// [* escale] [* w_scale].  lgf(e) gives logit e; PER experts a lane; lanes < n_used write ids_out / w_out.
template <int PER, class LG>
__device__ __forceinline__ void route_row_warp(const LG& lgf, int n_expert, int n_used, int gate, float in_scale,
                                               const float* __restrict__ bias, const float* __restrict__ escale,
                                               int norm, float w_scale, int lane, int32_t* ids_out, float* w_out) {
    float p[PER], pick[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int e = lane + k * 32;
        p[k] = e < n_expert ? lgf(e) * in_scale : -INFINITY;
        mx = fmaxf(mx, p[k]);
    }
    if (gate == 0) {
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            p[k] = lane + k * 32 < n_expert ? expf(p[k] - mx) : 0.0f;
            sum += p[k];
        }
        const float inv = __fdiv_rn(1.0f, warp_sum(sum));
#pragma unroll
        for (int k = 0; k < PER; ++k) p[k] *= inv;
    } else {
#pragma unroll
        for (int k = 0; k < PER; ++k) p[k] = __fdiv_rn(1.0f, 1.0f + expf(-p[k]));
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int e = lane + k * 32;
        pick[k] = e < n_expert ? p[k] + (bias ? bias[e] : 0.0f) : -INFINITY;
    }
    float sum = 0.0f, mine = 0.0f;
    int my_id = 0;
    for (int j = 0; j < n_used; ++j) {
        float best = -INFINITY;
        int at = n_expert;
#pragma unroll
        for (int k = 0; k < PER; ++k)
            if (pick[k] > best) best = pick[k], at = lane + k * 32;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float b = __shfl_xor_sync(0xffffffffu, best, o);
            const int a = __shfl_xor_sync(0xffffffffu, at, o);
            if (b > best || (b == best && a < at)) best = b, at = a;
        }
        float pw = 0.0f;
#pragma unroll
        for (int k = 0; k < PER; ++k)
            if (lane + k * 32 == at) pw = p[k], pick[k] = -INFINITY;
        pw = __shfl_sync(0xffffffffu, pw, at % 32);
        sum += pw;
        if (lane == j) mine = pw, my_id = at;
    }
    if (lane >= n_used) return;
    float v = mine;
    if (norm) v = __fdiv_rn(v, fmaxf(sum, 6.103515625e-5f));
    if (escale) v *= escale[my_id];
    if (w_scale != 0.0f) v *= w_scale;
    ids_out[lane] = my_id;
    w_out[lane] = v;
}

// ------------------------------------------------------------------------------------------------ row dots
// One warp, one row staged at `row` (shared memory): lane calls k = lane + 32 j (j < J) for C calls per row; the NC
// activations' per-lane partial sums in s[], then the xor tree.  The per-lane order and the tree are row_dot's
// (iq_kernels.cu:695-705), so each value is the reference's bit for bit.
template <int TY, int J, int NC>
__device__ __forceinline__ void row_dot(const uint8_t* row, int C, int lane, const typename Fmt<TY>::Act (&a)[NC][J],
                                        int nc, const IqTab& t, float (&s)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; ++c) s[c] = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int k = lane + 32 * j;
        if (k < C) {
            const typename Fmt<TY>::W w = decode_call<TY>(row, k, t);
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if (c < nc) s[c] += Fmt<TY>::apply(w, a[c][j]);
        }
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) s[c] = warp_sum(s[c]);
}

// P rows per pass (C < 32 calls per row, C a power of two): lane l takes call l % C of row l / C; segmented xor tree
// over C lanes (a whole-warp tree whose other lanes hold zeros gives the same bits).
template <int TY, int NC>
__device__ __forceinline__ void row_dot_packed(const uint8_t* rows, size_t row_bytes, int C, int lane,
                                               const typename Fmt<TY>::Act (&a)[NC][1], int nc, const IqTab& t,
                                               float (&s)[NC]) {
    const int r = lane / C, k = lane % C;
#pragma unroll
    for (int c = 0; c < NC; ++c) s[c] = 0.0f;
    const typename Fmt<TY>::W w = decode_call<TY>(rows + r * row_bytes, k, t);
#pragma unroll
    for (int c = 0; c < NC; ++c)
        if (c < nc) s[c] += Fmt<TY>::apply(w, a[c][0]);
#pragma unroll
    for (int c = 0; c < NC; ++c)
        for (int o = C >> 1; o > 0; o >>= 1) s[c] += __shfl_xor_sync(0xffffffffu, s[c], o);
}

// ------------------------------------------------------------------------------------------------ gate/up kernel
struct GuParams {
    int nst;               // stages per warp ring (1..kMaxStages)
    GroupArgs g;
    const BlockQ8_1* xq;   // [tokens][n_embd / 32]
    int n_embd, n_ff;
    uint64_t gu_row, up_off;
    float* h;              // [cap_entries][n_ff]: act(gate, up) of each grouped entry
    int act;
    float limit;
    unsigned* err;
};

constexpr int kWarps = 8;
constexpr int kMaxStages = 3;
constexpr size_t kSmemBudget = 200 * 1024;

// Task i of the call: group i / n_ff, row i % n_ff (its gate row and its up row).  Warp w of W takes tasks
// [w n / W, (w + 1) n / W): one group for long stretches, so its activations stay in registers.
template <int TY, int J, int NC>
__global__ void __launch_bounds__(kWarps * 32) k_expert_gu(GuParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = table_bytes<TY>();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t stage_bytes = (uint32_t) (2 * p.gu_row);
    uint64_t* bars = (uint64_t*) (smem + TB);
    uint8_t* stages = smem + TB + 128 * 8;
    const int nst = p.nst;
    WarpRing ring;
    ring.init(stages + (size_t) warp * nst * stage_bytes, bars + warp * kMaxStages, stage_bytes, nst, lane);

    const int ng = p.g.groups(p.err, 0x110u);
    const long long n_tasks = (long long) ng * p.n_ff;
    const long long W = (long long) gridDim.x * kWarps, wg = (long long) blockIdx.x * kWarps + warp;
    const long long lo = n_tasks * wg / W, hi = n_tasks * (wg + 1) / W;
    const int C = p.n_embd / Fmt<TY>::qk * Fmt<TY>::cpb;
    const int xb = p.n_embd / 32;

    auto src_of = [&](long long i, const uint8_t*& a) {
        const int g = (int) (i / p.n_ff), r = (int) (i % p.n_ff);
        a = (const uint8_t*) p.g.grp_ptr[g] + (size_t) r * p.gu_row;
    };
    // prologue: the first stages' copies go out before the tables are built
    for (int s = 0; s < nst; ++s)
        if (lo + s < hi) {
            const uint8_t* a;
            src_of(lo + s, a);
            ring.issue2(s, a, (uint32_t) p.gu_row, a + p.up_off, (uint32_t) p.gu_row, lane);
        }
    build_tables<TY>(smem);
    const IqTab tab = make_tab(smem, lane);
    if (lo >= hi) return;
    typename Fmt<TY>::Act act[NC][J];
    int cur_g = -1, cur_e = -1;
    for (long long i = lo; i < hi; ++i) {
        const int s = (int) ((i - lo) % nst);
        const int g = (int) (i / p.n_ff), r = (int) (i % p.n_ff);
        int e0, e1;
        p.g.entries(g, e0, e1);
        if (!ring.wait(s, p.err, 0x100u)) return;
        const uint8_t* gate = ring.stage(s);
        const uint8_t* up = gate + p.gu_row;
        for (int eb = e0; eb < e1; eb += NC) {
            const int nc = min(NC, e1 - eb);
            if (g != cur_g || eb != cur_e) {
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    if (c >= nc) break;
                    const BlockQ8_1* x = p.xq + (size_t) p.g.ent_tok[eb + c] * xb;
                    auto src = [&](int blk) { return qb_from_global(x + blk); };
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        const int k = lane + 32 * j;
                        if (k < C) act[c][j] = Fmt<TY>::act(src, k);
                    }
                }
                cur_g = g;
                cur_e = eb;
            }
            float sg[NC], su[NC];
            row_dot<TY, J, NC>(gate, C, lane, act, nc, tab, sg);
            row_dot<TY, J, NC>(up, C, lane, act, nc, tab, su);
#pragma unroll
            for (int c = 0; c < NC; ++c)
                if (c < nc && lane == c) p.h[(size_t) (eb + c) * p.n_ff + r] = act_value(p.act, sg[c], su[c], p.limit);
        }
        __syncwarp();
        if (i + nst < hi) {
            const uint8_t* a;
            src_of(i + nst, a);
            ring.issue2(s, a, (uint32_t) p.gu_row, a + p.up_off, (uint32_t) p.gu_row, lane);
        }
    }
}

// ------------------------------------------------------------------------------------------------ down kernel
struct DownParams {
    int nst;
    GroupArgs g;
    const float* h;        // [cap_entries][n_ff], quantised to q8_1 on the fly (the reference's swiglu_q8_1 step)
    int n_embd, n_ff;
    uint64_t d_row, down_off;
    int R;                 // rows per task (R * d_row a multiple of 16)
    float* out;            // [rows of ent_dst][n_embd]
    unsigned* err;
};

// Task i: group i / (n_embd / R), rows R (i % (n_embd / R)) .. + R.  J calls per lane (C >= 32) or P = 32 / C rows
// per pass (C < 32).
template <int TY, int J, int NC>
__global__ void __launch_bounds__(kWarps * 32) k_expert_down(DownParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = table_bytes<TY>();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t stage_bytes = (uint32_t) (p.R * p.d_row);
    uint64_t* bars = (uint64_t*) (smem + TB);
    uint8_t* stages = smem + TB + 128 * 8;
    const int nst = p.nst;
    WarpRing ring;
    ring.init(stages + (size_t) warp * nst * stage_bytes, bars + warp * kMaxStages, stage_bytes, nst, lane);

    const int ng = p.g.groups(p.err, 0x210u);
    const int chunks = p.n_embd / p.R;
    const long long n_tasks = (long long) ng * chunks;
    const long long W = (long long) gridDim.x * kWarps, wg = (long long) blockIdx.x * kWarps + warp;
    const long long lo = n_tasks * wg / W, hi = n_tasks * (wg + 1) / W;
    const int C = p.n_ff / Fmt<TY>::qk * Fmt<TY>::cpb;
    const int P = C < 32 ? 32 / C : 1;

    auto src_of = [&](long long i) {
        const int g = (int) (i / chunks), ch = (int) (i % chunks);
        return (const uint8_t*) p.g.grp_ptr[g] + p.down_off + (size_t) ch * p.R * p.d_row;
    };
    for (int s = 0; s < nst; ++s)
        if (lo + s < hi) ring.issue2(s, src_of(lo + s), stage_bytes, nullptr, 0, lane);
    build_tables<TY>(smem);
    const IqTab tab = make_tab(smem, lane);
    if (lo >= hi) return;

    typename Fmt<TY>::Act act[NC][J];
    int cur_g = -1, cur_e = -1;
    for (long long i = lo; i < hi; ++i) {
        const int s = (int) ((i - lo) % nst);
        const int g = (int) (i / chunks), r0 = (int) (i % chunks) * p.R;
        int e0, e1;
        p.g.entries(g, e0, e1);
        if (!ring.wait(s, p.err, 0x200u)) return;
        const uint8_t* rows = ring.stage(s);
        for (int eb = e0; eb < e1; eb += NC) {
            const int nc = min(NC, e1 - eb);
            if (g != cur_g || eb != cur_e) {
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    if (c >= nc) break;
                    const float* hx = p.h + (size_t) (eb + c) * p.n_ff;
                    auto src = [&](int blk) { return qb_from_f32(hx + 32 * blk); };
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        const int k = P > 1 ? lane % C : lane + 32 * j;
                        if (k < C) act[c][j] = Fmt<TY>::act(src, k);
                    }
                }
                cur_g = g;
                cur_e = eb;
            }
            if (P > 1) {
                if constexpr (J == 1) {
                    for (int rr = 0; rr < p.R; rr += P) {
                        float sv[NC];
                        row_dot_packed<TY, NC>(rows + (size_t) rr * p.d_row, p.d_row, C, lane, act, nc, tab, sv);
                        const int rl = lane / C, cl = lane % C;
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            if (c < nc && cl == c && rr + rl < p.R)
                                p.out[(size_t) p.g.ent_dst[eb + c] * p.n_embd + r0 + rr + rl] = sv[c];
                    }
                }
            } else {
                for (int rr = 0; rr < p.R; ++rr) {
                    float sv[NC];
                    row_dot<TY, J, NC>(rows + (size_t) rr * p.d_row, C, lane, act, nc, tab, sv);
#pragma unroll
                    for (int c = 0; c < NC; ++c)
                        if (c < nc && lane == c) p.out[(size_t) p.g.ent_dst[eb + c] * p.n_embd + r0 + rr] = sv[c];
                }
            }
        }
        __syncwarp();
        if (i + nst < hi) ring.issue2(s, src_of(i + nst), stage_bytes, nullptr, 0, lane);
    }
}

// stages per warp that fit the budget beside the tables (0: the stage itself does not fit)
template <int TY> inline int expert_stages(uint32_t stage_bytes) {
    const size_t avail = kSmemBudget - table_bytes<TY>() - 128 * 8;
    const size_t n = avail / ((size_t) kWarps * stage_bytes);
    return (int) (n < (size_t) kMaxStages ? n : (size_t) kMaxStages);
}
template <int TY> inline size_t expert_smem(uint32_t stage_bytes, int nst) {
    return (size_t) table_bytes<TY>() + 128 * 8 + (size_t) kWarps * nst * stage_bytes;
}

}  // namespace tsb
