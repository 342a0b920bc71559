// tsb_moe.cu - the B200 MoE expert path behind TinyStrata's expert-layer entry points: q8_1 quantiser, router GEMV,
// softmax / sigmoid top-k routers, decode grouping, grouped expert GEMVs, combine.  The C ABI is include/tsb_moe.h.
#include "tsb_kernels.cuh"
#include "tsb_prefill.cuh"
#include "tsb_prefill_k.cuh"
#include "tsb_mmq.cuh"
#include "tsb_mmvq.cuh"
#include "tsb_act_layout.cuh"
#include "../../include/tsb_moe.h"

#include <cuda_runtime.h>

#include <cfloat>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace tsb {

int decode_set_wait_limit(unsigned long long ns);   // tsb_decode.cu: that translation unit's copy of the bound
int decode_act_set_wait_limit(unsigned long long ns);   // tsb_decode_act.cu: its copy of the bound

// ================================================================================================ host error state
static thread_local char g_err[512] = "";

// The failure text of this thread's last call that failed in another translation unit of the library (tsb_ep.cu).
void set_last_error(const char* msg) { snprintf(g_err, sizeof g_err, "%s", msg); }

static int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}
static int cuda_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TSB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return TSB_OK;
}
static inline cudaStream_t cs(void* s) { return (cudaStream_t) s; }
static bool aligned(const void* p, size_t a) { return ((uintptr_t) p % a) == 0; }

// The device error word (a bounded wait that gave up records its site): one module global per device, zero when the
// module loads; tsb_device_error reads and clears it.
static __device__ unsigned g_dev_err;

struct DevInfo {
    int sms = 0;
    unsigned* err = nullptr;        // the device address of g_dev_err
    unsigned long long attr = 0;    // kernels whose large shared-memory opt-in is set on this device (bit per kernel)
};
static DevInfo g_dev[64];
static std::mutex g_dev_mu;

// The current device's entry, set up on its first use (the SM count and the error word's address; the lookup may load
// the module, so a process makes its first call on a device outside any stream capture).
static DevInfo* dev_info() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo& I = g_dev[d];
    if (I.sms == 0) {
        void* ep = nullptr;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess ||
            cudaGetSymbolAddress(&ep, g_dev_err) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        I.err = (unsigned*) ep;
        I.sms = sms;
    }
    return &I;
}

// The current device's error word, for the entry points of the other translation units.
unsigned* device_error_word() {
    DevInfo* di = dev_info();
    return di ? di->err : nullptr;
}

// Opt kernel `bit` of this device into `bytes` of dynamic shared memory once (the attribute is per device).
template <typename K>
static int smem_optin(DevInfo* di, int bit, K kern, size_t bytes, const char* what) {
    if (di->attr >> bit & 1ull) return TSB_OK;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) bytes) != cudaSuccess)
        return cuda_status(what);
    std::lock_guard<std::mutex> lk(g_dev_mu);
    di->attr |= 1ull << bit;
    return TSB_OK;
}

// ================================================================================================ formats (host)
static int qk_of(int t) {
    switch (t) {
        case T_Q4_0: case T_Q8_0: return 32;
        case T_Q4_K: case T_Q6_K: case T_IQ3_XXS: case T_IQ3_S: return 256;
        default: return 0;
    }
}
static int bb_of(int t) {
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
static int cpb_of(int t) {
    switch (t) {
        case T_Q4_0: return 2;
        case T_Q8_0: return 4;
        case T_Q4_K: return 16;
        case T_Q6_K: return 32;
        case T_IQ3_XXS: case T_IQ3_S: return 8;
        default: return 0;
    }
}

// ================================================================================================ small kernels
// q8_1 of rows (iq_kernels.cu:1483-1494): one warp per block, lane = value.
__global__ void k_quantize_q8_1(const float* __restrict__ x, BlockQ8_1* __restrict__ y, long long n) {
    const long long i = (long long) blockIdx.x * blockDim.x + threadIdx.x;
    if (i - (threadIdx.x & 31) >= n) return;   // whole warps only (n is a multiple of 32)
    float d, sum;
    const int8_t q = q8_1_warp(x[i], d, sum);
    BlockQ8_1* b = y + i / 32;
    b->qs[i % 32] = q;
    if ((i % 32) == 0) b->ds = make_half2(__float2half(q8_finite(d)), __float2half(q8_finite(sum)));
}

// fp32 router logits: logits[t * ld + o] = W[o] . h[t] (the router GEMV, q36_engine.cu:2106-2131).  Warp per row,
// float4 loads, up to 16 tokens per pass.
__global__ void __launch_bounds__(256) k_router_logits(const float* __restrict__ W, const float* __restrict__ h,
                                                       float* __restrict__ logits, int n_in, int n_out, int n_tok,
                                                       int ld) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); o < n_out; o += warps) {
        const float4* wr = (const float4*) (W + (size_t) o * n_in);
        for (int t0 = 0; t0 < n_tok; t0 += 16) {
            const int nt = min(16, n_tok - t0);
            float acc[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[t] = 0.0f;
            for (int i = lane; i < n_in / 4; i += 32) {
                const float4 w = __ldg(wr + i);
#pragma unroll
                for (int t = 0; t < 16; ++t)
                    if (t < nt) {
                        const float4 x = __ldg((const float4*) (h + (size_t) (t0 + t) * n_in) + i);
                        acc[t] += w.x * x.x + w.y * x.y + w.z * x.z + w.w * x.w;
                    }
            }
#pragma unroll
            for (int t = 0; t < 16; ++t)
                if (t < nt) {
                    const float v = warp_sum(acc[t]);
                    if (lane == 0) logits[(size_t) (t0 + t) * ld + o] = v;
                }
        }
    }
}

// Softmax top-k (native_router.cu:44-95, the same expressions under the reference's fast-math): a warp per token,
// V = n_expert / 32 values a lane, lowest id first among equal probabilities, weights renormalised with the
// 6.103515625e-5 floor.
template <int V>
__global__ void __launch_bounds__(256) k_route_topk(const float* __restrict__ logits, int ld, int32_t* __restrict__ ids,
                                                    float* __restrict__ weights, int n_tok, int K) {
    const int tk = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (tk >= n_tok) return;
    const int lane = threadIdx.x & 31;
    const float* lg = logits + (size_t) tk * ld;
    ids += (size_t) tk * K;
    weights += (size_t) tk * K;
    float values[V];
#pragma unroll
    for (int i = 0; i < V; ++i) values[i] = lg[lane + i * 32];
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
            ids[rank] = expert;
            selected_sum += best;
        }
        if (rank == lane) selected = best;
    }
    selected_sum = fmaxf(warp_sum(selected_sum), 6.103515625e-5f);
    const float inv = frcp_fm(selected_sum);
    if (lane < K) weights[lane] = selected * inv;
}

// Gemma / LFM routing (route_kernel, gemma4/kernels.cu:289-356; that file is built without fast-math): a warp per
// token, PER experts a lane (route_row_warp, tsb_kernels.cuh).
template <int PER>
__global__ void __launch_bounds__(256) k_route_rows(const float* __restrict__ logits, int n_expert, int n_used, int rows,
                                                    int gate, float in_scale, const float* __restrict__ bias,
                                                    const float* __restrict__ escale, int norm, float w_scale,
                                                    int32_t* __restrict__ ids, float* __restrict__ w) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* lg = logits + (size_t) row * n_expert;
    route_row_warp<PER>([&](int e) { return lg[e]; }, n_expert, n_used, gate, in_scale, bias, escale, norm, w_scale,
                        lane, ids + (size_t) row * n_used, w + (size_t) row * n_used);
}

// Decode grouping (k_group, q36_engine.cu:396-422): groups of ascending expert id, entries in entry order.  One CTA;
// an entry's slot is the number of entries before it in (expert, entry) order.
__global__ void __launch_bounds__(1024) k_group(const int32_t* __restrict__ ids, int n_ent, int K, int n_expert,
                                                const uint8_t* blobs, unsigned long long stride,
                                                unsigned long long* grp_ptr, int32_t* grp_start, int32_t* n_groups,
                                                int32_t* ent_dst, int32_t* ent_tok) {
    extern __shared__ int sh[];
    int* cnt = sh;                 // n_expert
    int* off = sh + n_expert;      // n_expert + 1 (exclusive scan)
    int* gidx = off + n_expert + 1;  // n_expert: group index of an expert
    for (int x = threadIdx.x; x < n_expert; x += blockDim.x) cnt[x] = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x) atomicAdd(&cnt[ids[e]], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
        int pos = 0, g = 0;
        for (int x = 0; x < n_expert; ++x) {
            off[x] = pos;
            gidx[x] = g;
            if (cnt[x]) {
                grp_ptr[g] = (unsigned long long) (blobs + (size_t) x * stride);
                grp_start[g] = pos;
                ++g;
            }
            pos += cnt[x];
        }
        off[n_expert] = pos;
        grp_start[g] = pos;
        *n_groups = g;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {
        const int id = ids[e];
        int before = 0;
        for (int e2 = 0; e2 < e; ++e2) before += ids[e2] == id;
        const int p = off[id] + before;
        ent_dst[p] = e;
        ent_tok[p] = e / K;
    }
}

// Combine (k_moe_out / k_moe_out_small, q36_engine.cu:307-332, q36_kernels.cuh:252-290): x += w0 p0 (+ fmaf over the
// picks in order) + sigmoid(sgate) shared; then with wn: h = rms(x) wn and hq = q8_1(h).  One CTA of 1024 per token; the
// squares are summed per 256-thread slot (element s, s + 256, ...) then the 256-wide tree, as the reference.
__global__ void __launch_bounds__(1024) k_combine(float* __restrict__ x, const float* __restrict__ parts,
                                                  const int32_t* __restrict__ prow, const float* __restrict__ wts, int K,
                                                  const float* __restrict__ shared, const float* __restrict__ sgate,
                                                  int sg_stride, const float* __restrict__ wn, float* __restrict__ h,
                                                  BlockQ8_1* __restrict__ hq, int n, float eps) {
    extern __shared__ float vv[];   // n values of x, then 256 partial sums
    float* sh = vv + n;
    __shared__ const float* pk[32];
    const int t = blockIdx.x;
    float* xr = x + (size_t) t * n;
    if ((int) threadIdx.x < K)
        pk[threadIdx.x] = parts + (size_t) (prow ? prow[t * K + threadIdx.x] : t * K + threadIdx.x) * n;
    __syncthreads();
    const float* wr = wts + (size_t) t * K;
    // sigmoid and the mean under the reference engine's fast-math build (CMakeLists.txt:204-207)
    const float gs = sgate ? frcp_fm(1.0f + fexp_fm(-sgate[(size_t) t * sg_stride])) : 1.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float acc = wr[0] * pk[0][i];
        for (int k = 1; k < K; ++k) acc = fmaf(wr[k], pk[k][i], acc);
        if (shared) acc += gs * shared[(size_t) t * n + i];
        const float v = xr[i] + acc;
        xr[i] = v;
        vv[i] = v;
    }
    if (wn == nullptr && h == nullptr) return;
    __syncthreads();
    if (threadIdx.x < 256) {
        float s = 0.0f;
        for (int i = threadIdx.x; i < n; i += 256) s += vv[i] * vv[i];
        sh[threadIdx.x] = s;
    }
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if ((int) threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    const float r = rsqrtf(fdiv_fm(sh[0], (float) n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float hv = __fmul_rn(__fmul_rn(vv[i], r), wn ? wn[i] : 1.0f);
        if (h) h[(size_t) t * n + i] = hv;
        if (hq) {
            float d, sum;
            const int8_t q = q8_1_warp(hv, d, sum);
            BlockQ8_1* b = hq + (size_t) t * (n >> 5) + (i >> 5);
            b->qs[i & 31] = q;
            if ((i & 31) == 0) b->ds = make_half2(__float2half(q8_finite(d)), __float2half(q8_finite(sum)));
        }
    }
}

// The combine without the norm epilogue (the prompt path): the same per-value expressions in the same order as
// k_combine, four values a thread (16-byte loads and stores), 256 threads a token row.
__global__ void __launch_bounds__(256) k_combine_v4(float* __restrict__ x, const float* __restrict__ parts,
                                                    const int32_t* __restrict__ prow, const float* __restrict__ wts,
                                                    int K, const float* __restrict__ shared,
                                                    const float* __restrict__ sgate, int sg_stride, int n) {
    __shared__ const float4* pk[32];
    __shared__ float ws[32];
    const int t = blockIdx.x;
    if ((int) threadIdx.x < K) {
        pk[threadIdx.x] = (const float4*) (parts + (size_t) (prow ? __ldg(prow + t * K + threadIdx.x)
                                                                   : t * K + threadIdx.x) * n);
        ws[threadIdx.x] = __ldg(wts + (size_t) t * K + threadIdx.x);
    }
    __syncthreads();
    const float gs = sgate ? frcp_fm(1.0f + fexp_fm(-sgate[(size_t) t * sg_stride])) : 1.0f;
    float4* xr = (float4*) (x + (size_t) t * n);
    const float4* sr = shared ? (const float4*) (shared + (size_t) t * n) : nullptr;
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        float4 p = __ldcs(pk[0] + i);
        float4 acc = make_float4(ws[0] * p.x, ws[0] * p.y, ws[0] * p.z, ws[0] * p.w);
        for (int k = 1; k < K; ++k) {
            p = __ldcs(pk[k] + i);
            acc = make_float4(fmaf(ws[k], p.x, acc.x), fmaf(ws[k], p.y, acc.y), fmaf(ws[k], p.z, acc.z),
                              fmaf(ws[k], p.w, acc.w));
        }
        if (sr) {
            const float4 v = __ldcs(sr + i);
            acc = make_float4(acc.x + gs * v.x, acc.y + gs * v.y, acc.z + gs * v.z, acc.w + gs * v.w);
        }
        const float4 xv = xr[i];
        xr[i] = make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w);
    }
}

// h = x * rsqrt(mean(x^2) + eps) * wn and hq = q8_1(h), one CTA of 1024 per row: the combine's epilogue alone (the
// reference's k_add_rms_q without the add, q36_kernels.cuh:222-250).
__global__ void __launch_bounds__(1024) k_rms_q8_1(const float* __restrict__ x, const float* __restrict__ wn,
                                                   float* __restrict__ h, BlockQ8_1* __restrict__ hq, int n, float eps) {
    __shared__ float sh[256];
    const float* xr = x + (size_t) blockIdx.x * n;
    if (threadIdx.x < 256) {
        float s = 0.0f;
        for (int i = threadIdx.x; i < n; i += 256) s += xr[i] * xr[i];
        sh[threadIdx.x] = s;
    }
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if ((int) threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    const float r = rsqrtf(fdiv_fm(sh[0], (float) n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float hv = __fmul_rn(__fmul_rn(xr[i], r), wn ? wn[i] : 1.0f);
        if (h) h[(size_t) blockIdx.x * n + i] = hv;
        if (hq) {
            float d, sum;
            const int8_t q = q8_1_warp(hv, d, sum);
            BlockQ8_1* b = hq + (size_t) blockIdx.x * (n >> 5) + (i >> 5);
            b->qs[i & 31] = q;
            if ((i & 31) == 0) b->ds = make_half2(__float2half(q8_finite(d)), __float2half(q8_finite(sum)));
        }
    }
}

// Gemma / LFM ordered weighted sum (moe_sum, gemma4/kernels.cu:358-366): acc[t] += sum_k w[t,k] x[t*K+k].
__global__ void k_moe_sum(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ acc, int n,
                          int n_used) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t first = (size_t) blockIdx.y * n_used;
    float s = 0.0f;
    for (int k = 0; k < n_used; ++k) s += w[first + k] * x[(first + k) * n + i];
    acc[(size_t) blockIdx.y * n + i] += s;
}

// acc[k][i] += x[k][i] * w[k] for k in order (the sums may alias: a thread adds its value of each vector in turn), the
// reference's add_scaled (src/gemma4/kernels.cu:245-249).
__global__ void k_add_scaled(tsb_scaled_rows rows, int count, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    for (int k = 0; k < count; ++k) rows.acc[k][i] = fmaf(rows.x[k][i], rows.w[k], rows.acc[k][i]);
}

// Sum of squares of one row, 256 threads: thread t adds values t, t + 256, ... in order, then a halving tree.
__device__ __forceinline__ float row_sumsq(const float* __restrict__ x, int n, float* red) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) s = fmaf(x[i], x[i], s);
    red[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if ((int) threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    const float v = red[0];
    __syncthreads();
    return v;
}
// The Gemma 4 layer tail after the routed experts (src/gemma4/gemma4.cpp:560-568), one row per CTA:
// cur = rms(moe) * post_moe (+ mlp); out = rms(cur) * post_ffn; r += out; r *= out_scale.  `cur` lives in shared memory.
__global__ void __launch_bounds__(256) k_layer_tail(const float* __restrict__ moe, const float* __restrict__ post_moe,
                                                    const float* __restrict__ mlp, const float* __restrict__ post_ffn,
                                                    float* __restrict__ r, float out_scale, int n, float eps) {
    extern __shared__ float cur[];   // n values, then 256 partial sums
    float* red = cur + n;
    const size_t off = (size_t) blockIdx.x * n;
    const float r1 = rsqrtf(row_sumsq(moe + off, n, red) / (float) n + eps);
    for (int i = threadIdx.x; i < n; i += 256) {
        float v = moe[off + i] * r1 * (post_moe ? post_moe[i] : 1.0f);
        if (mlp) v += mlp[off + i];
        cur[i] = v;
    }
    __syncthreads();
    const float r2 = rsqrtf(row_sumsq(cur, n, red) / (float) n + eps);
    for (int i = threadIdx.x; i < n; i += 256) {
        const float o = cur[i] * r2 * (post_ffn ? post_ffn[i] : 1.0f);
        r[off + i] = (r[off + i] + o) * out_scale;
    }
}

// Test hook: the per-call integer sums and float values of one row against one q8_1 activation.
template <int TY>
__global__ void k_row_calls(const uint8_t* __restrict__ row, const BlockQ8_1* __restrict__ x, int n_calls,
                            int32_t* __restrict__ sumi, float* __restrict__ val, int row_bytes) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = table_bytes<TY>();
    build_tables<TY>(smem);
    uint8_t* rs = smem + TB;
    for (int i = threadIdx.x; i < row_bytes; i += blockDim.x) rs[i] = row[i];
    __syncthreads();
    const IqTab tab = make_tab(smem, threadIdx.x & 31);
    auto src = [&](int blk) { return qb_from_global(x + blk); };
    for (int k = threadIdx.x; k < n_calls; k += blockDim.x) {
        const typename Fmt<TY>::Act a = Fmt<TY>::act(src, k);
        const typename Fmt<TY>::W w = decode_call<TY>(rs, k, tab);
        sumi[k] = Fmt<TY>::sumi(w, a);
        val[k] = Fmt<TY>::apply(w, a);
    }
}

// ================================================================================================ expert launches
// Bench-only phase selection, as the reference's native_expert_set_mode (iq_kernels.hpp:85): 0 both kernels,
// 1 gate/up + activation only, 2 down only.
static int g_phase = 0;
template <int TY, int J>
static int launch_gu_t(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const void* xq, float* h,
                       int act, float limit, cudaStream_t s, DevInfo* di) {
    GuParams p;
    p.g = g;
    p.xq = (const BlockQ8_1*) xq;
    p.n_embd = (int) L->n_embd;
    p.n_ff = (int) L->n_ff;
    p.gu_row = L->gu_row;
    p.up_off = L->up_off;
    p.h = h;
    p.act = act;
    p.limit = limit;
    p.err = di->err;
    const uint32_t sb = (uint32_t) (2 * L->gu_row);
    p.nst = expert_stages<TY>(sb);
    if (p.nst < 1) return fail(TSB_ERR_UNSUPPORTED, "expert gate/up: a %u-byte row pair does not fit", sb);
    const size_t smem = expert_smem<TY>(sb, p.nst);
    auto kern = k_expert_gu<TY, J, 4>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess)
        return cuda_status("expert gate/up: shared memory");
    const long long tasks = (long long) cap_groups * L->n_ff;
    const long long ctas = std::min<long long>((long long) di->sms * 2, (tasks + kWarps - 1) / kWarps);
    kern<<<(unsigned) std::max<long long>(ctas, 1), kWarps * 32, smem, s>>>(p);
    return cuda_status("expert gate/up");
}

template <int TY, int J>
static int launch_down_t(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const float* h, float* out,
                         cudaStream_t s, DevInfo* di) {
    DownParams p;
    p.g = g;
    p.h = h;
    p.n_embd = (int) L->n_embd;
    p.n_ff = (int) L->n_ff;
    p.d_row = L->d_row;
    p.down_off = L->down_off;
    int R = 1;
    while ((R * L->d_row) % 16 != 0) R *= 2;
    const int C = (int) (L->n_ff / qk_of(TY) * cpb_of(TY));
    const int P = C < 32 ? 32 / C : 1;
    while (R < P) R *= 2;
    if (L->n_embd % R != 0) return fail(TSB_ERR_UNSUPPORTED, "down rows: n_embd %% %d", R);
    p.R = R;
    p.out = out;
    p.err = di->err;
    const uint32_t sb = (uint32_t) (R * L->d_row);
    p.nst = expert_stages<TY>(sb);
    if (p.nst < 1) return fail(TSB_ERR_UNSUPPORTED, "expert down: a %u-byte chunk does not fit", sb);
    const size_t smem = expert_smem<TY>(sb, p.nst);
    auto kern = k_expert_down<TY, J, 4>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess)
        return cuda_status("expert down: shared memory");
    const long long tasks = (long long) cap_groups * (L->n_embd / R);
    const long long ctas = std::min<long long>((long long) di->sms * 2, (tasks + kWarps - 1) / kWarps);
    kern<<<(unsigned) std::max<long long>(ctas, 1), kWarps * 32, smem, s>>>(p);
    return cuda_status("expert down");
}

// J = calls per lane for C calls per row (1, 2, 4, 8 instantiated)
template <int TY>
static int launch_gu(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const void* xq, float* h,
                     int act, float limit, cudaStream_t s, DevInfo* di) {
    const int C = (int) (L->n_embd / qk_of(TY) * cpb_of(TY));
    const int J = (C + 31) / 32;
    if (J <= 1) return launch_gu_t<TY, 1>(L, g, cap_groups, xq, h, act, limit, s, di);
    if (J <= 2) return launch_gu_t<TY, 2>(L, g, cap_groups, xq, h, act, limit, s, di);
    if (J <= 4) return launch_gu_t<TY, 4>(L, g, cap_groups, xq, h, act, limit, s, di);
    if (J <= 8) return launch_gu_t<TY, 8>(L, g, cap_groups, xq, h, act, limit, s, di);
    return fail(TSB_ERR_UNSUPPORTED, "gate/up: %d calls per row (at most 256)", C);
}
template <int TY>
static int launch_down(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const float* h, float* out,
                       cudaStream_t s, DevInfo* di) {
    const int C = (int) (L->n_ff / qk_of(TY) * cpb_of(TY));
    if (C < 32 && (C & (C - 1)) != 0) return fail(TSB_ERR_UNSUPPORTED, "down: %d calls per row", C);
    const int J = (C + 31) / 32;
    if (J <= 1) return launch_down_t<TY, 1>(L, g, cap_groups, h, out, s, di);
    if (J <= 2) return launch_down_t<TY, 2>(L, g, cap_groups, h, out, s, di);
    if (J <= 4) return launch_down_t<TY, 4>(L, g, cap_groups, h, out, s, di);
    if (J <= 8) return launch_down_t<TY, 8>(L, g, cap_groups, h, out, s, di);
    return fail(TSB_ERR_UNSUPPORTED, "down: %d calls per row (at most 256)", C);
}

static int gu_dispatch(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const void* xq, float* h,
                       int act, float limit, cudaStream_t s, DevInfo* di) {
    switch (L->gu_type) {
        case T_IQ3_XXS: return launch_gu<T_IQ3_XXS>(L, g, cap_groups, xq, h, act, limit, s, di);
        case T_IQ3_S: return launch_gu<T_IQ3_S>(L, g, cap_groups, xq, h, act, limit, s, di);
        case T_Q4_0: return launch_gu<T_Q4_0>(L, g, cap_groups, xq, h, act, limit, s, di);
        case T_Q8_0: return launch_gu<T_Q8_0>(L, g, cap_groups, xq, h, act, limit, s, di);
        case T_Q4_K: return launch_gu<T_Q4_K>(L, g, cap_groups, xq, h, act, limit, s, di);
        case T_Q6_K: return launch_gu<T_Q6_K>(L, g, cap_groups, xq, h, act, limit, s, di);
        default: return fail(TSB_ERR_UNSUPPORTED, "gate/up type %d", L->gu_type);
    }
}
static int down_dispatch(const tsb_expert_layout* L, const GroupArgs& g, int64_t cap_groups, const float* h, float* out,
                         cudaStream_t s, DevInfo* di) {
    switch (L->d_type) {
        case T_IQ3_XXS: return launch_down<T_IQ3_XXS>(L, g, cap_groups, h, out, s, di);
        case T_IQ3_S: return launch_down<T_IQ3_S>(L, g, cap_groups, h, out, s, di);
        case T_Q4_0: return launch_down<T_Q4_0>(L, g, cap_groups, h, out, s, di);
        case T_Q8_0: return launch_down<T_Q8_0>(L, g, cap_groups, h, out, s, di);
        case T_Q4_K: return launch_down<T_Q4_K>(L, g, cap_groups, h, out, s, di);
        case T_Q6_K: return launch_down<T_Q6_K>(L, g, cap_groups, h, out, s, di);
        default: return fail(TSB_ERR_UNSUPPORTED, "down type %d", L->d_type);
    }
}

}  // namespace tsb

// ================================================================================================ C ABI
using namespace tsb;

extern "C" {

int tsb_moe_abi_version(void) { return TSB_MOE_ABI_VERSION; }

const char* tsb_last_error(void) { return g_err; }

int tsb_device_error(unsigned* code, int clear) {
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    unsigned v = 0;
    if (cudaMemcpy(&v, di->err, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_status("device error");
    if (clear && cudaMemset(di->err, 0, sizeof(unsigned)) != cudaSuccess) return cuda_status("device error: clear");
    if (code) *code = v;
    return TSB_OK;
}

int tsb_set_wait_limit_ns(uint64_t ns) {
    if (ns < 100000ull || ns > 60000000000ull) return fail(TSB_ERR_ARG, "set_wait_limit_ns: 1e5 .. 6e10 ns");
    const unsigned long long v = ns;
    if (cudaMemcpyToSymbol(g_wait_ns, &v, sizeof v) != cudaSuccess) return cuda_status("set_wait_limit_ns");
    if (decode_set_wait_limit(v) != TSB_OK) return cuda_status("set_wait_limit_ns (decode)");
    if (decode_act_set_wait_limit(v) != TSB_OK) return cuda_status("set_wait_limit_ns (decode_act)");
    return TSB_OK;
}

int tsb_type_supported(int ggml_type) { return qk_of(ggml_type) > 0; }

int64_t tsb_row_bytes(int ggml_type, int64_t n) {
    const int qk = qk_of(ggml_type);
    if (qk == 0 || n % qk != 0) return -1;
    return n / qk * bb_of(ggml_type);
}

int tsb_native_expert_layout(int gu_type, int d_type, int64_t n_embd, int64_t n_ff, tsb_expert_layout* L) {
    if (!L) return fail(TSB_ERR_ARG, "layout: null output");
    const int64_t gr = tsb_row_bytes(gu_type, n_embd), dr = tsb_row_bytes(d_type, n_ff);
    if (gr <= 0 || dr <= 0) return fail(TSB_ERR_UNSUPPORTED, "layout: types %d/%d at %lld/%lld", gu_type, d_type,
                                        (long long) n_embd, (long long) n_ff);
    L->gu_type = gu_type;
    L->d_type = d_type;
    L->n_embd = n_embd;
    L->n_ff = n_ff;
    L->gu_row = (uint64_t) gr;
    L->d_row = (uint64_t) dr;
    L->up_off = (uint64_t) (n_ff * gr);
    L->down_off = 2 * L->up_off;
    L->bytes = L->down_off + (uint64_t) (n_embd * dr);
    return TSB_OK;
}

int tsb_native_expert_supported(int gu_type, int d_type, int64_t n_embd, int64_t n_ff) {
    tsb_expert_layout L;
    if (tsb_native_expert_layout(gu_type, d_type, n_embd, n_ff, &L) != TSB_OK) return 0;
    if (L.gu_row % 16 != 0 || n_ff % 32 != 0) return 0;
    const int Cg = (int) (n_embd / qk_of(gu_type) * cpb_of(gu_type));
    const int Cd = (int) (n_ff / qk_of(d_type) * cpb_of(d_type));
    if (Cg > 256 || Cd > 256 || (Cd < 32 && (Cd & (Cd - 1)) != 0)) return 0;
    return 1;
}

uint64_t tsb_native_expert_scratch_bytes(int64_t cap_entries, int64_t n_ff) {
    return (uint64_t) ((cap_entries * n_ff * 4 + 255) & ~255LL);
}

int tsb_quantize_q8_1_rows(const float* x, int64_t n_rows, int64_t n_cols, void* y, void* stream) {
    if (n_rows == 0) return TSB_OK;
    if (!x || !y || n_rows < 0 || n_cols % 32 != 0) return fail(TSB_ERR_ARG, "quantize_q8_1_rows: arguments");
    const long long n = n_rows * n_cols;
    k_quantize_q8_1<<<(unsigned) ((n + 255) / 256), 256, 0, cs(stream)>>>(x, (BlockQ8_1*) y, n);
    return cuda_status("quantize_q8_1_rows");
}

// Many tokens (prefill): 64 tokens x 64 outputs per CTA, each thread 4 x 4 of them, K in smem tiles of 32; every
// logit is the plain fp32 sum over its inputs in order.
__global__ void __launch_bounds__(256) k_router_logits_tiled(const float* __restrict__ W, const float* __restrict__ h,
                                                             float* __restrict__ logits, int n_in, int n_out, int n_tok,
                                                             int ld) {
    __shared__ float xs[32][64 + 4], ws[32][64 + 4];   // [k][token], [k][output]
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int o0 = blockIdx.x * 64, t0 = blockIdx.y * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < n_in; k0 += 32) {
        for (int i = threadIdx.x; i < 64 * 8; i += 256) {   // 64 rows x 8 float4 of K
            const int row = i >> 3, c4 = i & 7;
            float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), wv = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + row < n_tok && k0 + 4 * c4 < n_in) xv = __ldg((const float4*) (h + (size_t) (t0 + row) * n_in + k0) + c4);
            if (o0 + row < n_out && k0 + 4 * c4 < n_in) wv = __ldg((const float4*) (W + (size_t) (o0 + row) * n_in + k0) + c4);
            xs[4 * c4][row] = xv.x; xs[4 * c4 + 1][row] = xv.y; xs[4 * c4 + 2][row] = xv.z; xs[4 * c4 + 3][row] = xv.w;
            ws[4 * c4][row] = wv.x; ws[4 * c4 + 1][row] = wv.y; ws[4 * c4 + 2][row] = wv.z; ws[4 * c4 + 3][row] = wv.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 a = *(const float4*) &xs[k][ty * 4];
            const float4 b = *(const float4*) &ws[k][tx * 4];
            const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = t0 + ty * 4 + i, o = o0 + tx * 4 + j;
            if (t < n_tok && o < n_out) logits[(size_t) t * ld + o] = acc[i][j];
        }
}

int tsb_router_logits_f32(const float* W, const float* h, float* logits, int n_in, int n_out, int n_tok, int ld,
                          void* stream) {
    if (!W || !h || !logits || n_in % 4 != 0 || n_tok < 0 || ld < n_out || !aligned(W, 16) || !aligned(h, 16))
        return fail(TSB_ERR_ARG, "router_logits_f32: arguments (n_in %% 4, 16-byte aligned W and h, ld >= n_out)");
    if (n_tok == 0) return TSB_OK;
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    if (n_tok > 64) {   // prefill: tiled over tokens and outputs
        k_router_logits_tiled<<<dim3((unsigned) ((n_out + 63) / 64), (unsigned) ((n_tok + 63) / 64)), 256, 0,
                                cs(stream)>>>(W, h, logits, n_in, n_out, n_tok, ld);
        return cuda_status("router_logits_f32");
    }
    const int ctas = std::min((n_out + 7) / 8, di->sms * 4);
    k_router_logits<<<ctas, 256, 0, cs(stream)>>>(W, h, logits, n_in, n_out, n_tok, ld);
    return cuda_status("router_logits_f32");
}

int tsb_native_router_topk(const float* logits, int32_t* ids, float* weights, int n_expert, int k, int n_tok, int ld,
                           void* stream) {
    if (!logits || !ids || !weights || n_tok < 0 || k < 1 || k > 32 || n_expert % 32 != 0 || n_expert < 32 ||
        n_expert > 512 || ld < n_expert || k > n_expert)
        return fail(TSB_ERR_ARG, "native_router_topk: 32..512 experts (a multiple of 32), 1..32 picks");
    if (n_tok == 0) return TSB_OK;
    const unsigned grid = (unsigned) ((n_tok + 7) / 8);
    switch (n_expert / 32) {
#define TSB_V(v) case v: k_route_topk<v><<<grid, 256, 0, cs(stream)>>>(logits, ld, ids, weights, n_tok, k); break;
        TSB_V(1) TSB_V(2) TSB_V(3) TSB_V(4) TSB_V(5) TSB_V(6) TSB_V(7) TSB_V(8)
        TSB_V(9) TSB_V(10) TSB_V(11) TSB_V(12) TSB_V(13) TSB_V(14) TSB_V(15) TSB_V(16)
#undef TSB_V
    }
    return cuda_status("native_router_topk");
}

int tsb_route_rows(const float* logits, int n_expert, int n_used, int rows, int gate, float in_scale, const float* bias,
                   const float* escale, int norm, float w_scale, int32_t* ids, float* w, void* stream) {
    if (rows <= 0) return TSB_OK;
    if (!logits || !ids || !w || n_expert > 512 || n_expert < 1 || n_used < 1 || n_used > 32 || n_used > n_expert ||
        (gate != 0 && gate != 1))
        return fail(TSB_ERR_ARG, "route_rows: at most 512 experts and 32 picks, gate 0 (softmax) or 1 (sigmoid)");
    const unsigned grid = (unsigned) ((rows + 7) / 8);
    auto go = [&](auto kern) {
        kern<<<grid, 256, 0, cs(stream)>>>(logits, n_expert, n_used, rows, gate, in_scale, bias, escale, norm, w_scale,
                                           ids, w);
    };
    if (n_expert <= 64) go(k_route_rows<2>);
    else if (n_expert <= 128) go(k_route_rows<4>);
    else if (n_expert <= 256) go(k_route_rows<8>);
    else go(k_route_rows<16>);
    return cuda_status("route_rows");
}

int tsb_moe_group(const int32_t* ids, int n_ent, int K, int n_expert, const void* blobs, uint64_t blob_stride,
                  uint64_t* grp_ptr, int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst, int32_t* ent_tok,
                  void* stream) {
    if (!ids || !grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok || K < 1 || n_ent < 0 || n_ent % K != 0 ||
        n_expert < 1 || n_expert > 4096)
        return fail(TSB_ERR_ARG, "moe_group: arguments");
    const size_t sh = sizeof(int) * (3 * (size_t) n_expert + 1);
    k_group<<<1, 1024, sh, cs(stream)>>>(ids, n_ent, K, n_expert, (const uint8_t*) blobs, blob_stride,
                                         (unsigned long long*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok);
    return cuda_status("moe_group");
}

int tsb_native_expert_grouped(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                              const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                              int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, void* scratch, float* out,
                              void* stream, int64_t grid_groups) {
    (void) grid_groups;   // the results never depend on it (iq_kernels.hpp:72-74); the launch is persistent anyway
    if (cap_groups <= 0 || cap_entries <= 0) return TSB_OK;
    if (!L || !grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok || !x_q8_1 || !scratch || !out)
        return fail(TSB_ERR_ARG, "native_expert_grouped: null argument");
    if (!tsb_native_expert_supported(L->gu_type, L->d_type, L->n_embd, L->n_ff))
        return fail(TSB_ERR_UNSUPPORTED, "native_expert_grouped: types %d/%d at %lld/%lld", L->gu_type, L->d_type,
                    (long long) L->n_embd, (long long) L->n_ff);
    if (L->up_off % 16 || L->down_off % 16 || L->bytes % 16)
        return fail(TSB_ERR_ALIGN, "native_expert_grouped: blob offsets must be multiples of 16 bytes");
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    const GroupArgs g{(const unsigned long long*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok,
                      (int) std::min<int64_t>(cap_groups, INT32_MAX), (int) std::min<int64_t>(cap_entries, INT32_MAX)};
    float* h = (float*) scratch;
    if (g_phase != 2) {
        const int rc = gu_dispatch(L, g, cap_groups, x_q8_1, h, ACT_SWIGLU, INFINITY, cs(stream), di);
        if (rc != TSB_OK) return rc;
    }
    if (g_phase == 1) return TSB_OK;
    return down_dispatch(L, g, cap_groups, h, out, cs(stream), di);
}

int tsb_native_expert_grouped_act(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                                  const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                                  int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, void* scratch,
                                  float* out, int act, float limit, void* stream) {
    if (cap_groups <= 0 || cap_entries <= 0) return TSB_OK;
    if (!L || !grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok || !x_q8_1 || !scratch || !out)
        return fail(TSB_ERR_ARG, "native_expert_grouped_act: null argument");
    if (act < 0 || act > 2) return fail(TSB_ERR_ARG, "native_expert_grouped_act: act 0 SwiGLU, 1 GELU-tanh, 2 clamped");
    if (!tsb_native_expert_supported(L->gu_type, L->d_type, L->n_embd, L->n_ff))
        return fail(TSB_ERR_UNSUPPORTED, "native_expert_grouped_act: unsupported layout");
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    const GroupArgs g{(const unsigned long long*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok,
                      (int) std::min<int64_t>(cap_groups, INT32_MAX), (int) std::min<int64_t>(cap_entries, INT32_MAX)};
    float* h = (float*) scratch;
    if (g_phase != 2) {
        const int rc = gu_dispatch(L, g, cap_groups, x_q8_1, h, act, limit, cs(stream), di);
        if (rc != TSB_OK) return rc;
    }
    if (g_phase == 1) return TSB_OK;
    return down_dispatch(L, g, cap_groups, h, out, cs(stream), di);
}

int tsb_native_expert_set_phase(int phase) {
    if (phase < 0 || phase > 2) return fail(TSB_ERR_ARG, "native_expert_set_phase: 0, 1 or 2");
    g_phase = phase;
    return TSB_OK;
}

int tsb_moe_combine(float* x, const float* parts, const int32_t* prow, const float* wts, int K, const float* shared,
                    const float* sgate, int sg_stride, const float* wn, float* h, void* hq, int n, float eps, int n_tok,
                    void* stream) {
    if (n_tok <= 0) return TSB_OK;
    if (!x || !parts || !wts || K < 1 || K > 32 || n % 32 != 0 || n <= 0)
        return fail(TSB_ERR_ARG, "moe_combine: arguments");
    if (!wn && !h && !hq && n % 4 == 0 && (uintptr_t) x % 16 == 0 && (uintptr_t) parts % 16 == 0 &&
        (!shared || (uintptr_t) shared % 16 == 0)) {   // no norm epilogue: the vectorised combine
        k_combine_v4<<<n_tok, 256, 0, cs(stream)>>>(x, parts, prow, wts, K, shared, sgate, sg_stride, n);
        return cuda_status("moe_combine");
    }
    const size_t sh = sizeof(float) * ((size_t) n + 256);
    if (sh > 200 * 1024) return fail(TSB_ERR_UNSUPPORTED, "moe_combine: n %d too large", n);
    if (sh > 48 * 1024 &&
        cudaFuncSetAttribute(k_combine, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sh) != cudaSuccess)
        return cuda_status("moe_combine: shared memory");
    k_combine<<<n_tok, 1024, sh, cs(stream)>>>(x, parts, prow, wts, K, shared, sgate, sg_stride, wn, h,
                                               (BlockQ8_1*) hq, n, eps);
    return cuda_status("moe_combine");
}

int tsb_rms_norm_q8_1(const float* x, const float* wn, float* h, void* hq, int n, float eps, int n_tok, void* stream) {
    if (n_tok <= 0) return TSB_OK;
    if (!x || n <= 0 || n % 32 != 0 || (!h && !hq)) return fail(TSB_ERR_ARG, "rms_norm_q8_1: arguments");
    k_rms_q8_1<<<n_tok, 1024, 0, cs(stream)>>>(x, wn, h, (BlockQ8_1*) hq, n, eps);
    return cuda_status("rms_norm_q8_1");
}

int tsb_moe_sum(const float* x, const float* w, float* acc, int n, int n_used, int rows, void* stream) {
    if (rows <= 0) return TSB_OK;
    if (!x || !w || !acc || n <= 0 || n_used < 1) return fail(TSB_ERR_ARG, "moe_sum: arguments");
    k_moe_sum<<<dim3((unsigned) ((n + 255) / 256), (unsigned) rows), 256, 0, cs(stream)>>>(x, w, acc, n, n_used);
    return cuda_status("moe_sum");
}

int tsb_add_scaled(const tsb_scaled_rows* rows, int count, int n, void* stream) {
    if (n <= 0) return TSB_OK;
    if (!rows || count < 1 || count > 32) return fail(TSB_ERR_ARG, "add_scaled: 1 to 32 vectors");
    for (int k = 0; k < count; ++k)
        if (!rows->x[k] || !rows->acc[k]) return fail(TSB_ERR_ARG, "add_scaled: null vector %d", k);
    k_add_scaled<<<(unsigned) ((n + 255) / 256), 256, 0, cs(stream)>>>(*rows, count, n);
    return cuda_status("add_scaled");
}

int tsb_moe_layer_tail(const float* moe, const float* post_moe, const float* mlp, const float* post_ffn, float* r,
                       float out_scale, int n, int rows, float eps, void* stream) {
    if (rows <= 0) return TSB_OK;
    if (!moe || !r || n <= 0) return fail(TSB_ERR_ARG, "moe_layer_tail: arguments");
    const size_t sh = sizeof(float) * ((size_t) n + 256);
    if (sh > 200 * 1024) return fail(TSB_ERR_UNSUPPORTED, "moe_layer_tail: n %d too large", n);
    if (sh > 48 * 1024 &&
        cudaFuncSetAttribute(k_layer_tail, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sh) != cudaSuccess)
        return cuda_status("moe_layer_tail: shared memory");
    k_layer_tail<<<(unsigned) rows, 256, sh, cs(stream)>>>(moe, post_moe, mlp, post_ffn, r, out_scale, n, eps);
    return cuda_status("moe_layer_tail");
}

// ------------------------------------------------------------------------------------------------ prefill
int tsb_moe_dispatch(const int32_t* ids, int n_ent, int K, int n_expert, int32_t* bounds, int32_t* row_ent,
                     int32_t* row_tok, int32_t* rinv, void* stream) {
    if (n_ent < 0 || K < 1 || n_expert < 1 || n_expert > 1024 || !bounds)
        return fail(TSB_ERR_ARG, "moe_dispatch: arguments");
    if (n_ent > 0 && (!ids || !row_ent || !row_tok || !rinv)) return fail(TSB_ERR_ARG, "moe_dispatch: null argument");
    k_dispatch_count<<<1, 1024, 0, cs(stream)>>>(ids, n_ent, n_expert, bounds, rinv);
    if (n_ent > 0) k_dispatch_scatter<<<n_expert, 1024, 0, cs(stream)>>>(ids, n_ent, K, bounds, row_ent, row_tok, rinv);
    return cuda_status("moe_dispatch");
}

}  // extern "C"
// ------------------------------------------------------------------------------------ prefill on the tensor cores
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn tmap_encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn) f;
        cudaGetLastError();
    });
    return fn;
}
// A 2-D map over [h][w] elements (row pitch `pitch` bytes) read in boxes of box_h x box_w; loads past the extent read 0.
static int tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t w, uint64_t h, uint64_t pitch,
                   uint32_t box_w, uint32_t box_h, CUtensorMapSwizzle sw) {
    EncodeTiledFn enc = tmap_encoder();
    if (!enc) return fail(TSB_ERR_CUDA, "prefill: cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[2] = {w, h};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_w, box_h};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TSB_ERR_CUDA, "prefill: tensor map (%llu x %llu, pitch %llu): error %d",
                                       (unsigned long long) h, (unsigned long long) w, (unsigned long long) pitch, (int) r);
    return TSB_OK;
}

template <int MODE, int WT>
static int mq_launch_t(const MqParams& pp, const MmqView& xa, cudaStream_t s, DevInfo* di) {
    using LY = MqLayout<WT>;
    auto kern = k_mmq<MODE, WT>;
    const int wi = WT == T_Q4_0 ? 0 : WT == T_Q8_0 ? 1 : WT == T_Q4_K ? 2 : WT == T_Q6_K ? 3 : WT == T_IQ3_XXS ? 4 : 5;
    int rc = smem_optin(di, 32 + wi * 2 + MODE, kern, LY::kSmem, "prefill: shared memory");
    if (rc != TSB_OK) return rc;
    CUtensorMap tx, tdx, tsx;
    rc = tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xa.codes, (uint64_t) pp.K, (uint64_t) pp.n_rows, (uint64_t) pp.K,
                 kMqBK, kMqBM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == TSB_OK)
        rc = tmap_2d(&tdx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xa.d, (uint64_t) (pp.K / 32), (uint64_t) pp.n_rows,
                     (uint64_t) xa.ldS * 4, kMqBlk, kMqBM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc == TSB_OK)
        rc = tmap_2d(&tsx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xa.s, (uint64_t) (pp.K / 32), (uint64_t) pp.n_rows,
                     (uint64_t) xa.ldS * 4, kMqBlk, kMqBM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != TSB_OK) return rc;
    kern<<<di->sms, kMqThreads, LY::kSmem, s>>>(tx, tdx, tsx, pp);
    return cuda_status(MODE == MQ_GU ? "moe_prefill_gu" : "moe_prefill_down");
}
template <int MODE>
static int mq_launch(int wt, const MqParams& pp, const MmqView& xa, cudaStream_t s, DevInfo* di) {
    switch (wt) {
        case T_Q4_0: return mq_launch_t<MODE, T_Q4_0>(pp, xa, s, di);
        case T_Q8_0: return mq_launch_t<MODE, T_Q8_0>(pp, xa, s, di);
        case T_Q4_K: return mq_launch_t<MODE, T_Q4_K>(pp, xa, s, di);
        case T_Q6_K: return mq_launch_t<MODE, T_Q6_K>(pp, xa, s, di);
        case T_IQ3_XXS: return mq_launch_t<MODE, T_IQ3_XXS>(pp, xa, s, di);
        case T_IQ3_S: return mq_launch_t<MODE, T_IQ3_S>(pp, xa, s, di);
        default: return fail(TSB_ERR_UNSUPPORTED, "moe_prefill: weight type %d", wt);
    }
}

extern "C" {

uint64_t tsb_mmq_act_bytes(int64_t rows, int64_t K) {
    if (rows < 0 || K <= 0 || K % 32) return 0;
    return mmq_act_bytes(rows, K);
}

int tsb_mmq_quantize(const float* x, int64_t ld_x, const int32_t* row_src, int n_rows, int K, void* act, void* stream) {
    if (n_rows == 0) return TSB_OK;
    if (!x || !act || n_rows < 0 || K <= 0 || K % 32 || ld_x < K) return fail(TSB_ERR_ARG, "mmq_quantize: arguments");
    if ((uintptr_t) act % 256) return fail(TSB_ERR_ALIGN, "mmq_quantize: the activation buffer must be 256-byte aligned");
    if ((uintptr_t) x % 16 || ld_x % 4) return fail(TSB_ERR_ALIGN, "mmq_quantize: 16-byte aligned rows");
    const MmqView v = mmq_view(act, n_rows, K);
    k_mmq_quantize<<<(unsigned) n_rows, 256, 0, cs(stream)>>>(x, ld_x, row_src, n_rows, K, v.codes, v.d, v.s, v.ldS);
    return cuda_status("mmq_quantize");
}

int tsb_mmq_from_q8_1(const void* x_q8_1, const int32_t* row_src, int n_rows, int K, void* act, void* stream) {
    if (n_rows == 0) return TSB_OK;
    if (!x_q8_1 || !act || n_rows < 0 || K <= 0 || K % 32) return fail(TSB_ERR_ARG, "mmq_from_q8_1: arguments");
    if ((uintptr_t) act % 256 || (uintptr_t) x_q8_1 % 4) return fail(TSB_ERR_ALIGN, "mmq_from_q8_1: alignment");
    const MmqView v = mmq_view(act, n_rows, K);
    const long long warps = (long long) n_rows * (K / 32);
    k_mmq_from_q8_1<<<(unsigned) ((warps + 7) / 8), 256, 0, cs(stream)>>>((const BlockQ8_1*) x_q8_1, row_src, n_rows, K,
                                                                           v.codes, v.d, v.s, v.ldS);
    return cuda_status("mmq_from_q8_1");
}

}  // extern "C"

static int mq_check(const tsb_expert_layout* L, const void* blobs, uint64_t blob_stride, int n_groups, int n_rows,
                    int mode) {
    if (!L || !blobs || n_rows < 0 || n_groups < 1 || n_groups > kMqMaxGroups)
        return fail(TSB_ERR_ARG, "moe_prefill: arguments (1 .. %d groups)", kMqMaxGroups);
    const int t = mode == MQ_GU ? L->gu_type : L->d_type;
    if (t != T_Q4_0 && t != T_Q8_0 && t != T_Q4_K && t != T_Q6_K && t != T_IQ3_XXS && t != T_IQ3_S)
        return fail(TSB_ERR_UNSUPPORTED, "moe_prefill: weight type %d (Q4_0, Q8_0, Q4_K, Q6_K, IQ3_XXS, IQ3_S)", t);
    if (L->n_embd % 64 || L->n_ff % 64 || L->n_embd < 128 || L->n_ff < 64)
        return fail(TSB_ERR_UNSUPPORTED, "moe_prefill: n_embd a multiple of 64 (>= 128), n_ff a multiple of 64");
    const int64_t k = mode == MQ_GU ? L->n_embd : L->n_ff;
    if (t != T_Q4_0 && t != T_Q8_0 && k % 256)
        return fail(TSB_ERR_UNSUPPORTED, "moe_prefill: K-quant / i-quant rows of 256-value blocks");
    // rows are read in aligned words: 4-byte (Q4_0, Q8_0: an even number of blocks), 16-byte (Q4_K), 2-byte (the rest)
    const int64_t row = mode == MQ_GU ? L->gu_row : L->d_row;
    const int64_t ra = (t == T_Q4_0 || t == T_Q8_0) ? 4 : t == T_Q4_K ? 16 : 2;
    if ((uintptr_t) blobs % 16 || blob_stride % 16 || L->up_off % 16 || L->down_off % 16 || row % ra)
        return fail(TSB_ERR_ALIGN, "moe_prefill: blob alignment (rows of %lld bytes)", (long long) row);
    return TSB_OK;
}

static MqParams mq_params(const tsb_expert_layout* L, int mode, const void* blobs, uint64_t blob_stride,
                          const int32_t* bounds, int n_groups, int n_rows) {
    MqParams pp{};
    pp.bounds = bounds;
    pp.n_groups = n_groups;
    pp.n_rows = n_rows;
    pp.blobs = (const uint8_t*) blobs;
    pp.blob_stride = blob_stride;
    if (mode == MQ_GU) {
        pp.w_off = 0;
        pp.up_off = L->up_off;
        pp.w_row = (uint32_t) L->gu_row;
        pp.K = (int) L->n_embd;
        pp.N = (int) L->n_ff;
    } else {
        pp.w_off = L->down_off;
        pp.w_row = (uint32_t) L->d_row;
        pp.K = (int) L->n_ff;
        pp.N = (int) L->n_embd;
    }
    pp.act = ACT_SWIGLU;
    pp.limit = INFINITY;
    return pp;
}

static int mq_run(const tsb_expert_layout* L, int mode, const void* blobs, uint64_t blob_stride, const int32_t* bounds,
                  int n_groups, int n_rows, const void* x_act, void* h_act, float* out, int act, float limit,
                  int32_t* dbg, cudaStream_t s) {
    int rc = mq_check(L, blobs, blob_stride, n_groups, n_rows, mode);
    if (rc != TSB_OK) return rc;
    if (n_rows == 0) return TSB_OK;
    if (!x_act || (mode == MQ_GU ? !h_act : !out) || (bounds == nullptr && n_groups != 1) || act < 0 || act > 2)
        return fail(TSB_ERR_ARG, "moe_prefill: arguments");
    if ((uintptr_t) x_act % 256 || (mode == MQ_GU ? (uintptr_t) h_act % 256 : (uintptr_t) out % 16))
        return fail(TSB_ERR_ALIGN, "moe_prefill: activation buffers 256-byte aligned, outputs 16-byte aligned");
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    MqParams pp = mq_params(L, mode, blobs, blob_stride, bounds, n_groups, n_rows);
    pp.err = di->err;
    pp.dbg = dbg;
    pp.act = act;
    pp.limit = limit;
    const MmqView xa = mmq_view(x_act, n_rows, pp.K);
    if (mode == MQ_GU) {
        const MmqView ha = mmq_view(h_act, n_rows, pp.N);
        pp.hc = ha.codes;
        pp.hd = ha.d;
        pp.hs = ha.s;
        pp.ldh = ha.ldS;
        return mq_launch<MQ_GU>(L->gu_type, pp, xa, s, di);
    }
    pp.D = out;
    pp.drow = nullptr;
    pp.ld_d = pp.N;
    return mq_launch<MQ_DOWN>(L->d_type, pp, xa, s, di);
}

extern "C" {

int tsb_moe_prefill_gu(const tsb_expert_layout* L, const void* blobs, uint64_t blob_stride, const int32_t* bounds,
                       int n_groups, int n_rows, const void* x_act, void* h_act, int act, float limit, void* stream) {
    return mq_run(L, MQ_GU, blobs, blob_stride, bounds, n_groups, n_rows, x_act, h_act, nullptr, act, limit, nullptr,
                  cs(stream));
}

int tsb_moe_prefill_down(const tsb_expert_layout* L, const void* blobs, uint64_t blob_stride, const int32_t* bounds,
                         int n_groups, int n_rows, const void* h_act, float* out, void* stream) {
    return mq_run(L, MQ_DOWN, blobs, blob_stride, bounds, n_groups, n_rows, h_act, nullptr, out, ACT_SWIGLU, INFINITY,
                  nullptr, cs(stream));
}

int tsb_mmq_product(const void* w, int ggml_type, int64_t w_rows, int64_t w_cols, uint64_t stride, int n,
                    const void* x_act, const int32_t* bounds, const int32_t* ids, int64_t total_rows, float* dst,
                    int64_t ld_dst, void* stream) {
    if (total_rows == 0 || n == 0) return TSB_OK;
    if (total_rows < 0 || total_rows > INT32_MAX || n < 0 || w_rows < 1 || w_rows > INT32_MAX || w_cols < 1 ||
        w_cols > INT32_MAX || !dst || ld_dst < w_rows || (n > 1 && !bounds))
        return fail(TSB_ERR_ARG, "mmq_product: arguments");
    if (ld_dst % 4) return fail(TSB_ERR_ALIGN, "mmq_product: ld_dst a multiple of 4 floats");
    // one expert blob per matrix: its rows are the "down" rows of a layout with n_ff = w_cols, n_embd = w_rows
    tsb_expert_layout L{};
    L.gu_type = ggml_type;
    L.d_type = ggml_type;
    L.n_embd = w_rows;
    L.n_ff = w_cols;
    L.gu_row = 0;
    L.d_row = (uint64_t) tsb_row_bytes(ggml_type, w_cols);
    L.up_off = 0;
    L.down_off = 0;
    L.bytes = L.d_row * (uint64_t) w_rows;
    if (L.d_row == 0) return fail(TSB_ERR_UNSUPPORTED, "mmq_product: weight type %d", ggml_type);
    int rc = mq_check(&L, w, stride, n, (int) total_rows, MQ_DOWN);
    if (rc != TSB_OK) return rc;
    if (!x_act) return fail(TSB_ERR_ARG, "mmq_product: null activations");
    if ((uintptr_t) x_act % 256 || (uintptr_t) dst % 16) return fail(TSB_ERR_ALIGN, "mmq_product: buffer alignment");
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    MqParams pp = mq_params(&L, MQ_DOWN, w, stride, bounds, n, (int) total_rows);
    pp.err = di->err;
    pp.dbg = nullptr;
    pp.D = dst;
    pp.drow = ids;
    pp.ld_d = ld_dst;
    const MmqView xa = mmq_view(x_act, total_rows, pp.K);
    return mq_launch<MQ_DOWN>(ggml_type, pp, xa, cs(stream), di);
}

}  // extern "C"

// ------------------------------------------------------------------------------------ many small matrix-vector products
template <int TY, int J>
static int mv_launch_t(const MvArgs& a, int count, cudaStream_t s, DevInfo* di) {
    constexpr int TB = table_bytes<TY>();
    auto kern = k_mmvq<TY, J>;
    if (TB > 48 * 1024) {   // the IQ3 tables: a per-device opt-in, bits 48..55
        const int bit = 48 + (TY == T_IQ3_S ? 4 : 0) + (J == 1 ? 0 : J == 2 ? 1 : J == 4 ? 2 : 3);
        const int rc = smem_optin(di, bit, kern, TB, "mmvq: shared memory");
        if (rc != TSB_OK) return rc;
    }
    const long long want = (2LL * di->sms + count - 1) / count;
    const long long gx = std::max<long long>(1, std::min<long long>((a.n_out + 7) / 8, want));
    kern<<<dim3((unsigned) gx, (unsigned) count), 256, TB, s>>>(a);
    return cuda_status("mmvq");
}
template <int TY>
static int mv_launch(const MvArgs& a, int count, cudaStream_t s, DevInfo* di) {
    const int C = a.n_in / qk_of(TY) * cpb_of(TY);
    if (C <= 32) return mv_launch_t<TY, 1>(a, count, s, di);
    if (C <= 64) return mv_launch_t<TY, 2>(a, count, s, di);
    if (C <= 128) return mv_launch_t<TY, 4>(a, count, s, di);
    if (C <= 256) return mv_launch_t<TY, 8>(a, count, s, di);
    return fail(TSB_ERR_UNSUPPORTED, "mmvq: %d calls per row (at most 256)", C);
}
static int mv_run(int t, MvArgs& a, int count, int n_in, int n_out, cudaStream_t s) {
    if (count < 0 || count > kMvMax || n_in <= 0 || n_out < 0)
        return fail(TSB_ERR_ARG, "mmvq: 0..%d matrices, positive n_in", kMvMax);
    if (qk_of(t) == 0) return fail(TSB_ERR_UNSUPPORTED, "mmvq: weight type %d", t);
    if (n_in % qk_of(t) || n_in % 32) return fail(TSB_ERR_UNSUPPORTED, "mmvq: rows of whole %d-value blocks", qk_of(t));
    if (count == 0 || n_out == 0) return TSB_OK;
    DevInfo* di = dev_info();
    if (!di) return fail(TSB_ERR_CUDA, "no CUDA device");
    a.n_in = n_in;
    a.n_out = n_out;
    a.row_bytes = (uint32_t) (n_in / qk_of(t) * bb_of(t));
    switch (t) {
        case T_Q4_0: return mv_launch<T_Q4_0>(a, count, s, di);
        case T_Q8_0: return mv_launch<T_Q8_0>(a, count, s, di);
        case T_Q4_K: return mv_launch<T_Q4_K>(a, count, s, di);
        case T_Q6_K: return mv_launch<T_Q6_K>(a, count, s, di);
        case T_IQ3_XXS: return mv_launch<T_IQ3_XXS>(a, count, s, di);
        case T_IQ3_S: return mv_launch<T_IQ3_S>(a, count, s, di);
        default: return fail(TSB_ERR_UNSUPPORTED, "mmvq: weight type %d", t);
    }
}

extern "C" {

int tsb_mmvq_supported(int ggml_type) { return qk_of(ggml_type) != 0 ? 1 : 0; }

int tsb_mmvq_run_slots(int ggml_type, const tsb_mmvq_slots* slots, int count, int n_in, int n_out, void* stream) {
    if (!slots) return fail(TSB_ERR_ARG, "mmvq_run_slots: null slots");
    MvArgs a{};
    for (int i = 0; i < count && i < kMvMax; ++i) {
        if (!slots->w[i] || !slots->x[i] || !slots->y[i]) return fail(TSB_ERR_ARG, "mmvq_slots: null pointer in slot %d", i);
        if ((uintptr_t) slots->w[i] % 2 || (uintptr_t) slots->x[i] % 4 || (uintptr_t) slots->y[i] % 4)
            return fail(TSB_ERR_ALIGN, "mmvq_slots: slot %d alignment", i);
        a.w[i] = slots->w[i];
        a.x[i] = slots->x[i];
        a.y[i] = slots->y[i];
    }
    a.by_ids = 0;
    return mv_run(ggml_type, a, count, n_in, n_out, cs(stream));
}

int tsb_mmvq_run_ids(int ggml_type, const tsb_mmvq_ids* m, int count, int n_in, int n_out, void* stream) {
    if (!m || !m->table || !m->ids || !m->x || !m->y || m->x_every < 1)
        return fail(TSB_ERR_ARG, "mmvq_ids: arguments");
    if (m->offset % 2 || (uintptr_t) m->x % 4 || m->x_stride % 4 || (uintptr_t) m->y % 4)
        return fail(TSB_ERR_ALIGN, "mmvq_ids: alignment");
    MvArgs a{};
    a.by_ids = 1;
    a.table = m->table;
    a.ids = m->ids;
    a.offset = m->offset;
    a.xb = (const uint8_t*) m->x;
    a.x_stride = m->x_stride;
    a.x_every = m->x_every;
    a.yb = m->y;
    a.y_stride = m->y_stride;
    return mv_run(ggml_type, a, count, n_in, n_out, cs(stream));
}

int tsb_debug_mmq_block_sums(const tsb_expert_layout* L, int mode, const void* blob, int n_rows, const void* x_act,
                             void* h_act, float* out, int32_t* sums, void* stream) {
    if (!sums || (mode != MQ_GU && mode != MQ_DOWN)) return fail(TSB_ERR_ARG, "debug_mmq_block_sums: arguments");
    return mq_run(L, mode, blob, L ? L->bytes : 0, nullptr, 1, n_rows, x_act, h_act, out, ACT_SWIGLU, INFINITY, sums,
                  cs(stream));
}

}  // extern "C"

extern "C" {
// ------------------------------------------------------------------------------------ no-allocation grouped experts
// tsb_native_expert_grouped with its scratch (the entries' hidden vectors, fp32 [cap_entries][n_ff]) in a fixed
// device array of this library instead of a caller buffer.  The array is zero when the module loads and needs no
// clearing between calls (the gate/up kernel writes every entry the down kernel then reads).  A bounded wait that gives
// up records its site in the device error word every entry point shares (tsb_device_error).  The cached addresses
// belong to the module instance of the device's current context: they do not survive a cudaDeviceReset.
// One copy per device: two calls in flight at the same time on one device (other streams, other threads) race on it.
static constexpr size_t kNoAllocScratchBytes = (size_t) 1 << 20;   // 1 MiB: 128 entries x n_ff 2048 fp32
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDev {
    bool ready = false;
    void* scratch = nullptr;
};
static NoAllocDev g_noalloc[64];
static std::mutex g_noalloc_mu;

// The current device's addresses of the fixed arrays, looked up once per device (cudaGetSymbolAddress; the first
// call may load the module, so it is made outside any stream capture).
static int noalloc_dev(NoAllocDev*& out) {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) {
        cudaGetLastError();
        return fail(TSB_ERR_CUDA, "native_expert_grouped_noalloc: no CUDA device");
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDev& N = g_noalloc[d];
    if (!N.ready) {
        void* sp = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&sp, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(TSB_ERR_CUDA, "native_expert_grouped_noalloc: device %d: %s", d, cudaGetErrorString(e));
        }
        N.scratch = sp;
        N.ready = true;
    }
    out = &N;
    return TSB_OK;
}

int tsb_native_expert_grouped_noalloc(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                                      const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                                      int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, float* out,
                                      void* stream) {
    if (cap_groups <= 0 || cap_entries <= 0) return TSB_OK;
    if (!L || !grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok || !x_q8_1 || !out)
        return fail(TSB_ERR_ARG, "native_expert_grouped_noalloc: null argument");
    if (!tsb_native_expert_supported(L->gu_type, L->d_type, L->n_embd, L->n_ff))
        return fail(TSB_ERR_UNSUPPORTED, "native_expert_grouped_noalloc: types %d/%d at %lld/%lld", L->gu_type,
                    L->d_type, (long long) L->n_embd, (long long) L->n_ff);
    if (L->up_off % 16 || L->down_off % 16 || L->bytes % 16)
        return fail(TSB_ERR_ALIGN, "native_expert_grouped_noalloc: blob offsets must be multiples of 16 bytes");
    const uint64_t need = tsb_native_expert_scratch_bytes(cap_entries, L->n_ff);
    if (need > kNoAllocScratchBytes)
        return fail(TSB_ERR_WORKSPACE,
                    "native_expert_grouped_noalloc: %lld entries x n_ff %lld need %llu bytes of scratch, more than the "
                    "fixed %zu; use tsb_native_expert_grouped with a caller buffer",
                    (long long) cap_entries, (long long) L->n_ff, (unsigned long long) need, kNoAllocScratchBytes);
    NoAllocDev* N = nullptr;
    const int rc = noalloc_dev(N);
    if (rc != TSB_OK) return rc;
    DevInfo* di = dev_info();   // the SM count and the device error word tsb_device_error reads
    if (!di) return fail(TSB_ERR_CUDA, "native_expert_grouped_noalloc: no CUDA device");
    const GroupArgs g{(const unsigned long long*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok,
                      (int) std::min<int64_t>(cap_groups, INT32_MAX), (int) std::min<int64_t>(cap_entries, INT32_MAX)};
    float* h = (float*) N->scratch;
    const int r1 = gu_dispatch(L, g, cap_groups, x_q8_1, h, ACT_SWIGLU, INFINITY, cs(stream), di);
    if (r1 != TSB_OK) return r1;
    return down_dispatch(L, g, cap_groups, h, out, cs(stream), di);
}

int tsb_debug_row_calls(int ggml_type, const void* row, const void* x_q8_1, int64_t n, int32_t* sumi, float* val,
                        void* stream) {
    const int64_t rb = tsb_row_bytes(ggml_type, n);
    if (rb <= 0 || !row || !x_q8_1 || !sumi || !val) return fail(TSB_ERR_ARG, "debug_row_calls: arguments");
    const int calls = (int) (n / qk_of(ggml_type) * cpb_of(ggml_type));
    auto go = [&](auto kern, int tb) {
        const size_t sh = (size_t) tb + (size_t) rb;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sh);
        kern<<<1, 256, sh, cs(stream)>>>((const uint8_t*) row, (const BlockQ8_1*) x_q8_1, calls, sumi, val, (int) rb);
    };
    switch (ggml_type) {
        case T_IQ3_XXS: go(k_row_calls<T_IQ3_XXS>, table_bytes<T_IQ3_XXS>()); break;
        case T_IQ3_S: go(k_row_calls<T_IQ3_S>, table_bytes<T_IQ3_S>()); break;
        case T_Q4_0: go(k_row_calls<T_Q4_0>, 0); break;
        case T_Q8_0: go(k_row_calls<T_Q8_0>, 0); break;
        case T_Q4_K: go(k_row_calls<T_Q4_K>, 0); break;
        case T_Q6_K: go(k_row_calls<T_Q6_K>, 0); break;
        default: return fail(TSB_ERR_UNSUPPORTED, "debug_row_calls: type %d", ggml_type);
    }
    return cuda_status("debug_row_calls");
}

}  // extern "C"
