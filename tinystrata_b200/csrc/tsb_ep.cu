// tsb_ep.cu - expert-parallel prefill over NCCL (one process per GPU of a node): the glue around the tensor-core
// grouped experts as kernels, and a host driver with one synchronisation per step (the exchanged row counts).
//
// Per step, for T tokens of this rank split into M micro-batches (token slices):
//   k_ep_plan    (1 CTA)  per micro-batch and destination rank: which tokens go there (a token goes to a rank once,
//                         whatever number of its picks live there), in (micro-batch, rank, token) order -> send_pos
//                         [T][G] (slot of token t in rank d's rows, -1 none) and the counts [G][M];
//   k_ep_pack             the q8_1 row of each slot, its picks' local expert ids on that rank (-1 for picks elsewhere)
//                         and their weights (0 elsewhere);
//   counts exchange       NCCL send/recv of the [M] counts per peer, copied to the host: the one synchronisation;
//   dispatch exchange     per micro-batch the rows, ids and weights to their ranks (the communicator's stream);
//   local experts         per micro-batch on the caller's stream as its rows arrive: the prompt-path dispatch of the
//                         received picks (tsb_moe_dispatch), k_ep_rows_to_mmq (the received q8_1 rows into the
//                         tensor-core layout in expert order), grouped gate/up and down (tsb_moe_prefill_gu / _down),
//                         k_ep_row_sum (each received row's weighted partial sum of its picks, fp32 or bf16);
//   return exchange      per micro-batch the partial rows back to the ranks they came from, in the slots' order;
//   k_ep_finish           per token: out (+)= the partials of the ranks it went to, in rank order, + the gated shared
//                         expert row.
// Micro-batch m + 1's dispatch exchange runs while micro-batch m computes, and m's return while m + 1 computes.
#include "tsb_act_layout.cuh"
#include "tsb_device.cuh"
#include "../../include/tsb_moe.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>

namespace tsb {

void set_last_error(const char* msg);   // tsb_moe.cu: the text tsb_last_error returns

namespace {

constexpr int kEpMaxWorld = 8;   // the GPUs of one node
constexpr int kEpMaxMb = 4;

int efail(int code, const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    set_last_error(b);
    return code;
}

// ------------------------------------------------------------------------------------------------------- kernels
__device__ __forceinline__ unsigned ep_token_mask(const int32_t* __restrict__ ids, int K, int E, int G, int per,
                                                  int cyclic) {
    unsigned m = 0;
    for (int k = 0; k < K; ++k) {
        const int id = __ldg(ids + k);
        if (id < 0 || id >= E) continue;
        m |= 1u << (cyclic ? id % G : id / per);
    }
    return m;
}

// One CTA: per micro-batch the destination ranks' token slots.  Each thread owns a contiguous run of the slice's
// tokens; a block-wide exclusive scan of the per-rank counts gives each thread's first slot per rank, so the slots of
// rank d are the slice's tokens bound for d in ascending order.  Slot index = the micro-batch's base (the slots of
// earlier micro-batches) + the counts of lower ranks in this micro-batch + the rank among d's tokens.
__global__ void __launch_bounds__(1024) k_ep_plan(const int32_t* __restrict__ ids, int T, int K, int E, int G, int per,
                                                  int cyclic, int n_mb, int32_t* __restrict__ send_pos,
                                                  int32_t* __restrict__ counts) {
    __shared__ int wsum[32][kEpMaxWorld];
    __shared__ int tot[kEpMaxWorld];
    __shared__ int region;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) region = 0;
    __syncthreads();
    for (int mb = 0; mb < n_mb; ++mb) {
        const int t0 = (int) ((long long) T * mb / n_mb), t1 = (int) ((long long) T * (mb + 1) / n_mb);
        const int n = t1 - t0, chunk = (n + 1023) / 1024;
        const int a = t0 + min(n, tid * chunk), b = t0 + min(n, (tid + 1) * chunk);
        int cnt[kEpMaxWorld], excl[kEpMaxWorld];
#pragma unroll
        for (int d = 0; d < kEpMaxWorld; ++d) cnt[d] = 0;
        for (int t = a; t < b; ++t) {
            const unsigned m = ep_token_mask(ids + (size_t) t * K, K, E, G, per, cyclic);
#pragma unroll
            for (int d = 0; d < kEpMaxWorld; ++d) cnt[d] += (m >> d) & 1u;
        }
#pragma unroll
        for (int d = 0; d < kEpMaxWorld; ++d) {
            int v = cnt[d];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            excl[d] = v - cnt[d];
            if (lane == 31) wsum[warp][d] = v;
        }
        __syncthreads();
        if (tid < kEpMaxWorld) {
            int s = 0;
            for (int w = 0; w < 32; ++w) {
                const int c = wsum[w][tid];
                wsum[w][tid] = s;
                s += c;
            }
            tot[tid] = s;
        }
        __syncthreads();
        int pos[kEpMaxWorld];
        int acc = region;
#pragma unroll
        for (int d = 0; d < kEpMaxWorld; ++d) {
            pos[d] = acc + wsum[warp][d] + excl[d];
            acc += tot[d];
        }
        for (int t = a; t < b; ++t) {
            const unsigned m = ep_token_mask(ids + (size_t) t * K, K, E, G, per, cyclic);
#pragma unroll
            for (int d = 0; d < kEpMaxWorld; ++d) {
                if (d >= G) break;
                int p = -1;
                if ((m >> d) & 1u) p = pos[d]++;
                send_pos[(size_t) t * G + d] = p;
            }
        }
        __syncthreads();
        if (tid < G) counts[tid * n_mb + mb] = tot[tid];
        if (tid == 0) {
            int s = 0;
            for (int d = 0; d < G; ++d) s += tot[d];
            region += s;
        }
        __syncthreads();
    }
}

// One warp per token: its q8_1 row into each of its slots (16-byte words when the row size allows), and per slot the
// picks' local expert ids on that rank (-1 for picks on other ranks) and weights (0 there).
__global__ void __launch_bounds__(256) k_ep_pack(const uint8_t* __restrict__ xq, int RB, const int32_t* __restrict__ ids,
                                                 const float* __restrict__ w, int T, int K, int E, int G, int per,
                                                 int cyclic, const int32_t* __restrict__ send_pos,
                                                 uint8_t* __restrict__ rows, int32_t* __restrict__ sids,
                                                 float* __restrict__ sw) {
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int id = lane < K ? __ldg(ids + (size_t) t * K + lane) : -1;
    const float wv = lane < K ? __ldg(w + (size_t) t * K + lane) : 0.0f;
    const bool valid = id >= 0 && id < E;
    const int dest = valid ? (cyclic ? id % G : id / per) : -1;
    const int loc = valid ? (cyclic ? id / G : id - dest * per) : -1;
    for (int d = 0; d < G; ++d) {
        const int p = __ldg(send_pos + (size_t) t * G + d);
        if (p < 0) continue;
        if ((RB & 15) == 0) {
            const uint4* s = (const uint4*) (xq + (size_t) t * RB);
            uint4* o = (uint4*) (rows + (size_t) p * RB);
            for (int i = lane; i < RB / 16; i += 32) o[i] = __ldg(s + i);
        } else {
            const uint32_t* s = (const uint32_t*) (xq + (size_t) t * RB);
            uint32_t* o = (uint32_t*) (rows + (size_t) p * RB);
            for (int i = lane; i < RB / 4; i += 32) o[i] = __ldg(s + i);
        }
        if (lane < K) {
            sids[(size_t) p * K + lane] = dest == d ? loc : -1;
            sw[(size_t) p * K + lane] = dest == d ? wv : 0.0f;
        }
    }
}

// One warp per dispatched pick (row r < *n_dev of the expert-ordered rows): the received q8_1 row it came from into
// the tensor-core layout: codes, d and d * sum(codes) per 32-value block (the q8_1 block's fp16 d widened, the sum of
// its int8 codes), as tsb_mmq_from_q8_1 writes them.
__global__ void __launch_bounds__(256) k_ep_rows_to_mmq(const uint8_t* __restrict__ rows, int RB,
                                                        const int32_t* __restrict__ row_tok,
                                                        const int32_t* __restrict__ n_dev, int cap, int H,
                                                        int8_t* __restrict__ codes, float* __restrict__ ds,
                                                        float* __restrict__ ss, int ldS) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= cap || r >= __ldg(n_dev)) return;
    const uint8_t* row = rows + (size_t) __ldg(row_tok + r) * RB;
    for (int b = lane; b < H / 32; b += 32) {
        const uint8_t* blk = row + 36 * b;
        const uint32_t* q = (const uint32_t*) (blk + 4);
        uint32_t v[8];
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[i] = __ldg(q + i);
            sum = __dp4a((int) v[i], 0x01010101, sum);
        }
        uint4* o = (uint4*) (codes + (size_t) r * H + 32 * b);
        o[0] = make_uint4(v[0], v[1], v[2], v[3]);
        o[1] = make_uint4(v[4], v[5], v[6], v[7]);
        const float d = __half2float(*(const __half*) blk);
        ds[(size_t) r * ldS + b] = d;
        ss[(size_t) r * ldS + b] = d * (float) sum;
    }
}

template <typename T>
__device__ __forceinline__ void st4(T* out, size_t i, float4 v);
template <>
__device__ __forceinline__ void st4<float>(float* out, size_t i, float4 v) {
    ((float4*) out)[i] = v;
}
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* out, size_t i, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *(uint32_t*) &a;
    u.y = *(uint32_t*) &b;
    ((uint2*) out)[i] = u;
}
template <typename T>
__device__ __forceinline__ float4 ld4(const T* in, size_t i);
template <>
__device__ __forceinline__ float4 ld4<float>(const float* in, size_t i) {
    return __ldcs((const float4*) in + i);
}
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* in, size_t i) {
    const uint2 u = __ldcs((const uint2*) in + i);
    const float2 a = __bfloat1622float2(*(const __nv_bfloat162*) &u.x), b = __bfloat1622float2(*(const __nv_bfloat162*) &u.y);
    return make_float4(a.x, a.y, b.x, b.y);
}

// One CTA per received row: the weighted sum of its picks' down rows in pick order (w0 p0, then fmaf), as the
// single-GPU combine sums them; picks on other ranks (rinv -1) are skipped.
template <typename OUT>
__global__ void __launch_bounds__(256) k_ep_row_sum(const float* __restrict__ parts, const int32_t* __restrict__ rinv,
                                                    const float* __restrict__ rw, int K, int H, OUT* __restrict__ out) {
    __shared__ int pr[32];
    __shared__ float pw[32];
    __shared__ int np;
    const int r = blockIdx.x;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int k = 0; k < K; ++k) {
            const int e = __ldg(rinv + (size_t) r * K + k);
            if (e >= 0) {
                pr[n] = e;
                pw[n] = __ldg(rw + (size_t) r * K + k);
                ++n;
            }
        }
        np = n;
    }
    __syncthreads();
    const int n = np;
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n > 0) {
            const float4 p = __ldcs((const float4*) (parts + (size_t) pr[0] * H) + i);
            acc = make_float4(pw[0] * p.x, pw[0] * p.y, pw[0] * p.z, pw[0] * p.w);
        }
        for (int k = 1; k < n; ++k) {
            const float4 p = __ldcs((const float4*) (parts + (size_t) pr[k] * H) + i);
            acc = make_float4(fmaf(pw[k], p.x, acc.x), fmaf(pw[k], p.y, acc.y), fmaf(pw[k], p.z, acc.z),
                              fmaf(pw[k], p.w, acc.w));
        }
        st4<OUT>(out, (size_t) r * (H / 4) + i, acc);
    }
}

// One CTA per token: out (+)= the returned partials of the ranks it went to, in rank order, + sigmoid(sgate) shared.
template <typename IN>
__global__ void __launch_bounds__(256) k_ep_finish(float* __restrict__ out, int accumulate, const IN* __restrict__ back,
                                                   const int32_t* __restrict__ send_pos, int G, int H,
                                                   const float* __restrict__ shared, const float* __restrict__ sgate,
                                                   int sg_stride) {
    __shared__ int sp[kEpMaxWorld];
    const int t = blockIdx.x;
    if ((int) threadIdx.x < G) sp[threadIdx.x] = __ldg(send_pos + (size_t) t * G + threadIdx.x);
    __syncthreads();
    const float gs = sgate ? frcp_fm(1.0f + fexp_fm(-sgate[(size_t) t * sg_stride])) : 1.0f;
    float4* xr = (float4*) (out + (size_t) t * H);
    const float4* sr = shared ? (const float4*) (shared + (size_t) t * H) : nullptr;
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        bool any = false;
        for (int d = 0; d < G; ++d) {
            if (sp[d] < 0) continue;
            const float4 p = ld4<IN>(back, (size_t) sp[d] * (H / 4) + i);
            acc = any ? make_float4(acc.x + p.x, acc.y + p.y, acc.z + p.z, acc.w + p.w) : p;
            any = true;
        }
        if (sr) {
            const float4 v = __ldcs(sr + i);
            acc = make_float4(acc.x + gs * v.x, acc.y + gs * v.y, acc.z + gs * v.z, acc.w + gs * v.w);
        }
        if (accumulate) {
            const float4 xv = xr[i];
            acc = make_float4(xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w);
        }
        xr[i] = acc;
    }
}

// ------------------------------------------------------------------------------------------------------- NCCL
// The process's NCCL (the one the framework around the library loaded, else the system's), resolved at run time so
// that the library never carries a second copy.
struct Nccl {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

const Nccl* nccl_lib() {
    static Nccl N;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        bool ok = true;
        auto get = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            ok = ok && fn != nullptr;
        };
        get(N.GetUniqueId, "ncclGetUniqueId");
        get(N.CommInitRank, "ncclCommInitRank");
        get(N.CommDestroy, "ncclCommDestroy");
        get(N.CommAbort, "ncclCommAbort");
        get(N.CommGetAsyncError, "ncclCommGetAsyncError");
        get(N.GroupStart, "ncclGroupStart");
        get(N.GroupEnd, "ncclGroupEnd");
        get(N.Send, "ncclSend");
        get(N.Recv, "ncclRecv");
        get(N.GetErrorString, "ncclGetErrorString");
        N.ok = ok;
    });
    return N.ok ? &N : nullptr;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

struct tsb_ep {
    int rank = 0, world = 1, E = 0, per = 0, K = 0, cyclic = 1, max_tok = 0, act = 0;
    float limit = INFINITY;
    tsb_expert_layout L{};
    const uint8_t* blobs = nullptr;
    uint64_t stride = 0;
    int H = 0, RB = 0, kloc = 0;              // hidden size, q8_1 row bytes, picks a row can have on one rank
    int64_t S_cap = 0, R_cap = 0, P_cap = 0;  // send slots, received rows, local picks
    const Nccl* N = nullptr;
    ncclComm_t comm = nullptr;
    cudaStream_t cs = nullptr;                // the communicator's stream
    cudaEvent_t ev_ready = nullptr, ev_counts = nullptr, ev_ret = nullptr;
    cudaEvent_t ev_disp[kEpMaxMb] = {}, ev_comp[kEpMaxMb] = {};
    int32_t *send_pos = nullptr, *counts = nullptr, *counts_h = nullptr;
    uint8_t* rows_s = nullptr;
    int32_t* ids_s = nullptr;
    float* w_s = nullptr;
    uint8_t* rows_r = nullptr;
    int32_t* ids_r = nullptr;
    float* w_r = nullptr;
    int32_t *bounds = nullptr, *row_ent = nullptr, *row_tok = nullptr, *rinv = nullptr;
    void *xa = nullptr, *ha = nullptr;
    float* parts = nullptr;
    void *ret_s = nullptr, *back = nullptr;
    // the step between tsb_ep_dispatch and tsb_ep_combine
    bool pending = false, broken = false;
    int n_tok = 0, n_mb = 1;
    int64_t off_s[kEpMaxMb][kEpMaxWorld], cnt_s[kEpMaxMb][kEpMaxWorld];
    int64_t off_r[kEpMaxMb][kEpMaxWorld], cnt_r[kEpMaxMb][kEpMaxWorld];
    uint64_t timeout_ns = 120000000000ull;
    int64_t st_sent = 0, st_recv = 0, st_picks = 0;
};

namespace {

int nccl_check(tsb_ep* ep, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return TSB_OK;
    return efail(TSB_ERR_COMM, "expert parallel: %s: %s", what, ep->N->GetErrorString(r));
}

// Wait for `ev` (work on the communicator's stream) with the host's bound; past it, or on an asynchronous
// communicator error, abort the communicator so that its kernels end, and mark the handle broken.
int ep_wait(tsb_ep* ep, cudaEvent_t ev, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return TSB_OK;
        if (e != cudaErrorNotReady) return efail(TSB_ERR_CUDA, "expert parallel: %s: %s", what, cudaGetErrorString(e));
        ncclResult_t ae = ncclSuccess;
        ep->N->CommGetAsyncError(ep->comm, &ae);
        const uint64_t ns = (uint64_t) std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::steady_clock::now() - t0).count();
        if ((ae != ncclSuccess && ae != ncclInProgress) || ns > ep->timeout_ns) {
            ep->N->CommAbort(ep->comm);
            ep->comm = nullptr;
            ep->broken = true;
            ep->pending = false;
            if (ae != ncclSuccess && ae != ncclInProgress)
                return efail(TSB_ERR_COMM, "expert parallel: %s: %s", what, ep->N->GetErrorString(ae));
            return efail(TSB_ERR_COMM, "expert parallel: %s: no answer within %.3f s (communicator aborted)", what,
                         ep->timeout_ns * 1e-9);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

void ep_free(tsb_ep* ep) {
    void* dev[] = {ep->send_pos, ep->counts, ep->rows_s, ep->ids_s, ep->w_s, ep->rows_r, ep->ids_r, ep->w_r,
                   ep->bounds, ep->row_ent, ep->row_tok, ep->rinv, ep->xa, ep->ha, ep->parts, ep->ret_s, ep->back};
    for (void* p : dev)
        if (p) cudaFree(p);
    if (ep->counts_h) cudaFreeHost(ep->counts_h);
    cudaEvent_t evs[] = {ep->ev_ready, ep->ev_counts, ep->ev_ret};
    for (cudaEvent_t e : evs)
        if (e) cudaEventDestroy(e);
    for (int m = 0; m < kEpMaxMb; ++m) {
        if (ep->ev_disp[m]) cudaEventDestroy(ep->ev_disp[m]);
        if (ep->ev_comp[m]) cudaEventDestroy(ep->ev_comp[m]);
    }
    if (ep->cs) cudaStreamDestroy(ep->cs);
}

}  // namespace

extern "C" {

int tsb_ep_unique_id(void* id128) {
    if (!id128) return efail(TSB_ERR_ARG, "ep_unique_id: null argument");
    const Nccl* N = nccl_lib();
    if (!N) return efail(TSB_ERR_COMM, "ep_unique_id: libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    const ncclResult_t r = N->GetUniqueId(&id);
    if (r != ncclSuccess) return efail(TSB_ERR_COMM, "ep_unique_id: %s", N->GetErrorString(r));
    memcpy(id128, &id, sizeof id);
    return TSB_OK;
}

int tsb_ep_create(const void* id128, int rank, int world, const tsb_expert_layout* L, const void* blobs,
                  uint64_t blob_stride, int n_expert, int n_used, int cyclic, int max_tokens, int act, float limit,
                  tsb_ep** out) {
    if (!out) return efail(TSB_ERR_ARG, "ep_create: null handle");
    *out = nullptr;
    if (!id128 || !L || !blobs || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || n_expert < world ||
        n_expert % world || n_used < 1 || n_used > 32 || max_tokens < 1 || act < 0 || act > 2)
        return efail(TSB_ERR_ARG, "ep_create: arguments (1..%d ranks, experts a multiple of the ranks, 1..32 picks)",
                     kEpMaxWorld);
    if (L->n_embd % 128) return efail(TSB_ERR_UNSUPPORTED, "ep_create: n_embd a multiple of 128");
    if (n_expert / world > 512) return efail(TSB_ERR_UNSUPPORTED, "ep_create: at most 512 experts per rank");
    const Nccl* N = nccl_lib();
    if (!N) return efail(TSB_ERR_COMM, "ep_create: libnccl.so.2 could not be loaded");
    tsb_ep* ep = new tsb_ep();
    ep->rank = rank;
    ep->world = world;
    ep->E = n_expert;
    ep->per = n_expert / world;
    ep->K = n_used;
    ep->cyclic = cyclic ? 1 : 0;
    ep->max_tok = max_tokens;
    ep->act = act;
    ep->limit = limit;
    ep->L = *L;
    ep->blobs = (const uint8_t*) blobs;
    ep->stride = blob_stride;
    ep->H = (int) L->n_embd;
    ep->RB = ep->H / 32 * 36;
    ep->kloc = n_used;   // a row's picks on one rank: up to all of them (a token may pick an expert twice)
    ep->S_cap = (int64_t) max_tokens * (n_used < world ? n_used : world);
    ep->R_cap = (int64_t) max_tokens * world;
    ep->P_cap = ep->R_cap * ep->kloc;
    ep->N = N;
    const int G = world, F = (int) L->n_ff;
    bool ok = true;
    auto dmal = [&](auto& p, size_t bytes) {
        if (ok && cudaMalloc((void**) &p, bytes < 256 ? 256 : bytes) != cudaSuccess) ok = false;
    };
    dmal(ep->send_pos, (size_t) max_tokens * G * 4);
    dmal(ep->counts, (size_t) 2 * G * kEpMaxMb * 4);
    dmal(ep->rows_s, (size_t) ep->S_cap * ep->RB);
    dmal(ep->ids_s, (size_t) ep->S_cap * n_used * 4);
    dmal(ep->w_s, (size_t) ep->S_cap * n_used * 4);
    dmal(ep->rows_r, (size_t) ep->R_cap * ep->RB);
    dmal(ep->ids_r, (size_t) ep->R_cap * n_used * 4);
    dmal(ep->w_r, (size_t) ep->R_cap * n_used * 4);
    dmal(ep->bounds, (size_t) (ep->per + 1) * 4);
    dmal(ep->row_ent, (size_t) ep->P_cap * 4);
    dmal(ep->row_tok, (size_t) ep->P_cap * 4);
    dmal(ep->rinv, (size_t) ep->R_cap * n_used * 4);
    dmal(ep->xa, (size_t) mmq_act_bytes(ep->P_cap, ep->H));
    dmal(ep->ha, (size_t) mmq_act_bytes(ep->P_cap, F));
    dmal(ep->parts, (size_t) ep->P_cap * ep->H * 4);
    dmal(ep->ret_s, (size_t) ep->R_cap * ep->H * 4);
    dmal(ep->back, (size_t) ep->S_cap * ep->H * 4);
    if (ok && cudaMallocHost((void**) &ep->counts_h, (size_t) 2 * G * kEpMaxMb * 4) != cudaSuccess) ok = false;
    if (ok && cudaStreamCreateWithFlags(&ep->cs, cudaStreamNonBlocking) != cudaSuccess) ok = false;
    for (cudaEvent_t* e : {&ep->ev_ready, &ep->ev_counts, &ep->ev_ret})
        if (ok && cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) ok = false;
    for (int m = 0; m < kEpMaxMb && ok; ++m)
        if (cudaEventCreateWithFlags(&ep->ev_disp[m], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ep->ev_comp[m], cudaEventDisableTiming) != cudaSuccess)
            ok = false;
    if (!ok) {
        const cudaError_t e = cudaGetLastError();
        ep_free(ep);
        delete ep;
        return efail(TSB_ERR_CUDA, "ep_create: device buffers for %d tokens per rank: %s", max_tokens,
                     cudaGetErrorString(e));
    }
    ncclUniqueId uid;
    memcpy(&uid, id128, sizeof uid);
    const ncclResult_t r = N->CommInitRank(&ep->comm, world, uid, rank);
    if (r != ncclSuccess) {
        ep_free(ep);
        delete ep;
        return efail(TSB_ERR_COMM, "ep_create: ncclCommInitRank: %s", N->GetErrorString(r));
    }
    *out = ep;
    return TSB_OK;
}

int tsb_ep_set_timeout_ns(tsb_ep* ep, uint64_t ns) {
    if (!ep || ns < 1000000ull) return efail(TSB_ERR_ARG, "ep_set_timeout_ns: arguments (>= 1 ms)");
    ep->timeout_ns = ns;
    return TSB_OK;
}

int tsb_ep_dispatch(tsb_ep* ep, const void* x_q8_1, const int32_t* ids, const float* w, int n_tok, int micro_batches,
                    void* stream) {
    if (!ep) return efail(TSB_ERR_ARG, "ep_dispatch: null handle");
    if (ep->broken) return efail(TSB_ERR_COMM, "ep_dispatch: the communicator was aborted");
    if (ep->pending) return efail(TSB_ERR_ARG, "ep_dispatch: the previous step was not combined");
    if (n_tok < 0 || n_tok > ep->max_tok || micro_batches < 1 || micro_batches > kEpMaxMb ||
        (n_tok > 0 && (!x_q8_1 || !ids || !w)))
        return efail(TSB_ERR_ARG, "ep_dispatch: arguments (0..%d tokens, 1..%d micro-batches)", ep->max_tok, kEpMaxMb);
    if ((uintptr_t) x_q8_1 % 16) return efail(TSB_ERR_ALIGN, "ep_dispatch: q8_1 rows 16-byte aligned");
    cudaStream_t s = (cudaStream_t) stream;
    // every rank exchanges M counts with every peer: M is the caller's (the same on every rank), never derived from
    // this rank's token count (a slice may hold no tokens)
    const int G = ep->world, M = micro_batches, K = ep->K;
    if (n_tok > 0) {
        k_ep_plan<<<1, 1024, 0, s>>>(ids, n_tok, K, ep->E, G, ep->per, ep->cyclic, M, ep->send_pos, ep->counts);
        k_ep_pack<<<(unsigned) ((n_tok + 7) / 8), 256, 0, s>>>((const uint8_t*) x_q8_1, ep->RB, ids, w, n_tok, K, ep->E,
                                                                G, ep->per, ep->cyclic, ep->send_pos, ep->rows_s,
                                                                ep->ids_s, ep->w_s);
    } else {
        cudaMemsetAsync(ep->counts, 0, (size_t) G * M * 4, s);
    }
    cudaEventRecord(ep->ev_ready, s);
    cudaStreamWaitEvent(ep->cs, ep->ev_ready, 0);
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) return efail(TSB_ERR_CUDA, "ep_dispatch: %s", cudaGetErrorString(le));
    // the counts: [G][M] of this rank's slots per destination, then [G][M] received per source
    int rc = nccl_check(ep, ep->N->GroupStart(), "group");
    for (int d = 0; d < G && rc == TSB_OK; ++d) {
        rc = nccl_check(ep, ep->N->Send(ep->counts + d * M, M, ncclInt32, d, ep->comm, ep->cs), "counts send");
        if (rc == TSB_OK)
            rc = nccl_check(ep, ep->N->Recv(ep->counts + G * M + d * M, M, ncclInt32, d, ep->comm, ep->cs),
                            "counts recv");
    }
    const int rg = nccl_check(ep, ep->N->GroupEnd(), "group");
    if (rc != TSB_OK || rg != TSB_OK) return rc != TSB_OK ? rc : rg;
    cudaMemcpyAsync(ep->counts_h, ep->counts, (size_t) 2 * G * M * 4, cudaMemcpyDeviceToHost, ep->cs);
    cudaEventRecord(ep->ev_counts, ep->cs);
    rc = ep_wait(ep, ep->ev_counts, "counts exchange");
    if (rc != TSB_OK) return rc;
    int64_t so = 0, ro = 0;
    for (int m = 0; m < M; ++m) {
        for (int d = 0; d < G; ++d) {
            ep->cnt_s[m][d] = ep->counts_h[d * M + m];
            ep->off_s[m][d] = so;
            so += ep->cnt_s[m][d];
        }
        for (int d = 0; d < G; ++d) {
            ep->cnt_r[m][d] = ep->counts_h[G * M + d * M + m];
            ep->off_r[m][d] = ro;
            ro += ep->cnt_r[m][d];
        }
    }
    if (so > ep->S_cap || ro > ep->R_cap)
        return efail(TSB_ERR_ARG, "ep_dispatch: %lld rows received > %lld (a peer's tokens exceed max_tokens)",
                     (long long) ro, (long long) ep->R_cap);
    for (int m = 0; m < M; ++m) {
        rc = nccl_check(ep, ep->N->GroupStart(), "group");
        for (int d = 0; d < G && rc == TSB_OK; ++d) {
            const int64_t ns = ep->cnt_s[m][d], os = ep->off_s[m][d], nr = ep->cnt_r[m][d], orr = ep->off_r[m][d];
            if (ns > 0) {
                rc = nccl_check(ep, ep->N->Send(ep->rows_s + os * ep->RB, ns * ep->RB, ncclUint8, d, ep->comm, ep->cs),
                                "rows send");
                if (rc == TSB_OK)
                    rc = nccl_check(ep, ep->N->Send(ep->ids_s + os * K, ns * K, ncclInt32, d, ep->comm, ep->cs),
                                    "ids send");
                if (rc == TSB_OK)
                    rc = nccl_check(ep, ep->N->Send(ep->w_s + os * K, ns * K, ncclFloat32, d, ep->comm, ep->cs),
                                    "weights send");
            }
            if (nr > 0 && rc == TSB_OK) {
                rc = nccl_check(ep, ep->N->Recv(ep->rows_r + orr * ep->RB, nr * ep->RB, ncclUint8, d, ep->comm, ep->cs),
                                "rows recv");
                if (rc == TSB_OK)
                    rc = nccl_check(ep, ep->N->Recv(ep->ids_r + orr * K, nr * K, ncclInt32, d, ep->comm, ep->cs),
                                    "ids recv");
                if (rc == TSB_OK)
                    rc = nccl_check(ep, ep->N->Recv(ep->w_r + orr * K, nr * K, ncclFloat32, d, ep->comm, ep->cs),
                                    "weights recv");
            }
        }
        const int rg2 = nccl_check(ep, ep->N->GroupEnd(), "group");
        if (rc != TSB_OK || rg2 != TSB_OK) return rc != TSB_OK ? rc : rg2;
        cudaEventRecord(ep->ev_disp[m], ep->cs);
    }
    ep->n_tok = n_tok;
    ep->n_mb = M;
    ep->pending = true;
    ep->st_sent = so;
    ep->st_recv = ro;
    ep->st_picks = 0;
    const cudaError_t e2 = cudaGetLastError();
    if (e2 != cudaSuccess) return efail(TSB_ERR_CUDA, "ep_dispatch: %s", cudaGetErrorString(e2));
    return TSB_OK;
}

int tsb_ep_combine(tsb_ep* ep, float* out, int accumulate, const float* shared, const float* sgate, int sg_stride,
                   int return_bf16, void* stream) {
    if (!ep) return efail(TSB_ERR_ARG, "ep_combine: null handle");
    if (ep->broken) return efail(TSB_ERR_COMM, "ep_combine: the communicator was aborted");
    if (!ep->pending) return efail(TSB_ERR_ARG, "ep_combine: no step dispatched");
    if (ep->n_tok > 0 && !out) return efail(TSB_ERR_ARG, "ep_combine: null output");
    if ((uintptr_t) out % 16 || (uintptr_t) shared % 16) return efail(TSB_ERR_ALIGN, "ep_combine: rows 16-byte aligned");
    cudaStream_t s = (cudaStream_t) stream;
    const int G = ep->world, K = ep->K, H = ep->H, M = ep->n_mb;
    const size_t esz = return_bf16 ? 2 : 4;
    const ncclDataType_t et = return_bf16 ? ncclBfloat16 : ncclFloat32;
    for (int m = 0; m < M; ++m) {
        int64_t R = 0;
        for (int d = 0; d < G; ++d) R += ep->cnt_r[m][d];
        const int64_t base = ep->off_r[m][0];
        cudaStreamWaitEvent(s, ep->ev_disp[m], 0);
        if (R > 0) {
            const int64_t P = R * ep->kloc;
            int rc = tsb_moe_dispatch(ep->ids_r + base * K, (int) (R * K), K, ep->per, ep->bounds, ep->row_ent,
                                      ep->row_tok, ep->rinv, s);
            if (rc != TSB_OK) return rc;
            const MmqView xv = mmq_view(ep->xa, P, H);
            k_ep_rows_to_mmq<<<(unsigned) ((P + 7) / 8), 256, 0, s>>>(ep->rows_r + base * ep->RB, ep->RB, ep->row_tok,
                                                                      ep->bounds + ep->per, (int) P, H, xv.codes, xv.d,
                                                                      xv.s, xv.ldS);
            rc = tsb_moe_prefill_gu(&ep->L, ep->blobs, ep->stride, ep->bounds, ep->per, (int) P, ep->xa, ep->ha,
                                    ep->act, ep->limit, s);
            if (rc == TSB_OK)
                rc = tsb_moe_prefill_down(&ep->L, ep->blobs, ep->stride, ep->bounds, ep->per, (int) P, ep->ha,
                                          ep->parts, s);
            if (rc != TSB_OK) return rc;
            uint8_t* dst = (uint8_t*) ep->ret_s + (size_t) base * H * esz;
            if (return_bf16)
                k_ep_row_sum<__nv_bfloat16><<<(unsigned) R, 256, 0, s>>>(ep->parts, ep->rinv, ep->w_r + base * K, K, H,
                                                                         (__nv_bfloat16*) dst);
            else
                k_ep_row_sum<float><<<(unsigned) R, 256, 0, s>>>(ep->parts, ep->rinv, ep->w_r + base * K, K, H,
                                                                 (float*) dst);
            ep->st_picks += P;
        }
        cudaEventRecord(ep->ev_comp[m], s);
        cudaStreamWaitEvent(ep->cs, ep->ev_comp[m], 0);
        int rc = nccl_check(ep, ep->N->GroupStart(), "group");
        for (int d = 0; d < G && rc == TSB_OK; ++d) {
            const int64_t nr = ep->cnt_r[m][d], orr = ep->off_r[m][d], ns = ep->cnt_s[m][d], os = ep->off_s[m][d];
            if (nr > 0)
                rc = nccl_check(ep, ep->N->Send((uint8_t*) ep->ret_s + (size_t) orr * H * esz, (size_t) nr * H, et, d,
                                                ep->comm, ep->cs), "partials send");
            if (ns > 0 && rc == TSB_OK)
                rc = nccl_check(ep, ep->N->Recv((uint8_t*) ep->back + (size_t) os * H * esz, (size_t) ns * H, et, d,
                                                ep->comm, ep->cs), "partials recv");
        }
        const int rg = nccl_check(ep, ep->N->GroupEnd(), "group");
        if (rc != TSB_OK || rg != TSB_OK) return rc != TSB_OK ? rc : rg;
    }
    cudaEventRecord(ep->ev_ret, ep->cs);
    cudaStreamWaitEvent(s, ep->ev_ret, 0);
    if (ep->n_tok > 0) {
        if (return_bf16)
            k_ep_finish<__nv_bfloat16><<<(unsigned) ep->n_tok, 256, 0, s>>>(out, accumulate, (const __nv_bfloat16*) ep->back,
                                                                           ep->send_pos, G, H, shared, sgate, sg_stride);
        else
            k_ep_finish<float><<<(unsigned) ep->n_tok, 256, 0, s>>>(out, accumulate, (const float*) ep->back,
                                                                   ep->send_pos, G, H, shared, sgate, sg_stride);
    }
    ep->pending = false;
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return efail(TSB_ERR_CUDA, "ep_combine: %s", cudaGetErrorString(e));
    return TSB_OK;
}

int tsb_ep_synchronize(tsb_ep* ep) {
    if (!ep) return efail(TSB_ERR_ARG, "ep_synchronize: null handle");
    if (ep->broken) return efail(TSB_ERR_COMM, "ep_synchronize: the communicator was aborted");
    cudaEventRecord(ep->ev_counts, ep->cs);
    return ep_wait(ep, ep->ev_counts, "synchronize");
}

int tsb_ep_stats(const tsb_ep* ep, int64_t* sent, int64_t* received, int64_t* picks) {
    if (!ep) return efail(TSB_ERR_ARG, "ep_stats: null handle");
    if (sent) *sent = ep->st_sent;
    if (received) *received = ep->st_recv;
    if (picks) *picks = ep->st_picks;
    return TSB_OK;
}

int tsb_ep_destroy(tsb_ep* ep) {
    if (!ep) return TSB_OK;
    int rc = TSB_OK;
    if (ep->comm) {
        cudaEventRecord(ep->ev_ret, ep->cs);
        rc = ep_wait(ep, ep->ev_ret, "destroy");
        if (ep->comm) {
            const ncclResult_t r = ep->N->CommDestroy(ep->comm);
            if (r != ncclSuccess && rc == TSB_OK) rc = efail(TSB_ERR_COMM, "ep_destroy: %s", ep->N->GetErrorString(r));
        }
    }
    ep_free(ep);
    delete ep;
    return rc;
}

}  // extern "C"
