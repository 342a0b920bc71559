// tsb_staged.cu - host-staged experts: an HBM expert cache (slots) with the layer's other experts in pinned host memory.
//
// The reference's hybrid mode (src/qwen35/q36_engine.cu) keeps n_slots experts of a layer in VRAM slots
// (slot_of[x] >= 0: the blob at slots + slot_of[x] * stride), groups only their entries on the GPU (k_group_hy,
// :423-452) and runs the other entries on a CPU thread pool whose rows are merged back (moe_hybrid_cpu, :3088-3210,
// k_merge_cpu :455-459); its prompt path copies a whole layer into a staging ring, runs of resident experts device to
// device and the others over PCIe (stream_kick, :3001-3033); between steps the most-used experts take the slots
// (rebalance, :3215-3265, with the halving age of include/strata/qwen35/cache_policy.hpp:28-30).
//
// Here every entry runs on the GPU through the same grouped expert kernels as a resident layer, so a staged layer's
// outputs equal the resident layer's bit for bit:
//   k_group_staged  (1 CTA)  the grouping of every entry (as k_group); a group's blob is its expert's slot, or, for an
//                            expert without one, the next free blob of the caller's stage buffer; usage counts += 1
//                            per entry;
//   k_fetch_staged           the staged groups' blobs pulled from mapped pinned host memory by the GPU itself (16-byte
//                            loads over the host link, 32 KB per CTA): no host synchronisation, graph-capturable.
// The placement (tsb_staged_rebalance) and the slot loads (tsb_staged_load) are host calls between steps; the
// streamed layer of the prompt path (tsb_stage_layer) issues the reference's runs of copies.
#include "../../include/tsb_moe.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <numeric>
#include <vector>

namespace tsb {

void set_last_error(const char* msg);   // tsb_moe.cu: the text tsb_last_error returns

namespace {

int sfail(int code, const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    set_last_error(b);
    return code;
}
int scuda(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return sfail(TSB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return TSB_OK;
}

constexpr int kFetchThreads = 256;
constexpr int kFetchUnroll = 8;                                      // 16-byte loads in flight per thread
constexpr uint64_t kFetchChunk = (uint64_t) kFetchThreads * kFetchUnroll * 16;   // 32 KB per CTA

// Groups of ascending expert id, entries in entry order (the order of k_group).  Ids outside [0, n_expert) are
// dropped (no row).  A group's blob: slots + slot_of[x] * stride when 0 <= slot_of[x] < n_slots, else stage + m * stride
// for the m-th group without a slot (the host checks stage_cap >= min(n_ent, n_expert), so m < stage_cap).
__global__ void __launch_bounds__(1024) k_group_staged(const int32_t* __restrict__ ids, int n_ent, int K, int n_expert,
                                                       const int32_t* __restrict__ slot_of, int n_slots,
                                                       const uint8_t* slots, const uint8_t* stage,
                                                       unsigned long long stride, unsigned long long* grp_ptr,
                                                       int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst,
                                                       int32_t* ent_tok, unsigned* counts) {
    extern __shared__ int sh[];
    int* cnt = sh;                   // n_expert
    int* off = sh + n_expert;        // n_expert: first row of an expert's group
    for (int x = threadIdx.x; x < n_expert; x += blockDim.x) cnt[x] = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {
        const int id = ids[e];
        if (id >= 0 && id < n_expert) {
            atomicAdd(&cnt[id], 1);
            if (counts) atomicAdd(counts + id, 1u);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int pos = 0, g = 0, m = 0;
        for (int x = 0; x < n_expert; ++x) {
            off[x] = pos;
            if (!cnt[x]) continue;
            const int s = slot_of[x];
            const uint8_t* b = (s >= 0 && s < n_slots) ? slots + (size_t) s * stride : stage + (size_t) (m++) * stride;
            grp_ptr[g] = (unsigned long long) b;
            grp_start[g] = pos;
            ++g;
            pos += cnt[x];
        }
        grp_start[g] = pos;
        *n_groups = g;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_ent; e += blockDim.x) {
        const int id = ids[e];
        if (id < 0 || id >= n_expert) continue;
        int before = 0;
        for (int e2 = 0; e2 < e; ++e2) before += ids[e2] == id;
        const int p = off[id] + before;
        ent_dst[p] = e;
        ent_tok[p] = e / K;
    }
}

// grid (groups, blob chunks): CTA (g, c) copies bytes [c * 32 KB, (c + 1) * 32 KB) of group g's expert blob from host
// memory into the group's stage blob, when the group's blob lies in the stage buffer.  stride is a multiple of 16.
__global__ void __launch_bounds__(kFetchThreads) k_fetch_staged(const int32_t* __restrict__ ids,
                                                                const unsigned long long* __restrict__ grp_ptr,
                                                                const int32_t* __restrict__ grp_start,
                                                                const int32_t* __restrict__ n_groups,
                                                                const int32_t* __restrict__ ent_dst,
                                                                const uint8_t* host, const uint8_t* stage,
                                                                unsigned long long stride, int stage_cap) {
    const int g = blockIdx.x;
    if (g >= *n_groups) return;
    const unsigned long long p = grp_ptr[g];
    const unsigned long long s0 = (unsigned long long) stage;
    if (p < s0 || p >= s0 + (unsigned long long) stage_cap * stride) return;
    const int x = ids[ent_dst[grp_start[g]]];
    const uint4* src = (const uint4*) (host + (size_t) x * stride);
    uint4* dst = (uint4*) p;
    const uint64_t n16 = stride / 16;
    const uint64_t base = (uint64_t) blockIdx.y * (kFetchChunk / 16);
    uint4 v[kFetchUnroll];
#pragma unroll
    for (int i = 0; i < kFetchUnroll; ++i) {
        const uint64_t j = base + (uint64_t) i * kFetchThreads + threadIdx.x;
        if (j < n16) v[i] = src[j];
    }
#pragma unroll
    for (int i = 0; i < kFetchUnroll; ++i) {
        const uint64_t j = base + (uint64_t) i * kFetchThreads + threadIdx.x;
        if (j < n16) dst[j] = v[i];
    }
}

// Host memory the device can read at the same address (pinned and mapped: cudaHostAlloc / cudaMallocHost under
// unified addressing, or cudaHostRegister with cudaHostRegisterMapped).
bool device_readable_host(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost && a.devicePointer == p;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" {

int tsb_moe_group_staged(const int32_t* ids, int n_ent, int K, int n_expert, const int32_t* slot_of, int n_slots,
                         const void* slots, const void* host_blobs, uint64_t stride, void* stage, int stage_cap,
                         uint64_t* grp_ptr, int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst, int32_t* ent_tok,
                         uint32_t* counts, void* stream) {
    if (!ids || !slot_of || !host_blobs || !grp_ptr || !grp_start || !n_groups || !ent_dst || !ent_tok)
        return sfail(TSB_ERR_ARG, "group_staged: null argument");
    if (n_ent < 1 || K < 1 || n_expert < 1 || n_expert > 4096 || n_slots < 0 || (n_slots > 0 && !slots))
        return sfail(TSB_ERR_ARG, "group_staged: n_ent %d, K %d, n_expert %d, n_slots %d", n_ent, K, n_expert, n_slots);
    if (stride == 0 || stride % 16 || (uintptr_t) host_blobs % 16 || (uintptr_t) slots % 16 || (uintptr_t) stage % 16)
        return sfail(TSB_ERR_ALIGN, "group_staged: stride and blob bases must be multiples of 16 bytes");
    const int need = std::min(n_ent, n_expert);
    if (stage_cap < need || !stage)
        return sfail(TSB_ERR_WORKSPACE, "group_staged: stage holds %d blobs, a step may miss %d experts", stage_cap, need);
    cudaStream_t s = (cudaStream_t) stream;
    // checked outside stream capture (a captured call was checked when the caller ran it eagerly, or fails on replay
    // with a CUDA error rather than a fault: unmapped host memory has no device address to read)
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) return scuda("group_staged: capture status");
    if (cap == cudaStreamCaptureStatusNone && !device_readable_host(host_blobs))
        return sfail(TSB_ERR_ARG, "group_staged: host_blobs is not pinned host memory mapped for the device");
    k_group_staged<<<1, 1024, (size_t) 2 * n_expert * sizeof(int), s>>>(
        ids, n_ent, K, n_expert, slot_of, n_slots, (const uint8_t*) slots, (const uint8_t*) stage,
        (unsigned long long) stride, (unsigned long long*) grp_ptr, grp_start, n_groups, ent_dst, ent_tok, counts);
    int rc = scuda("group_staged: grouping");
    if (rc != TSB_OK) return rc;
    const dim3 grid((unsigned) need, (unsigned) ((stride + kFetchChunk - 1) / kFetchChunk));
    k_fetch_staged<<<grid, kFetchThreads, 0, s>>>(ids, (const unsigned long long*) grp_ptr, grp_start, n_groups,
                                                  ent_dst, (const uint8_t*) host_blobs, (const uint8_t*) stage,
                                                  (unsigned long long) stride, stage_cap);
    return scuda("group_staged: fetch");
}

int tsb_staged_rebalance(double* score, int n_expert, int n_slots, int32_t* slot_of, int32_t* exp_in_slot,
                         int max_swaps, int32_t* move_expert, int32_t* move_slot) {
    if (!score || !slot_of || !exp_in_slot || n_expert < 1 || n_slots < 0 || n_slots > n_expert || max_swaps < 0 ||
        (max_swaps > 0 && (!move_expert || !move_slot)))
        return sfail(TSB_ERR_ARG, "staged_rebalance: bad argument");
    for (int s = 0; s < n_slots; ++s) {
        const int y = exp_in_slot[s];
        if (y < 0 || y >= n_expert || slot_of[y] != s)
            return sfail(TSB_ERR_ARG, "staged_rebalance: slot %d holds expert %d, whose slot_of is not %d", s, y, s);
    }
    int moves = 0;
    if (n_slots > 0 && n_slots < n_expert) {
        // experts by score, highest first (ties: the lower id); slots by their resident's score, lowest first (ties:
        // the lower slot): the residents to give away
        std::vector<int> order((size_t) n_expert);
        std::iota(order.begin(), order.end(), 0);
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return score[a] > score[b]; });
        std::vector<int> victims((size_t) n_slots);
        std::iota(victims.begin(), victims.end(), 0);
        std::stable_sort(victims.begin(), victims.end(),
                         [&](int a, int b) { return score[exp_in_slot[a]] < score[exp_in_slot[b]]; });
        size_t vi = 0;
        for (int i = 0; i < n_slots && moves < max_swaps && vi < victims.size(); ++i) {
            const int x = order[(size_t) i];
            if (slot_of[x] >= 0) continue;
            const int s = victims[vi];
            const int y = exp_in_slot[s];
            if (score[y] >= score[x]) break;   // no resident left that scores below a top expert
            ++vi;
            slot_of[y] = -1;
            slot_of[x] = s;
            exp_in_slot[s] = x;
            move_expert[moves] = x;
            move_slot[moves] = s;
            ++moves;
        }
        for (int x = 0; x < n_expert; ++x) score[x] *= 0.5;   // aged only where a placement is chosen, as the reference
    }
    return moves;
}

int tsb_staged_load(const void* host_blobs, void* slots, uint64_t stride, uint64_t blob_bytes, const int32_t* move_expert,
                    const int32_t* move_slot, int n_moves, int n_expert, int n_slots, void* stream) {
    if (n_moves < 0 || (n_moves > 0 && (!host_blobs || !slots || !move_expert || !move_slot)) || blob_bytes > stride)
        return sfail(TSB_ERR_ARG, "staged_load: bad argument");
    cudaStream_t s = (cudaStream_t) stream;
    for (int i = 0; i < n_moves; ++i) {
        const int x = move_expert[i], sl = move_slot[i];
        if (x < 0 || x >= n_expert || sl < 0 || sl >= n_slots)
            return sfail(TSB_ERR_ARG, "staged_load: move %d (expert %d -> slot %d) out of range", i, x, sl);
        if (cudaMemcpyAsync((uint8_t*) slots + (size_t) sl * stride, (const uint8_t*) host_blobs + (size_t) x * stride,
                            blob_bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return scuda("staged_load: copy");
    }
    return TSB_OK;
}

int tsb_stage_layer(const int32_t* slot_of, int n_expert, int n_slots, const void* slots, const void* host_blobs,
                    uint64_t stride, void* stage, int whole, void* stream) {
    if (!slot_of || !host_blobs || !stage || n_expert < 1 || stride == 0 || n_slots < 0 || (n_slots > 0 && !slots))
        return sfail(TSB_ERR_ARG, "stage_layer: bad argument");
    cudaStream_t s = (cudaStream_t) stream;
    const uint8_t* hb = (const uint8_t*) host_blobs;
    const uint8_t* sb = (const uint8_t*) slots;
    uint8_t* dst = (uint8_t*) stage;
    int copies = 0;
    auto resident = [&](int x) { return slot_of[x] >= 0 && slot_of[x] < n_slots; };
    if (whole || 2 * n_slots < n_expert) {
        // fewer than half the experts resident: one whole-layer copy beats many small ones
        if (cudaMemcpyAsync(dst, hb, stride * (size_t) n_expert, cudaMemcpyHostToDevice, s) != cudaSuccess)
            return scuda("stage_layer: whole layer");
        return 1;
    }
    for (int x = 0; x < n_expert;) {
        const bool dev = resident(x);
        int y = x + 1;
        if (dev)   // consecutive slots holding consecutive experts
            while (y < n_expert && resident(y) && slot_of[y] == slot_of[y - 1] + 1) ++y;
        else
            while (y < n_expert && !resident(y)) ++y;
        const size_t n = (size_t) (y - x) * stride;
        const cudaError_t e =
            dev ? cudaMemcpyAsync(dst + (size_t) x * stride, sb + (size_t) slot_of[x] * stride, n, cudaMemcpyDeviceToDevice, s)
                : cudaMemcpyAsync(dst + (size_t) x * stride, hb + (size_t) x * stride, n, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return scuda("stage_layer: copy");
        ++copies;
        x = y;
    }
    return copies;
}

}  // extern "C"
