// tsb_decode.cu - host side of the fused decode kernel (tsb_decode.cuh): validation, workspace, cooperative launch.
#include <algorithm>
#include "tsb_decode.cuh"
#include "../../include/tsb_moe.h"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

namespace tsb {
namespace {
thread_local char g_derr[512];
unsigned long long* g_trace = nullptr;
int g_withhold = 0;
int dfail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_derr, sizeof g_derr, fmt, ap);
    va_end(ap);
    return code;
}

// Every exchange buffer holds tagged 8-byte words (value, layer + 1); the whole workspace is zeroed before each launch
// so that no word carries a tag of this launch before it is written.
struct WsLayout {
    size_t logits, hsh, hbuf, sh_out, xt, err, total;
};
WsLayout ws_layout(const tsb_decode_desc* d) {
    auto al = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    WsLayout w;
    size_t o = 0;
    w.logits = o; o += al((size_t) d->n_tok * (d->n_expert + 1) * 2 * 8);
    w.hsh = o;    o += al((size_t) d->n_tok * d->sh_n_ff * 8);
    w.hbuf = o;   o += al((size_t) d->n_tok * d->n_used * d->n_ff * 8);
    w.sh_out = o; o += al((size_t) d->n_tok * d->n_embd * 8);
    w.xt = o;     o += al((size_t) d->n_tok * d->n_embd * 8);
    w.err = o;    o += 8192;   // error word, its context (words 1..127), one progress word per CTA from word 128
    w.total = o;
    return w;
}
}  // namespace

// The decode kernel's requirements on a layer description (the Qwen3.6 MoE block).
int decode_check(const tsb_decode_desc* d, DecParams& p, size_t& smem) {
    if (!d || d->struct_size != sizeof(tsb_decode_desc)) return dfail(TSB_ERR_ARG, "decode: descriptor size");
    if (d->gu_type != T_IQ3_XXS || d->d_type != T_IQ3_XXS || d->sh_gu_type != T_Q8_0 || d->sh_d_type != T_Q8_0)
        return dfail(TSB_ERR_UNSUPPORTED, "decode: IQ3_XXS routed experts with a Q8_0 shared expert only");
    const int T = d->n_tok, H = d->n_embd, F = d->n_ff, E = d->n_expert, K = d->n_used, FS = d->sh_n_ff;
    if (T < 1 || T > kDecMaxT || K < 1 || T * K > kDecMaxEnt || E < 32 || E % 32 || E / 32 != 8 || K > E)
        return dfail(TSB_ERR_UNSUPPORTED, "decode: 1..16 tokens, 256 experts, T*K <= 128");
    if (H % 2048 || H > 2048 || F != 512 || FS % 128)
        return dfail(TSB_ERR_UNSUPPORTED, "decode: hidden 2048, expert FF 512, shared FF a multiple of 128");
    p.n_layers = d->n_layers;
    p.T = T; p.H = H; p.F = F; p.E = E; p.K = K; p.FS = FS;
    p.gu_row = (uint32_t) (H / 256 * 98);
    p.d_row = (uint32_t) (F / 256 * 98);
    p.up_off = (uint64_t) F * p.gu_row;
    p.down_off = 2 * p.up_off;
    p.blob_bytes = p.down_off + (uint64_t) H * p.d_row;
    p.sgu_row = (uint32_t) (H / 32 * 34);
    p.sd_row = (uint32_t) (FS / 32 * 34);
    p.s_up_off = (uint64_t) FS * p.sgu_row;
    p.s_down_off = 2 * p.s_up_off;
    p.R = 4;   // four rows per routed down task: one pass of 32 lanes over their two blocks each (F = 512)
    p.rt_per_unit = std::min(2, (int) (kSlotBytes / (2 * p.gu_row)));   // two row pairs: units for every warp at T = 1
    p.sd_per_unit = (int) (kSlotBytes / p.sd_row);
    while (p.sd_per_unit > 1 && H % p.sd_per_unit) --p.sd_per_unit;
    // Two routed down tasks (4 rows of one expert each) per slot: about one unit per consumer warp at T = 1.
    p.dn_per_unit = std::min(2, (int) (kSlotBytes / (p.R * p.d_row)));
    if (p.gu_row % 16 || p.sgu_row % 16 || p.sd_row % 16 || p.blob_bytes % 16 || p.rt_per_unit < 1 || F % p.rt_per_unit ||
        2 * p.sgu_row > kSlotBytes || p.dn_per_unit < 1 || H % p.R)
        return dfail(TSB_ERR_UNSUPPORTED, "decode: rows do not fit the ring slots");
    int dev = 0, reserved = 0, max_smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    p.smem_base = (uint32_t) reserved;
    if (p.smem_base + (uint32_t) (2 * kLowWarps) * kSlotBytes > 0x10000u || (uint32_t) kDecWarps * kSlotBytes > 2 * kLowWarps * kSlotBytes)
        return dfail(TSB_ERR_UNSUPPORTED, "decode: %d reserved bytes leave no room for the slots", reserved);
    // two slots a warp (a unit in flight ahead of the one computing) when shared memory allows, else one
    p.nslot = dec_smem(p.smem_base, T, H, F, FS, K, 2).total <= (uint32_t) max_smem ? 2 : 1;
    smem = dec_smem(p.smem_base, T, H, F, FS, K, p.nslot).total;
    return TSB_OK;
}

// This translation unit's copy of the wait bound (tsb_set_wait_limit_ns sets every copy on the current device).
int decode_set_wait_limit(unsigned long long ns) {
    return cudaMemcpyToSymbol(g_wait_ns, &ns, sizeof ns) == cudaSuccess ? TSB_OK : TSB_ERR_CUDA;
}

}  // namespace tsb

using namespace tsb;

extern "C" {

uint64_t tsb_moe_decode_workspace_bytes(const tsb_decode_desc* d) {
    if (!d) return 0;
    return ws_layout(d).total;
}

int tsb_moe_decode_layers(const tsb_decode_desc* d, const tsb_decode_layer* layers, float* x, int32_t* ids_rec,
                          float* w_rec, float* x_rec, void* workspace, uint64_t ws_bytes, void* stream) {
    static_assert(sizeof(tsb_decode_layer) == sizeof(DecLayer), "tsb_decode_layer mirrors DecLayer");
    DecParams p{};
    size_t smem = 0;
    int rc = decode_check(d, p, smem);
    if (rc != TSB_OK) return rc;
    if (!layers || !x || !workspace) return dfail(TSB_ERR_ARG, "decode: null argument");
    const WsLayout w = ws_layout(d);
    if (ws_bytes < w.total) return dfail(TSB_ERR_WORKSPACE, "decode: workspace %llu < %llu bytes",
                                         (unsigned long long) ws_bytes, (unsigned long long) w.total);
    if ((uintptr_t) workspace % 256 || (uintptr_t) x % 16) return dfail(TSB_ERR_ALIGN, "decode: workspace / x alignment");
    int dev = 0, sms = 0, coop = 0, max_smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (!coop) return dfail(TSB_ERR_UNSUPPORTED, "decode: device without cooperative launch");
    if ((int) smem > max_smem) return dfail(TSB_ERR_UNSUPPORTED, "decode: %zu bytes of shared memory > %d", smem, max_smem);
    if ((p.H / p.R + sms - 1) / sms * p.R > kDecMaxRows) return dfail(TSB_ERR_UNSUPPORTED, "decode: too few SMs");
    // every CTA computes some of P1 (router or shared gate/up rows): the reuse of the exchange buffers relies on it
    if (2 * (p.E + 1) + p.FS < sms) return dfail(TSB_ERR_UNSUPPORTED, "decode: fewer P1 rows than SMs");
    uint8_t* ws = (uint8_t*) workspace;
    p.layers = (const DecLayer*) layers;
    p.x = x;
    p.logits = (uint64_t*) (ws + w.logits);
    p.hsh = (uint64_t*) (ws + w.hsh);
    p.hbuf = (uint64_t*) (ws + w.hbuf);
    p.sh_out = (uint64_t*) (ws + w.sh_out);
    p.xt = (uint64_t*) (ws + w.xt);
    p.err = (unsigned*) (ws + w.err);
    p.ids_rec = ids_rec;
    p.w_rec = w_rec;
    p.x_rec = x_rec;
    p.trace = g_trace;
    p.dbg_withhold = g_withhold;
    p.eps = d->eps;
    cudaStream_t s = (cudaStream_t) stream;
    auto kern = k_decode_layers<8>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess)
        return dfail(TSB_ERR_CUDA, "decode: shared memory attribute: %s", cudaGetErrorString(cudaGetLastError()));
    if (cudaMemsetAsync(ws, 0, w.total, s) != cudaSuccess)
        return dfail(TSB_ERR_CUDA, "decode: memset: %s", cudaGetErrorString(cudaGetLastError()));
    void* args[] = {&p};
    const cudaError_t e = cudaLaunchCooperativeKernel((const void*) kern, dim3(sms), dim3(kDecThreads), args, smem, s);
    if (e != cudaSuccess) return dfail(TSB_ERR_CUDA, "decode: launch: %s", cudaGetErrorString(e));
    return TSB_OK;
}

int tsb_moe_decode_error(const tsb_decode_desc* d, const void* workspace, unsigned* code) {
    if (!d || !workspace || !code) return dfail(TSB_ERR_ARG, "decode_error: null argument");
    const WsLayout w = ws_layout(d);
    if (cudaMemcpy(code, (const uint8_t*) workspace + w.err, sizeof(unsigned) * 128, cudaMemcpyDeviceToHost) != cudaSuccess)
        return dfail(TSB_ERR_CUDA, "decode_error: %s", cudaGetErrorString(cudaGetLastError()));
    return TSB_OK;
}

const char* tsb_decode_last_error(void) { return g_derr; }

int tsb_moe_decode_set_trace(unsigned long long* buf) {
    g_trace = buf;
    return TSB_OK;
}

int tsb_moe_decode_set_debug(int withhold_cta) {
    if (withhold_cta < 0) return dfail(TSB_ERR_ARG, "decode_set_debug: a CTA index + 1, or 0");
    g_withhold = withhold_cta;
    return TSB_OK;
}

}  // extern "C"
