/*
 * tsb_moe.h - C ABI of the B200 MoE expert-layer path (libtsb_moe.so).
 *
 * Drop-in boundary for TinyStrata's expert-layer entry points.  Each function names the reference interface it
 * replaces (paths inside the TinyStrata tree).  Conventions, as the reference's:
 *   - every pointer argument is a DEVICE pointer unless stated; buffers are caller-owned, calls allocate nothing on the
 *     stream path and never synchronise it (counts such as n_groups stay on the device, so calls are graph-capturable);
 *   - ggml type ids: Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q6_K = 14, IQ3_XXS = 18, IQ3_S = 21; weights are raw GGUF blocks;
 *   - activations are q8_1 blocks (fp16 d, fp16 sum, 32 int8 codes: 36 bytes per 32 values);
 *   - `stream` is a cudaStream_t (0 = the legacy default stream).
 * Every call returns TSB_OK (0) or a negative tsb_status; tsb_last_error() describes the last failure of the calling
 * thread.  Nothing here exits or throws.
 */
#ifndef TSB_MOE_H
#define TSB_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSB_MOE_ABI_VERSION 1

enum tsb_status {
    TSB_OK = 0,
    TSB_ERR_ARG = -1,          /* a null pointer, a bad size or count */
    TSB_ERR_UNSUPPORTED = -2,  /* a format or shape without a kernel */
    TSB_ERR_CUDA = -3,         /* a CUDA launch or runtime error (see tsb_last_error) */
    TSB_ERR_ALIGN = -4,        /* a buffer or blob offset not aligned as the kernel needs */
    TSB_ERR_WORKSPACE = -5,    /* caller workspace smaller than the query said */
    TSB_ERR_COMM = -6          /* a communicator call failed or a peer did not answer within the bound */
};

/* The layout of one expert blob: [gate rows | up rows | down rows] of raw GGUF blocks.
 * Replaces strata::kernels::NativeExpertLayout (include/strata/kernels/iq_kernels.hpp:45-53). */
typedef struct tsb_expert_layout {
    int32_t gu_type, d_type;
    int64_t n_embd, n_ff;
    uint64_t gu_row, d_row;      /* bytes per row */
    uint64_t up_off, down_off;   /* byte offsets inside the blob */
    uint64_t bytes;              /* the whole blob */
} tsb_expert_layout;

int tsb_moe_abi_version(void);
/* The calling thread's last error message ("" when none). */
const char* tsb_last_error(void);
/* The current device's error word: non-zero when a kernel's bounded wait gave up (the kernel then returned early) or
 * a device-side count exceeded the capacity the caller passed (the kernel clamped it).  `clear` resets it.  Reads
 * device memory (synchronous).  The word is a module global of the library, zero when it loads: the library's first
 * call on a device looks up its address (and may load the module), so make that first call outside stream capture. */
int tsb_device_error(unsigned* code, int clear);
/* The bound of every spin-wait in this library's kernels on the current device (default 2 s, accepted 1e5 .. 6e10 ns):
 * a wait that runs past it records its site in the error word and the kernel returns early.  Synchronous; set it outside
 * stream capture.  No counterpart in the reference (its kernels do not wait on one another). */
int tsb_set_wait_limit_ns(uint64_t ns);

/* --------------------------------------------------------------------------------------------- formats */
/* Replaces iq_supported / iq_row_bytes (iq_kernels.hpp:17-21). */
int tsb_type_supported(int ggml_type);
int64_t tsb_row_bytes(int ggml_type, int64_t n);
/* Replaces native_expert_layout / native_expert_supported / native_expert_scratch_bytes (iq_kernels.hpp:53-62). */
int tsb_native_expert_layout(int gu_type, int d_type, int64_t n_embd, int64_t n_ff, tsb_expert_layout* out);
int tsb_native_expert_supported(int gu_type, int d_type, int64_t n_embd, int64_t n_ff);
uint64_t tsb_native_expert_scratch_bytes(int64_t cap_entries, int64_t n_ff);

/* --------------------------------------------------------------------------------------------- activations */
/* q8_1 blocks of n_rows rows of n_cols floats (n_cols % 32 == 0).  Replaces quantize_q8_1_rows (iq_kernels.hpp:24)
 * and native_quantize_q8_1 (native_mmvq.hpp:38): the same blocks bit for bit. */
int tsb_quantize_q8_1_rows(const float* x, int64_t n_rows, int64_t n_cols, void* y, void* stream);

/* --------------------------------------------------------------------------------------------- router */
/* fp32 router logits: logits[t * ld + o] = W[o] . h[t] for o < n_out (W row-major [n_out][n_in], 16-byte aligned).
 * Replaces the f32mm router GEMV (src/qwen35/q36_engine.cu:2106-2131; the shared-expert gate is row n_expert). */
int tsb_router_logits_f32(const float* W, const float* h, float* logits, int n_in, int n_out, int n_tok, int ld,
                          void* stream);
/* Softmax top-k with renormalised weights, ids and weights [n_tok][k], logits row stride ld.
 * Replaces native_router_topk (include/strata/kernels/native_router.hpp:5-6), generalised from (256, 8) to any
 * multiple of 32 experts up to 512 and k <= 32; the (256, 8) case gives the same ids and weights bit for bit. */
int tsb_native_router_topk(const float* logits, int32_t* ids, float* weights, int n_expert, int k, int n_tok, int ld,
                           void* stream);
/* Gemma 4 / LFM2 routing: gate 0 = softmax(logit * in_scale), 1 = sigmoid; the n_used largest of p + bias; weights
 * the bare p, divided by max(sum, 6.103515625e-5) when norm, times escale[id] when given, times w_scale when non-zero.
 * Replaces route_rows (include/strata/gemma4/kernels.hpp; src/gemma4/kernels.cu:289-356). */
int tsb_route_rows(const float* logits, int n_expert, int n_used, int rows, int gate, float in_scale, const float* bias,
                   const float* escale, int norm, float w_scale, int32_t* ids, float* w, void* stream);

/* --------------------------------------------------------------------------------------------- dispatch */
/* Decode grouping: one group per expert used (ascending id) with blob address blobs + id * blob_stride, its entries
 * (entry e = t * K + k) in entry order: grp_ptr[<= n_ent], grp_start[<= n_ent + 1], *n_groups, ent_dst[e'] = e,
 * ent_tok[e'] = e / K.  Replaces k_group / k_group_small (src/qwen35/q36_engine.cu:396-422,
 * src/qwen35/q36_kernels.cuh:347-381). */
int tsb_moe_group(const int32_t* ids, int n_ent, int K, int n_expert, const void* blobs, uint64_t blob_stride,
                  uint64_t* grp_ptr, int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst, int32_t* ent_tok,
                  void* stream);

/* Prefill permutation: entries e = t * K + k (ids [n_ent]) sorted stably by expert.  bounds[x] = first row of expert
 * x (bounds[n_expert] = entries placed), row_ent[row] = e, row_tok[row] = e / K, rinv[e] = row (-1 for an id outside
 * [0, n_expert), which is dropped).  Replaces k_route_count / k_route_scan / k_route_scatter
 * (src/qwen35/q36_engine.cu:486-510) without their device-to-host copy: the bounds stay on the device. */
int tsb_moe_dispatch(const int32_t* ids, int n_ent, int K, int n_expert, int32_t* bounds, int32_t* row_ent,
                     int32_t* row_tok, int32_t* rinv, void* stream);
/* --------------------------------------------------------------------------------------------- experts */
/* Grouped experts, SwiGLU: for each group g (blob grp_ptr[g]) and entry e in [grp_start[g], grp_start[g+1]):
 * out[ent_dst[e]] = down(q8_1(silu(gate . x) * (up . x))) with x = token ent_tok[e] of x_q8_1 (n_embd / 32 blocks per
 * token).  Counts are read on the device.  scratch: tsb_native_expert_scratch_bytes(cap_entries, n_ff) bytes.
 * Replaces native_expert_grouped (include/strata/kernels/iq_kernels.hpp:75-78); grid_groups is accepted and, as
 * there, never changes the results. */
int tsb_native_expert_grouped(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                              const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                              int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, void* scratch, float* out,
                              void* stream, int64_t grid_groups);
/* The same with the activation chosen: act 0 SwiGLU, 1 GELU-tanh (Gemma 4), 2 SwiGLU with the inputs clamped to
 * `limit` (LFM2).  Replaces gemma_native_mmvq_ids + geglu_rows / swiglu_clamp_rows + gemma_native_quantize_q8_1 +
 * the down gemma_native_mmvq_ids (src/gemma4/matvec.hpp:150-171, include/strata/gemma4/kernels.hpp). */
int tsb_native_expert_grouped_act(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                                  const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                                  int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, void* scratch,
                                  float* out, int act, float limit, void* stream);

/* tsb_native_expert_grouped (SwiGLU) without a caller scratch buffer: the hidden vectors live in a fixed 1 MiB device
 * array inside this library (cap_entries * n_ff * 4 bytes, rounded up to 256, must fit: 128 entries at n_ff 2048;
 * larger calls return TSB_ERR_WORKSPACE and launch nothing).  For callers that hold no workspace and must not
 * allocate one on the call path.  The array starts at zero when the module loads; the hidden vectors need no clearing
 * between calls.  A bounded wait that gives up is recorded in the device error word (tsb_device_error), as for every
 * other entry point.  There is ONE array per device: calls that overlap in time on a device (other streams or threads)
 * race on it.  Its address is looked up once per device with cudaGetSymbolAddress at the first call, which may load
 * the module: make that first call outside any stream capture; the looked-up address does not survive a
 * cudaDeviceReset.  No counterpart in the reference (native_expert_grouped, iq_kernels.hpp:75-78, always takes the
 * caller's scratch). */
int tsb_native_expert_grouped_noalloc(const tsb_expert_layout* L, const uint64_t* grp_ptr, const int32_t* grp_start,
                                      const int32_t* n_groups, const int32_t* ent_dst, const int32_t* ent_tok,
                                      int64_t cap_groups, int64_t cap_entries, const void* x_q8_1, float* out,
                                      void* stream);

/* --------------------------------------------------------------------------------------------- prefill (prompt path)
 * The activations of the tensor-core products live in the "mmq" layout, the role of the reference's block_q8_1_mmq
 * (include/strata/prefill/moe_mmq.hpp:37): int8 codes [rows][K], then fp32 block scales d [rows][ldS] (the q8_1 fp16
 * scale, as a float) and d * (sum of the block's codes) [rows][ldS], ldS = K / 32 rounded up to a multiple of 4, each
 * part starting on 256 bytes.  Codes and scales are the q8_1 quantiser's, bit for bit.  Buffers 256-byte aligned. */
uint64_t tsb_mmq_act_bytes(int64_t rows, int64_t K);
/* fp32 rows -> mmq layout: output row r quantises row row_src[r] of x (null: row r; row stride ld_x floats).  The gather
 * puts the entries in expert order for the grouped products.  Replaces mmq::quantize(x, ids, xq, ...) (moe_mmq.hpp:37,
 * src/prefill/moe_mmq.cu:322) and Mmq::quantize (src/gemma4/mmq.hpp:31-41). */
int tsb_mmq_quantize(const float* x, int64_t ld_x, const int32_t* row_src, int n_rows, int K, void* act, void* stream);
/* q8_1 blocks (quantize_q8_1_rows's) -> mmq layout, output row r from row row_src[r] (null: r); the same codes and scales.
 * For activations that arrive already quantised (an expert-parallel exchange). */
int tsb_mmq_from_q8_1(const void* x_q8_1, const int32_t* row_src, int n_rows, int K, void* act, void* stream);
/* Prefill grouped gate/up on the tensor cores (tcgen05.mma.kind::i8, TMA-loaded activation tiles): for group g (rows
 * [bounds[g], bounds[g+1]) of x_act, weights blobs + g * blob_stride in layout L; bounds null: one group of n_rows rows),
 * h[row] = q8_1(act(gate . x, up . x)) written to h_act in the mmq layout (tsb_mmq_act_bytes(n_rows, n_ff)).  Per
 * 32-value block the integer dot is exact (int32 in tensor memory) and is scaled and summed in fp32 block after block,
 * as the reference's.  act as tsb_native_expert_grouped_act.  Weights Q4_0, Q8_0, Q4_K, Q6_K, IQ3_XXS or IQ3_S (L's
 * gu_type); n_embd a multiple of 64 (>= 128) and of 256 for the K-quant and i-quant formats, n_ff a multiple of 64;
 * at most 512 groups.  Replaces the gate/up mmq::Context::run + mmq::swiglu + the re-quantisation of the prompt path
 * (include/strata/prefill/moe_mmq.hpp:58-81, src/prefill/moe_mmq.cu:334-384, 123-131; src/gemma4/mmq.cu:74-110). */
int tsb_moe_prefill_gu(const tsb_expert_layout* L, const void* blobs, uint64_t blob_stride, const int32_t* bounds,
                       int n_groups, int n_rows, const void* x_act, void* h_act, int act, float limit, void* stream);
/* Prefill grouped down: out[row] = down . h[row] (fp32 [n_rows][n_embd], 16-byte aligned) with the groups as above and
 * h_act the hidden rows tsb_moe_prefill_gu wrote.  Replaces the down mmq::Context::run (src/prefill/moe_mmq.cu:334-384). */
int tsb_moe_prefill_down(const tsb_expert_layout* L, const void* blobs, uint64_t blob_stride, const int32_t* bounds,
                         int n_groups, int n_rows, const void* h_act, float* out, void* stream);
/* A grouped product on the tensor cores with fp32 output: for each of n matrices of [w_rows][w_cols] weights of
 * ggml_type, `stride` bytes apart from w, the activation rows [bounds[e], bounds[e+1]) of x_act (the tensor-core layout
 * of total_rows rows of w_cols values) times matrix e; row i's product goes to row ids[i] of dst (row i when ids is
 * null), ld_dst floats a row.  With one matrix, bounds may be null (every row).  Replaces mmq::Context::run
 * (include/strata/prefill/moe_mmq.hpp:69-98, src/prefill/moe_mmq.cu) and gemma4::Mmq::mul (src/gemma4/mmq.hpp:36-41,
 * mmq.cu:74-110). */
int tsb_mmq_product(const void* w, int ggml_type, int64_t w_rows, int64_t w_cols, uint64_t stride, int n,
                    const void* x_act, const int32_t* bounds, const int32_t* ids, int64_t total_rows, float* dst,
                    int64_t ld_dst, void* stream);

/* Bench only: 0 = both expert kernels (default), 1 = gate/up + activation only, 2 = down only (reads the scratch the
 * previous call left).  Replaces native_expert_set_mode's phase argument (iq_kernels.hpp:85).  Process-wide; set
 * outside graph capture. */
int tsb_native_expert_set_phase(int phase);

/* --------------------------------------------------------------------------------------------- combine */
/* x[t] += sum_k wts[t,k] parts[prow ? prow[t*K+k] : t*K+k] (fma in pick order) + sigmoid(sgate[t*sg_stride]) *
 * shared[t] (shared / sgate may be null); with wn or h: h = x * rsqrt(mean(x^2) + eps) * wn (wn null = 1) and, with hq,
 * hq = q8_1(h).  Replaces k_moe_out / k_moe_out_small (src/qwen35/q36_engine.cu:307-332,
 * src/qwen35/q36_kernels.cuh:252-290). */
int tsb_moe_combine(float* x, const float* parts, const int32_t* prow, const float* wts, int K, const float* shared,
                    const float* sgate, int sg_stride, const float* wn, float* h, void* hq, int n, float eps, int n_tok,
                    void* stream);
/* h = x * rsqrt(mean(x^2) + eps) * wn (wn null = 1) and hq = q8_1(h) for n_tok rows (either output may be null).
 * Replaces k_add_rms_q without the add (src/qwen35/q36_kernels.cuh:222-250): the layer input's norm and q8_1 image. */
int tsb_rms_norm_q8_1(const float* x, const float* wn, float* h, void* hq, int n, float eps, int n_tok, void* stream);
/* acc[t] += sum_k w[t,k] x[t*K+k], n values per row.  Replaces moe_sum (src/gemma4/kernels.cu:358-366). */
int tsb_moe_sum(const float* x, const float* w, float* acc, int n, int n_used, int rows, void* stream);

/* Up to 32 scaled vectors added into sums: acc[k][i] += x[k][i] * w[k] for k in order (the sums may be one and the same
 * vector).  Replaces add_scaled and its ScaledRows (include/strata/gemma4/kernels.hpp:51-56, src/gemma4/kernels.cu:
 * 245-249, 1444-1447): the host structure holds device pointers and the weights. */
typedef struct tsb_scaled_rows {
    const float* x[32];
    float* acc[32];
    float w[32];
} tsb_scaled_rows;
int tsb_add_scaled(const tsb_scaled_rows* rows, int count, int n, void* stream);
/* The Gemma 4 layer tail after the routed experts, per row of n values: cur = rms(moe) * post_moe + mlp (mlp may be
 * null), out = rms(cur) * post_ffn, r = (r + out) * out_scale (norm weights may be null: 1).  Replaces the
 * rms_norm / axpy / rms_norm / axpy / scale sequence of Gemma4::layer_tail (src/gemma4/gemma4.cpp:560-568). */
int tsb_moe_layer_tail(const float* moe, const float* post_moe, const float* mlp, const float* post_ffn, float* r,
                       float out_scale, int n, int rows, float eps, void* stream);

/* --------------------------------------------------------------------------------------------- fused decode */
/* One layer of the fused decode path: device pointers to its expert blobs ([n_expert][blob bytes], the
 * NativeExpertLayout of each), its fp32 router ([n_expert + 1][n_embd]: the expert rows, then the shared-expert gate
 * row, as q36_engine.cu:1139-1142 appends it) and its shared expert blob. */
typedef struct tsb_decode_layer {
    const void* blobs;
    const float* router;
    const void* sh_blob;
    const float* logit_prior;   /* optional [n_tok][n_expert] fp32 added to the router logits before the softmax (an
                                   additive routing prior, e.g. a benchmark's fixed expert choice); null: none */
} tsb_decode_layer;

typedef struct tsb_decode_desc {
    uint32_t struct_size;            /* sizeof(tsb_decode_desc) */
    int32_t n_layers, n_tok;         /* layers of the step; tokens (1..16) */
    int32_t n_embd, n_ff, n_expert, n_used, sh_n_ff;
    int32_t gu_type, d_type, sh_gu_type, sh_d_type;
    float eps;                       /* the RMS epsilon of the layer input's norm */
} tsb_decode_desc;

/* Workspace bytes tsb_moe_decode_layers needs for this description. */
uint64_t tsb_moe_decode_workspace_bytes(const tsb_decode_desc* d);
/* Every layer's MoE block for n_tok decode tokens in one persistent launch (one CTA per SM, cooperative):
 * per layer h = rms(x), router GEMV, softmax top-k, grouping, routed and shared experts, and x += the gated combine
 * (q36_engine.cu:2821-2925 with k_moe_out_small, per layer).  x: [n_tok][n_embd] fp32, in / out.  layers: a DEVICE
 * array of n_layers tsb_decode_layer.  ids_rec / w_rec (optional, [n_layers][n_tok][n_used]) record the routing and
 * x_rec (optional, [n_layers][n_tok][n_embd]) x after every layer (a step that checks itself layer by layer).
 * Supported: IQ3_XXS routed experts (n_ff 512), 256 experts, Q8_0 shared expert, SwiGLU.  Replaces the per-layer
 * sequence f32mm + route_group + native_expert_grouped + shared expert + moe_end of the Qwen3.6 engine. */
int tsb_moe_decode_layers(const tsb_decode_desc* d, const tsb_decode_layer* layers, float* x, int32_t* ids_rec,
                          float* w_rec, float* x_rec, void* workspace, uint64_t ws_bytes, void* stream);
/* The decode kernel's error record in `workspace`: code[0] non-zero when a bounded wait gave up (its site), code[1..4]
 * that wait's context (unit sequence and layer, producer progress, claim counter, CTA, raw barrier words).  `code`
 * holds 128 words.
 * Synchronous read. */
int tsb_moe_decode_error(const tsb_decode_desc* d, const void* workspace, unsigned* code);
/* The calling thread's last decode-path error message. */
const char* tsb_decode_last_error(void);
/* Profiling: launches made after this call stamp %globaltimer (ns) into `buf` (device, [n_layers][16][n_CTAs]
 * u64) at each phase boundary of every layer (consumer stamps 0-8, producer stamps 9-12, see tsb_decode.cuh); null
 * turns it off.  Process-wide; a captured graph keeps the buffer it was captured with. */
int tsb_moe_decode_set_trace(unsigned long long* buf);
/* Tests of the bounded waits: launches made after this call have CTA withhold_cta - 1 skip publishing its layer-0
 * router logits, so every other CTA's wait for them runs out (their site lands in the error record); 0 turns it off.
 * Process-wide.  No counterpart in the reference. */
int tsb_moe_decode_set_debug(int withhold_cta);

/* ---- the Gemma 4 / LFM2 decode MoE block in one launch.  Replaces the per-layer decode sequence of those engines
 * (src/gemma4/engine.cpp:2436-2457: route_rows, gemma_native_mmvq_ids gate/up, geglu_rows / swiglu_clamp_rows, the
 * hidden rows' q8_1, gemma_native_mmvq_ids down, moe_sum; and the dense shared MLP's gate/up, activation, q8_1 and
 * down).  Per token t: logits = router . h[t] (router fp32 [n_expert][n_embd]); picks and weights as tsb_route_rows
 * (gate, in_scale, bias, escale, norm, w_scale); out[t] (+)= sum_k w[t,k] down_k(q8_1(act(gate_k . hq[t], up_k .
 * hq[t]))) in pick order, as tsb_moe_sum; with a shared MLP (sh_n_ff > 0, blob in the expert layout of the same
 * formats) sh_out[t] = its output (sh_act).  Every value equals the layer-by-layer entry points' bit for bit.  The
 * workspace begins with the router logits [n_tok][n_expert].  Weights Q4_0 / Q4_0 or Q4_K / Q6_K (gate-up / down);
 * 1..16 tokens, n_tok * n_used <= 128, n_expert a multiple of 32 up to 512, rows of up to 256 calls. */
typedef struct tsb_decode_act_desc {
    uint32_t struct_size;   /* sizeof(tsb_decode_act_desc) */
    int32_t n_tok, n_embd, n_ff, n_expert, n_used, sh_n_ff;
    int32_t gu_type, d_type;
    int32_t act, sh_act;    /* 0 SwiGLU, 1 GELU-tanh, 2 clamped SwiGLU (limit) */
    float limit;
    int32_t gate;           /* 0 softmax of logit * in_scale, 1 sigmoid */
    float in_scale;
    int32_t norm;
    float w_scale;
} tsb_decode_act_desc;
uint64_t tsb_moe_decode_act_workspace_bytes(const tsb_decode_act_desc* d);
/* Phase stamps of tsb_moe_decode_act: with a device buffer of (SM count) * 8 u64, every CTA stores the global timer
 * at its start, end of phase A, after barrier 1, after routing, end of phase B, after barrier 2, after quantising the
 * hidden rows and at its end; null turns it off.  Process-wide; a captured graph keeps the buffer it was captured
 * with.  No counterpart in the reference. */
int tsb_moe_decode_act_set_trace(unsigned long long* buf);
int tsb_moe_decode_act(const tsb_decode_act_desc* d, const float* router, const float* bias, const float* escale,
                       const float* h, const void* hq, const void* blobs, uint64_t blob_stride, const void* sh_blob,
                       float* out, int accumulate, float* sh_out, int32_t* ids, float* w, void* workspace,
                       uint64_t ws_bytes, void* stream);

/* --------------------------------------------------------------------------------------------- small products */
/* Up to TSB_MMVQ_MAX matrices of one ggml type and shape [n_out][n_in] in one launch, each times its own q8_1 column
 * (n_in / 32 blocks): y[i][r] = row r of w[i] . x[i], each value the reference's iq_mmvq row dot bit for bit (the
 * same calls, lanes and sum order).  Replaces gemma_native_mmvq_slots / gemma_native_mmvq_ids
 * (include/strata/gemma4/matvec.hpp:143-171: the Gemma 4 / LFM2 cached-expert decode step).  Formats Q4_0, Q8_0,
 * Q4_K, Q6_K, IQ3_XXS, IQ3_S (tsb_mmvq_supported); others return TSB_ERR_UNSUPPORTED and launch nothing, where the
 * reference's call returns false. */
#define TSB_MMVQ_MAX 32
typedef struct tsb_mmvq_slots {
    const void* w[TSB_MMVQ_MAX];
    const void* x[TSB_MMVQ_MAX];
    float* y[TSB_MMVQ_MAX];
} tsb_mmvq_slots;
/* The same with the matrices the device picked: matrix j = table[ids[j]] + offset bytes (table and ids on the device),
 * column x + (j / x_every) * x_stride bytes, output y + j * y_stride floats. */
typedef struct tsb_mmvq_ids {
    const void* const* table;
    const int32_t* ids;
    uint64_t offset;
    const void* x;
    uint64_t x_stride;
    int32_t x_every;
    float* y;
    uint64_t y_stride;
} tsb_mmvq_ids;
int tsb_mmvq_supported(int ggml_type);
int tsb_mmvq_run_slots(int ggml_type, const tsb_mmvq_slots* slots, int count, int n_in, int n_out, void* stream);
int tsb_mmvq_run_ids(int ggml_type, const tsb_mmvq_ids* m, int count, int n_in, int n_out, void* stream);

/* ------------------------------------------------------------------------------------------- host-staged experts */
/* A layer whose experts do not all sit in HBM: n_slots of them in device slots (expert x in slot slot_of[x] >= 0, at
 * slots + slot_of[x] * stride), every expert's blob in host memory at host_blobs + x * stride (n_expert * stride bytes,
 * pinned and mapped for the device: cudaHostAlloc, or cudaHostRegister with cudaHostRegisterMapped).  Replaces the
 * reference's hybrid mode (src/qwen35/q36_engine.cu: k_group_hy 423-452, moe_hybrid_gpu / moe_hybrid_cpu /
 * k_merge_cpu 3052-3210, rebalance 3215-3265, the streamed layer 2995-3049).  Where the reference runs the entries
 * of experts without a slot on a CPU thread pool, here the GPU pulls those experts' blobs over the host link itself
 * and runs every entry through the grouped expert kernels: outputs equal a resident layer's bit for bit. */

/* Grouping as tsb_moe_group (slot_of, device array [n_expert]; ids outside [0, n_expert) are dropped), each group's
 * blob at its expert's slot or, for an expert without one, at the next free blob of stage (stage_cap blobs of stride
 * bytes, stage_cap >= min(n_ent, n_expert)), which the same call fills from host_blobs on `stream` (device loads of
 * the mapped host memory: no host synchronisation, graph-capturable).  counts (optional, device [n_expert]) += the
 * entries of each expert: the usage a placement reads between steps.  stride a multiple of 16. */
int tsb_moe_group_staged(const int32_t* ids, int n_ent, int K, int n_expert, const int32_t* slot_of, int n_slots,
                         const void* slots, const void* host_blobs, uint64_t stride, void* stage, int stage_cap,
                         uint64_t* grp_ptr, int32_t* grp_start, int32_t* n_groups, int32_t* ent_dst, int32_t* ent_tok,
                         uint32_t* counts, void* stream);
/* Host arrays.  The reference's rebalance for one layer: experts by score (highest first, ties the lower id), slots
 * by their resident's score (lowest first, ties the lower slot); each top-n_slots expert without a slot takes the
 * next such slot while its resident scores lower, up to max_swaps moves; then every score is halved (the age).
 * Writes the moves (expert, slot) and updates slot_of / exp_in_slot; returns the number of moves (>= 0).  With no
 * partial residency (n_slots 0 or n_expert) nothing changes, scores included. */
int tsb_staged_rebalance(double* score, int n_expert, int n_slots, int32_t* slot_of, int32_t* exp_in_slot,
                         int max_swaps, int32_t* move_expert, int32_t* move_slot);
/* The moves' blobs (blob_bytes each) host to device into their slots on `stream`; upload slot_of after them on the
 * same stream so that no step reads a slot before its blob. */
int tsb_staged_load(const void* host_blobs, void* slots, uint64_t stride, uint64_t blob_bytes, const int32_t* move_expert,
                    const int32_t* move_slot, int n_moves, int n_expert, int n_slots, void* stream);
/* The streamed layer of the prompt path: every expert's blob into stage in expert order (n_expert * stride bytes),
 * runs of consecutive slots holding consecutive experts device to device and runs of experts without a slot host to
 * device; the whole layer in one host copy when fewer than half the experts are resident or `whole` is set.
 * slot_of is a HOST array here.  Returns the number of copies issued (> 0) or a negative status. */
int tsb_stage_layer(const int32_t* slot_of, int n_expert, int n_slots, const void* slots, const void* host_blobs,
                    uint64_t stride, void* stage, int whole, void* stream);

/* --------------------------------------------------------------------------------------------- expert parallelism */
/* Prompt-path experts sharded over the ranks of one node (one process per GPU), dispatch and return over NCCL
 * point-to-point exchanges on NVLink.  The reference runs one GPU per engine; the per-rank body is its prompt branch
 * (src/gemma4/engine.cpp:2436-2457 with src/prefill/moe_mmq.cu:334-384) over the rank's experts.  Expert e lives on
 * rank e % world as local expert e / world (cyclic) or on rank e / (n_expert / world) (block).  A token goes to a rank
 * once, whatever number of its picks live there.  Per step one host synchronisation (the exchanged row counts); every
 * other step of the glue (plan, pack, unpack, per-row partial sums, the ordered sum of the returns) is a kernel. */
typedef struct tsb_ep tsb_ep;
/* An NCCL unique id (128 bytes) for tsb_ep_create, made on one rank and handed to every rank by the caller. */
int tsb_ep_unique_id(void* id128);
/* Join the ranks' communicator (collective: every rank calls it with the same id) on the current device and size the
 * buffers for max_tokens tokens per rank.  blobs: this rank's n_expert / world expert blobs (stride blob_stride) in
 * local order.  The NCCL library the process already loaded is used (dlopen of libnccl.so.2). */
int tsb_ep_create(const void* id128, int rank, int world, const tsb_expert_layout* L, const void* blobs,
                  uint64_t blob_stride, int n_expert, int n_used, int cyclic, int max_tokens, int act, float limit,
                  tsb_ep** out);
/* Route this rank's n_tok tokens: x_q8_1 [n_tok][n_embd / 32 blocks] q8_1 rows, ids / w [n_tok][n_used] (the
 * router's picks).  Plans and packs on `stream`, exchanges the counts (the one host synchronisation, bounded by the
 * wait limit), and starts the dispatch exchange of every micro-batch (1..4 slices of the tokens) on the
 * communicator's stream.  Returns once the exchanges are queued; the caller may queue more work on `stream` (the
 * shared expert) before tsb_ep_combine. */
int tsb_ep_dispatch(tsb_ep* ep, const void* x_q8_1, const int32_t* ids, const float* w, int n_tok, int micro_batches,
                    void* stream);
/* micro_batches is collective: every rank passes the same value (a rank's slice may hold no tokens). */
/* Finish the step tsb_ep_dispatch started: per micro-batch the local grouped experts on the tensor cores as its rows
 * arrive, the weighted partial row per received token, its return exchange; then per token, on `stream`,
 * out = (accumulate ? out : 0) + the partials of the ranks it went to in rank order (+ sigmoid(sgate[t * sg_stride])
 * shared[t] when shared is given).  return_bf16: partial rows travel as bf16 instead of fp32 (half the return bytes;
 * the rounding moves single outputs by up to ~2 % of the RMS, past the layer tolerance fp32 returns meet).
 * return_bf16 is collective: the same on every rank. */
int tsb_ep_combine(tsb_ep* ep, float* out, int accumulate, const float* shared, const float* sgate, int sg_stride,
                   int return_bf16, void* stream);
/* The bound of the host's waits on the exchanges (default 120 s): past it the communicator is aborted and the call
 * returns TSB_ERR_COMM (the handle is then only good for tsb_ep_destroy). */
int tsb_ep_set_timeout_ns(tsb_ep* ep, uint64_t ns);
/* Wait, within the bound, for every exchange issued so far (host-synchronous; a caller that reads results on the host
 * calls it before synchronising its own stream, so that a peer that never answers ends in TSB_ERR_COMM). */
int tsb_ep_synchronize(tsb_ep* ep);
/* The last step's rows: rows sent to other ranks and to this one, rows received, picks computed here. */
int tsb_ep_stats(const tsb_ep* ep, int64_t* sent, int64_t* received, int64_t* picks);
/* Free the buffers and the communicator (collective). */
int tsb_ep_destroy(tsb_ep* ep);

/* --------------------------------------------------------------------------------------------- GGUF files */
/* A GGUF (v2 / v3) model file, memory-mapped read-only: metadata, tensor directory, and the repack of a layer's
 * expert tensors into the native expert blobs above.  Replaces the parts of include/strata/artifact/gguf_reader.hpp the
 * expert path needs and the blob build of src/qwen35/q36_engine.cu:1144-1167, 1196-1200.  Host memory only. */
typedef struct tsb_gguf tsb_gguf;
typedef struct tsb_gguf_tensor_info {
    int32_t type, n_dims;
    int64_t ne[4];         /* ne[0] innermost (values per row), as the file stores them */
    uint64_t bytes;
    const void* data;      /* inside the mapping; valid until tsb_gguf_close */
} tsb_gguf_tensor_info;
int tsb_gguf_open(const char* path, tsb_gguf** out);
int tsb_gguf_close(tsb_gguf* g);
int tsb_gguf_tensor_count(const tsb_gguf* g);
int tsb_gguf_tensor_name(const tsb_gguf* g, int i, char* buf, int buf_bytes);
int tsb_gguf_tensor(const tsb_gguf* g, const char* name, tsb_gguf_tensor_info* out);
int tsb_gguf_kv_int(const tsb_gguf* g, const char* key, int64_t* value);
int tsb_gguf_kv_float(const tsb_gguf* g, const char* key, double* value);
int tsb_gguf_kv_str(const tsb_gguf* g, const char* key, char* buf, int buf_bytes);
/* The layer whose tensors start with `prefix` (e.g. "blk.3."): its ffn_{gate,up,down}_exps types and shapes as a
 * native expert layout, the blob stride (the blob rounded up to whole blocks of both types and 16 bytes, as the
 * reference's engine places them) and the expert count. */
int tsb_gguf_expert_layer(const tsb_gguf* g, const char* prefix, tsb_expert_layout* L, uint64_t* stride,
                          int32_t* n_expert);
/* Experts [first, first + count) of that layer as native expert blobs at dst + q * stride (host memory, zero bytes
 * between a blob's end and the next), dst_bytes >= count * stride. */
int tsb_gguf_repack_experts(const tsb_gguf* g, const char* prefix, int first, int count, void* dst,
                            uint64_t dst_bytes);

/* --------------------------------------------------------------------------------------------- test hook */
/* The per-call integer sums and float values of one weight row (n values) against one q8_1 activation, as the
 * expert kernels compute them (calls in row_dot order, src/kernels/cuda/iq_kernels.cu:695-705).  Parity tests only. */
int tsb_debug_row_calls(int ggml_type, const void* row, const void* x_q8_1, int64_t n, int32_t* sumi, float* val,
                        void* stream);
/* The tensor-core block sums of the prefill products: one launch of the gate/up (mode 0, output h_act) or down (mode 1,
 * output out) kernel over one expert blob and n_rows rows of x_act, which also stores the int32 block sums of its first
 * tile (rows 0..127, tile columns 0..127) in sums: [K / 32][split][128 rows][128 columns], split 2 for Q6_K (its 16-value
 * halves) and 1 otherwise.  Gate/up tile columns interleave gate and up rows in 32-row groups (columns 0-31 gate rows
 * 0-31, 32-63 up rows 0-31, 64-95 gate rows 32-63, 96-127 up rows 32-63).  Parity tests only. */
int tsb_debug_mmq_block_sums(const tsb_expert_layout* L, int mode, const void* blob, int n_rows, const void* x_act,
                             void* h_act, float* out, int32_t* sums, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TSB_MOE_H */
