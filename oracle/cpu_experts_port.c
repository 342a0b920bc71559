/*
 * oracle/cpu_experts_port.c - TEST INFRASTRUCTURE (the benchmark's CPU baseline, never the product): a C restatement
 * of the reference's host-side expert path for Q4_0 weights, src/gemma4/cpu_experts.cpp:145-235 (cpu_experts), which
 * the reference runs through ggml-cpu's row quantiser and dot products.  ggml-cpu is a dependency the reference builds
 * from an external llama.cpp tree (STRATA_LLAMA_SOURCE_DIR, cmake/gemma4.cmake:5; only ggml-common.h of ggml commit
 * 3cf03257f219 is vendored, third_party/ggml/VERSION.txt), so its published Q4_0 x Q8_0 algorithm is restated here
 * (quantize_row_q8_0 and ggml_vec_dot_q4_0_q8_0: per 32-value block d = max|x| / 127, q = round(x / d), fp16 d; the
 * dot of a block is (sum of (nibble - 8) * q) * d_w * d_x in fp32), as scalar C that the compiler vectorises.
 *
 * The task structure is the reference's: the activation rows quantised in parallel; the uses (token, expert) sorted
 * stably by expert into runs; gate/up tasks of 32 rows of one expert over all of its uses, GELU-tanh or clamped SiLU;
 * the hidden vectors quantised in parallel; down tasks of 16 output rows over every run; a token's output the sum of
 * its uses in the order they were given.  Workers take task indices from one atomic counter per phase.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK 32
#define Q4_BYTES 18   /* fp16 d, 16 bytes of nibbles */
#define Q8_BYTES 34   /* fp16 d, 32 int8 */
#define ROWS_PER_TASK 32
#define ROWS_PER_DOWN_TASK 16

static uint16_t f2h(float f) {   /* round to nearest even, finite inputs of a quantiser's scale */
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t s = (x >> 16) & 0x8000u;
    int e = (int) ((x >> 23) & 255) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (e >= 31) return (uint16_t) (s | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t) s;
        m |= 0x800000u;
        const int sh = 14 - e;
        uint32_t r = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1))) ++r;
        return (uint16_t) (s | r);
    }
    uint32_t r = ((uint32_t) e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) ++r;
    return (uint16_t) (s | r);
}

static void quantize_q8_0(const float* x, uint8_t* y, int n) {
    for (int b = 0; b < n / QK; ++b) {
        float amax = 0.f;
        for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(x[b * QK + j]));
        const float d = amax / 127.f, id = d != 0.f ? 1.f / d : 0.f;
        uint8_t* blk = y + (size_t) b * Q8_BYTES;
        const uint16_t dh = f2h(d);
        memcpy(blk, &dh, 2);
        int8_t* q = (int8_t*) (blk + 2);
        for (int j = 0; j < QK; ++j) q[j] = (int8_t) roundf(x[b * QK + j] * id);
    }
}

/* The block dot in AVX2 (the form ggml's x86 path takes): the 32 weight values as int8 (nibble - 8), their absolute
 * values times the activation codes with the weights' signs (vpmaddubsw), pairs summed to int32 (vpmaddwd), eight
 * lanes to fp32 and scaled by d_w * d_x into a running fp32 vector; one horizontal sum per row. */
static float dot_q4_0_q8_0(int n, const uint8_t* w, const uint8_t* x) {
    __m256 acc = _mm256_setzero_ps();
    const __m128i lo_mask = _mm_set1_epi8(0x0F);
    const __m256i eight = _mm256_set1_epi8(8);
    const __m256i ones = _mm256_set1_epi16(1);
    for (int b = 0; b < n / QK; ++b) {
        const uint8_t* wb = w + (size_t) b * Q4_BYTES;
        const uint8_t* xb = x + (size_t) b * Q8_BYTES;
        uint16_t dw, dx;
        memcpy(&dw, wb, 2);
        memcpy(&dx, xb, 2);
        const __m128i nib = _mm_loadu_si128((const __m128i*) (wb + 2));
        const __m128i lo = _mm_and_si128(nib, lo_mask), hi = _mm_and_si128(_mm_srli_epi16(nib, 4), lo_mask);
        const __m256i wv = _mm256_sub_epi8(_mm256_set_m128i(hi, lo), eight);
        const __m256i xv = _mm256_loadu_si256((const __m256i*) (xb + 2));
        const __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(wv, wv), _mm256_sign_epi8(xv, wv));
        const __m256 p = _mm256_cvtepi32_ps(_mm256_madd_epi16(p16, ones));
        acc = _mm256_fmadd_ps(_mm256_set1_ps(_cvtsh_ss(dw) * _cvtsh_ss(dx)), p, acc);
    }
    __m128 s4 = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    s4 = _mm_add_ps(s4, _mm_movehl_ps(s4, s4));
    s4 = _mm_add_ss(s4, _mm_shuffle_ps(s4, s4, 1));
    return _mm_cvtss_f32(s4);
}

/* ------------------------------------------------------------------------------------------------ workers */
typedef struct Job Job;
typedef void (*TaskFn)(Job*, int);
struct Job {
    TaskFn fn;
    int n_tasks;
    volatile int next;
    /* the call */
    const uint8_t* blobs;
    size_t stride, gu_row, d_row, up_off, down_off;
    int n_embd, n_ff, rows, n, K, gelu;
    float limit;
    const float* x;
    const int32_t* ids;
    const float* w;
    float* out;
    uint8_t *act, *hq;
    float* h;
    int *by, *run, n_run;
};

static void* worker(void* arg) {
    Job* j = (Job*) arg;
    for (;;) {
        const int t = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (t >= j->n_tasks) break;
        j->fn(j, t);
    }
    return NULL;
}

static void run_phase(Job* j, TaskFn fn, int n_tasks, int threads) {
    j->fn = fn;
    j->n_tasks = n_tasks;
    j->next = 0;
    pthread_t th[256];
    int nt = threads < 256 ? threads : 256;
    for (int i = 1; i < nt; ++i) pthread_create(&th[i], NULL, worker, j);
    worker(j);
    for (int i = 1; i < nt; ++i) pthread_join(th[i], NULL);
}

static void t_quant_act(Job* j, int t) {
    quantize_q8_0(j->x + (size_t) t * j->n_embd, j->act + (size_t) t * (j->n_embd / QK) * Q8_BYTES, j->n_embd);
}

static void t_gate_up(Job* j, int t) {
    const int gu_tasks = (j->n_ff + ROWS_PER_TASK - 1) / ROWS_PER_TASK;
    const int i0 = j->run[t / gu_tasks], i1 = j->run[t / gu_tasks + 1];
    const int e = j->ids[j->by[i0]];
    const uint8_t* blob = j->blobs + (size_t) e * j->stride;
    const int r0 = (t % gu_tasks) * ROWS_PER_TASK, r1 = r0 + ROWS_PER_TASK < j->n_ff ? r0 + ROWS_PER_TASK : j->n_ff;
    const size_t a_bytes = (size_t) (j->n_embd / QK) * Q8_BYTES;
    for (int r = r0; r < r1; ++r) {
        const uint8_t* gate = blob + (size_t) r * j->gu_row;
        const uint8_t* up = blob + j->up_off + (size_t) r * j->gu_row;
        for (int i = i0; i < i1; ++i) {
            const int u = j->by[i];
            const uint8_t* a = j->act + (size_t) (u / j->K) * a_bytes;
            float g = dot_q4_0_q8_0(j->n_embd, gate, a), v = dot_q4_0_q8_0(j->n_embd, up, a);
            float hv;
            if (j->gelu) {
                hv = 0.5f * g * (1.f + tanhf(0.7978845608f * g * (1.f + 0.044715f * g * g))) * v;
            } else {
                g = fminf(g, j->limit);
                v = fminf(fmaxf(v, -j->limit), j->limit);
                hv = g / (1.f + expf(-g)) * v;
            }
            j->h[(size_t) u * j->n_ff + r] = hv;
        }
    }
}

static void t_quant_h(Job* j, int u) {
    quantize_q8_0(j->h + (size_t) u * j->n_ff, j->hq + (size_t) u * (j->n_ff / QK) * Q8_BYTES, j->n_ff);
}

static void t_down(Job* j, int t) {
    float* s = (float*) malloc(sizeof(float) * (size_t) j->n);
    const size_t h_bytes = (size_t) (j->n_ff / QK) * Q8_BYTES;
    const int r0 = t * ROWS_PER_DOWN_TASK;
    const int r1 = r0 + ROWS_PER_DOWN_TASK < j->n_embd ? r0 + ROWS_PER_DOWN_TASK : j->n_embd;
    for (int r = r0; r < r1; ++r) {
        for (int q = 0; q < j->n_run; ++q) {
            const int e = j->ids[j->by[j->run[q]]];
            const uint8_t* down = j->blobs + (size_t) e * j->stride + j->down_off + (size_t) r * j->d_row;
            for (int i = j->run[q]; i < j->run[q + 1]; ++i)
                s[j->by[i]] = dot_q4_0_q8_0(j->n_ff, down, j->hq + (size_t) j->by[i] * h_bytes);
        }
        for (int row = 0; row < j->rows; ++row) {   /* a token's uses in the order given */
            float acc = 0.f;
            for (int k = 0; k < j->K; ++k) acc += j->w[(size_t) row * j->K + k] * s[row * j->K + k];
            j->out[(size_t) row * j->n_embd + r] = acc;
        }
    }
    free(s);
}

static const int32_t* g_sort_ids;
static int cmp_use(const void* a, const void* b) {
    const int ua = *(const int*) a, ub = *(const int*) b;
    const int ea = g_sort_ids[ua], eb = g_sort_ids[ub];
    if (ea != eb) return ea < eb ? -1 : 1;
    return ua < ub ? -1 : ua > ub;   /* stable: the uses of one expert in their given order */
}

/* out[row] = sum over k of w[row][k] * expert ids[row][k] (x[row]) for `rows` tokens of n_embd values, Q4_0 experts
 * (blob: gate rows at 0, up rows at up_off, down rows at down_off; blob_stride bytes apart).  Returns 0 or -1. */
int cx_moe_experts_q4_0(const uint8_t* blobs, size_t blob_stride, size_t up_off, size_t down_off, int n_embd,
                        int n_ff, const float* x, int rows, const int32_t* ids, const float* w, int K, int gelu,
                        float limit, int threads, float* out) {
    if (n_embd % QK || n_ff % QK || rows < 0 || K < 1 || threads < 1) return -1;
    Job j;
    memset(&j, 0, sizeof j);
    j.blobs = blobs;
    j.stride = blob_stride;
    j.gu_row = (size_t) (n_embd / QK) * Q4_BYTES;
    j.d_row = (size_t) (n_ff / QK) * Q4_BYTES;
    j.up_off = up_off;
    j.down_off = down_off;
    j.n_embd = n_embd;
    j.n_ff = n_ff;
    j.rows = rows;
    j.n = rows * K;
    j.K = K;
    j.gelu = gelu;
    j.limit = limit;
    j.x = x;
    j.ids = ids;
    j.w = w;
    j.out = out;
    j.act = (uint8_t*) malloc((size_t) rows * (n_embd / QK) * Q8_BYTES + 1);
    j.hq = (uint8_t*) malloc((size_t) j.n * (n_ff / QK) * Q8_BYTES + 1);
    j.h = (float*) malloc(sizeof(float) * (size_t) j.n * n_ff + 4);
    j.by = (int*) malloc(sizeof(int) * (size_t) (j.n + 1));
    j.run = (int*) malloc(sizeof(int) * (size_t) (j.n + 2));
    for (int i = 0; i < j.n; ++i) j.by[i] = i;
    g_sort_ids = ids;
    qsort(j.by, (size_t) j.n, sizeof(int), cmp_use);
    j.n_run = 0;
    for (int i = 0; i < j.n; ++i)
        if (i == 0 || ids[j.by[i]] != ids[j.by[i - 1]]) j.run[j.n_run++] = i;
    j.run[j.n_run] = j.n;
    run_phase(&j, t_quant_act, rows, threads);
    run_phase(&j, t_gate_up, j.n_run * ((n_ff + ROWS_PER_TASK - 1) / ROWS_PER_TASK), threads);
    run_phase(&j, t_quant_h, j.n, threads);
    run_phase(&j, t_down, (n_embd + ROWS_PER_DOWN_TASK - 1) / ROWS_PER_DOWN_TASK, threads);
    free(j.act);
    free(j.hq);
    free(j.h);
    free(j.by);
    free(j.run);
    return 0;
}
