// tsb_gguf.cpp - GGUF model files for the expert path: a reader (mmap, header, metadata, tensor directory) and the
// repack of one layer's expert tensors into the native expert blobs the kernels take.
//
// Reference: the engines read GGUF v3 through include/strata/artifact/gguf_reader.hpp (mmap, metadata of every value
// type, tensor directory, data at the aligned offset after the directory) and build each layer's expert blobs in
// src/qwen35/q36_engine.cu:1144-1167 and 1196-1200: expert e's gate rows, up rows and down rows copied from the
// ffn_{gate,up,down}_exps tensors ([n_expert][rows][row bytes], contiguous per expert) into
// [gate | up | down] at e * stride, the stride the blob size rounded up to a whole number of blocks of both types and
// of 16 bytes.  Host code only: no CUDA.  The format is the published GGUF one (the file as ggml writes it); the
// multi-shard (split.*) files of the reference's loader are one reader per shard here.
#include "../../include/tsb_moe.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace tsb {
void set_last_error(const char* msg);   // tsb_moe.cu
}

namespace {

int gfail(int code, const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    tsb::set_last_error(b);
    return code;
}

// GGUF metadata value types
enum : uint32_t {
    GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case GV_U8: case GV_I8: case GV_BOOL: return 1;
        case GV_U16: case GV_I16: return 2;
        case GV_U32: case GV_I32: case GV_F32: return 4;
        case GV_U64: case GV_I64: case GV_F64: return 8;
        default: return 0;
    }
}

// (values per block, bytes per block) of the ggml types a GGUF expert file holds
bool block_geometry(uint32_t t, uint64_t& qk, uint64_t& bytes) {
    switch (t) {
        case 0: qk = 1; bytes = 4; return true;      // F32
        case 1: case 30: qk = 1; bytes = 2; return true;   // F16, BF16
        case 2: qk = 32; bytes = 18; return true;    // Q4_0
        case 3: qk = 32; bytes = 20; return true;    // Q4_1
        case 6: qk = 32; bytes = 22; return true;    // Q5_0
        case 7: qk = 32; bytes = 24; return true;    // Q5_1
        case 8: qk = 32; bytes = 34; return true;    // Q8_0
        case 10: qk = 256; bytes = 84; return true;  // Q2_K
        case 11: qk = 256; bytes = 110; return true; // Q3_K
        case 12: qk = 256; bytes = 144; return true; // Q4_K
        case 13: qk = 256; bytes = 176; return true; // Q5_K
        case 14: qk = 256; bytes = 210; return true; // Q6_K
        case 16: qk = 256; bytes = 66; return true;  // IQ2_XXS
        case 17: qk = 256; bytes = 74; return true;  // IQ2_XS
        case 18: qk = 256; bytes = 98; return true;  // IQ3_XXS
        case 19: qk = 256; bytes = 50; return true;  // IQ1_S
        case 20: qk = 32; bytes = 18; return true;   // IQ4_NL
        case 21: qk = 256; bytes = 110; return true; // IQ3_S
        case 22: qk = 256; bytes = 82; return true;  // IQ2_S
        case 23: qk = 256; bytes = 136; return true; // IQ4_XS
        case 24: qk = 1; bytes = 1; return true;     // I8
        case 25: qk = 1; bytes = 2; return true;     // I16
        case 26: qk = 1; bytes = 4; return true;     // I32
        case 27: qk = 1; bytes = 8; return true;     // I64
        case 28: qk = 1; bytes = 8; return true;     // F64
        default: return false;
    }
}

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <typename T> T get() {
        T v{};
        if (end - p < (ptrdiff_t) sizeof(T)) {
            ok = false;
            p = end;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t) (end - p) < n) {
            ok = false;
            p = end;
            return {};
        }
        std::string s((const char*) p, (size_t) n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if ((uint64_t) (end - p) < n) {
            ok = false;
            p = end;
        } else {
            p += n;
        }
    }
};

struct Tensor {
    uint32_t type = 0, n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0, bytes = 0;
};

struct Kv {
    uint32_t type = 0;
    int64_t i = 0;       // integer and bool values
    double f = 0.0;      // float values
    std::string s;       // string values
    uint32_t arr_type = 0;
    uint64_t arr_n = 0;
};

}  // namespace

struct tsb_gguf {
    int fd = -1;
    uint8_t* map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_off = 0;
    std::map<std::string, Kv> kv;
    std::map<std::string, Tensor> tensors;
    std::vector<std::string> names;
};

namespace {

int parse(tsb_gguf* g) {
    Cursor c{g->map, g->map + g->size};
    if (g->size < 24 || memcmp(g->map, "GGUF", 4) != 0) return gfail(TSB_ERR_ARG, "gguf: not a GGUF file");
    c.skip(4);
    g->version = c.get<uint32_t>();
    if (g->version < 2 || g->version > 3) return gfail(TSB_ERR_UNSUPPORTED, "gguf: version %u", g->version);
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) return gfail(TSB_ERR_ARG, "gguf: implausible counts");
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        const std::string key = c.str();
        Kv v;
        v.type = c.get<uint32_t>();
        switch (v.type) {
            case GV_U8: v.i = c.get<uint8_t>(); break;
            case GV_I8: v.i = c.get<int8_t>(); break;
            case GV_U16: v.i = c.get<uint16_t>(); break;
            case GV_I16: v.i = c.get<int16_t>(); break;
            case GV_U32: v.i = c.get<uint32_t>(); break;
            case GV_I32: v.i = c.get<int32_t>(); break;
            case GV_F32: v.f = c.get<float>(); break;
            case GV_BOOL: v.i = c.get<uint8_t>(); break;
            case GV_STR: v.s = c.str(); break;
            case GV_U64: v.i = (int64_t) c.get<uint64_t>(); break;
            case GV_I64: v.i = c.get<int64_t>(); break;
            case GV_F64: v.f = c.get<double>(); break;
            case GV_ARR: {
                v.arr_type = c.get<uint32_t>();
                v.arr_n = c.get<uint64_t>();
                if (v.arr_type == GV_STR) {
                    for (uint64_t k = 0; k < v.arr_n && c.ok; ++k) c.str();
                } else {
                    const size_t es = scalar_size(v.arr_type);
                    if (es == 0) return gfail(TSB_ERR_ARG, "gguf: array of type %u under %s", v.arr_type, key.c_str());
                    c.skip(v.arr_n * es);
                }
                break;
            }
            default: return gfail(TSB_ERR_ARG, "gguf: value type %u under %s", v.type, key.c_str());
        }
        g->kv[key] = v;
    }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        const std::string name = c.str();
        Tensor t;
        t.n_dims = c.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) return gfail(TSB_ERR_ARG, "gguf: %s has %u dimensions", name.c_str(), t.n_dims);
        for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = c.get<uint64_t>();
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        uint64_t qk = 0, bb = 0;
        if (!block_geometry(t.type, qk, bb) || t.ne[0] % qk)
            return gfail(TSB_ERR_UNSUPPORTED, "gguf: %s: type %u, row of %llu values", name.c_str(), t.type,
                         (unsigned long long) t.ne[0]);
        t.bytes = t.ne[0] / qk * bb * t.ne[1] * t.ne[2] * t.ne[3];
        g->tensors[name] = t;
        g->names.push_back(name);
    }
    if (!c.ok) return gfail(TSB_ERR_ARG, "gguf: truncated header");
    auto al = g->kv.find("general.alignment");
    if (al != g->kv.end() && al->second.i > 0) g->alignment = (uint64_t) al->second.i;
    const uint64_t here = (uint64_t) (c.p - g->map);
    g->data_off = (here + g->alignment - 1) / g->alignment * g->alignment;
    for (auto& [name, t] : g->tensors)
        if (g->data_off + t.offset + t.bytes > g->size)
            return gfail(TSB_ERR_ARG, "gguf: %s lies past the end of the file", name.c_str());
    return TSB_OK;
}

uint64_t gcd64(uint64_t a, uint64_t b) {
    while (b) {
        const uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

}  // namespace

extern "C" {

int tsb_gguf_open(const char* path, tsb_gguf** out) {
    if (!path || !out) return gfail(TSB_ERR_ARG, "gguf_open: null argument");
    *out = nullptr;
    tsb_gguf* g = new tsb_gguf();
    g->fd = open(path, O_RDONLY);
    struct stat st{};
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        delete g;
        return gfail(TSB_ERR_ARG, "gguf_open: %s: cannot open", path);
    }
    g->size = (size_t) st.st_size;
    void* m = g->size ? mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0) : MAP_FAILED;
    if (m == MAP_FAILED) {
        close(g->fd);
        delete g;
        return gfail(TSB_ERR_ARG, "gguf_open: %s: cannot map", path);
    }
    g->map = (uint8_t*) m;
    const int rc = parse(g);
    if (rc != TSB_OK) {
        tsb_gguf_close(g);
        return rc;
    }
    *out = g;
    return TSB_OK;
}

int tsb_gguf_close(tsb_gguf* g) {
    if (!g) return TSB_OK;
    if (g->map) munmap(g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return TSB_OK;
}

int tsb_gguf_tensor_count(const tsb_gguf* g) { return g ? (int) g->names.size() : -1; }

int tsb_gguf_tensor_name(const tsb_gguf* g, int i, char* buf, int buf_bytes) {
    if (!g || i < 0 || i >= (int) g->names.size() || !buf || buf_bytes < 1)
        return gfail(TSB_ERR_ARG, "gguf_tensor_name: arguments");
    snprintf(buf, (size_t) buf_bytes, "%s", g->names[(size_t) i].c_str());
    return TSB_OK;
}

int tsb_gguf_tensor(const tsb_gguf* g, const char* name, tsb_gguf_tensor_info* out) {
    if (!g || !name || !out) return gfail(TSB_ERR_ARG, "gguf_tensor: null argument");
    auto it = g->tensors.find(name);
    if (it == g->tensors.end()) return gfail(TSB_ERR_ARG, "gguf_tensor: no tensor %s", name);
    const Tensor& t = it->second;
    out->type = (int32_t) t.type;
    out->n_dims = (int32_t) t.n_dims;
    for (int d = 0; d < 4; ++d) out->ne[d] = (int64_t) t.ne[d];
    out->bytes = t.bytes;
    out->data = g->map + g->data_off + t.offset;
    return TSB_OK;
}

int tsb_gguf_kv_int(const tsb_gguf* g, const char* key, int64_t* value) {
    if (!g || !key || !value) return gfail(TSB_ERR_ARG, "gguf_kv_int: null argument");
    auto it = g->kv.find(key);
    if (it == g->kv.end()) return gfail(TSB_ERR_ARG, "gguf_kv_int: no key %s", key);
    const Kv& v = it->second;
    if (v.type == GV_F32 || v.type == GV_F64 || v.type == GV_STR || v.type == GV_ARR)
        return gfail(TSB_ERR_ARG, "gguf_kv_int: %s is not an integer", key);
    *value = v.i;
    return TSB_OK;
}

int tsb_gguf_kv_float(const tsb_gguf* g, const char* key, double* value) {
    if (!g || !key || !value) return gfail(TSB_ERR_ARG, "gguf_kv_float: null argument");
    auto it = g->kv.find(key);
    if (it == g->kv.end()) return gfail(TSB_ERR_ARG, "gguf_kv_float: no key %s", key);
    const Kv& v = it->second;
    if (v.type == GV_F32 || v.type == GV_F64) *value = v.f;
    else if (v.type == GV_STR || v.type == GV_ARR) return gfail(TSB_ERR_ARG, "gguf_kv_float: %s is not a number", key);
    else *value = (double) v.i;
    return TSB_OK;
}

int tsb_gguf_kv_str(const tsb_gguf* g, const char* key, char* buf, int buf_bytes) {
    if (!g || !key || !buf || buf_bytes < 1) return gfail(TSB_ERR_ARG, "gguf_kv_str: arguments");
    auto it = g->kv.find(key);
    if (it == g->kv.end() || it->second.type != GV_STR) return gfail(TSB_ERR_ARG, "gguf_kv_str: no string %s", key);
    snprintf(buf, (size_t) buf_bytes, "%s", it->second.s.c_str());
    return TSB_OK;
}

int tsb_gguf_expert_layer(const tsb_gguf* g, const char* prefix, tsb_expert_layout* L, uint64_t* stride,
                          int32_t* n_expert) {
    if (!g || !prefix || !L || !stride || !n_expert) return gfail(TSB_ERR_ARG, "gguf_expert_layer: null argument");
    const std::string p(prefix);
    tsb_gguf_tensor_info tg{}, tu{}, td{};
    int rc = tsb_gguf_tensor(g, (p + "ffn_gate_exps.weight").c_str(), &tg);
    if (rc == TSB_OK) rc = tsb_gguf_tensor(g, (p + "ffn_up_exps.weight").c_str(), &tu);
    if (rc == TSB_OK) rc = tsb_gguf_tensor(g, (p + "ffn_down_exps.weight").c_str(), &td);
    if (rc != TSB_OK) return rc;
    // ne: gate / up [n_embd, n_ff, n_expert], down [n_ff, n_embd, n_expert]
    if (tg.type != tu.type) return gfail(TSB_ERR_UNSUPPORTED, "gguf_expert_layer: %sffn_gate_exps / ffn_up_exps differ in type", prefix);
    if (tg.n_dims != 3 || tu.n_dims != 3 || td.n_dims != 3 || tg.ne[0] != tu.ne[0] || tg.ne[1] != tu.ne[1] ||
        tg.ne[2] != tu.ne[2] || td.ne[0] != tg.ne[1] || td.ne[1] != tg.ne[0] || td.ne[2] != tg.ne[2])
        return gfail(TSB_ERR_ARG, "gguf_expert_layer: %s: expert tensor shapes do not agree", prefix);
    rc = tsb_native_expert_layout(tg.type, td.type, tg.ne[0], tg.ne[1], L);
    if (rc != TSB_OK) return rc;
    uint64_t qk = 0, bg = 0, bd = 0;
    block_geometry((uint32_t) tg.type, qk, bg);
    block_geometry((uint32_t) td.type, qk, bd);
    uint64_t al = bg / gcd64(bg, bd) * bd;
    al = al / gcd64(al, 16) * 16;
    *stride = (L->bytes + al - 1) / al * al;
    *n_expert = (int32_t) tg.ne[2];
    return TSB_OK;
}

int tsb_gguf_repack_experts(const tsb_gguf* g, const char* prefix, int first, int count, void* dst,
                            uint64_t dst_bytes) {
    tsb_expert_layout L{};
    uint64_t stride = 0;
    int32_t n_expert = 0;
    int rc = tsb_gguf_expert_layer(g, prefix, &L, &stride, &n_expert);
    if (rc != TSB_OK) return rc;
    if (!dst || first < 0 || count < 0 || first + count > n_expert)
        return gfail(TSB_ERR_ARG, "gguf_repack_experts: experts [%d, %d) of %d", first, first + count, n_expert);
    if (dst_bytes < (uint64_t) count * stride)
        return gfail(TSB_ERR_WORKSPACE, "gguf_repack_experts: %llu bytes < %llu", (unsigned long long) dst_bytes,
                     (unsigned long long) ((uint64_t) count * stride));
    const std::string p(prefix);
    tsb_gguf_tensor_info tg{}, tu{}, td{};
    tsb_gguf_tensor(g, (p + "ffn_gate_exps.weight").c_str(), &tg);
    tsb_gguf_tensor(g, (p + "ffn_up_exps.weight").c_str(), &tu);
    tsb_gguf_tensor(g, (p + "ffn_down_exps.weight").c_str(), &td);
    const uint64_t gsz = (uint64_t) L.n_ff * L.gu_row, dsz = (uint64_t) L.n_embd * L.d_row;
    uint8_t* o = (uint8_t*) dst;
    for (int q = 0; q < count; ++q) {
        const uint64_t e = (uint64_t) (first + q);
        uint8_t* blob = o + (uint64_t) q * stride;
        memcpy(blob, (const uint8_t*) tg.data + e * gsz, gsz);
        memcpy(blob + L.up_off, (const uint8_t*) tu.data + e * gsz, gsz);
        memcpy(blob + L.down_off, (const uint8_t*) td.data + e * dsz, dsz);
        if (stride > L.bytes) memset(blob + L.bytes, 0, stride - L.bytes);
    }
    return TSB_OK;
}

}  // extern "C"
