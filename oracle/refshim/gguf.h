// Minimal stand-in for gguf.h: TEST INFRASTRUCTURE ONLY (oracle/_ref).
//
// Implements the handful of gguf/ggml calls the reference runtime's model
// section makes (board/tp/tp_llama.cpp:149-188: gguf_init_from_file,
// ggml_get_tensor, gguf_find_tensor, gguf_get_data_offset,
// gguf_get_tensor_offset, gguf_find_key, gguf_get_val_u32, gguf_get_val_f32)
// over the published GGUF v2/v3 layout: the "GGUF" magic, version, tensor and
// key counts, the key/value pairs, the tensor infos (name, dims, type,
// offset), then the data section at the next multiple of general.alignment
// (32 when absent). Only what the runtime reads is kept.
#pragma once

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <string>
#include <vector>

#include "ggml.h"

struct gguf_init_params {
    bool no_alloc;
    struct ggml_context **ctx;
};

struct ggml_tensor {
    std::string name;
    uint32_t type;
    std::vector<uint64_t> ne;
    uint64_t offset;
};

struct ggml_context {
    std::vector<ggml_tensor> tensors;
};

struct gguf_kv {
    std::string key;
    uint32_t type;
    uint64_t u;   // integer / bool values
    double f;     // float values
};

struct gguf_context {
    uint32_t version = 0;
    std::vector<gguf_kv> kv;
    ggml_context *meta = nullptr;
    size_t data_offset = 0;
};

namespace gguf_shim {

enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 };

struct reader {
    FILE *f;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (fread(&v, sizeof v, 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) { ok = false; return {}; }
        std::string s(n, '\0');
        if (n && fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
    size_t scalar_size(uint32_t t) {
        switch (t) {
            case T_U8: case T_I8: case T_BOOL: return 1;
            case T_U16: case T_I16: return 2;
            case T_U32: case T_I32: case T_F32: return 4;
            case T_U64: case T_I64: case T_F64: return 8;
            default: return 0;
        }
    }
    void value(uint32_t t, gguf_kv *out) {
        switch (t) {
            case T_U8: out->u = get<uint8_t>(); break;
            case T_I8: out->u = (uint64_t)(int64_t)get<int8_t>(); break;
            case T_U16: out->u = get<uint16_t>(); break;
            case T_I16: out->u = (uint64_t)(int64_t)get<int16_t>(); break;
            case T_U32: out->u = get<uint32_t>(); break;
            case T_I32: out->u = (uint64_t)(int64_t)get<int32_t>(); break;
            case T_BOOL: out->u = get<uint8_t>(); break;
            case T_U64: out->u = get<uint64_t>(); break;
            case T_I64: out->u = (uint64_t)get<int64_t>(); break;
            case T_F32: out->f = get<float>(); break;
            case T_F64: out->f = get<double>(); break;
            case T_STRING: str(); break;
            case T_ARRAY: {
                const uint32_t et = get<uint32_t>();
                const uint64_t n = get<uint64_t>();
                if (!ok) return;
                if (et == T_STRING) {
                    for (uint64_t i = 0; i < n && ok; ++i) str();
                } else if (et == T_ARRAY || !scalar_size(et)) {
                    ok = false;
                } else if (fseek(f, (long)(n * scalar_size(et)), SEEK_CUR)) {
                    ok = false;
                }
                break;
            }
            default: ok = false;
        }
    }
};

}  // namespace gguf_shim

static inline gguf_context *gguf_init_from_file(const char *path, gguf_init_params params) {
    FILE *f = fopen(path, "rb");
    if (!f) return nullptr;
    gguf_shim::reader r{f};
    gguf_context *g = new gguf_context();
    g->meta = new ggml_context();
    char magic[4] = {0, 0, 0, 0};
    if (fread(magic, 1, 4, f) != 4 || magic[0] != 'G' || magic[1] != 'G' || magic[2] != 'U' || magic[3] != 'F')
        r.ok = false;
    g->version = r.get<uint32_t>();
    if (g->version < 2) r.ok = false;
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        gguf_kv kv{};
        kv.key = r.str();
        kv.type = r.get<uint32_t>();
        r.value(kv.type, &kv);
        if (kv.key == "general.alignment" && kv.type == gguf_shim::T_U32) alignment = kv.u;
        g->kv.push_back(kv);
    }
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        ggml_tensor t;
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd > 4) r.ok = false;
        for (uint32_t d = 0; d < nd && r.ok; ++d) t.ne.push_back(r.get<uint64_t>());
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        g->meta->tensors.push_back(t);
    }
    const long end = ftell(f);
    fclose(f);
    if (!r.ok || end < 0 || !alignment || (alignment & (alignment - 1))) {
        delete g->meta;
        delete g;
        return nullptr;
    }
    g->data_offset = ((size_t)end + alignment - 1) / alignment * alignment;
    if (params.ctx) *params.ctx = g->meta;
    return g;
}

static inline const ggml_tensor *ggml_get_tensor(const ggml_context *ctx, const char *name) {
    for (const ggml_tensor &t : ctx->tensors)
        if (t.name == name) return &t;
    return nullptr;
}

static inline int64_t gguf_find_tensor(const gguf_context *g, const char *name) {
    for (size_t i = 0; i < g->meta->tensors.size(); ++i)
        if (g->meta->tensors[i].name == name) return (int64_t)i;
    return -1;
}

static inline size_t gguf_get_data_offset(const gguf_context *g) { return g->data_offset; }

static inline size_t gguf_get_tensor_offset(const gguf_context *g, int64_t i) {
    return (size_t)g->meta->tensors[(size_t)i].offset;
}

static inline int64_t gguf_find_key(const gguf_context *g, const char *key) {
    for (size_t i = 0; i < g->kv.size(); ++i)
        if (g->kv[i].key == key) return (int64_t)i;
    return -1;
}

static inline uint32_t gguf_get_val_u32(const gguf_context *g, int64_t i) { return (uint32_t)g->kv[(size_t)i].u; }

static inline float gguf_get_val_f32(const gguf_context *g, int64_t i) { return (float)g->kv[(size_t)i].f; }

static inline void gguf_shim_free(gguf_context *g) {
    if (!g) return;
    delete g->meta;
    delete g;
}
