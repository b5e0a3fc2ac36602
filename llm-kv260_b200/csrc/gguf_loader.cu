// GGUF model loading (include/b200_gguf.h): the reference runtime's
// gguf_file and load_model (board/tp/tp_llama.cpp:149-188, 226-283) as host
// code of this library. The file is mapped read-only and parsed with every
// read bounds-checked against the mapping; the tensors go to the decoder's
// own set_layer / set_output / set_rope_freqs, which cut the rank's shard as
// load_model does (copy_rows / copy_cols, tp_llama.cpp:191-207).
//
// GGUF v2/v3 layout: "GGUF", u32 version, u64 tensor count, u64 key count;
// key/value pairs (u64-length string key, u32 type, value; arrays are u32
// element type, u64 count, elements); tensor infos (name, u32 dims, u64 ne[],
// u32 ggml type, u64 offset into the data section); the data section at the
// next multiple of general.alignment (32 when absent).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/b200_gguf.h"
#include "decode.h"

using namespace b200;

namespace {

constexpr int kErrNoEnt = -2;  // -ENOENT

enum : uint32_t { kU8, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64 };

struct Kv {
    std::string key;
    uint32_t type = 0;
    uint64_t u = 0;  // integer and bool values
    double f = 0;    // float values
};

struct TensorInfo {
    std::string name;
    uint32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;  // from the data section
    uint64_t bytes = 0;   // 0: a type whose size this loader does not know
};

int gfail(int code, const char *fmt, ...) {
    char msg[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    return report_error(code, msg);
}

// Bytes of n elements of a ggml type (0 when unknown).
uint64_t type_bytes(uint32_t type, uint64_t n) {
    switch (type) {
        case B200_GGML_F32: return 4 * n;
        case B200_GGML_F16: return 2 * n;
        case B200_GGML_Q4_0: return n % 32 ? 0 : n / 32 * 18;
        case B200_GGML_Q8_0: return n % 32 ? 0 : n / 32 * 34;
        default: return 0;
    }
}

// A bounds-checked cursor over the mapped header.
struct Cursor {
    const uint8_t *p, *end;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (static_cast<size_t>(end - p) < sizeof v) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof v);
        p += sizeof v;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > static_cast<uint64_t>(end - p)) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(p), n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if (n > static_cast<uint64_t>(end - p)) ok = false;
        else p += n;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

void read_value(Cursor &c, uint32_t t, Kv *kv) {
    switch (t) {
        case kU8: kv->u = c.get<uint8_t>(); break;
        case kI8: kv->u = static_cast<uint64_t>(static_cast<int64_t>(c.get<int8_t>())); break;
        case kU16: kv->u = c.get<uint16_t>(); break;
        case kI16: kv->u = static_cast<uint64_t>(static_cast<int64_t>(c.get<int16_t>())); break;
        case kU32: kv->u = c.get<uint32_t>(); break;
        case kI32: kv->u = static_cast<uint64_t>(static_cast<int64_t>(c.get<int32_t>())); break;
        case kBool: kv->u = c.get<uint8_t>(); break;
        case kU64: kv->u = c.get<uint64_t>(); break;
        case kI64: kv->u = static_cast<uint64_t>(c.get<int64_t>()); break;
        case kF32: kv->f = c.get<float>(); break;
        case kF64: kv->f = c.get<double>(); break;
        case kString: c.skip(c.get<uint64_t>()); break;
        case kArray: {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (!c.ok) return;
            if (et == kString) {
                for (uint64_t i = 0; i < n && c.ok; ++i) c.skip(c.get<uint64_t>());
            } else if (scalar_size(et) && n <= UINT64_MAX / 8) {
                c.skip(n * scalar_size(et));
            } else {
                c.ok = false;  // nested arrays do not occur in llama GGUFs
            }
            break;
        }
        default: c.ok = false;
    }
}

}  // namespace

struct b200_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t data_offset = 0;
    std::vector<Kv> kv;
    std::vector<TensorInfo> tensors;

    const Kv *find_key(const char *key) const {
        for (const Kv &k : kv)
            if (k.key == key) return &k;
        return nullptr;
    }
    const TensorInfo *find_tensor(const char *name) const {
        for (const TensorInfo &t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
};

extern "C" void b200_gguf_close(b200_gguf_t *g) {
    if (!g) return;
    if (g->map) munmap(const_cast<uint8_t *>(g->map), g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
}

extern "C" int b200_gguf_open(b200_gguf_t **out, const char *path) {
    if (!out || !path) return gfail(kErrInval, "gguf: null argument");
    *out = nullptr;
    b200_gguf_t *g = new (std::nothrow) b200_gguf_t();
    if (!g) return gfail(kErrNoMem, "gguf: out of host memory");
    g->fd = open(path, O_RDONLY);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0) {
        b200_gguf_close(g);
        return gfail(kErrNoEnt, "gguf: cannot open %s", path);
    }
    g->size = static_cast<size_t>(st.st_size);
    void *m = g->size ? mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0) : MAP_FAILED;
    if (m == MAP_FAILED) {
        b200_gguf_close(g);
        return gfail(kErrInval, "gguf: cannot map %s", path);
    }
    g->map = static_cast<const uint8_t *>(m);
    Cursor c{g->map, g->map + g->size};
    const uint32_t magic = c.get<uint32_t>();
    g->version = c.get<uint32_t>();
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (!c.ok || memcmp(&magic, "GGUF", 4) != 0 || g->version < 2 || g->version > 3) {
        b200_gguf_close(g);
        return gfail(kErrInval, "gguf: %s is not a GGUF v2/v3 file", path);
    }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        Kv kv;
        kv.key = c.str();
        kv.type = c.get<uint32_t>();
        read_value(c, kv.type, &kv);
        if (kv.key == "general.alignment" && kv.type == kU32) alignment = kv.u;
        g->kv.push_back(std::move(kv));
    }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        TensorInfo t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd > 4) c.ok = false;
        uint64_t n = 1;
        for (uint32_t d = 0; d < nd && c.ok; ++d) {
            t.ne[d] = static_cast<int64_t>(c.get<uint64_t>());
            if (t.ne[d] < 0 || (t.ne[d] && n > UINT64_MAX / static_cast<uint64_t>(t.ne[d]))) c.ok = false;
            else n *= static_cast<uint64_t>(t.ne[d]);
        }
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        t.bytes = type_bytes(t.type, n);
        g->tensors.push_back(std::move(t));
    }
    if (!c.ok || !alignment || (alignment & (alignment - 1))) {
        b200_gguf_close(g);
        return gfail(kErrInval, "gguf: %s has a malformed header", path);
    }
    const uint64_t end = static_cast<uint64_t>(c.p - g->map);
    g->data_offset = (end + alignment - 1) / alignment * alignment;
    for (const TensorInfo &t : g->tensors)
        if (t.offset > g->size || g->data_offset > g->size - t.offset || t.bytes > g->size - g->data_offset - t.offset) {
            const std::string name = t.name;
            b200_gguf_close(g);
            return gfail(kErrInval, "gguf: tensor %s lies outside %s", name.c_str(), path);
        }
    *out = g;
    return 0;
}

extern "C" int b200_gguf_tensor(const b200_gguf_t *g, const char *name, const void **data, uint64_t *bytes, int *type,
                                int64_t ne[4]) {
    if (!g || !name) return gfail(kErrInval, "gguf: null argument");
    const TensorInfo *t = g->find_tensor(name);
    if (!t) return gfail(kErrNoEnt, "gguf: tensor %s missing", name);
    if (data) *data = g->map + g->data_offset + t->offset;
    if (bytes) *bytes = t->bytes;
    if (type) *type = static_cast<int>(t->type);
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = t->ne[d];
    return 0;
}

extern "C" int b200_gguf_config(const b200_gguf_t *g, b200_decoder_config_t *cfg) {
    if (!g || !cfg) return gfail(kErrInval, "gguf: null argument");
    auto u32 = [&](const char *key, int *out) -> int {
        const Kv *k = g->find_key(key);
        if (!k || (k->type != kU32 && k->type != kI32 && k->type != kU64 && k->type != kI64) || k->u == 0 ||
            k->u > 0x7fffffffu)
            return gfail(kErrInval, "gguf: key %s missing or not a positive integer", key);
        *out = static_cast<int>(k->u);
        return 0;
    };
    auto f32 = [&](const char *key, float dflt) -> float {
        const Kv *k = g->find_key(key);
        return k && (k->type == kF32 || k->type == kF64) ? static_cast<float>(k->f) : dflt;
    };
    b200_decoder_config_t c = *cfg;
    if (int rc = u32("llama.block_count", &c.n_layer)) return rc;
    if (int rc = u32("llama.embedding_length", &c.n_embd)) return rc;
    if (int rc = u32("llama.feed_forward_length", &c.n_ff)) return rc;
    if (int rc = u32("llama.attention.head_count", &c.n_head)) return rc;
    if (int rc = u32("llama.attention.head_count_kv", &c.n_head_kv)) return rc;
    if (g->find_key("llama.vocab_size")) {
        if (int rc = u32("llama.vocab_size", &c.n_vocab)) return rc;
    } else {
        const TensorInfo *te = g->find_tensor("token_embd.weight");
        if (!te || te->ne[1] <= 0 || te->ne[1] > 0x7fffffff)
            return gfail(kErrInval, "gguf: neither llama.vocab_size nor token_embd.weight gives the vocabulary");
        c.n_vocab = static_cast<int>(te->ne[1]);
    }
    if (c.n_embd % c.n_head) return gfail(kErrInval, "gguf: embedding_length %d not a multiple of head_count", c.n_embd);
    c.head_dim = c.n_embd / c.n_head;
    c.rope_base = f32("llama.rope.freq_base", 10000.0f);
    c.rms_eps = f32("llama.attention.layer_norm_rms_epsilon", 1e-5f);
    *cfg = c;
    return 0;
}

namespace {

// The tensor `name`, checked for type and shape [ne0, ne1].
int want_tensor(const b200_gguf_t *g, const char *name, uint32_t type, int64_t ne0, int64_t ne1, const void **data) {
    const TensorInfo *t = g->find_tensor(name);
    if (!t) return gfail(kErrNoEnt, "gguf: tensor %s missing", name);
    if (t->type != type)
        return gfail(kErrInval, "gguf: tensor %s has ggml type %u, the decoder needs %u", name, t->type, type);
    if (t->ne[0] != ne0 || t->ne[1] != ne1 || t->ne[2] != 1 || t->ne[3] != 1)
        return gfail(kErrInval, "gguf: tensor %s is [%lld, %lld], expected [%lld, %lld]", name,
                     static_cast<long long>(t->ne[0]), static_cast<long long>(t->ne[1]), static_cast<long long>(ne0),
                     static_cast<long long>(ne1));
    *data = g->map + g->data_offset + t->offset;
    return 0;
}

}  // namespace

extern "C" int b200_decoder_load_gguf(b200_decoder_t *d, const b200_gguf_t *g) {
    if (!d || !g) return gfail(kErrInval, "gguf: null argument");
    b200_decoder_config_t c{}, f{};
    if (int rc = decoder_config(d, &c)) return rc;
    if (int rc = b200_gguf_config(g, &f)) return rc;
    if (f.n_layer != c.n_layer || f.n_embd != c.n_embd || f.n_ff != c.n_ff || f.n_head != c.n_head ||
        f.n_head_kv != c.n_head_kv || f.n_vocab != c.n_vocab)
        return gfail(kErrInval, "gguf: the file's hyperparameters differ from the decoder's");
    const int e = c.n_embd, kv = c.n_head_kv * c.head_dim;
    // check everything before the first upload
    std::vector<const void *> p(static_cast<size_t>(c.n_layer) * 9);
    char name[96];
    struct Spec {
        const char *what;
        uint32_t type;
        int64_t ne0, ne1;
    };
    const Spec specs[9] = {{"attn_q", B200_GGML_Q4_0, e, e},        {"attn_k", B200_GGML_Q4_0, e, kv},
                           {"attn_v", B200_GGML_Q4_0, e, kv},       {"attn_output", B200_GGML_Q4_0, e, e},
                           {"ffn_gate", B200_GGML_Q4_0, e, c.n_ff}, {"ffn_up", B200_GGML_Q4_0, e, c.n_ff},
                           {"ffn_down", B200_GGML_Q4_0, c.n_ff, e}, {"attn_norm", B200_GGML_F32, e, 1},
                           {"ffn_norm", B200_GGML_F32, e, 1}};
    for (int l = 0; l < c.n_layer; ++l)
        for (int i = 0; i < 9; ++i) {
            snprintf(name, sizeof name, "blk.%d.%s.weight", l, specs[i].what);
            if (int rc = want_tensor(g, name, specs[i].type, specs[i].ne0, specs[i].ne1, &p[9 * l + i])) return rc;
        }
    const void *te = nullptr, *on = nullptr, *rf = nullptr;
    if (int rc = want_tensor(g, "token_embd.weight", B200_GGML_Q4_0, e, c.n_vocab, &te)) return rc;
    if (int rc = want_tensor(g, "output_norm.weight", B200_GGML_F32, e, 1, &on)) return rc;
    if (g->find_tensor("rope_freqs.weight"))
        if (int rc = want_tensor(g, "rope_freqs.weight", B200_GGML_F32, c.head_dim / 2, 1, &rf)) return rc;
    for (int l = 0; l < c.n_layer; ++l) {
        const void *const *q = &p[9 * l];
        if (int rc = b200_decoder_set_layer(d, l, q[0], q[1], q[2], q[3], q[4], q[5], q[6],
                                            static_cast<const float *>(q[7]), static_cast<const float *>(q[8])))
            return rc;
    }
    if (int rc = b200_decoder_set_output(d, te, static_cast<const float *>(on))) return rc;
    if (rf)
        if (int rc = b200_decoder_set_rope_freqs(d, static_cast<const float *>(rf))) return rc;
    return 0;
}
