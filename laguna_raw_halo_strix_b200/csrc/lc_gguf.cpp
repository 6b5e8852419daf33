// lc_gguf.cpp -- GGUF v3 reader, the C++ counterpart of the reference's
// GGUFReader (src/gguf.rs:321-421) and of Model::from_reader's
// hyper-parameter lookup (src/model.rs:29-129, src/gguf.rs:516-653).
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "laguna_cuda.h"

int lc_fail(int code, const char *fmt, ...);

namespace {

struct Value {
    enum Kind { NUM_U, NUM_I, NUM_F, BOOL, STR, ARR } kind = NUM_U;
    uint32_t type = 0;  // GGUF value type id (0..12)
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<Value> arr;
    // GGUF ids of the 32- and 64-bit numbers, the only ones the accessors take
    static bool wide_int(uint32_t t) { return t == 4 || t == 5 || t == 10 || t == 11; }
    static bool wide_float(uint32_t t) { return t == 6 || t == 12; }
    bool as_u64(uint64_t *out) const {
        // GGUFValue::as_u64 (src/gguf.rs:228-237): U32/U64/I32/I64 only
        if (!wide_int(type)) return false;
        *out = kind == NUM_U ? u : (uint64_t)i;
        return true;
    }
    bool as_f32(float *out) const {
        // GGUFValue::as_f32 (src/gguf.rs:239-249): F32/F64 and the wide integers
        if (wide_float(type)) return *out = (float)f, true;
        if (!wide_int(type)) return false;
        *out = kind == NUM_U ? (float)u : (float)i;
        return true;
    }
    bool as_bool(bool *out) const {
        // GGUFValue::as_bool (src/gguf.rs:251-262): Bool, wide integers, floats
        if (type == 7) return *out = u != 0, true;
        if (wide_int(type)) return *out = (kind == NUM_U ? u : (uint64_t)i) != 0, true;
        if (wide_float(type)) return *out = f != 0.0, true;
        return false;
    }
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> shape;
    int dtype = 0;
    uint64_t offset = 0;
};

}  // namespace

// The whole file is mapped read-only; tensor data is read (or handed out) from
// the mapping, so a tensor costs no read() copy and the page cache feeds the
// upload directly.
struct lc_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t size = 0;
    uint32_t version = 0;
    std::vector<std::pair<std::string, Value>> meta;
    std::map<std::string, size_t> meta_index;
    std::vector<Tensor> tensors;
    uint64_t data_offset = 0;
};

namespace {

// Bounds-checked cursor over the mapping: every header read fails instead of
// running past the end of a truncated file.
struct Src {
    const uint8_t *p;
    uint64_t n, pos;
};

bool rd(Src &f, void *p, size_t n) {
    if (n > f.n - f.pos) return false;
    memcpy(p, f.p + f.pos, n);
    f.pos += n;
    return true;
}

template <typename T>
bool rdv(Src &f, T *v) {
    return rd(f, v, sizeof(T));
}

bool read_string(Src &f, std::string *s) {
    uint64_t n;
    if (!rdv(f, &n) || n > (1ull << 32)) return false;
    s->resize(n);
    return n == 0 || rd(f, &(*s)[0], n);
}

// read_value (src/gguf.rs:441-514): GGUF value type ids 0..12.
bool read_value(Src &f, uint32_t type, Value *v, int depth = 0) {
    if (depth > 4) return false;
    v->type = type;
    switch (type) {
    case 0: { uint8_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_U; v->u = x; return true; }
    case 1: { int8_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_I; v->i = x; return true; }
    case 2: { uint16_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_U; v->u = x; return true; }
    case 3: { int16_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_I; v->i = x; return true; }
    case 4: { uint32_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_U; v->u = x; return true; }
    case 5: { int32_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_I; v->i = x; return true; }
    case 6: { float x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_F; v->f = x; return true; }
    case 7: { uint8_t x; if (!rdv(f, &x)) return false; v->kind = Value::BOOL; v->u = x != 0; return true; }
    case 8: v->kind = Value::STR; return read_string(f, &v->s);
    case 9: {
        uint32_t at;
        uint64_t n;
        if (!rdv(f, &at) || !rdv(f, &n) || n > (1ull << 28)) return false;
        v->kind = Value::ARR;
        v->arr.resize(n);
        for (uint64_t i = 0; i < n; i++)
            if (!read_value(f, at, &v->arr[i], depth + 1)) return false;
        return true;
    }
    case 10: { uint64_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_U; v->u = x; return true; }
    case 11: { int64_t x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_I; v->i = x; return true; }
    case 12: { double x; if (!rdv(f, &x)) return false; v->kind = Value::NUM_F; v->f = x; return true; }
    default: return false;
    }
}

const Value *find_meta(const lc_gguf *g, const char *key) {
    auto it = g->meta_index.find(key);
    return it == g->meta_index.end() ? nullptr : &g->meta[it->second].second;
}

// One of the laguna./dflash./bare spellings of a key (populate_metadata,
// src/gguf.rs:516-653).  The reference applies fields in file order, so when
// several spellings are present the one stored last wins; same here.
const Value *find_any(const lc_gguf *g, std::initializer_list<const char *> keys) {
    const Value *v = nullptr;
    size_t best = 0;
    for (const char *k : keys) {
        auto it = g->meta_index.find(k);
        if (it != g->meta_index.end() && (!v || it->second >= best)) {
            v = &g->meta[it->second].second;
            best = it->second;
        }
    }
    return v;
}

}  // namespace

extern "C" uint64_t lc_type_block_bytes(int dtype) {
    switch (dtype) {
    case LC_F32: return 4;
    case LC_F16: case LC_BF16: return 2;
    case LC_Q8_0: return 34;
    case LC_Q4_K: return 144;
    default: return 0;
    }
}

extern "C" uint64_t lc_type_block_elements(int dtype) {
    switch (dtype) {
    case LC_F32: case LC_F16: case LC_BF16: return 1;
    case LC_Q8_0: return 32;
    case LC_Q4_K: return 256;
    default: return 0;
    }
}

extern "C" uint64_t lc_tensor_bytes(int dtype, uint64_t n) {
    const uint64_t be = lc_type_block_elements(dtype);
    if (!be) return 0;
    return (n + be - 1) / be * lc_type_block_bytes(dtype);
}

extern "C" int lc_gguf_open(const char *path, lc_gguf **out) {
    if (!path || !out) return lc_fail(LC_ERR_INVALID, "lc_gguf_open: null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return lc_fail(LC_ERR_IO, "lc_gguf_open: cannot open %s", path);
    lc_gguf *g = new lc_gguf();
    g->fd = fd;
    struct stat st;
    if (fstat(fd, &st) != 0) {
        lc_gguf_close(g);
        return lc_fail(LC_ERR_IO, "lc_gguf_open: cannot stat %s", path);
    }
    g->size = (uint64_t)st.st_size;
    if (g->size) {
        void *p = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            lc_gguf_close(g);
            return lc_fail(LC_ERR_IO, "lc_gguf_open: cannot map %s", path);
        }
        g->map = (const uint8_t *)p;
        madvise(p, g->size, MADV_SEQUENTIAL);  // tensors are read front to back
    }
    Src f{g->map, g->size, 0};
    auto bad = [&](const char *what) {
        lc_gguf_close(g);
        return lc_fail(LC_ERR_IO, "lc_gguf_open(%s): %s", path, what);
    };
    char magic[4];
    if (!rd(f, magic, 4) || memcmp(magic, "GGUF", 4) != 0) return bad("not a GGUF file");
    if (!rdv(f, &g->version)) return bad("truncated header");
    if (g->version != 3) return bad("only GGUF v3 is supported");
    uint64_t n_tensors, n_fields;
    if (!rdv(f, &n_tensors) || !rdv(f, &n_fields) || n_tensors > (1ull << 24) || n_fields > (1ull << 24))
        return bad("bad counts");
    for (uint64_t i = 0; i < n_fields; i++) {
        std::string key;
        uint32_t type;
        Value v;
        if (!read_string(f, &key) || !rdv(f, &type) || !read_value(f, type, &v)) return bad("bad metadata");
        g->meta_index[key] = g->meta.size();
        g->meta.emplace_back(std::move(key), std::move(v));
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        Tensor t;
        uint32_t nd, dt;
        if (!read_string(f, &t.name) || !rdv(f, &nd) || nd > 4) return bad("bad tensor info");
        t.shape.resize(nd);
        for (uint32_t d = 0; d < nd; d++)
            if (!rdv(f, &t.shape[d])) return bad("bad tensor shape");
        if (!rdv(f, &dt) || !rdv(f, &t.offset)) return bad("bad tensor info");
        t.dtype = (int)dt;
        g->tensors.push_back(std::move(t));
    }
    const uint64_t pos = f.pos;
    uint64_t align = 32;
    if (const Value *a = find_meta(g, "general.alignment")) {
        uint64_t v;
        if (a->as_u64(&v) && v > 0) align = v;
    }
    g->data_offset = ((uint64_t)pos + align - 1) / align * align;
    *out = g;
    return LC_OK;
}

extern "C" int lc_gguf_close(lc_gguf *g) {
    if (!g) return LC_OK;
    if (g->map) munmap((void *)g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    delete g;
    return LC_OK;
}

extern "C" uint64_t lc_gguf_tensor_count(const lc_gguf *g) { return g ? g->tensors.size() : 0; }

extern "C" int lc_gguf_tensor_info(const lc_gguf *g, uint64_t i, const char **name, int *dtype, uint32_t *n_dims,
                                   uint64_t shape[4], uint64_t *offset, uint64_t *n_bytes) {
    if (!g || i >= g->tensors.size()) return lc_fail(LC_ERR_INVALID, "lc_gguf_tensor_info: bad index");
    const Tensor &t = g->tensors[i];
    uint64_t n = 1;
    for (uint64_t d : t.shape) n *= d;
    if (name) *name = t.name.c_str();
    if (dtype) *dtype = t.dtype;
    if (n_dims) *n_dims = (uint32_t)t.shape.size();
    if (shape)
        for (int d = 0; d < 4; d++) shape[d] = d < (int)t.shape.size() ? t.shape[d] : 1;
    if (offset) *offset = t.offset;
    if (n_bytes) *n_bytes = lc_tensor_bytes(t.dtype, n);
    return LC_OK;
}

extern "C" int lc_gguf_find(const lc_gguf *g, const char *name, uint64_t *index) {
    if (!g || !name || !index) return lc_fail(LC_ERR_INVALID, "lc_gguf_find: null argument");
    for (uint64_t i = 0; i < g->tensors.size(); i++)
        if (g->tensors[i].name == name) return *index = i, LC_OK;
    return lc_fail(LC_ERR_INVALID, "lc_gguf_find: no tensor named %s", name);
}

extern "C" int lc_gguf_read(lc_gguf *g, uint64_t index, void *dst, uint64_t bytes) {
    if (!g || !dst || index >= g->tensors.size()) return lc_fail(LC_ERR_INVALID, "lc_gguf_read: bad argument");
    uint64_t need;
    lc_gguf_tensor_info(g, index, nullptr, nullptr, nullptr, nullptr, nullptr, &need);
    if (bytes < need) return lc_fail(LC_ERR_INVALID, "lc_gguf_read: buffer of %llu < %llu bytes",
                                     (unsigned long long)bytes, (unsigned long long)need);
    const void *src;
    if (int s = lc_gguf_tensor_data(g, index, &src, nullptr)) return s;
    memcpy(dst, src, need);
    return LC_OK;
}

extern "C" int lc_gguf_tensor_data(const lc_gguf *g, uint64_t index, const void **data, uint64_t *bytes) {
    if (!g || !data || index >= g->tensors.size()) return lc_fail(LC_ERR_INVALID, "lc_gguf_tensor_data: bad argument");
    uint64_t need;
    lc_gguf_tensor_info(g, index, nullptr, nullptr, nullptr, nullptr, nullptr, &need);
    const uint64_t at = g->data_offset + g->tensors[index].offset;
    if (at < g->data_offset || at > g->size || need > g->size - at)
        return lc_fail(LC_ERR_IO, "lc_gguf: %s lies past the end of the file (%llu + %llu > %llu bytes)",
                       g->tensors[index].name.c_str(), (unsigned long long)at, (unsigned long long)need,
                       (unsigned long long)g->size);
    *data = g->map + at;
    if (bytes) *bytes = need;
    return LC_OK;
}

extern "C" int lc_gguf_meta_u64(const lc_gguf *g, const char *key, uint64_t *out) {
    const Value *v = g && key ? find_meta(g, key) : nullptr;
    if (!v || !out || !v->as_u64(out)) return lc_fail(LC_ERR_INVALID, "lc_gguf_meta_u64: no integer %s", key);
    return LC_OK;
}

extern "C" int lc_gguf_meta_f32(const lc_gguf *g, const char *key, float *out) {
    const Value *v = g && key ? find_meta(g, key) : nullptr;
    if (!v || !out || !v->as_f32(out)) return lc_fail(LC_ERR_INVALID, "lc_gguf_meta_f32: no number %s", key);
    return LC_OK;
}

extern "C" int lc_gguf_meta_str(const lc_gguf *g, const char *key, const char **out) {
    const Value *v = g && key ? find_meta(g, key) : nullptr;
    if (!v || !out || v->kind != Value::STR) return lc_fail(LC_ERR_INVALID, "lc_gguf_meta_str: no string %s", key);
    *out = v->s.c_str();
    return LC_OK;
}

extern "C" int lc_gguf_dflash_hparams(const lc_gguf *g, lc_dflash_hparams *hp) {
    if (!g || !hp) return lc_fail(LC_ERR_INVALID, "lc_gguf_dflash_hparams: null argument");
    memset(hp, 0, sizeof(*hp));
    auto u64 = [&](std::initializer_list<const char *> keys, int arr_index = -1) -> uint64_t {
        const Value *v = find_any(g, keys);
        uint64_t r = 0;
        if (!v) return 0;
        if (v->kind == Value::ARR) {
            // head_count arrays: first element; head_count_kv arrays: second (src/gguf.rs:540-560)
            size_t i = arr_index < 0 ? 0 : (size_t)arr_index;
            if (i < v->arr.size()) v->arr[i].as_u64(&r);
            return r;
        }
        v->as_u64(&r);
        return r;
    };
    hp->n_layers = (uint32_t)u64({"block_count", "laguna.block_count", "dflash.block_count"});
    hp->n_embd = (uint32_t)u64({"embedding_length", "laguna.embedding_length", "dflash.embedding_length"});
    hp->n_ff = (uint32_t)u64({"feed_forward_length", "laguna.feed_forward_length", "dflash.feed_forward_length"});
    hp->n_heads = (uint32_t)u64({"attention.head_count", "laguna.attention.head_count", "dflash.attention.head_count"}, 0);
    {
        const Value *v = find_any(g, {"attention.head_count_kv", "laguna.attention.head_count_kv",
                                      "dflash.attention.head_count_kv"});
        uint64_t r = 0;
        if (v && v->kind == Value::ARR) {
            if (v->arr.size() > 1) v->arr[1].as_u64(&r);
        } else if (v) {
            v->as_u64(&r);
        }
        hp->n_kv_heads = (uint32_t)r;
    }
    hp->head_dim = (uint32_t)u64({"laguna.attention.key_length", "dflash.attention.key_length"});
    if (hp->head_dim == 0 && hp->n_heads) hp->head_dim = hp->n_embd / hp->n_heads;  // key_length absent
    hp->rope_dim = (uint32_t)u64({"rope.dimension_count", "laguna.rope.dimension_count", "dflash.rope.dimension_count"});
    hp->rope_base = 500000.0f;
    if (const Value *v = find_any(g, {"rope.freq_base", "laguna.rope.freq_base", "dflash.rope.freq_base"})) {
        float f;
        if (v->as_f32(&f)) hp->rope_base = f;
    }
    if (const Value *v = find_any(g, {"target_layers", "laguna.target_layers", "dflash.target_layers"}))
        if (v->kind == Value::ARR) hp->n_aux = (uint32_t)v->arr.size();
    hp->norm_eps = 1e-5f;
    hp->qk_eps = 1e-6f;
    return LC_OK;
}

extern "C" int lc_gguf_target_hparams(const lc_gguf *g, lc_target_hparams *hp) {
    if (!g || !hp) return lc_fail(LC_ERR_INVALID, "lc_gguf_target_hparams: null argument");
    memset(hp, 0, sizeof(*hp));
    // Model::from_reader (src/model.rs:29-129) over populate_metadata's aliases
    // (src/gguf.rs:516-653); the DFlash reader shares the dense keys.
    lc_dflash_hparams d;
    lc_gguf_dflash_hparams(g, &d);
    auto u64 = [&](std::initializer_list<const char *> keys) -> uint64_t {
        const Value *v = find_any(g, keys);
        uint64_t r = 0;
        if (v) v->as_u64(&r);
        return r;
    };
    hp->n_layers = d.n_layers;
    hp->n_embd = d.n_embd;
    hp->n_ff = d.n_ff;
    hp->n_heads = d.n_heads;
    hp->n_kv_heads = d.n_kv_heads;
    hp->head_dim = (uint32_t)u64({"laguna.attention.key_length", "dflash.attention.key_length"});  // no fallback
    hp->rope_dim = d.rope_dim;
    hp->rope_dim_swa = (uint32_t)u64({"rope.dimension_count_swa", "laguna.rope.dimension_count_swa",
                                      "dflash.rope.dimension_count_swa"});
    const uint64_t window = u64({"laguna.attention.sliding_window", "dflash.attention.sliding_window"});
    hp->swa = hp->rope_dim_swa > 0 || window > 0;  // src/target.rs:328
    hp->rope_base = d.rope_base;
    hp->rope_base_swa = 10000.0f;  // src/target.rs:362-367
    if (const Value *v = find_any(g, {"rope.freq_base_swa", "laguna.rope.freq_base_swa", "dflash.rope.freq_base_swa"})) {
        float f;
        if (v->as_f32(&f)) hp->rope_base_swa = f;
    }
    hp->expert_weights_scale = 1.0f;  // src/target.rs:672
    if (const Value *v = find_any(g, {"expert_weights_scale", "laguna.expert_weights_scale",
                                      "dflash.expert_weights_scale"})) {
        float f;
        if (v->as_f32(&f)) hp->expert_weights_scale = f;
    }
    if (const Value *v = find_any(g, {"expert_weights_norm", "laguna.expert_weights_norm",
                                      "dflash.expert_weights_norm"})) {
        bool b;
        if (v->as_bool(&b)) hp->expert_weights_norm = b;
    }
    // expert sizes: metadata first, else the tensors' shapes (src/model.rs:43-107)
    uint64_t ffn_from_shape = 0, exp_from_shape = 0;
    bool has_moe = false, has_shexp = false;
    for (const Tensor &t : g->tensors) {
        const bool gate_exps = t.name.find("ffn_gate_exps") != std::string::npos;
        const bool gate_shexp = t.name.find("ffn_gate_shexp") != std::string::npos;
        if ((gate_exps || gate_shexp) && t.shape.size() >= 2) ffn_from_shape = std::max<uint64_t>(ffn_from_shape, t.shape[1]);
        if (gate_exps && t.shape.size() == 3) exp_from_shape = std::max<uint64_t>(exp_from_shape, t.shape[2]);
        has_moe |= gate_exps;
        has_shexp |= gate_shexp;
        if (t.name == "token_embd.weight" && hp->n_embd) {
            uint64_t n = 1;
            for (uint64_t dim : t.shape) n *= dim;
            hp->n_vocab = (uint32_t)(n / hp->n_embd);  // TargetModel::vocab_size (src/target.rs:287-291)
        }
    }
    const uint64_t exp_count = u64({"expert.count", "expert_count"});
    const uint64_t exp_used = u64({"expert.used_count", "expert_used_count"});
    const uint64_t ffn_exp = u64({"expert.feed_forward_length", "expert_feed_forward_length"});
    const uint64_t ffn_sh = u64({"expert.shared_feed_forward_length", "expert_shared_feed_forward_length"});
    hp->n_ff_exp = (uint32_t)(ffn_exp ? ffn_exp : ffn_from_shape);
    hp->n_ff_shexp = (uint32_t)(ffn_sh ? ffn_sh : ffn_from_shape);
    hp->n_expert = (uint32_t)(exp_count ? exp_count : exp_from_shape);
    hp->n_expert_used = (uint32_t)(exp_used ? exp_used : (exp_from_shape ? 10 : 0));
    hp->has_moe = has_moe;
    hp->has_shexp = has_shexp;
    hp->norm_eps = 1e-5f;  // dispatch_rmsnorm (src/target.rs:970)
    hp->qk_eps = 1e-6f;    // dispatch_qk_norm_rope (src/target.rs:897)
    return LC_OK;
}

extern "C" int lc_gguf_target_layers(const lc_gguf *g, int64_t *out, uint32_t cap, uint32_t *n) {
    if (!g || !n || (cap && !out)) return lc_fail(LC_ERR_INVALID, "lc_gguf_target_layers: null argument");
    // populate_metadata (src/gguf.rs:633-638): the array's integer elements
    *n = 0;
    const Value *v = find_any(g, {"target_layers", "laguna.target_layers", "dflash.target_layers"});
    if (!v || v->kind != Value::ARR) return LC_OK;
    for (const Value &e : v->arr) {
        uint64_t u;
        if (!e.as_u64(&u)) continue;
        if (*n < cap) out[*n] = (int64_t)u;
        ++*n;
    }
    return LC_OK;
}
