// lc_model.cu -- the DFlash draft model driver: the C++ counterpart of the
// reference's DFlashModel (src/dflash.rs:6-976) built on the C ABI kernels.
//
// Weights keep their GGUF layout on the device (raw Q8_0 / Q4_K blocks or f32);
// every projection runs the fused dequant kernels.  The host round trips of the
// reference (K/V concatenation with read_f32/upload, src/dflash.rs:945-952, and
// the softplus gate, :956-958) are on the device: block K/V rows are written by
// the projections straight into the per-layer K/V cache after the context rows.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "lc_internal.cuh"

namespace {

using Weight = lc::DevTensor;

struct LayerW {
    Weight attn_norm, q, k, v, o, q_norm, k_norm, gate_attn, ffn_norm, gate, up, down;
};

// repeat_v.comp: out[i] = v[i % n_kv] (forward_from_input's attention stand-in).
__global__ void repeat_v_kernel(const float *v, float *out, int n_kv, int n_out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_out; i += gridDim.x * blockDim.x) out[i] = v[i % n_kv];
}

// forward_token's embedding lookup (src/dflash.rs:482-485): x[i] = emb[i*vocab + tok].
__global__ void gather_column_kernel(const float *emb, float *x, int n_embd, int vocab, int tok) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_embd; i += gridDim.x * blockDim.x)
        x[i] = emb[(size_t)i * vocab + tok];
}

}  // namespace

struct lc_dflash {
    lc_ctx *ctx = nullptr;
    lc_dflash_hparams hp{};
    uint32_t max_ctx = 0, max_block = 0;
    std::vector<LayerW> layers;
    Weight tok_embd, output_norm, fc, enc_aux_norm, enc_output_norm;
    float *freq = nullptr;
    float *kcache = nullptr, *vcache = nullptr;  // [layers][max_ctx + max_block][n_kv*head_dim]
    uint32_t n_ctx = 0;
    // block workspace
    float *x = nullptr, *nx = nullptr, *q = nullptr, *attn = nullptr, *gate = nullptr, *tmp = nullptr;
    float *ffg = nullptr, *ffu = nullptr, *ffh = nullptr;
    // grown on demand: encoder / context inputs, legacy decoder vectors
    float *ctx_nx = nullptr;
    size_t ctx_nx_cap = 0;
    float *host_io = nullptr;
    size_t host_io_cap = 0;
    std::vector<void *> allocs;

    ~lc_dflash() {
        for (void *p : allocs) cudaFree(p);
        if (ctx_nx) cudaFree(ctx_nx);
        if (host_io) cudaFree(host_io);
    }
    size_t kv_dim() const { return (size_t)hp.n_kv_heads * hp.head_dim; }
    size_t cache_rows() const { return (size_t)max_ctx + max_block; }
    float *kl(uint32_t l) const { return kcache + (size_t)l * cache_rows() * kv_dim(); }
    float *vl(uint32_t l) const { return vcache + (size_t)l * cache_rows() * kv_dim(); }
};

#define LC_TRY(expr)               \
    do {                           \
        int _s = (expr);           \
        if (_s != LC_OK) return _s; \
    } while (0)

static int dalloc(lc_dflash *m, size_t bytes, void **out) {
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 256);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return lc_fail(LC_ERR_OOM, "lc_dflash: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    m->allocs.push_back(p);
    *out = p;
    return LC_OK;
}

template <typename T>
static int dalloc_t(lc_dflash *m, size_t count, T **out) {
    void *p = nullptr;
    LC_TRY(dalloc(m, count * sizeof(T), &p));
    *out = (T *)p;
    return LC_OK;
}

static int grow(float **buf, size_t *cap, size_t count) {
    if (count <= *cap) return LC_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc((void **)buf, count * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *buf = nullptr;
        return lc_fail(LC_ERR_OOM, "lc_dflash: cudaMalloc(%zu): %s", count * 4, cudaGetErrorString(e));
    }
    *cap = count;
    return LC_OK;
}

// A projection by the weight's own dtype, with the shape checked against it.
int lc::proj_w(lc_ctx *c, const DevTensor &w, const char *what, const float *x, float *y, uint32_t rows, uint32_t k,
               uint32_t n) {
    if (!w.ptr) return lc_fail(LC_ERR_INVALID, "missing tensor %s", what);
    if (w.n_el < (uint64_t)k * n)
        return lc_fail(LC_ERR_INVALID, "%s has %llu elements, need %u x %u", what, (unsigned long long)w.n_el, n, k);
    return lc_proj_m(c, w.dtype, x, w.ptr, y, rows, k, n, 0);
}

// Projections of one activation block (lc::gemm_dq_group): one packing and one
// tcgen05 GEMM launch when every weight has the same quantized dtype and the
// block size runs that GEMM.  Otherwise one projection per weight, with the
// element-wise input op and the residual adds as their own launches, in the
// reference's order; `materialized` (rows x k) receives the op's result there
// and `tmp` (rows x the widest accumulated output) the summands.
int lc::proj_w_block(lc_ctx *c, float *tmp, const PackSrc &src, float *materialized, ProjOut *outs,
                     const DevTensor *const *ws, const char *const *names, int ng, uint32_t rows, uint32_t k) {
    bool grouped = lc::routes_to_gemm_dq(c, rows);
    for (int i = 0; i < ng; i++) {
        if (!ws[i]->ptr) return lc_fail(LC_ERR_INVALID, "missing tensor %s", names[i]);
        if (ws[i]->n_el < (uint64_t)k * outs[i].n)
            return lc_fail(LC_ERR_INVALID, "%s has %llu elements, need %u x %u", names[i],
                           (unsigned long long)ws[i]->n_el, outs[i].n, k);
        outs[i].w = ws[i]->ptr;
        if (ws[i]->dtype != ws[0]->dtype) grouped = false;
    }
    const int dtype = ws[0]->dtype;
    if (grouped && (dtype == LC_Q4_K || dtype == LC_Q8_0)) {
        const int s = lc::gemm_dq_group(c, dtype, src, outs, ng, rows, k);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    const float *x = src.x;
    if (src.op == lc::LC_PACK_RMSNORM) {
        LC_TRY(lc_rmsnorm(c, src.x2, src.x, materialized, rows, k, src.eps));
        x = materialized;
    } else if (src.op == lc::LC_PACK_SWIGLU) {
        LC_TRY(lc_activation(c, src.x, src.x2, materialized, rows * k));
        x = materialized;
    } else if (src.op == lc::LC_PACK_HEADGATE) {
        const uint32_t heads = k / (uint32_t)src.head_dim;
        float *gate = const_cast<float *>(src.x2);  // the block's own gate buffer
        LC_TRY(lc_softplus(c, gate, gate, rows * heads));
        LC_TRY(lc_gate_mul(c, src.x, gate, materialized, rows * k, heads, (uint32_t)src.head_dim));
        x = materialized;
    }
    for (int i = 0; i < ng; i++) {
        if (!outs[i].accumulate) {
            LC_TRY(proj_w(c, *ws[i], names[i], x, outs[i].y, rows, k, outs[i].n));
        } else {
            LC_TRY(proj_w(c, *ws[i], names[i], x, tmp, rows, k, outs[i].n));
            LC_TRY(lc_add(c, outs[i].y, tmp, outs[i].y, rows * outs[i].n));
        }
    }
    return LC_OK;
}

static int proj(lc_dflash *m, const Weight &w, const char *what, const float *x, float *y, uint32_t rows, uint32_t k,
                uint32_t n) {
    return lc::proj_w(m->ctx, w, what, x, y, rows, k, n);
}

static int proj_block(lc_dflash *m, const lc::PackSrc &src, float *materialized, lc::ProjOut *outs,
                      const Weight *const *ws, const char *const *names, int ng, uint32_t rows, uint32_t k) {
    return lc::proj_w_block(m->ctx, m->tmp, src, materialized, outs, ws, names, ng, rows, k);
}

static const float *need(const Weight &w, const char *what, int *status) {
    if (!w.ptr || w.dtype != LC_F32) {
        *status = lc_fail(LC_ERR_INVALID, "lc_dflash: missing f32 tensor %s", what);
        return nullptr;
    }
    return (const float *)w.ptr;
}

extern "C" int lc_dflash_create(lc_ctx *ctx, const lc_dflash_hparams *hp, uint32_t max_ctx, uint32_t max_block,
                                lc_dflash **out) {
    LC_REQUIRE(ctx && hp && out, LC_ERR_INVALID, "lc_dflash_create: null argument");
    *out = nullptr;
    LC_REQUIRE(hp->n_layers && hp->n_embd && hp->n_heads && hp->n_kv_heads && hp->head_dim && hp->n_ff,
               LC_ERR_INVALID, "lc_dflash_create: incomplete hyper-parameters");
    LC_REQUIRE(hp->n_heads % hp->n_kv_heads == 0, LC_ERR_UNSUPPORTED,
               "lc_dflash_create: n_heads %u not a multiple of n_kv_heads %u", hp->n_heads, hp->n_kv_heads);
    LC_REQUIRE(max_block >= 1 && max_ctx >= 1, LC_ERR_INVALID, "lc_dflash_create: max_ctx/max_block must be >= 1");
    LC_TRY(lc_use_device(ctx));
    lc_dflash *m = new lc_dflash();
    m->ctx = ctx;
    m->hp = *hp;
    m->max_ctx = max_ctx;
    m->max_block = max_block;
    m->layers.resize(hp->n_layers);
    const size_t E = hp->n_embd, QD = (size_t)hp->n_heads * hp->head_dim, F = hp->n_ff, B = max_block;
    int s = LC_OK;
    float *freq_host = nullptr;
    do {
        if ((s = dalloc_t(m, hp->rope_dim / 2 + 1, &m->freq))) break;
        if ((s = dalloc_t(m, (size_t)hp->n_layers * m->cache_rows() * m->kv_dim(), &m->kcache))) break;
        if ((s = dalloc_t(m, (size_t)hp->n_layers * m->cache_rows() * m->kv_dim(), &m->vcache))) break;
        if ((s = dalloc_t(m, B * E, &m->x))) break;
        if ((s = dalloc_t(m, B * E, &m->nx))) break;
        if ((s = dalloc_t(m, B * std::max(QD, E), &m->q))) break;
        if ((s = dalloc_t(m, B * std::max(QD, E), &m->attn))) break;
        if ((s = dalloc_t(m, B * hp->n_heads, &m->gate))) break;
        if ((s = dalloc_t(m, B * E, &m->tmp))) break;
        if ((s = dalloc_t(m, B * F, &m->ffg))) break;
        if ((s = dalloc_t(m, B * F, &m->ffu))) break;
        if ((s = dalloc_t(m, B * F, &m->ffh))) break;
        freq_host = new float[hp->rope_dim / 2 + 1];
        lc_rope_freq(freq_host, hp->rope_dim, hp->rope_base);  // src/dflash.rs:901-907
        cudaError_t e = cudaMemcpy(m->freq, freq_host, (hp->rope_dim / 2 + 1) * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) s = lc_fail(LC_ERR_CUDA, "lc_dflash_create: %s", cudaGetErrorString(e));
    } while (0);
    delete[] freq_host;
    if (s) {
        delete m;
        return s;
    }
    *out = m;
    return LC_OK;
}

extern "C" int lc_dflash_destroy(lc_dflash *m) {
    if (!m) return LC_OK;
    lc_use_device(m->ctx);
    cudaStreamSynchronize(m->ctx->stream);
    delete m;
    return LC_OK;
}

extern "C" int lc_dflash_get_hparams(const lc_dflash *m, lc_dflash_hparams *out) {
    LC_REQUIRE(m && out, LC_ERR_INVALID, "lc_dflash_get_hparams: null argument");
    *out = m->hp;
    return LC_OK;
}

static Weight *slot_for(lc_dflash *m, const char *name) {
    if (!strcmp(name, "token_embd.weight")) return &m->tok_embd;
    if (!strcmp(name, "output_norm.weight")) return &m->output_norm;
    if (!strcmp(name, "fc.weight")) return &m->fc;
    if (!strcmp(name, "enc.aux_norm.weight")) return &m->enc_aux_norm;
    if (!strcmp(name, "enc.output_norm.weight")) return &m->enc_output_norm;
    unsigned layer;
    int off = 0;
    if (sscanf(name, "blk.%u.%n", &layer, &off) != 1 || off == 0 || layer >= m->layers.size()) return nullptr;
    const char *suf = name + off;
    LayerW &L = m->layers[layer];
    struct {
        const char *s;
        Weight *w;
    } tab[] = {{"attn_norm.weight", &L.attn_norm}, {"attn_q.weight", &L.q},          {"attn_k.weight", &L.k},
               {"attn_v.weight", &L.v},            {"attn_output.weight", &L.o},     {"attn_q_norm.weight", &L.q_norm},
               {"attn_k_norm.weight", &L.k_norm},  {"attn_gate.weight", &L.gate_attn}, {"ffn_norm.weight", &L.ffn_norm},
               {"ffn_gate.weight", &L.gate},       {"ffn_up.weight", &L.up},         {"ffn_down.weight", &L.down}};
    for (auto &e : tab)
        if (!strcmp(suf, e.s)) return e.w;
    return nullptr;
}

extern "C" int lc_dflash_set_tensor(lc_dflash *m, const char *name, int dtype, const void *host, size_t bytes) {
    LC_REQUIRE(m && name && (host || !bytes), LC_ERR_INVALID, "lc_dflash_set_tensor: null argument");
    Weight *w = slot_for(m, name);
    if (!w) return LC_OK;  // tensors the draft path does not use are skipped, like DFlashModel::load
    const uint64_t be = lc_type_block_elements(dtype), bb = lc_type_block_bytes(dtype);
    LC_REQUIRE(be && bb, LC_ERR_UNSUPPORTED, "lc_dflash_set_tensor: %s has unsupported type %d", name, dtype);
    LC_TRY(lc_use_device(m->ctx));
    const uint64_t n_el = bytes / bb * be;
    void *raw = nullptr;
    LC_TRY(dalloc(m, bytes, &raw));
    cudaError_t e = cudaMemcpyAsync(raw, host, bytes, cudaMemcpyHostToDevice, m->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->ctx->stream);
    if (e != cudaSuccess) return lc_fail(LC_ERR_CUDA, "lc_dflash_set_tensor(%s): %s", name, cudaGetErrorString(e));
    if (dtype == LC_F16 || dtype == LC_BF16) {
        // dequant_to_f32 rules (src/dflash.rs:351-378, :437-462), as the reference uploads them
        void *f = nullptr;
        LC_TRY(dalloc(m, n_el * 4, &f));
        LC_TRY(lc_dequant(m->ctx, dtype, raw, bytes, n_el, (float *)f));
        raw = f;
        dtype = LC_F32;
        bytes = n_el * 4;
    }
    w->ptr = raw;
    w->bytes = bytes;
    w->dtype = dtype;
    w->n_el = n_el;
    return LC_OK;
}

extern "C" int lc_dflash_load_gguf_ex(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block,
                                      uint32_t flags, lc_dflash **out) {
    LC_REQUIRE(ctx && path && out, LC_ERR_INVALID, "lc_dflash_load_gguf: null argument");
    LC_REQUIRE((flags & ~(uint32_t)LC_LOAD_BF16_NATIVE) == 0, LC_ERR_INVALID, "lc_dflash_load_gguf: unknown flags %#x",
               flags);
    *out = nullptr;
    lc_gguf *g;
    LC_TRY(lc_gguf_open(path, &g));
    lc_dflash_hparams hp;
    int s = lc_gguf_dflash_hparams(g, &hp);
    lc_dflash *m = nullptr;
    if (!s) s = lc_dflash_create(ctx, &hp, max_ctx, max_block, &m);
    if (!s)
        s = lc::load_tensors(ctx, g, [m](const char *name) { return slot_for(m, name); }, flags, &m->allocs);
    lc_gguf_close(g);
    if (s) {
        lc_dflash_destroy(m);
        return s;
    }
    *out = m;
    return LC_OK;
}

extern "C" int lc_dflash_load_gguf(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block,
                                   lc_dflash **out) {
    return lc_dflash_load_gguf_ex(ctx, path, max_ctx, max_block, 0, out);
}

extern "C" int lc_dflash_weight(const lc_dflash *m, const char *name, const void **data, int *dtype,
                                uint64_t *bytes) {
    LC_REQUIRE(m && name && data, LC_ERR_INVALID, "lc_dflash_weight: null argument");
    const Weight *w = slot_for(const_cast<lc_dflash *>(m), name);
    LC_REQUIRE(w && w->ptr, LC_ERR_INVALID, "lc_dflash_weight: no tensor %s", name);
    *data = w->ptr;
    if (dtype) *dtype = w->dtype;
    if (bytes) *bytes = w->bytes;
    return LC_OK;
}

extern "C" int lc_dflash_encode(lc_dflash *m, const float *features, uint32_t n_ctx, float *enc_out) {
    LC_REQUIRE(m && features && enc_out, LC_ERR_INVALID, "lc_dflash_encode: null argument");
    LC_REQUIRE(n_ctx >= 1, LC_ERR_INVALID, "lc_dflash_encode: n_ctx must be >= 1");
    LC_REQUIRE(m->hp.n_aux >= 1, LC_ERR_INVALID, "lc_dflash_encode: model has no target_layers (n_aux = 0)");
    LC_TRY(lc_use_device(m->ctx));
    const lc_dflash_hparams &h = m->hp;
    const uint32_t E = h.n_embd, IN = h.n_aux * h.n_embd;
    int s = LC_OK;
    const float *aux_w = need(m->enc_aux_norm, "enc.aux_norm.weight", &s);
    const float *out_w = need(m->enc_output_norm, "enc.output_norm.weight", &s);
    if (s) return s;
    LC_TRY(grow(&m->ctx_nx, &m->ctx_nx_cap, (size_t)n_ctx * IN));
    LC_TRY(lc_enc_aux_norm(m->ctx, features, aux_w, m->ctx_nx, E, h.n_aux, n_ctx, h.norm_eps));
    LC_TRY(proj(m, m->fc, "fc.weight", m->ctx_nx, enc_out, n_ctx, IN, E));
    LC_TRY(lc_rmsnorm(m->ctx, out_w, enc_out, enc_out, n_ctx, E, h.norm_eps));
    return LC_OK;
}

extern "C" int lc_dflash_set_context(lc_dflash *m, const float *enc_out, uint32_t n_ctx) {
    LC_REQUIRE(m && enc_out, LC_ERR_INVALID, "lc_dflash_set_context: null argument");
    LC_REQUIRE(n_ctx >= 1 && n_ctx <= m->max_ctx, LC_ERR_INVALID, "lc_dflash_set_context: n_ctx %u not in 1..%u",
               n_ctx, m->max_ctx);
    LC_TRY(lc_use_device(m->ctx));
    const lc_dflash_hparams &h = m->hp;
    const uint32_t E = h.n_embd, KVD = (uint32_t)m->kv_dim();
    LC_TRY(grow(&m->ctx_nx, &m->ctx_nx_cap, (size_t)n_ctx * E));
    for (uint32_t l = 0; l < h.n_layers; l++) {
        const LayerW &L = m->layers[l];
        int s = LC_OK;
        const float *an = need(L.attn_norm, "attn_norm.weight", &s);
        const float *kn = need(L.k_norm, "attn_k_norm.weight", &s);
        if (s) return s;
        // src/dflash.rs:933-936: rmsnorm(enc) -> k, v projections -> k QK-norm + RoPE
        LC_TRY(lc_rmsnorm(m->ctx, an, enc_out, m->ctx_nx, n_ctx, E, h.norm_eps));
        LC_TRY(proj(m, L.k, "attn_k.weight", m->ctx_nx, m->kl(l), n_ctx, E, KVD));
        LC_TRY(proj(m, L.v, "attn_v.weight", m->ctx_nx, m->vl(l), n_ctx, E, KVD));
        LC_TRY(lc_qk_norm_rope(m->ctx, m->kl(l), kn, m->freq, m->kl(l), n_ctx, h.n_kv_heads, h.head_dim, h.rope_dim,
                               h.qk_eps, 0));
    }
    m->n_ctx = n_ctx;
    return LC_OK;
}

extern "C" int lc_dflash_decode_block(lc_dflash *m, const float *x_in, uint32_t mt, float *hidden) {
    LC_REQUIRE(m && x_in && hidden, LC_ERR_INVALID, "lc_dflash_decode_block: null argument");
    LC_REQUIRE(mt >= 1 && mt <= m->max_block, LC_ERR_INVALID, "lc_dflash_decode_block: %u tokens not in 1..%u", mt,
               m->max_block);
    LC_REQUIRE(m->n_ctx >= 1, LC_ERR_INVALID, "lc_dflash_decode_block: no context (call lc_dflash_set_context)");
    LC_TRY(lc_use_device(m->ctx));
    const lc_dflash_hparams &h = m->hp;
    const uint32_t E = h.n_embd, QD = h.n_heads * h.head_dim, KVD = (uint32_t)m->kv_dim(), F = h.n_ff;
    const uint32_t pos0 = m->n_ctx;
    const float scale = 1.0f / sqrtf((float)h.head_dim);  // src/dflash.rs:1173
    lc_ctx *c = m->ctx;
    LC_CUDA(cudaMemcpyAsync(m->x, x_in, (size_t)mt * E * 4, cudaMemcpyDeviceToDevice, c->stream));
    for (uint32_t l = 0; l < h.n_layers; l++) {
        const LayerW &L = m->layers[l];
        int s = LC_OK;
        const float *an = need(L.attn_norm, "attn_norm.weight", &s);
        const float *qn = need(L.q_norm, "attn_q_norm.weight", &s);
        const float *kn = need(L.k_norm, "attn_k_norm.weight", &s);
        const float *fn = need(L.ffn_norm, "ffn_norm.weight", &s);
        if (s) return s;
        float *kblk = m->kl(l) + (size_t)pos0 * KVD, *vblk = m->vl(l) + (size_t)pos0 * KVD;
        // src/dflash.rs:938-943 (+ the head-gate projection of :955, which reads
        // the same normalised block): one activation block, four projections
        // attn_norm is formed while the block is packed (m->nx only on the
        // per-projection route)
        {
            lc::PackSrc src;
            src.x = m->x;
            src.x2 = an;
            src.op = lc::LC_PACK_RMSNORM;
            src.eps = h.norm_eps;
            lc::ProjOut outs[4] = {{nullptr, m->q, QD, false}, {nullptr, kblk, KVD, false},
                                   {nullptr, vblk, KVD, false}, {nullptr, m->gate, h.n_heads, false}};
            const Weight *ws[4] = {&L.q, &L.k, &L.v, &L.gate_attn};
            const char *names[4] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_gate.weight"};
            LC_TRY(proj_block(m, src, m->nx, outs, ws, names, 4, mt, E));
        }
        LC_TRY(lc::qk_norm_rope_pair(c, m->q, qn, m->q, h.n_heads, kblk, kn, kblk, h.n_kv_heads, m->freq, mt,
                                     h.head_dim, h.rope_dim, h.qk_eps, pos0));
        // :945-954 -- K/V rows [context; block] are already adjacent in the cache
        LC_TRY(lc_mha_attn(c, m->q, m->kl(l), m->vl(l), m->attn, mt, h.n_heads, h.n_kv_heads, h.head_dim,
                           pos0 + mt, scale, pos0, 1));
        // :955-969 -- attn * softplus(head gate), output projection, residual add
        {
            lc::PackSrc src;
            src.x = m->attn;
            src.x2 = m->gate;
            src.op = lc::LC_PACK_HEADGATE;
            src.head_dim = (int)h.head_dim;
            lc::ProjOut outs[1] = {{nullptr, m->x, E, true}};
            const Weight *ws[1] = {&L.o};
            const char *names[1] = {"attn_output.weight"};
            LC_TRY(proj_block(m, src, m->attn, outs, ws, names, 1, mt, QD));
        }
        {  // ffn_norm, likewise
            lc::PackSrc src;
            src.x = m->x;
            src.x2 = fn;
            src.op = lc::LC_PACK_RMSNORM;
            src.eps = h.norm_eps;
            lc::ProjOut outs[2] = {{nullptr, m->ffg, F, false}, {nullptr, m->ffu, F, false}};
            const Weight *ws[2] = {&L.gate, &L.up};
            const char *names[2] = {"ffn_gate.weight", "ffn_up.weight"};
            LC_TRY(proj_block(m, src, m->nx, outs, ws, names, 2, mt, E));
        }
        {
            lc::PackSrc src;
            src.x = m->ffg;
            src.x2 = m->ffu;
            src.op = lc::LC_PACK_SWIGLU;
            lc::ProjOut outs[1] = {{nullptr, m->x, E, true}};
            const Weight *ws[1] = {&L.down};
            const char *names[1] = {"ffn_down.weight"};
            LC_TRY(proj_block(m, src, m->ffh, outs, ws, names, 1, mt, F));
        }
    }
    // :972-975
    int s = LC_OK;
    const float *on = need(m->output_norm, "output_norm.weight", &s);
    if (s) return s;
    LC_TRY(lc_rmsnorm(c, on, m->x, hidden, mt, E, h.norm_eps));
    return lc_after_launch(c, "lc_dflash_decode_block");
}

extern "C" int lc_dflash_forward_injected_decode_hidden(lc_dflash *m, const float *features_host,
                                                        const float *token_host, float *hidden_host) {
    LC_REQUIRE(m && features_host && token_host && hidden_host, LC_ERR_INVALID,
               "lc_dflash_forward_injected_decode_hidden: null argument");
    LC_TRY(lc_use_device(m->ctx));
    const uint32_t E = m->hp.n_embd, IN = m->hp.n_aux * m->hp.n_embd;
    LC_TRY(grow(&m->host_io, &m->host_io_cap, (size_t)IN + 3 * E));
    float *feat = m->host_io, *enc = feat + IN, *tok = enc + E, *hid = tok + E;
    cudaStream_t st = m->ctx->stream;
    LC_CUDA(cudaMemcpyAsync(feat, features_host, (size_t)IN * 4, cudaMemcpyHostToDevice, st));
    LC_CUDA(cudaMemcpyAsync(tok, token_host, (size_t)E * 4, cudaMemcpyHostToDevice, st));
    LC_TRY(lc_dflash_encode(m, feat, 1, enc));
    LC_TRY(lc_dflash_set_context(m, enc, 1));
    LC_TRY(lc_dflash_decode_block(m, tok, 1, hid));
    LC_CUDA(cudaMemcpyAsync(hidden_host, hid, (size_t)E * 4, cudaMemcpyDeviceToHost, st));
    LC_CUDA(cudaStreamSynchronize(st));
    return LC_OK;
}

extern "C" int lc_dflash_forward_from_input(lc_dflash *m, const float *input, float *hidden, float *logits,
                                            uint32_t *n_vocab) {
    LC_REQUIRE(m && input && hidden, LC_ERR_INVALID, "lc_dflash_forward_from_input: null argument");
    LC_TRY(lc_use_device(m->ctx));
    const lc_dflash_hparams &h = m->hp;
    const uint32_t E = h.n_embd, QD = h.n_heads * h.head_dim, KVD = (uint32_t)m->kv_dim(), F = h.n_ff;
    lc_ctx *c = m->ctx;
    LC_CUDA(cudaMemcpyAsync(m->x, input, (size_t)E * 4, cudaMemcpyDeviceToDevice, c->stream));
    for (uint32_t l = 0; l < h.n_layers; l++) {
        const LayerW &L = m->layers[l];
        int s = LC_OK;
        const float *an = need(L.attn_norm, "attn_norm.weight", &s);
        const float *fn = need(L.ffn_norm, "ffn_norm.weight", &s);
        if (s) return s;
        // src/dflash.rs:769-833.  The q/k projections and their QK-norm+RoPE
        // feed nothing downstream in this decoder (the head gate multiplies the
        // repeated v), so they are not computed.
        LC_TRY(lc_rmsnorm(c, an, m->x, m->nx, 1, E, h.norm_eps));
        LC_TRY(proj(m, L.v, "attn_v.weight", m->nx, m->tmp, 1, E, KVD));
        repeat_v_kernel<<<(QD + 255) / 256, 256, 0, c->stream>>>(m->tmp, m->q, (int)KVD, (int)QD);
        LC_TRY(proj(m, L.gate_attn, "attn_gate.weight", m->nx, m->gate, 1, E, h.n_heads));
        LC_TRY(lc_softplus(c, m->gate, m->gate, h.n_heads));
        LC_TRY(lc_gate_mul(c, m->q, m->gate, m->attn, QD, h.n_heads, h.head_dim));
        LC_TRY(proj(m, L.o, "attn_output.weight", m->attn, m->tmp, 1, QD, E));
        LC_TRY(lc_add(c, m->x, m->tmp, m->x, E));
        LC_TRY(lc_rmsnorm(c, fn, m->x, m->nx, 1, E, h.norm_eps));
        LC_TRY(proj(m, L.gate, "ffn_gate.weight", m->nx, m->ffg, 1, E, F));
        LC_TRY(proj(m, L.up, "ffn_up.weight", m->nx, m->ffu, 1, E, F));
        LC_TRY(lc_activation(c, m->ffg, m->ffu, m->ffh, F));
        LC_TRY(proj(m, L.down, "ffn_down.weight", m->ffh, m->tmp, 1, F, E));
        LC_TRY(lc_add(c, m->x, m->tmp, m->x, E));
    }
    int s = LC_OK;
    const float *on = need(m->output_norm, "output_norm.weight", &s);
    if (s) return s;
    LC_TRY(lc_rmsnorm(c, on, m->x, hidden, 1, E, h.norm_eps));
    if (logits) {
        // src/dflash.rs:839-847: fc.weight as a [size/(n_embd) rows, n_embd] head
        LC_REQUIRE(m->fc.ptr, LC_ERR_INVALID, "lc_dflash_forward_from_input: logits need fc.weight");
        const uint32_t vocab = (uint32_t)(m->fc.n_el / E);
        if (n_vocab) *n_vocab = vocab;
        LC_TRY(lc_proj_m(c, m->fc.dtype, hidden, m->fc.ptr, logits, 1, E, vocab, 0));
    }
    return lc_after_launch(c, "lc_dflash_forward_from_input");
}

extern "C" int lc_dflash_forward_token(lc_dflash *m, uint32_t token_id, float *hidden, float *logits,
                                       uint32_t *n_vocab) {
    LC_REQUIRE(m && hidden, LC_ERR_INVALID, "lc_dflash_forward_token: null argument");
    LC_TRY(lc_use_device(m->ctx));
    const uint32_t E = m->hp.n_embd;
    LC_REQUIRE(m->tok_embd.ptr && m->tok_embd.dtype == LC_F32, LC_ERR_UNSUPPORTED,
               "lc_dflash_forward_token: needs an F32/F16/BF16 token_embd.weight");
    const uint32_t vocab = (uint32_t)(m->tok_embd.n_el / E);
    LC_REQUIRE(token_id < vocab, LC_ERR_INVALID, "lc_dflash_forward_token: token_id %u >= vocab_size %u", token_id,
               vocab);
    LC_TRY(grow(&m->host_io, &m->host_io_cap, (size_t)E));
    gather_column_kernel<<<(E + 255) / 256, 256, 0, m->ctx->stream>>>((const float *)m->tok_embd.ptr, m->host_io,
                                                                      (int)E, (int)vocab, (int)token_id);
    return lc_dflash_forward_from_input(m, m->host_io, hidden, logits, n_vocab);
}
