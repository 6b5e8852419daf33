// laguna-cuda -- command-line driver with the reference's subcommand surface
// (src/main.rs:24-105, src/lib.rs:24-255) for the commands on the quantized
// projection path, running on the CUDA backend through the C ABI.
//
//   info <gguf>            model metadata + tensors      (run_info, lib.rs:24)
//   shapes <gguf>          tensor shapes                 (run_shapes, lib.rs:50)
//   forward <gguf> <tok>   legacy single-token forward   (run_forward, lib.rs:57)
//   encode <gguf>          encode + decode, zero feats   (run_forward_encode, lib.rs:81)
//   test-dequant           dequant self-test             (run_test_dequant, lib.rs:94)
//   test-matmul            8x3 f32 projection self-test  (run_test_matmul, lib.rs:120)
//   test-rmsnorm           4-element rmsnorm self-test   (run_test_rmsnorm, lib.rs:167)
//   draft <gguf> [ctx] [m] block draft forward: encode ctx rows of synthetic
//                          target features, then decode an m-token block
//   target-info <gguf>     target metadata + layer kinds (run_target_info, lib.rs:257)
//   target-forward <gguf> [tok]  forward_token, all layers captured (lib.rs:284)
//   target-generate <gguf> [start] [n]  greedy, K/V cached (lib.rs:335)
//   target-dflash <t> <d> [tok]  one draft step's logits (lib.rs:384)
//   target-dflash-verify <t> <d> [tok] [n]  draft / verify loop (lib.rs:466)
//   project-ref <gguf> <file>    lm_head of an f32 hidden state (lib.rs:530)
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "laguna_cuda.h"

#include <cuda_runtime.h>

static const char *kTypeNames(int t) {
    switch (t) {
    case LC_F32: return "F32";
    case LC_F16: return "F16";
    case LC_Q8_0: return "Q8_0";
    case LC_Q4_K: return "Q4_K";
    case LC_BF16: return "BF16";
    default: return "?";
    }
}

static void die(const char *what) {
    fprintf(stderr, "%s: %s\n", what, lc_last_error());
    exit(1);
}

#define CHECK(expr)                  \
    do {                             \
        if ((expr) != LC_OK) die(#expr); \
    } while (0)

static lc_ctx *ctx_open() {
    lc_ctx *c;
    CHECK(lc_init(0, &c));
    CHECK(lc_set_sync(c, 1));
    return c;
}

static int run_info(const char *path, bool shapes_only) {
    lc_gguf *g;
    CHECK(lc_gguf_open(path, &g));
    if (!shapes_only) {
        lc_dflash_hparams hp;
        CHECK(lc_gguf_dflash_hparams(g, &hp));
        const char *arch = "";
        lc_gguf_meta_str(g, "general.architecture", &arch);
        printf("GGUF v3\narchitecture: %s\n", arch);
        printf("block_count: %u\nembedding_length: %u\nfeed_forward_length: %u\n", hp.n_layers, hp.n_embd, hp.n_ff);
        printf("attention_head_count: %u\nattention_head_count_kv: %u\nattention_key_length: %u\n", hp.n_heads,
               hp.n_kv_heads, hp.head_dim);
        printf("rope_dimension_count: %u\nrope_freq_base: %g\ntarget_layers: %u\n", hp.rope_dim, hp.rope_base,
               hp.n_aux);
        printf("tensor_count: %llu\n\ntensors:\n", (unsigned long long)lc_gguf_tensor_count(g));
    }
    for (uint64_t i = 0; i < lc_gguf_tensor_count(g); i++) {
        const char *name;
        int dt;
        uint32_t nd;
        uint64_t shape[4], off, nb;
        CHECK(lc_gguf_tensor_info(g, i, &name, &dt, &nd, shape, &off, &nb));
        printf("  %s [", name);
        for (uint32_t d = 0; d < nd; d++) printf(d ? ", %llu" : "%llu", (unsigned long long)shape[d]);
        printf("] %s (%llu bytes @ %llu)\n", kTypeNames(dt), (unsigned long long)nb, (unsigned long long)off);
    }
    lc_gguf_close(g);
    return 0;
}

static void print_logits(const float *dev, uint32_t n, const char *what) {
    std::vector<float> h(n);
    cudaMemcpy(h.data(), dev, n * 4, cudaMemcpyDeviceToHost);
    printf("%s complete, %u logits\n", what, n);
    for (uint32_t i = 0; i < n && i < 10; i++) printf("  logit[%u] = %g\n", i, h[i]);
}

static int run_forward(const char *path, uint32_t tok, bool encode) {
    lc_ctx *c = ctx_open();
    lc_dflash *m;
    CHECK(lc_dflash_load_gguf(c, path, 1, 1, &m));
    lc_dflash_hparams hp;
    CHECK(lc_dflash_get_hparams(m, &hp));
    float *hidden, *logits, *feat, *enc;
    const size_t in = (size_t)hp.n_aux * hp.n_embd;
    cudaMalloc(&hidden, hp.n_embd * 4);
    cudaMalloc(&logits, (size_t)1 << 28);
    cudaMalloc(&feat, (in ? in : 1) * 4);
    cudaMalloc(&enc, hp.n_embd * 4);
    uint32_t vocab = 0;
    if (encode) {
        // run_forward_encode (lib.rs:81-92): zero target features
        cudaMemset(feat, 0, in * 4);
        CHECK(lc_dflash_encode(m, feat, 1, enc));
        CHECK(lc_dflash_forward_from_input(m, enc, hidden, logits, &vocab));
        print_logits(logits, vocab, "encode+decode");
    } else {
        CHECK(lc_dflash_forward_token(m, tok, hidden, logits, &vocab));
        print_logits(logits, vocab, "forward pass");
    }
    lc_dflash_destroy(m);
    lc_destroy(c);
    return 0;
}

// Known answers of the reference's dequant unit tests (src/dflash.rs:1334-1365)
// and the Q8_0 block of run_test_dequant, on the device.
static int run_test_dequant() {
    lc_ctx *c = ctx_open();
    void *src;
    float *out;
    cudaMalloc(&src, 256);
    cudaMalloc(&out, 64 * 4);
    float h[64];
    // "BF16" branch with f16 patterns 0x3C00 -> 1.0 and 0x3E00 -> 1.5
    uint16_t bf[2] = {0x3C00, 0x3E00};
    cudaMemcpy(src, bf, 4, cudaMemcpyHostToDevice);
    CHECK(lc_dequant(c, LC_BF16, src, 4, 2, out));
    cudaMemcpy(h, out, 8, cudaMemcpyDeviceToHost);
    if (fabsf(h[0] - 1.0f) > 1e-6f || fabsf(h[1] - 1.5f) > 1e-6f) {
        fprintf(stderr, "test-dequant: bf16 mismatch %g %g\n", h[0], h[1]);
        return 1;
    }
    printf("test-dequant: PASS (bf16, 2 elements)\n");
    unsigned char q8[34] = {0};
    q8[0] = 0x00;
    q8[1] = 0x3C;  // d = 1.0
    for (int i = 0; i < 32; i++) q8[2 + i] = 1;
    cudaMemcpy(src, q8, 34, cudaMemcpyHostToDevice);
    CHECK(lc_dequant(c, LC_Q8_0, src, 34, 32, out));
    cudaMemcpy(h, out, 32 * 4, cudaMemcpyDeviceToHost);
    for (int i = 0; i < 32; i++)
        if (fabsf(h[i] - 1.0f) > 1e-3f) {
            fprintf(stderr, "test-dequant: q8_0 mismatch at %d: %g\n", i, h[i]);
            return 1;
        }
    printf("test-dequant: PASS (q8_0, 32 elements)\n");
    lc_destroy(c);
    return 0;
}

static int run_test_matmul() {
    lc_ctx *c = ctx_open();
    float a[8], b[24], r[3];
    for (int i = 0; i < 8; i++) a[i] = i * 0.1f;
    for (int i = 0; i < 24; i++) b[i] = i * 0.01f;
    float *da, *db, *dc;
    cudaMalloc(&da, 32);
    cudaMalloc(&db, 96);
    cudaMalloc(&dc, 12);
    cudaMemcpy(da, a, 32, cudaMemcpyHostToDevice);
    cudaMemcpy(db, b, 96, cudaMemcpyHostToDevice);
    CHECK(lc_proj_f32(c, da, db, dc, 8, 3, 0));
    cudaMemcpy(r, dc, 12, cudaMemcpyDeviceToHost);
    for (int j = 0; j < 3; j++) {
        float e = 0;
        for (int i = 0; i < 8; i++) e += a[i] * b[j * 8 + i];
        if (fabsf(r[j] - e) > 1e-4f) {
            fprintf(stderr, "matmul mismatch at %d: %g vs %g\n", j, r[j], e);
            return 1;
        }
    }
    printf("test-matmul: PASS (8x3, 3 outputs)\n");
    lc_destroy(c);
    return 0;
}

static int run_test_rmsnorm() {
    lc_ctx *c = ctx_open();
    float x[4], w[4] = {0.5f, 1.0f, 1.5f, 2.0f}, y[4];
    for (int i = 0; i < 4; i++) x[i] = (i + 1.0f) * 0.5f;
    float *dx, *dw, *dy;
    cudaMalloc(&dx, 16);
    cudaMalloc(&dw, 16);
    cudaMalloc(&dy, 16);
    cudaMemcpy(dx, x, 16, cudaMemcpyHostToDevice);
    cudaMemcpy(dw, w, 16, cudaMemcpyHostToDevice);
    CHECK(lc_rmsnorm(c, dw, dx, dy, 1, 4, 1e-5f));
    cudaMemcpy(y, dy, 16, cudaMemcpyDeviceToHost);
    float ms = 0;
    for (int i = 0; i < 4; i++) ms += x[i] * x[i];
    ms /= 4;
    const float nf = 1.0f / sqrtf(ms + 1e-5f);
    for (int i = 0; i < 4; i++)
        if (fabsf(y[i] - x[i] * nf * w[i]) > 1e-4f) {
            fprintf(stderr, "rmsnorm mismatch at %d\n", i);
            return 1;
        }
    printf("test-rmsnorm: PASS (4 elements)\n");
    lc_destroy(c);
    return 0;
}

static int run_draft(const char *path, uint32_t n_ctx, uint32_t mt) {
    lc_ctx *c = ctx_open();
    CHECK(lc_set_sync(c, 0));
    lc_dflash *m;
    CHECK(lc_dflash_load_gguf(c, path, n_ctx, mt, &m));
    lc_dflash_hparams hp;
    CHECK(lc_dflash_get_hparams(m, &hp));
    const size_t in = (size_t)hp.n_aux * hp.n_embd;
    std::vector<float> feats((size_t)n_ctx * in), toks((size_t)mt * hp.n_embd);
    for (size_t i = 0; i < feats.size(); i++) feats[i] = sinf(i * 0.01f) * 0.1f;  // examples/test_encode.rs:8-10
    for (size_t i = 0; i < toks.size(); i++) toks[i] = cosf(i * 0.013f) * 0.05f;
    float *df, *de, *dx, *dh;
    cudaMalloc(&df, feats.size() * 4);
    cudaMalloc(&de, (size_t)n_ctx * hp.n_embd * 4);
    cudaMalloc(&dx, toks.size() * 4);
    cudaMalloc(&dh, toks.size() * 4);
    cudaMemcpy(df, feats.data(), feats.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dx, toks.data(), toks.size() * 4, cudaMemcpyHostToDevice);
    CHECK(lc_dflash_encode(m, df, n_ctx, de));
    CHECK(lc_dflash_set_context(m, de, n_ctx));
    CHECK(lc_dflash_decode_block(m, dx, mt, dh));
    CHECK(lc_synchronize(c));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaStream_t st = (cudaStream_t)lc_get_stream(c);
    const int iters = 20;
    cudaEventRecord(e0, st);
    for (int i = 0; i < iters; i++) CHECK(lc_dflash_decode_block(m, dx, mt, dh));
    cudaEventRecord(e1, st);
    CHECK(lc_synchronize(c));
    float ms;
    cudaEventElapsedTime(&ms, e0, e1);
    std::vector<float> h(toks.size());
    cudaMemcpy(h.data(), dh, h.size() * 4, cudaMemcpyDeviceToHost);
    double s = 0, mx = 0;
    bool finite = true;
    for (float v : h) {
        s += v * v;
        mx = fmax(mx, fabs(v));
        finite = finite && isfinite(v);
    }
    printf("draft: ctx %u, block %u: hidden rms %.6g max %.6g finite %d; %.3f ms per block forward (%.1f fwd/s)\n",
           n_ctx, mt, sqrt(s / h.size()), mx, (int)finite, ms / iters, 1000.0 * iters / ms);
    lc_dflash_destroy(m);
    lc_destroy(c);
    return finite ? 0 : 1;
}

// ---- target model (src/lib.rs:257-560) ---------------------------------------

// Device buffers of the target commands; freed at exit.
template <typename T>
static T *dev_alloc(size_t n) {
    void *p = nullptr;
    if (cudaMalloc(&p, (n ? n : 1) * sizeof(T)) != cudaSuccess) {
        fprintf(stderr, "cudaMalloc failed\n");
        exit(1);
    }
    return (T *)p;
}

template <typename T>
static std::vector<T> to_host(const T *d, size_t n) {
    std::vector<T> h(n);
    if (cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost) != cudaSuccess) {
        fprintf(stderr, "cudaMemcpy failed\n");
        exit(1);
    }
    return h;
}

static lc_target *target_open(lc_ctx *c, const char *path, uint32_t max_ctx, uint32_t max_block) {
    lc_target *t;
    CHECK(lc_target_load_gguf(c, path, max_ctx, max_block, 0, &t));
    return t;
}

static std::vector<int64_t> gguf_target_layers(const char *path) {
    lc_gguf *g;
    CHECK(lc_gguf_open(path, &g));
    uint32_t n = 0;
    CHECK(lc_gguf_target_layers(g, nullptr, 0, &n));
    std::vector<int64_t> v(n);
    if (n) CHECK(lc_gguf_target_layers(g, v.data(), n, &n));
    lc_gguf_close(g);
    return v;
}

static void print_list(const char *label, const std::vector<int64_t> &v) {
    printf("%s[", label);
    for (size_t i = 0; i < v.size(); i++) printf(i ? ", %lld" : "%lld", (long long)v[i]);
    printf("]\n");
}

// An f32 as Rust's Display writes it: the fewest significant digits that read
// back as the same f32, in plain decimal notation (no exponent).
static std::string rust_f32(float v) {
    if (std::isnan(v)) return "NaN";
    if (std::isinf(v)) return v < 0 ? "-inf" : "inf";
    if (v == 0) return std::signbit(v) ? "-0" : "0";
    char b[64];
    for (int p = 0; p < 9; p++) {
        snprintf(b, sizeof b, "%.*e", p, (double)v);
        if (strtof(b, nullptr) == v) break;
    }
    std::string s(b), digits;
    const bool neg = s[0] == '-';
    if (neg) s.erase(0, 1);
    const size_t e = s.find('e');
    for (size_t i = 0; i < e; i++)
        if (s[i] != '.') digits += s[i];
    const int point = atoi(s.c_str() + e + 1) + 1;  // digits left of the decimal point
    std::string out;
    if (point <= 0) out = "0." + std::string(-point, '0') + digits;
    else if (point >= (int)digits.size()) out = digits + std::string(point - digits.size(), '0');
    else out = digits.substr(0, point) + "." + digits.substr(point);
    return neg ? "-" + out : out;
}

static void print_logit(size_t i, float v) { printf("  logit[%zu] = %s\n", i, rust_f32(v).c_str()); }

// The n largest logits, in the order of a stable descending sort (equal
// values keep index order), as the reference prints them.
static void print_top(const std::vector<float> &lg, int n) {
    std::vector<int> idx(lg.size());
    for (size_t i = 0; i < idx.size(); i++) idx[i] = (int)i;
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return lg[a] > lg[b]; });
    for (int i = 0; i < n && i < (int)idx.size(); i++) print_logit(idx[i], lg[idx[i]]);
}

// The argmax of a row (the last maximum), lib.rs:456-464.
static uint32_t key_token(const uint64_t *keys_dev) {
    return lc_key_index(to_host(keys_dev, 1)[0]);
}

static int run_target_info(const char *path) {
    lc_ctx *c = ctx_open();
    lc_target *t = target_open(c, path, 1, 1);
    lc_target_hparams h;
    CHECK(lc_target_get_hparams(t, &h));
    printf("Target Model Info:\n");
    printf("  layers: %u\n  embedding_length: %u\n  ffn_length: %u\n  head_count: %u\n  head_count_kv: %u\n",
           h.n_layers, h.n_embd, h.n_ff, h.n_heads, h.n_kv_heads);
    printf("  head_dim: %u\n  rope_dim: %u\n  rope_dim_swa: %u\n", h.head_dim, h.rope_dim, h.rope_dim_swa);
    printf("  expert_count: %u\n  expert_used_count: %u\n  expert_ffn_length: %u\n  shared_ffn_length: %u\n",
           h.n_expert, h.n_expert_used, h.n_ff_exp, h.n_ff_shexp);
    printf("  has_moe: %s\n  has_shexp: %s\n  vocab_size: %u\n", h.has_moe ? "true" : "false",
           h.has_shexp ? "true" : "false", h.n_vocab);
    print_list("  target_layers: ", gguf_target_layers(path));
    for (uint32_t l = 0; l < h.n_layers; l++) {
        uint32_t moe;
        CHECK(lc_target_layer_info(t, l, &moe, nullptr));
        printf("  layer %u [%s]\n", l, moe ? "MoE" : "Dense");
    }
    lc_target_destroy(t);
    lc_destroy(c);
    return 0;
}

// target-forward: forward_token of the token's embedding, every layer's input
// captured (run_target_forward, lib.rs:284-331).
static int run_target_forward(const char *path, uint32_t tok) {
    lc_ctx *c = ctx_open();
    lc_target *t = target_open(c, path, 1, 1);
    lc_target_hparams h;
    CHECK(lc_target_get_hparams(t, &h));
    const uint32_t E = h.n_embd, V = h.n_vocab ? h.n_vocab : E;
    const void *emb_w;
    const bool has_emb = lc_target_weight(t, "token_embd.weight", &emb_w, nullptr, nullptr) == LC_OK;
    float *x = dev_alloc<float>(E), *cap = dev_alloc<float>((size_t)h.n_layers * E);
    float *logits = dev_alloc<float>(std::max(V, E));
    if (has_emb) {
        if (tok >= h.n_vocab) {
            fprintf(stderr, "token_id %u >= vocab_size %u\n", tok, h.n_vocab);
            return 1;
        }
        CHECK(lc_target_embed(t, &tok, 1, x));
        printf("Running target model forward pass with token_id=%u\n", tok);
    } else {
        std::vector<float> d(E, 0.1f);
        cudaMemcpy(x, d.data(), E * 4, cudaMemcpyHostToDevice);
    }
    std::vector<uint32_t> layers(h.n_layers);
    for (uint32_t l = 0; l < h.n_layers; l++) layers[l] = l;
    CHECK(lc_target_forward(t, x, 1, 0, layers.data(), h.n_layers, cap, nullptr, logits, nullptr));
    const uint32_t n_logits = lc_target_weight(t, "output.weight", &emb_w, nullptr, nullptr) == LC_OK ? V : E;
    std::vector<float> lg = to_host(logits, n_logits);
    printf("Forward pass complete: %u logits, %u captured states\n", n_logits, h.n_layers);
    if (has_emb) {
        printf("Top logits:\n");
        print_top(lg, 10);
        printf("Specific indices:\n");
    }
    for (uint32_t i = 0; i < 10 && i < n_logits; i++) print_logit(i, lg[i]);
    lc_target_destroy(t);
    lc_destroy(c);
    return 0;
}

// target-generate: greedy tokens through the K/V cache (run_target_generate,
// lib.rs:335-380).
static int run_target_generate(const char *path, uint32_t start, uint32_t n) {
    lc_ctx *c = ctx_open();
    lc_target *t = target_open(c, path, n + 1, 1);
    lc_target_hparams h;
    CHECK(lc_target_get_hparams(t, &h));
    const void *w;
    if (lc_target_weight(t, "token_embd.weight", &w, nullptr, nullptr) != LC_OK) {
        fprintf(stderr, "model has no token embeddings; cannot generate\n");
        return 1;
    }
    float *x = dev_alloc<float>(h.n_embd);
    uint64_t *keys = dev_alloc<uint64_t>(1);
    std::vector<int64_t> out;
    uint32_t cur = start;
    printf("Generating %u tokens from start_token=%u\n", n, start);
    for (uint32_t step = 0; step < n; step++) {
        if (cur >= h.n_vocab) {
            fprintf(stderr, "token %u out of range\n", cur);
            break;
        }
        CHECK(lc_target_embed(t, &cur, 1, x));
        CHECK(lc_target_forward(t, x, 1, LC_TARGET_CACHED, nullptr, 0, nullptr, nullptr, nullptr, keys));
        const uint32_t next = key_token(keys);
        printf("  step %u: input=%u -> next=%u\n", step, cur, next);
        out.push_back(next);
        cur = next;
    }
    print_list("Generated tokens: ", out);
    lc_target_destroy(t);
    lc_destroy(c);
    return 0;
}

// One draft step of the verify loops: the target's forward_token with the
// draft's target layers captured, the draft's forward_injected_decode_hidden,
// the target's lm_head on the draft's hidden state (lib.rs:404-426, :486-496).
struct DraftPair {
    lc_ctx *c;
    lc_target *t;
    lc_dflash *d;
    lc_target_hparams h;
    std::vector<int64_t> draft_layers;  // as the draft lists them
    std::vector<uint32_t> layers;       // captured: sorted, distinct
    const void *out_w = nullptr;
    int out_dt = 0;
    float *x, *cap, *enc, *dh, *logits;
    uint64_t *keys;
};

static DraftPair pair_open(const char *tpath, const char *dpath) {
    DraftPair p;
    p.c = ctx_open();
    p.t = target_open(p.c, tpath, 1, 1);
    CHECK(lc_target_get_hparams(p.t, &p.h));
    CHECK(lc_dflash_load_gguf(p.c, dpath, 1, 1, &p.d));
    // forward_token captures the layers in layer order, each once, and the
    // final state for index n_layers (src/target.rs:398-407, :550-551).
    p.draft_layers = gguf_target_layers(dpath);
    for (int64_t v : p.draft_layers)
        if (v >= 0 && v <= p.h.n_layers) p.layers.push_back((uint32_t)v);
    std::sort(p.layers.begin(), p.layers.end());
    p.layers.erase(std::unique(p.layers.begin(), p.layers.end()), p.layers.end());
    lc_dflash_hparams dh;
    CHECK(lc_dflash_get_hparams(p.d, &dh));
    if (dh.n_embd != p.h.n_embd || dh.n_aux != p.layers.size()) {
        fprintf(stderr, "draft (n_embd %u, %u target layers) does not fit the target (n_embd %u, %zu capture layers)\n",
                dh.n_embd, dh.n_aux, p.h.n_embd, p.layers.size());
        exit(1);
    }
    CHECK(lc_target_weight(p.t, "output.weight", &p.out_w, &p.out_dt, nullptr));
    const uint32_t E = p.h.n_embd, n = (uint32_t)p.layers.size();
    p.x = dev_alloc<float>(E), p.cap = dev_alloc<float>((size_t)(n ? n : 1) * E), p.enc = dev_alloc<float>(E);
    p.dh = dev_alloc<float>(E), p.logits = dev_alloc<float>(p.h.n_vocab), p.keys = dev_alloc<uint64_t>(2);
    return p;
}

// Returns (target token, draft token); the draft's logits stay in p.logits.
static void pair_step(DraftPair &p, uint32_t tok, uint32_t *target_tok, uint32_t *draft_tok) {
    const uint32_t E = p.h.n_embd, n = (uint32_t)p.layers.size();
    CHECK(lc_target_embed(p.t, &tok, 1, p.x));
    CHECK(lc_target_forward(p.t, p.x, 1, 0, p.layers.data(), n, p.cap, nullptr, nullptr, p.keys));
    CHECK(lc_dflash_encode(p.d, p.cap, 1, p.enc));
    CHECK(lc_dflash_set_context(p.d, p.enc, 1));
    CHECK(lc_dflash_decode_block(p.d, p.x, 1, p.dh));
    CHECK(lc_lm_head_argmax(p.c, p.out_dt, p.dh, p.out_w, 1, E, p.h.n_vocab, 0, p.keys + 1, p.logits));
    std::vector<uint64_t> k = to_host(p.keys, 2);
    *target_tok = lc_key_index(k[0]);
    *draft_tok = lc_key_index(k[1]);
}

// target-dflash: one draft step, the draft's logits (run_target_dflash,
// lib.rs:384-429).
static int run_target_dflash(const char *tpath, const char *dpath, uint32_t tok) {
    DraftPair p = pair_open(tpath, dpath);
    if (tok >= p.h.n_vocab) {
        fprintf(stderr, "token_id %u >= vocab_size %u\n", tok, p.h.n_vocab);
        return 1;
    }
    print_list("DFlash target layers: ", p.draft_layers);
    uint32_t tt, dt;
    pair_step(p, tok, &tt, &dt);
    printf("Captured %zu states, %zu feature floats\n", p.layers.size(), p.layers.size() * p.h.n_embd);
    printf("DFlash draft logits: %u\n", p.h.n_vocab);
    printf("Top draft logits:\n");
    print_top(to_host(p.logits, p.h.n_vocab), 10);
    lc_dflash_destroy(p.d);
    lc_target_destroy(p.t);
    lc_destroy(p.c);
    return 0;
}

// target-dflash-verify: the draft / verify loop (run_target_dflash_verify,
// lib.rs:466-528).
static int run_target_dflash_verify(const char *tpath, const char *dpath, uint32_t tok, uint32_t steps) {
    DraftPair p = pair_open(tpath, dpath);
    std::vector<int64_t> accepted;
    print_list("DFlash target layers: ", p.draft_layers);
    uint32_t exact = 0;
    for (uint32_t s = 0; s < steps; s++) {
        if (tok >= p.h.n_vocab) {
            fprintf(stderr, "token_id %u >= vocab_size %u\n", tok, p.h.n_vocab);
            return 1;
        }
        uint32_t tt, dt;
        pair_step(p, tok, &tt, &dt);
        const bool ok = dt == tt;
        exact += ok;
        const uint32_t next = ok ? dt : tt;
        accepted.push_back(next);
        printf("step %u: input=%u draft=%u target=%u %s -> accepted=%u\n", s, tok, dt, tt, ok ? "ACCEPT" : "REJECT",
               next);
        tok = next;
    }
    print_list("accepted tokens: ", accepted);
    printf("exact draft accept rate: %u/%u\n", exact, steps);
    lc_dflash_destroy(p.d);
    lc_target_destroy(p.t);
    lc_destroy(p.c);
    return 0;
}

// project-ref: the lm_head on a hidden state read from a file of n_embd f32
// (run_project_ref, lib.rs:530-556).
static int run_project_ref(const char *path, const char *hidden_path) {
    lc_ctx *c = ctx_open();
    lc_target *t = target_open(c, path, 1, 1);
    lc_target_hparams h;
    CHECK(lc_target_get_hparams(t, &h));
    std::vector<float> hid(h.n_embd);
    FILE *f = fopen(hidden_path, "rb");
    if (!f || fread(hid.data(), 4, h.n_embd, f) != h.n_embd || fgetc(f) != EOF) {
        fprintf(stderr, "%s: expected %u f32 values\n", hidden_path, h.n_embd);
        return 1;
    }
    fclose(f);
    const void *w;
    int dt;
    CHECK(lc_target_weight(t, "output.weight", &w, &dt, nullptr));
    float *x = dev_alloc<float>(h.n_embd), *logits = dev_alloc<float>(h.n_vocab);
    uint64_t *keys = dev_alloc<uint64_t>(1);
    cudaMemcpy(x, hid.data(), h.n_embd * 4, cudaMemcpyHostToDevice);
    CHECK(lc_lm_head_argmax(c, dt, x, w, 1, h.n_embd, h.n_vocab, 0, keys, logits));
    std::vector<float> lg = to_host(logits, h.n_vocab);
    printf("Top logits:\n");
    print_top(lg, 10);
    printf("Specific indices:\n");
    for (uint32_t i = 0; i < 8 && i < h.n_vocab; i++) print_logit(i, lg[i]);
    lc_target_destroy(t);
    lc_destroy(c);
    return 0;
}

int main(int argc, char **argv) {
    if (argc < 2) {
        fprintf(stderr,
                "usage: %s <command> [args...]\ncommands:\n"
                "  info <gguf_path>          - show model metadata\n"
                "  shapes <gguf_path>        - show tensor shapes\n"
                "  forward <gguf_path> <tok> - run forward pass\n"
                "  encode <gguf_path>        - encode + decode with zero features\n"
                "  draft <gguf_path> [ctx] [block] - block draft forward\n"
                "  test-dequant              - test dequantization\n"
                "  test-matmul               - test matmul on GPU\n"
                "  test-rmsnorm              - test rmsnorm on GPU\n"
                "  target-info <gguf>        - show target model metadata\n"
                "  target-forward <gguf> [tok] - target forward pass\n"
                "  target-generate <gguf> [start] [n] - greedy cached generation\n"
                "  target-dflash <target> <dflash> [tok] - one DFlash draft step\n"
                "  target-dflash-verify <target> <dflash> [tok] [n] - draft/verify loop\n"
                "  project-ref <gguf> <hidden_f32_file> - lm_head of a hidden state\n",
                argv[0]);
        return 1;
    }
    const char *cmd = argv[1];
    auto arg = [&](int i) -> const char * {
        if (i >= argc) {
            fprintf(stderr, "%s: missing argument\n", cmd);
            exit(1);
        }
        return argv[i];
    };
    if (!strcmp(cmd, "info")) return run_info(arg(2), false);
    if (!strcmp(cmd, "shapes")) return run_info(arg(2), true);
    if (!strcmp(cmd, "forward")) return run_forward(arg(2), argc > 3 ? (uint32_t)atoi(argv[3]) : 0, false);
    if (!strcmp(cmd, "encode")) return run_forward(arg(2), 0, true);
    if (!strcmp(cmd, "draft"))
        return run_draft(arg(2), argc > 3 ? (uint32_t)atoi(argv[3]) : 2048, argc > 4 ? (uint32_t)atoi(argv[4]) : 16);
    if (!strcmp(cmd, "test-dequant")) return run_test_dequant();
    if (!strcmp(cmd, "test-matmul")) return run_test_matmul();
    if (!strcmp(cmd, "test-rmsnorm")) return run_test_rmsnorm();
    auto num = [&](int i, uint32_t dflt) { return argc > i ? (uint32_t)strtoul(argv[i], nullptr, 10) : dflt; };
    if (!strcmp(cmd, "target-info")) return run_target_info(arg(2));
    if (!strcmp(cmd, "target-forward")) return run_target_forward(arg(2), num(3, 0));
    if (!strcmp(cmd, "target-generate")) return run_target_generate(arg(2), num(3, 0), num(4, 16));
    if (!strcmp(cmd, "target-dflash")) return run_target_dflash(arg(2), arg(3), num(4, 0));
    if (!strcmp(cmd, "target-dflash-verify")) return run_target_dflash_verify(arg(2), arg(3), num(4, 0), num(5, 4));
    if (!strcmp(cmd, "project-ref")) return run_project_ref(arg(2), arg(3));
    fprintf(stderr, "unknown command: %s\n", cmd);
    return 1;
}
