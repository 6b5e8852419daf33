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
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

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
                "  test-rmsnorm              - test rmsnorm on GPU\n",
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
    fprintf(stderr, "unknown command: %s\n", cmd);
    return 1;
}
