// lc_runtime.cu -- context, buffers, errors: the part of the C ABI that
// replaces the reference's VulkanContext / GpuBuffer (src/vulkan.rs).
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>

#include <stdlib.h>

#include "lc_internal.cuh"
#include "lc_sm100.cuh"

static thread_local char g_err[1024] = "";

int lc_fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

extern "C" const char *lc_last_error(void) { return g_err; }

extern "C" const char *lc_version(void) { return "laguna-cuda 0.1 (sm_100a)"; }

extern "C" int lc_device_count(int *count) {
    LC_REQUIRE(count, LC_ERR_INVALID, "lc_device_count: null out");
    LC_CUDA(cudaGetDeviceCount(count));
    return LC_OK;
}

int lc_use_device(lc_ctx *ctx) {
    int cur = -1;
    LC_CUDA(cudaGetDevice(&cur));
    if (cur != ctx->device) LC_CUDA(cudaSetDevice(ctx->device));
    return LC_OK;
}

extern "C" int lc_init(int device, lc_ctx **out) {
    LC_REQUIRE(out, LC_ERR_INVALID, "lc_init: null out");
    *out = nullptr;
    int n = 0;
    LC_CUDA(cudaGetDeviceCount(&n));
    LC_REQUIRE(device >= 0 && device < n, LC_ERR_INVALID, "lc_init: device %d out of range (%d devices)", device, n);
    LC_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    LC_CUDA(cudaGetDeviceProperties(&prop, device));
    LC_REQUIRE(prop.major == 10 && prop.minor == 0, LC_ERR_UNSUPPORTED,
               "lc_init: device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
               prop.minor);
    lc_ctx *ctx = new lc_ctx();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    ctx->smem_optin = prop.sharedMemPerBlockOptin;
    if (const char *e = getenv("LC_GEMM_TC")) ctx->gemm_tc = e[0] != '0';
    if (const char *e = getenv("LC_GEMV_I8_MIN")) ctx->gemv_i8_min = atoi(e) < 1 ? 1 : atoi(e);
    if (const char *e = getenv("LC_GEMV_I8_MAX")) ctx->gemv_i8_max = atoi(e) < 0 ? 0 : atoi(e) > 16 ? 16 : atoi(e);
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return lc_fail(LC_ERR_CUDA, "lc_init: cudaStreamCreate: %s", cudaGetErrorString(e));
    }
    ctx->stream = ctx->own_stream;
    e = cudaMalloc((void **)&ctx->dev_status, 256);
    if (e == cudaSuccess) e = cudaMemset(ctx->dev_status, 0, 256);
    if (e != cudaSuccess) {
        if (ctx->dev_status) cudaFree(ctx->dev_status);
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return lc_fail(LC_ERR_CUDA, "lc_init: status word: %s", cudaGetErrorString(e));
    }
    const int sp = lc_static_pack_resolve(ctx);
    if (sp) {
        cudaFree(ctx->dev_status);
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return sp;
    }
    *out = ctx;
    return LC_OK;
}

extern "C" int lc_ctx_scratch_bytes(lc_ctx *ctx, size_t *bytes) {
    LC_REQUIRE(ctx && bytes, LC_ERR_INVALID, "lc_ctx_scratch_bytes: null argument");
    size_t t = 0;
    for (int i = 0; i < LC_SCRATCH_COUNT; i++) t += ctx->scratch_bytes[i];
    *bytes = t;
    return LC_OK;
}

extern "C" int lc_device_status(lc_ctx *ctx) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_device_status: null ctx");
    int s = lc_use_device(ctx);
    if (s) return s;
    unsigned v = 0;
    LC_CUDA(cudaMemcpyAsync(&v, ctx->dev_status, sizeof(v), cudaMemcpyDeviceToHost, ctx->stream));
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    if (!v) return LC_OK;
    LC_CUDA(cudaMemsetAsync(ctx->dev_status, 0, sizeof(v), ctx->stream));
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    return lc_fail(LC_ERR_TIMEOUT, "a bounded device-side wait expired (status 0x%x); results of that launch are invalid",
                   v);
}

extern "C" int lc_destroy(lc_ctx *ctx) {
    if (!ctx) return LC_OK;
    lc_use_device(ctx);
    if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
    if (ctx->stream && ctx->stream != ctx->own_stream) cudaStreamSynchronize(ctx->stream);
    for (int i = 0; i < LC_SCRATCH_COUNT; i++)
        if (ctx->scratch[i]) cudaFree(ctx->scratch[i]);
    if (ctx->dev_status) cudaFree(ctx->dev_status);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return LC_OK;
}

extern "C" int lc_set_stream(lc_ctx *ctx, void *stream) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_set_stream: null ctx");
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return LC_OK;
}

extern "C" void *lc_get_stream(lc_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

extern "C" int lc_synchronize(lc_ctx *ctx) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_synchronize: null ctx");
    int s = lc_use_device(ctx);
    if (s) return s;
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    return LC_OK;
}

extern "C" int lc_set_sync(lc_ctx *ctx, int sync) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_set_sync: null ctx");
    ctx->sync = sync ? 1 : 0;
    return LC_OK;
}

extern "C" int lc_set_half_mode(lc_ctx *ctx, int mode) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_set_half_mode: null ctx");
    LC_REQUIRE(mode == LC_HALF_REF || mode == LC_HALF_IEEE, LC_ERR_INVALID, "lc_set_half_mode: bad mode %d", mode);
    ctx->half_mode = mode;
    return LC_OK;
}

extern "C" int lc_ctx_device(lc_ctx *ctx, int *device) {
    LC_REQUIRE(ctx && device, LC_ERR_INVALID, "lc_ctx_device: null argument");
    *device = ctx->device;
    return LC_OK;
}

int lc_set_smem_attr(const void *kernel, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, size_t> done;
    int dev = 0;
    LC_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    size_t &have = done[{dev, kernel}];
    if (have >= bytes) return LC_OK;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return lc_fail(LC_ERR_CUDA, "cudaFuncSetAttribute(%zu): %s", bytes, cudaGetErrorString(e));
    have = bytes;
    return LC_OK;
}

int lc_after_launch(lc_ctx *ctx, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return lc_fail(LC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    if (ctx->sync) {
        e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return lc_fail(LC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
        return lc_device_status(ctx);
    }
    return LC_OK;
}

void *lc_scratch(lc_ctx *ctx, int slot, size_t bytes) {
    if (bytes <= ctx->scratch_bytes[slot]) return ctx->scratch[slot];
    size_t want = (bytes + 255) & ~(size_t)255;
    if (want < ((size_t)1 << 20)) want = (size_t)1 << 20;
    if (ctx->scratch[slot]) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            lc_fail(LC_ERR_CUDA, "scratch: %s", cudaGetErrorString(e));
            return nullptr;
        }
        cudaFree(ctx->scratch[slot]);
        ctx->scratch[slot] = nullptr;
        ctx->scratch_bytes[slot] = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->scratch[slot], want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        lc_fail(LC_ERR_OOM, "scratch: cudaMalloc(%zu): %s", want, cudaGetErrorString(e));
        ctx->scratch[slot] = nullptr;
        return nullptr;
    }
    ctx->scratch_bytes[slot] = want;
    return ctx->scratch[slot];
}

void *lc_scratch_zeroed(lc_ctx *ctx, int slot, size_t bytes) {
    const bool grow = bytes > ctx->scratch_bytes[slot];
    void *p = lc_scratch(ctx, slot, bytes);
    if (p && grow) {
        cudaError_t e = cudaMemsetAsync(p, 0, ctx->scratch_bytes[slot], ctx->stream);
        if (e != cudaSuccess) {
            lc_fail(LC_ERR_CUDA, "scratch memset: %s", cudaGetErrorString(e));
            return nullptr;
        }
    }
    return p;
}

// ---- buffers ---------------------------------------------------------------

extern "C" int lc_buf_alloc(lc_ctx *ctx, size_t bytes, lc_buf **out) {
    LC_REQUIRE(ctx && out, LC_ERR_INVALID, "lc_buf_alloc: null argument");
    *out = nullptr;
    int s = lc_use_device(ctx);
    if (s) return s;
    lc_buf *b = new lc_buf();
    b->ctx = ctx;
    b->size = bytes;
    if (bytes) {
        cudaError_t e = cudaMalloc(&b->ptr, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            delete b;
            return lc_fail(LC_ERR_OOM, "lc_buf_alloc(%zu): %s", bytes, cudaGetErrorString(e));
        }
        e = cudaMemsetAsync(b->ptr, 0, bytes, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            cudaFree(b->ptr);
            delete b;
            return lc_fail(LC_ERR_CUDA, "lc_buf_alloc: memset: %s", cudaGetErrorString(e));
        }
    }
    *out = b;
    return LC_OK;
}

extern "C" int lc_buf_free(lc_buf *b) {
    if (!b) return LC_OK;
    if (b->ptr) {
        lc_use_device(b->ctx);
        cudaStreamSynchronize(b->ctx->stream);
        cudaFree(b->ptr);
    }
    delete b;
    return LC_OK;
}

extern "C" void *lc_buf_device_ptr(const lc_buf *b) { return b ? b->ptr : nullptr; }

extern "C" size_t lc_buf_size(const lc_buf *b) { return b ? b->size : 0; }

extern "C" int lc_buf_upload_at(lc_buf *b, size_t offset, const void *src, size_t bytes) {
    LC_REQUIRE(b && (src || !bytes), LC_ERR_INVALID, "lc_buf_upload: null argument");
    LC_REQUIRE(offset <= b->size && bytes <= b->size - offset, LC_ERR_INVALID,
               "lc_buf_upload: %zu bytes at offset %zu exceed buffer of %zu", bytes, offset, b->size);
    if (!bytes) return LC_OK;
    int s = lc_use_device(b->ctx);
    if (s) return s;
    LC_CUDA(cudaMemcpyAsync((char *)b->ptr + offset, src, bytes, cudaMemcpyHostToDevice, b->ctx->stream));
    LC_CUDA(cudaStreamSynchronize(b->ctx->stream));
    return LC_OK;
}

extern "C" int lc_buf_upload(lc_buf *b, const void *src, size_t bytes) { return lc_buf_upload_at(b, 0, src, bytes); }

extern "C" int lc_buf_read(lc_buf *b, size_t offset, void *dst, size_t bytes) {
    LC_REQUIRE(b && (dst || !bytes), LC_ERR_INVALID, "lc_buf_read: null argument");
    LC_REQUIRE(offset <= b->size && bytes <= b->size - offset, LC_ERR_INVALID,
               "lc_buf_read: %zu bytes at offset %zu exceed buffer of %zu", bytes, offset, b->size);
    if (!bytes) return LC_OK;
    int s = lc_use_device(b->ctx);
    if (s) return s;
    LC_CUDA(cudaMemcpyAsync(dst, (const char *)b->ptr + offset, bytes, cudaMemcpyDeviceToHost, b->ctx->stream));
    LC_CUDA(cudaStreamSynchronize(b->ctx->stream));
    return LC_OK;
}

extern "C" int lc_buf_read_f32(lc_buf *b, float *dst, size_t n) {
    LC_REQUIRE(n <= ((size_t)-1) / 4, LC_ERR_INVALID, "lc_buf_read_f32: n too large");
    return lc_buf_read(b, 0, dst, n * 4);
}

// ---- keys -------------------------------------------------------------------

extern "C" uint64_t lc_pack_key(float value, uint32_t index) { return lc_make_key(value, index); }

extern "C" float lc_key_value(uint64_t key) {
    uint32_t o = (uint32_t)((key ^ 0x8000000000000000ull) >> 32);
    uint32_t b = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

extern "C" uint32_t lc_key_index(uint64_t key) { return (uint32_t)(key & 0xFFFFFFFFull); }

extern "C" int lc_rope_freq(float *freq, uint32_t rope_dim, float base) {
    LC_REQUIRE(freq || rope_dim < 2, LC_ERR_INVALID, "lc_rope_freq: null out");
    for (uint32_t i = 0; i < rope_dim / 2; i++)
        freq[i] = 1.0f / powf(base, (2.0f * (float)i) / (float)rope_dim);
    return LC_OK;
}

// One CTA waits on a barrier that nobody arrives on, with a bound of `spins`
// polls, and records the expiry like every bounded wait of the library.
__global__ void bounded_wait_check_kernel(unsigned *status, uint32_t spins) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
    }
    __syncthreads();
    bool ok = false;
    for (uint32_t i = 0; i < spins && !ok; ++i) ok = mbar_test(&bar, 0u);
    if (!ok && threadIdx.x == 0) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
}

extern "C" int lc_check_bounded_wait(lc_ctx *ctx, uint32_t spins) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_check_bounded_wait: null ctx");
    LC_REQUIRE(spins > 0 && spins <= (1u << 20), LC_ERR_INVALID, "lc_check_bounded_wait: spins %u not in 1..2^20",
               spins);
    int s = lc_use_device(ctx);
    if (s) return s;
    bounded_wait_check_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_status, spins);
    return lc_after_launch(ctx, "lc_check_bounded_wait");
}
