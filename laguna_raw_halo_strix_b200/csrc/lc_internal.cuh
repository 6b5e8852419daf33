// lc_internal.cuh -- shared declarations of the CUDA backend (not installed).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <functional>
#include <vector>

#include "laguna_cuda.h"

// Context: one device, one stream, one grow-only scratch arena.
struct lc_ctx {
    int device = 0;
    int num_sms = 148;
    size_t smem_optin = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int sync = 0;
    int half_mode = LC_HALF_REF;
    // 1: 5..32-token Q4_K / Q8_0 projections run the tcgen05 GEMM (lc_gemm.cu);
    // 0: the mma.sync tiled kernels.  Set from LC_GEMM_TC at lc_init (default 1).
    int gemm_tc = 1;
    // Token counts sent to the int8 tcgen05 GEMV: gemv_i8_min..gemv_i8_max
    // (LC_GEMV_I8_MIN, default 3; LC_GEMV_I8_MAX, default 8, at most 16).
    int gemv_i8_min = 3;
    int gemv_i8_max = 8;
    // Grow-only scratch slots (see LC_SCRATCH_*).
    void *scratch[8] = {};
    size_t scratch_bytes[8] = {};
    // Device word that kernels set (atomicOr of LC_DEV_*) when a bounded wait
    // gives up; read and cleared by lc_device_status().  Allocated at init.
    unsigned *dev_status = nullptr;
    // Device address of lc_proj.cu's static scratch array on this device,
    // resolved at lc_init (lc_static_pack_resolve).
    void *static_pack = nullptr;
};

// Bits of lc_ctx::dev_status.
enum { LC_DEV_WAIT_TIMEOUT = 1u };

struct lc_buf {
    lc_ctx *ctx = nullptr;
    void *ptr = nullptr;
    size_t size = 0;
};

// Record an error message for lc_last_error() and return `code`.
int lc_fail(int code, const char *fmt, ...);
// After enqueuing kernels: check the launch, and wait if the context is sync.
int lc_after_launch(lc_ctx *ctx, const char *what);
// Scratch slots: packed activation fragments, logits of the argmax path,
// the DFlash block-forward workspace, attention partials.
// LC_SCRATCH_FIXUP holds the split-tile sums of the stream-K projections and
// must read zero between calls (the kernels leave it zeroed).
enum {
    LC_SCRATCH_PACK = 0,
    LC_SCRATCH_LOGITS = 1,
    LC_SCRATCH_MODEL = 2,
    LC_SCRATCH_ATTN = 3,
    LC_SCRATCH_FIXUP = 4,
    LC_SCRATCH_FFN = 5,
    LC_SCRATCH_HOSTIO = 6,
    LC_SCRATCH_COUNT = 8
};
// Grow-only scratch slot of at least `bytes` (256-byte aligned).  Returns
// nullptr and sets the error on failure.  Waits for the stream before
// reallocating.
void *lc_scratch(lc_ctx *ctx, int slot, size_t bytes);
// Same, and a newly allocated slot is zero-filled (on the context's stream).
void *lc_scratch_zeroed(lc_ctx *ctx, int slot, size_t bytes);
// Resolve ctx->static_pack with ctx->device current (lc_proj.cu; called by lc_init).
int lc_static_pack_resolve(lc_ctx *ctx);
// Make ctx->device current on this thread.
int lc_use_device(lc_ctx *ctx);
// Raise a kernel's dynamic shared memory limit to at least `bytes` on the
// current device; remembered per (device, kernel) so repeated calls (and calls
// made while a stream is being captured into a CUDA graph) do not touch the
// driver again.
int lc_set_smem_attr(const void *kernel, size_t bytes);

#define LC_REQUIRE(cond, code, ...)             \
    do {                                        \
        if (!(cond)) return lc_fail((code), __VA_ARGS__); \
    } while (0)

#define LC_CUDA(expr)                                                        \
    do {                                                                     \
        cudaError_t _e = (expr);                                             \
        if (_e != cudaSuccess)                                               \
            return lc_fail(_e == cudaErrorMemoryAllocation ? LC_ERR_OOM : LC_ERR_CUDA, \
                           "%s: %s", #expr, cudaGetErrorString(_e));         \
    } while (0)

// ---- device helpers -------------------------------------------------------

// f16 bits -> f32.  LC_HALF_REF keeps the implicit one on subnormals exactly
// like kernels/proj_q8_0.comp:27-45 (sign | 113<<23 | mant<<13); otherwise IEEE.
__device__ __forceinline__ float lc_half_to_f32(uint32_t h, int mode) {
    h &= 0xFFFFu;
    if (mode == LC_HALF_IEEE) return __half2float(__ushort_as_half((unsigned short)h));
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = (h & 0x3FFu) << 13;
    uint32_t ebits = (e == 0u) ? (mant ? (113u << 23) : 0u) : (e == 31u ? 0x7F800000u : (e + 112u) << 23);
    return __uint_as_float(sign | ebits | mant);
}

__device__ __forceinline__ uint32_t lc_h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 lc_u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Split a float into f16 hi + f16 lo with hi + lo == v to ~22 bits.
// part 0 -> hi, part 1 -> lo.
__device__ __forceinline__ __half lc_split_part(float v, int part) {
    __half hi = __float2half_rn(v);
    if (part == 0) return hi;
    return __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ uint32_t lc_pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Order-preserving (value, index) key; see lc_pack_key in laguna_cuda.h.
__host__ __device__ __forceinline__ uint64_t lc_make_key(float v, uint32_t idx) {
    uint32_t b;
#ifdef __CUDA_ARCH__
    b = __float_as_uint(v);
#else
    memcpy(&b, &v, 4);
#endif
    uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    uint64_t k = ((uint64_t)o << 32) | idx;
    return k ^ 0x8000000000000000ull;
}

// mma.sync m16n8k16 f16 x f16 -> f32 (row.col).
__device__ __forceinline__ void lc_mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// mma.sync m16n8k8 f16 x f16 -> f32 (row.col).
__device__ __forceinline__ void lc_mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// Element-wise functions shared by the stand-alone kernels and the fused
// activation packing: kernels/activation.comp (SiLU(g) * up) and the host
// softplus of src/dflash.rs:956-958 (log(1 + e^v), identity above 20).
__device__ __forceinline__ float lc_swiglu(float g, float up) { return g * (1.0f / (1.0f + expf(-g))) * up; }
__device__ __forceinline__ float lc_softplus_f(float v) { return v > 20.0f ? v : logf(1.0f + expf(v)); }

// Host-side launch helpers defined in the kernel files.
namespace lc {
int proj_q4k(lc_ctx *ctx, const float *x, const void *w, float *c, uint32_t m, uint32_t k, uint32_t n,
             uint32_t expert_offset);
int proj_q8_0(lc_ctx *ctx, const float *x, const void *w, float *c, uint32_t m, uint32_t k, uint32_t n);
int proj_f32(lc_ctx *ctx, const float *x, const float *w, float *c, uint32_t m, uint32_t k, uint32_t n,
             uint32_t row_major);
// tcgen05 GEMM for 5..32 tokens (lc_gemm.cu); LC_ERR_UNSUPPORTED when the
// shape is not covered.
int gemm_dq(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n);
// Projections that read one activation block: up to kGroupMax weight matrices
// of one dtype and one k in a single packing launch and a single tcgen05 GEMM
// launch (lc_gemm.cu).  The packed activation is src.x, or a function of two
// inputs applied while packing:
//   LC_PACK_SWIGLU:   x * sigmoid(x) * x2                (activation.comp)
//   LC_PACK_HEADGATE: x * softplus(x2[row * k / hd + col / hd])  (softplus, gate_mul.comp)
//   LC_PACK_RMSNORM:  (x * x2) * rsqrt(mean(x_row^2) + eps), x2 the norm weight
//                     of length k                           (rmsnorm.comp)
// Each output is y = src . W^T, or y += src . W^T when `accumulate` (the residual
// add of the decoder).  LC_ERR_UNSUPPORTED when the shape is not covered.
enum { LC_PACK_PLAIN = 0, LC_PACK_SWIGLU = 1, LC_PACK_HEADGATE = 2, LC_PACK_RMSNORM = 3 };
constexpr int kGroupMax = 4;
struct PackSrc {
    const float *x = nullptr;
    const float *x2 = nullptr;
    int op = LC_PACK_PLAIN;
    int head_dim = 0;
    float eps = 0.f;  // LC_PACK_RMSNORM
};
struct ProjOut {
    const void *w = nullptr;
    float *y = nullptr;
    uint32_t n = 0;
    bool accumulate = false;
};
int gemm_dq_group(lc_ctx *ctx, int dtype, const PackSrc &src, const ProjOut *outs, int ng, uint32_t m, uint32_t k);
// lc_qk_norm_rope of the block's Q and K in one launch where possible; row r
// is rotated at position pos0 + r * pos_step (lc_ops.cu).
int qk_norm_rope_pair(lc_ctx *ctx, const float *xa, const float *wa, float *ya, uint32_t n_heads_a, const float *xb,
                      const float *wb, float *yb, uint32_t n_heads_b, const float *freq, uint32_t m,
                      uint32_t head_dim, uint32_t rope_dim, float eps, uint32_t pos0, uint32_t pos_step = 1);
// Projections of 1 or 2 tokens with f32 activations (lc_gemv.cu): up to
// kGroupMax weight matrices of one format and one k sharing the activations
// (src.x, or SiLU(src.x) * src.x2 for LC_PACK_SWIGLU), rows streamed from HBM
// once.  LC_ERR_UNSUPPORTED when the shape is not covered (gemv_rows_covers).
bool gemv_rows_covers(const lc_ctx *ctx, int dtype, uint32_t m, uint32_t k);
int gemv_rows(lc_ctx *ctx, int dtype, const PackSrc &src, const ProjOut *outs, int ng, uint32_t m, uint32_t k);
// gate and up (n rows each) of one FFN in one gemv_rows launch, rows
// interleaved; h [m][n] = SiLU(x . gate^T) * (x . up^T) (activation.comp).
int gemv_rows_swiglu(lc_ctx *ctx, int dtype, const PackSrc &src, const void *w_gate, const void *w_up, float *h,
                     uint32_t m, uint32_t k, uint32_t n);
// lc_dequant, or with bf16_native a BF16 tensor decoded as bfloat16 (f32 =
// bits << 16) instead of the reference's f16 reading (lc_ops.cu).
int dequant_f32(lc_ctx *ctx, int dtype, const void *src, size_t src_bytes, size_t n, float *out, bool bf16_native);
// A tensor held on the device by a model: raw GGUF blocks (F32 / Q8_0 / Q4_K)
// or f32 decoded from F16 / BF16; shape is GGUF's (ne0 first).
struct DevTensor {
    void *ptr = nullptr;
    size_t bytes = 0;
    int dtype = -1;
    uint64_t n_el = 0;
    uint64_t shape[4] = {1, 1, 1, 1};
    uint32_t n_dims = 0;
};
// Upload every tensor of g for which slot(name) returns a DevTensor into one
// device allocation (appended to *allocs), through pinned staging; F16 / BF16
// are decoded to f32 (bfloat16 proper with LC_LOAD_BF16_NATIVE).  Waits for
// the copies before returning (lc_load.cu).
int load_tensors(lc_ctx *ctx, lc_gguf *g, const std::function<DevTensor *(const char *)> &slot, uint32_t flags,
                 std::vector<void *> *allocs);
// A projection by the tensor's own dtype with its size checked (lc_model.cu).
int proj_w(lc_ctx *c, const DevTensor &w, const char *what, const float *x, float *y, uint32_t rows, uint32_t k,
           uint32_t n);
// Projections of one activation block: grouped into one tcgen05 launch where
// the shapes allow, else one projection per weight with the input op
// materialised in `materialized` and accumulated outputs summed through `tmp`
// (lc_model.cu).
int proj_w_block(lc_ctx *c, float *tmp, const PackSrc &src, float *materialized, ProjOut *outs,
                 const DevTensor *const *ws, const char *const *names, int ng, uint32_t rows, uint32_t k);
// True when a projection of m rows would run the tcgen05 GEMM (gemm_dq).
bool routes_to_gemm_dq(const lc_ctx *ctx, uint32_t m);
// 3..16-token projections on tcgen05 kind::i8 (lc_gemm.cu); LC_ERR_UNSUPPORTED when
// the shape is not covered.
int gemv_i8(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n);
// y = x . W^T for more than 32 rows on the lm_head tiles (lc_gemm.cu);
// LC_ERR_UNSUPPORTED when the shape is not covered.
int gemm_large(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n);
// lm_head logits + argmax keys on tcgen05 (lc_gemm.cu); LC_ERR_UNSUPPORTED when
// the shape is not covered.
int lm_head_tc(lc_ctx *ctx, int dtype, const float *x, const void *w, uint32_t m, uint32_t k, uint32_t n,
               uint32_t row_offset, uint64_t *keys, float *logits);
}  // namespace lc
