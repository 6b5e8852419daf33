// lc_ops.cu -- the kernels interleaved with the projections in the DFlash
// encoder/decoder (kernels/rmsnorm.comp, qk_norm_rope.comp, activation.comp,
// add.comp, gate_mul.comp, enc_aux_norm.comp, the host softplus of
// src/dflash.rs:956-958) plus dequant_to_f32 (src/dflash.rs:331-465) and the
// row argmax of src/lib.rs:456-464.
//
// The reference recomputes each row's sum of squares in every invocation
// (O(n^2)); here one CTA reduces a row once and then writes it, which also
// makes the in-place calls of the reference (output_norm x -> x,
// src/dflash.rs:973) race-free.
#include <algorithm>

#include "lc_internal.cuh"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum; every thread gets the result.  `sh` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float r = lane < nw ? sh[lane] : 0.f;
    r = warp_sum(r);
    return r;
}

// rmsnorm.comp:22-35 over m rows: y = x * w * inversesqrt(mean(x^2) + eps).
__global__ void rmsnorm_kernel(const float *__restrict__ w, const float *x, float *y, int n, float eps) {
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        s += v * v;
    }
    s = block_sum(s, sh);
    const float rms = rsqrtf(s / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * w[i] * rms;
}

// rmsnorm for rows of n % 4 == 0, n <= 16 * blockDim: the row stays in
// registers (4 float4 per thread at most), one read of x.
__global__ void rmsnorm4_kernel(const float *__restrict__ w, const float *x, float *y, int n, float eps) {
    __shared__ float sh[32];
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * n);
    float4 *yr = reinterpret_cast<float4 *>(y + (size_t)blockIdx.x * n);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    const int n4 = n >> 2;
    float4 v[4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
    s = block_sum(s, sh);
    const float rms = rsqrtf(s / (float)n + eps);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < n4) {
            const float4 ww = w4[i];
            yr[i] = make_float4(v[j].x * ww.x * rms, v[j].y * ww.y * rms, v[j].z * ww.z * rms, v[j].w * ww.w * rms);
        }
    }
}

// qk_norm_rope.comp:29-67 for head_dim 128 and rope_dim 0 or 128: one CTA per
// (row, 4 heads), one warp per head, lane l holding dims 4l..4l+3.  The rope
// partner of dim d (d +/- 64) sits in lane l ^ 16, fetched with a shuffle, so
// the head is read once into registers and out may alias x.  The row's 64
// (cos, sin) pairs are computed once per CTA (the same sincosf of the same
// argument as the per-element form) instead of once per element.  Two
// tensors of the same rows (the block's Q and K) go in one launch: CTAs with
// blockIdx.y < nb0 take set 0, the rest set 1.
struct QkPair {
    const float *x[2];
    const float *w[2];
    float *y[2];
    int n_heads[2];
    int nb0;
};

__global__ void qk_norm_rope128_kernel(const QkPair p, const float *__restrict__ freq, int rope, float eps,
                                       uint32_t pos0, uint32_t pos_step) {
    __shared__ float2 cs[64];
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool second = (int)blockIdx.y >= p.nb0;
    const float *x = second ? p.x[1] : p.x[0];
    const float *__restrict__ w = second ? p.w[1] : p.w[0];
    float *y = second ? p.y[1] : p.y[0];
    const int n_heads = second ? p.n_heads[1] : p.n_heads[0];
    const int h = ((int)blockIdx.y - (second ? p.nb0 : 0)) * 4 + warp;
    const uint32_t pos = pos0 + row * pos_step;
    if (rope && threadIdx.x < 64) {
        float sf, cf;
        sincosf(freq[threadIdx.x] * (float)pos, &sf, &cf);
        cs[threadIdx.x] = make_float2(cf, sf);
    }
    __syncthreads();
    if (h >= n_heads) return;
    const size_t base = ((size_t)row * n_heads + h) * 128 + 4 * lane;
    const float4 v = *reinterpret_cast<const float4 *>(x + base);
    const float sq = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    const float r = rsqrtf(warp_sum(sq) / 128.f + eps);
    const float4 wv = *reinterpret_cast<const float4 *>(w + 4 * lane);
    const float nv[4] = {v.x * wv.x * r, v.y * wv.y * r, v.z * wv.z * r, v.w * wv.w * r};
    float o[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const float pn = __shfl_xor_sync(0xffffffffu, nv[c], 16);  // dim +/- 64
        if (!rope) {
            o[c] = nv[c];
        } else {
            const float2 t = cs[4 * (lane & 15) + c];
            o[c] = lane < 16 ? nv[c] * t.x - pn * t.y : nv[c] * t.x + pn * t.y;
        }
    }
    *reinterpret_cast<float4 *>(y + base) = make_float4(o[0], o[1], o[2], o[3]);
}

// qk_norm_rope.comp:29-67 for one row (n_heads*head_dim) per CTA at position
// pos0 + row * pos_step.  The row is staged in shared memory first so out may
// alias x.
__global__ void qk_norm_rope_kernel(const float *x, const float *__restrict__ w, const float *__restrict__ freq,
                                    float *y, int n_heads, int head_dim, int rope_dim, float eps, uint32_t pos0,
                                    uint32_t pos_step) {
    extern __shared__ float srow[];  // total + n_heads
    const int total = n_heads * head_dim;
    float *rms = srow + total;
    const float *xr = x + (size_t)blockIdx.x * total;
    float *yr = y + (size_t)blockIdx.x * total;
    const uint32_t pos = pos0 + blockIdx.x * pos_step;
    for (int i = threadIdx.x; i < total; i += blockDim.x) srow[i] = xr[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int h = warp; h < n_heads; h += nw) {
        float s = 0.f;
        for (int d = lane; d < head_dim; d += 32) {
            float v = srow[h * head_dim + d];
            s += v * v;
        }
        s = warp_sum(s);
        if (lane == 0) rms[h] = rsqrtf(s / (float)head_dim + eps);
    }
    __syncthreads();
    const int rh = rope_dim / 2, hh = head_dim / 2;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int head = i / head_dim, dim = i % head_dim;
        const float r = rms[head];
        const float normed = srow[i] * w[dim] * r;
        if (dim >= rope_dim) {
            yr[i] = normed;
        } else {
            const int hf = dim % rh;
            float sf, cf;
            sincosf(freq[hf] * (float)pos, &sf, &cf);
            if (dim < rh) {
                const int pi = i + hh;
                const float pn = srow[pi] * w[pi % head_dim] * r;
                yr[i] = normed * cf - pn * sf;
            } else {
                const int pi = i - hh;
                const float pn = srow[pi] * w[pi % head_dim] * r;
                yr[i] = normed * cf + pn * sf;
            }
        }
    }
}

__global__ void activation_kernel(const float *gate, const float *up, float *h, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        h[i] = lc_swiglu(gate[i], up[i]);
    }
}

__global__ void add_kernel(const float *a, const float *b, float *c, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) c[i] = a[i] + b[i];
}

__global__ void gate_mul_kernel(const float *v, const float *gate, float *out, int n, int head_dim) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = v[i] * gate[i / head_dim];
}

__global__ void softplus_kernel(const float *g, float *out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        out[i] = lc_softplus_f(g[i]);
    }
}

// enc_aux_norm.comp:24-43: one CTA per (token, aux) segment of n_feat;
// y = x * rms * w[aux segment].
__global__ void enc_aux_norm_kernel(const float *x, const float *__restrict__ w, float *y, int n_feat, int n_aux,
                                     float eps) {
    __shared__ float sh[32];
    const int seg = blockIdx.x;
    const int aux = seg % n_aux;
    const float *xr = x + (size_t)seg * n_feat;
    float *yr = y + (size_t)seg * n_feat;
    float s = 0.f;
    for (int i = threadIdx.x; i < n_feat; i += blockDim.x) {
        float v = xr[i];
        s += v * v;
    }
    s = block_sum(s, sh);
    const float rms = rsqrtf(s / (float)n_feat + eps);
    for (int i = threadIdx.x; i < n_feat; i += blockDim.x) yr[i] = xr[i] * rms * w[i + aux * n_feat];
}

// ---- dequant_to_f32 ---------------------------------------------------------

__device__ __forceinline__ uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// dequant_kernel's dtype code for BF16 decoded as bfloat16 (the loader's
// LC_LOAD_BF16_NATIVE); not a GGUF type id.
constexpr int kDeqBf16Native = 0x10000 | LC_BF16;

// One thread per output element; reads bounded by nbytes like the Rust code.
__global__ void dequant_kernel(const uint8_t *__restrict__ src, size_t nbytes, int dtype, size_t n,
                               float *__restrict__ out, int half_mode) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = 0.f;
        switch (dtype) {
        case LC_F32:  // src/dflash.rs:333-350
            if (i * 4 + 4 <= nbytes) {
                uint32_t b = (uint32_t)src[4 * i] | ((uint32_t)src[4 * i + 1] << 8) |
                             ((uint32_t)src[4 * i + 2] << 16) | ((uint32_t)src[4 * i + 3] << 24);
                v = __uint_as_float(b);
            }
            break;
        case LC_BF16:  // src/dflash.rs:351-378 decodes these bits with the f16 layout
            if (i * 2 + 2 <= nbytes) v = lc_half_to_f32(rd16(src + 2 * i), LC_HALF_REF);
            break;
        case kDeqBf16Native:  // bfloat16 proper: the top half of an f32
            if (i * 2 + 2 <= nbytes) v = __uint_as_float(rd16(src + 2 * i) << 16);
            break;
        case LC_F16:  // src/dflash.rs:437-462 (IEEE; NaN -> 0x7FC00000)
            if (i * 2 + 2 <= nbytes) {
                uint32_t h = rd16(src + 2 * i);
                if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu))
                    v = __uint_as_float(0x7FC00000u);
                else
                    v = __half2float(__ushort_as_half((unsigned short)h));
            }
            break;
        case LC_Q8_0: {  // src/dflash.rs:379-397 == proj_q8_0.comp:54-63
            size_t b = i / 32, off = b * 34;
            if (off + 34 <= nbytes) {
                float d = lc_half_to_f32(rd16(src + off), half_mode);
                v = __fmul_rn((float)(int8_t)src[off + 2 + (i % 32)], d);
            }
            break;
        }
        case LC_Q4_K: {  // proj_q4k.comp:67-87 (GGUF Q4_K, shader formula)
            size_t b = i / 256, base = b * 144;
            if (base + 144 <= nbytes) {
                const uint8_t *p = src + base;
                uint32_t elm = (uint32_t)(i % 256);
                float d = lc_half_to_f32(rd16(p), half_mode), dmin = lc_half_to_f32(rd16(p + 2), half_mode);
                uint32_t sb = elm / 32u, g64 = elm / 64u, w64 = elm % 64u;
                uint32_t qb = p[16u + g64 * 32u + (w64 % 32u)];
                float q = (float)((w64 < 32u) ? (qb & 0xFu) : ((qb >> 4) & 0xFu));
                const uint8_t *s = p + 4;
                uint32_t sc, mn;
                if (sb < 4u) {
                    sc = s[sb] & 63u;
                    mn = s[sb + 4u] & 63u;
                } else {
                    sc = (s[sb + 4u] & 15u) | ((s[sb - 4u] >> 6) << 4);
                    mn = (s[sb + 4u] >> 4) | ((s[sb] >> 6) << 4);
                }
                v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), q), __fmul_rn(dmin, (float)mn));
            }
            break;
        }
        case LC_Q4_K_DFLASH_CPU: {  // src/dflash.rs:398-436 as written
            size_t b = i / 256, base = b * 144;
            if (base + 144 <= nbytes) {
                const uint8_t *p = src + base;
                float d = __uint_as_float(rd16(p) << 16);
                float k4 = __uint_as_float(rd16(p + 2) << 16);
                float signs = __uint_as_float(rd16(p + 4) << 16);
                size_t e = i % 256;
                uint8_t byte = p[6 + e / 2];
                uint32_t q = (e % 2 == 0) ? ((byte >> 4) & 7u) : (byte & 7u);
                float sgn = signs < 0.0f ? -1.0f : 1.0f;
                v = __fadd_rn(__fmul_rn((float)q, d), __fmul_rn(sgn, k4));
            }
            break;
        }
        default: break;
        }
        out[i] = v;
    }
}

// ---- argmax ------------------------------------------------------------------

// Keys order as signed int64 (see lc_pack_key).
__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return (long long)a > (long long)b ? a : b; }
constexpr uint64_t kKeyMin = 0x8000000000000000ull;

// One CTA per row: keys[row] = max over j of key(logits[row, j], row_offset + j).
__global__ void argmax_rows_kernel(const float *__restrict__ logits, int n, uint32_t row_offset,
                                   uint64_t *__restrict__ keys) {
    __shared__ uint64_t sh[32];
    const float *lr = logits + (size_t)blockIdx.x * n;
    uint64_t best = kKeyMin;
    for (int j = threadIdx.x; j < n; j += blockDim.x) best = umax64(best, lc_make_key(lr[j], row_offset + j));
    for (int o = 16; o; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sh[warp] = best;
    __syncthreads();
    if (warp == 0) {
        best = lane < (int)(blockDim.x >> 5) ? sh[lane] : kKeyMin;
        for (int o = 16; o; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0) keys[blockIdx.x] = best;
    }
}

int grid_for(lc_ctx *ctx, size_t n, int block = 256) {
    size_t g = (n + block - 1) / block;
    size_t cap = (size_t)ctx->num_sms * 16;
    if (g > cap) g = cap;
    return (int)std::max<size_t>(1, g);
}

}  // namespace

// ---- C ABI ---------------------------------------------------------------------

#define LC_BEGIN(ctx, name)                                   \
    LC_REQUIRE(ctx, LC_ERR_INVALID, name ": null ctx");      \
    do {                                                      \
        int _s = lc_use_device(ctx);                          \
        if (_s) return _s;                                    \
    } while (0)

extern "C" int lc_rmsnorm(lc_ctx *ctx, const float *w, const float *x, float *out, uint32_t m, uint32_t n,
                          float eps) {
    LC_BEGIN(ctx, "lc_rmsnorm");
    if (m == 0 || n == 0) return LC_OK;
    LC_REQUIRE(w && x && out, LC_ERR_INVALID, "lc_rmsnorm: null pointer");
    const int bd = n > 4096 ? 1024 : 256;
    if (n % 4 == 0 && n <= 16u * bd && (((uintptr_t)w | (uintptr_t)x | (uintptr_t)out) & 15) == 0)
        rmsnorm4_kernel<<<m, bd, 0, ctx->stream>>>(w, x, out, (int)n, eps);
    else
        rmsnorm_kernel<<<m, n >= 4096 ? 1024 : 256, 0, ctx->stream>>>(w, x, out, (int)n, eps);
    return lc_after_launch(ctx, "lc_rmsnorm");
}

static int qk_norm_rope_steps(lc_ctx *ctx, const float *x, const float *w, const float *freq, float *out,
                              uint32_t m, uint32_t n_heads, uint32_t head_dim, uint32_t rope_dim, float eps,
                              uint32_t pos0, uint32_t pos_step) {
    LC_BEGIN(ctx, "lc_qk_norm_rope");
    if (m == 0 || n_heads == 0) return LC_OK;
    LC_REQUIRE(x && w && out && (freq || rope_dim == 0), LC_ERR_INVALID, "lc_qk_norm_rope: null pointer");
    LC_REQUIRE(head_dim > 0 && head_dim % 2 == 0, LC_ERR_INVALID, "lc_qk_norm_rope: head_dim %u must be even",
               head_dim);
    // qk_norm_rope.comp pairs dim with dim +/- head_dim/2 while rotating only
    // dims < rope_dim; for 0 < rope_dim < head_dim that pair index leaves the
    // head (head 0 reads before the buffer), and rope_dim > head_dim reads the
    // frequency table past its end.  Only the well-defined forms are accepted.
    LC_REQUIRE(rope_dim == 0 || rope_dim == head_dim, LC_ERR_UNSUPPORTED,
               "lc_qk_norm_rope: rope_dim %u must be 0 or head_dim %u", rope_dim, head_dim);
    if (head_dim == 128 && (((uintptr_t)x | (uintptr_t)w | (uintptr_t)out) & 15) == 0) {
        QkPair p = {{x, x}, {w, w}, {out, out}, {(int)n_heads, 0}, (int)(n_heads + 3) / 4};
        qk_norm_rope128_kernel<<<dim3(m, p.nb0), 128, 0, ctx->stream>>>(p, freq, rope_dim ? 1 : 0, eps, pos0, pos_step);
        return lc_after_launch(ctx, "lc_qk_norm_rope");
    }
    const size_t smem = ((size_t)n_heads * head_dim + n_heads) * 4;
    LC_REQUIRE(smem <= ctx->smem_optin, LC_ERR_UNSUPPORTED, "lc_qk_norm_rope: row of %u values too large",
               n_heads * head_dim);
    if (smem > 48 * 1024)
        if (int s = lc_set_smem_attr((const void *)qk_norm_rope_kernel, smem)) return s;
    qk_norm_rope_kernel<<<m, 256, smem, ctx->stream>>>(x, w, freq, out, (int)n_heads, (int)head_dim, (int)rope_dim,
                                                        eps, pos0, pos_step);
    return lc_after_launch(ctx, "lc_qk_norm_rope");
}

extern "C" int lc_qk_norm_rope(lc_ctx *ctx, const float *x, const float *w, const float *freq, float *out,
                               uint32_t m, uint32_t n_heads, uint32_t head_dim, uint32_t rope_dim, float eps,
                               uint32_t pos0) {
    return qk_norm_rope_steps(ctx, x, w, freq, out, m, n_heads, head_dim, rope_dim, eps, pos0, 1);
}

namespace lc {
// lc_qk_norm_rope of two tensors over the same m rows (the block's Q with
// n_heads_a heads and K with n_heads_b), in one launch when both take the
// head_dim 128 kernel.
int qk_norm_rope_pair(lc_ctx *ctx, const float *xa, const float *wa, float *ya, uint32_t n_heads_a, const float *xb,
                      const float *wb, float *yb, uint32_t n_heads_b, const float *freq, uint32_t m,
                      uint32_t head_dim, uint32_t rope_dim, float eps, uint32_t pos0, uint32_t pos_step) {
    const bool fused = m > 0 && n_heads_a > 0 && n_heads_b > 0 && head_dim == 128 &&
                       (rope_dim == 0 || rope_dim == head_dim) && xa && wa && ya && xb && wb && yb &&
                       (freq || rope_dim == 0) &&
                       (((uintptr_t)xa | (uintptr_t)wa | (uintptr_t)ya | (uintptr_t)xb | (uintptr_t)wb |
                         (uintptr_t)yb) & 15) == 0;
    if (!fused) {
        const int s = qk_norm_rope_steps(ctx, xa, wa, freq, ya, m, n_heads_a, head_dim, rope_dim, eps, pos0, pos_step);
        if (s) return s;
        return qk_norm_rope_steps(ctx, xb, wb, freq, yb, m, n_heads_b, head_dim, rope_dim, eps, pos0, pos_step);
    }
    LC_BEGIN(ctx, "lc_qk_norm_rope");
    const int nb0 = (int)(n_heads_a + 3) / 4, nb1 = (int)(n_heads_b + 3) / 4;
    QkPair p = {{xa, xb}, {wa, wb}, {ya, yb}, {(int)n_heads_a, (int)n_heads_b}, nb0};
    qk_norm_rope128_kernel<<<dim3(m, nb0 + nb1), 128, 0, ctx->stream>>>(p, freq, rope_dim ? 1 : 0, eps, pos0,
                                                                         pos_step);
    return lc_after_launch(ctx, "lc_qk_norm_rope");
}
}  // namespace lc

extern "C" int lc_activation(lc_ctx *ctx, const float *gate, const float *up, float *h, uint32_t n) {
    LC_BEGIN(ctx, "lc_activation");
    if (n == 0) return LC_OK;
    LC_REQUIRE(gate && up && h, LC_ERR_INVALID, "lc_activation: null pointer");
    activation_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(gate, up, h, (int)n);
    return lc_after_launch(ctx, "lc_activation");
}

extern "C" int lc_add(lc_ctx *ctx, const float *a, const float *b, float *c, uint32_t n) {
    LC_BEGIN(ctx, "lc_add");
    if (n == 0) return LC_OK;
    LC_REQUIRE(a && b && c, LC_ERR_INVALID, "lc_add: null pointer");
    add_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(a, b, c, (int)n);
    return lc_after_launch(ctx, "lc_add");
}

extern "C" int lc_gate_mul(lc_ctx *ctx, const float *v, const float *gate, float *out, uint32_t n_hd,
                           uint32_t n_heads, uint32_t head_dim) {
    LC_BEGIN(ctx, "lc_gate_mul");
    (void)n_heads;
    if (n_hd == 0) return LC_OK;
    LC_REQUIRE(v && gate && out, LC_ERR_INVALID, "lc_gate_mul: null pointer");
    LC_REQUIRE(head_dim > 0, LC_ERR_INVALID, "lc_gate_mul: head_dim must be > 0");
    gate_mul_kernel<<<grid_for(ctx, n_hd), 256, 0, ctx->stream>>>(v, gate, out, (int)n_hd, (int)head_dim);
    return lc_after_launch(ctx, "lc_gate_mul");
}

extern "C" int lc_softplus(lc_ctx *ctx, const float *g, float *out, uint32_t n) {
    LC_BEGIN(ctx, "lc_softplus");
    if (n == 0) return LC_OK;
    LC_REQUIRE(g && out, LC_ERR_INVALID, "lc_softplus: null pointer");
    softplus_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(g, out, (int)n);
    return lc_after_launch(ctx, "lc_softplus");
}

extern "C" int lc_enc_aux_norm(lc_ctx *ctx, const float *x, const float *w, float *y, uint32_t n_feat,
                               uint32_t n_aux, uint32_t n_tokens, float eps) {
    LC_BEGIN(ctx, "lc_enc_aux_norm");
    if (n_feat == 0 || n_aux == 0 || n_tokens == 0) return LC_OK;
    LC_REQUIRE(x && w && y, LC_ERR_INVALID, "lc_enc_aux_norm: null pointer");
    enc_aux_norm_kernel<<<n_aux * n_tokens, n_feat >= 4096 ? 1024 : 256, 0, ctx->stream>>>(x, w, y, (int)n_feat,
                                                                                           (int)n_aux, eps);
    return lc_after_launch(ctx, "lc_enc_aux_norm");
}

extern "C" int lc_dequant(lc_ctx *ctx, int dtype, const void *src, size_t src_bytes, size_t n, float *out) {
    LC_BEGIN(ctx, "lc_dequant");
    if (n == 0) return LC_OK;
    LC_REQUIRE(out && (src || src_bytes == 0), LC_ERR_INVALID, "lc_dequant: null pointer");
    dequant_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>((const uint8_t *)src, src ? src_bytes : 0, dtype, n,
                                                              out, ctx->half_mode);
    return lc_after_launch(ctx, "lc_dequant");
}

int lc::dequant_f32(lc_ctx *ctx, int dtype, const void *src, size_t src_bytes, size_t n, float *out,
                    bool bf16_native) {
    if (!(bf16_native && dtype == LC_BF16)) return lc_dequant(ctx, dtype, src, src_bytes, n, out);
    LC_BEGIN(ctx, "lc_dequant");
    if (n == 0) return LC_OK;
    LC_REQUIRE(out && src, LC_ERR_INVALID, "lc_dequant: null pointer");
    dequant_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>((const uint8_t *)src, src_bytes, kDeqBf16Native, n, out,
                                                              ctx->half_mode);
    return lc_after_launch(ctx, "lc_dequant");
}

extern "C" int lc_argmax_rows(lc_ctx *ctx, const float *logits, uint32_t m, uint32_t n, uint32_t row_offset,
                              uint64_t *keys) {
    LC_BEGIN(ctx, "lc_argmax_rows");
    if (m == 0) return LC_OK;
    LC_REQUIRE(logits && keys, LC_ERR_INVALID, "lc_argmax_rows: null pointer");
    LC_REQUIRE(n > 0, LC_ERR_INVALID, "lc_argmax_rows: n must be > 0");
    argmax_rows_kernel<<<m, 1024, 0, ctx->stream>>>(logits, (int)n, row_offset, keys);
    return lc_after_launch(ctx, "lc_argmax_rows");
}

extern "C" int lc_lm_head_argmax(lc_ctx *ctx, int dtype, const float *x, const void *w, uint32_t m, uint32_t k,
                                 uint32_t n_local, uint32_t row_offset, uint64_t *keys, float *logits) {
    LC_BEGIN(ctx, "lc_lm_head_argmax");
    if (m == 0) return LC_OK;
    LC_REQUIRE(x && w && keys, LC_ERR_INVALID, "lc_lm_head_argmax: null pointer");
    LC_REQUIRE(n_local > 0, LC_ERR_INVALID, "lc_lm_head_argmax: n_local must be > 0");
    // Blocks of more than 32 rows: tensor-core tiles with the argmax fused in
    // the epilogue (the choice depends on m only, so every vocab shard of a
    // call computes its logits the same way).
    if (ctx->gemm_tc && m > 32) {
        const int s = lc::lm_head_tc(ctx, dtype, x, w, m, k, n_local, row_offset, keys, logits);
        if (s != LC_ERR_UNSUPPORTED) return s ? s : lc_after_launch(ctx, "lc_lm_head_argmax");
    }
    float *lg = logits;
    if (!lg) {
        lg = (float *)lc_scratch(ctx, LC_SCRATCH_LOGITS, (size_t)m * n_local * 4);
        if (!lg) return LC_ERR_OOM;
    }
    int s = lc_proj_m(ctx, dtype, x, w, lg, m, k, n_local, 0);
    if (s) return s;
    argmax_rows_kernel<<<m, 1024, 0, ctx->stream>>>(lg, (int)n_local, row_offset, keys);
    return lc_after_launch(ctx, "lc_lm_head_argmax");
}
