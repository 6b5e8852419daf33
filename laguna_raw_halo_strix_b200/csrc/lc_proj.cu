// lc_proj.cu -- fused GGUF dequant + projection (GEMV / small-M GEMM).
//
// Reference: kernels/proj_q4k.comp:127-159, kernels/proj_q8_0.comp:47-67 and
// kernels/proj.comp:23-33 compute c[i] = sum_j x[j] * w(i, j) one output per
// invocation with a serial K loop.  Here each warp owns a 16-row tile of W and
// streams its raw blocks from HBM exactly once; the dot products run on the
// tensor cores (mma.sync m16n8k16, f16 inputs, f32 accumulate):
//
//  * A (16 rows x 16 k) is built in registers from the raw block bytes with
//    exact f16 values only: Q4_K nibble*scale (<= 15*63 = 945) via
//    (0x6400|q) magic + one HFMA2; Q8_0 int8 via (0x64xx) magic + HSUB2.
//  * B (16 k x 8 columns) holds the activations.  Column 2*t + p is token t's
//    x split into f16 hi (p = 0) and f16 lo (p = 1), so hi + lo reproduces the
//    f32 activation to ~22 bits and every product is exact in the f32
//    accumulator.  One n-tile carries 4 tokens; NT n-tiles carry 4*NT.
//  * Per-block f16 scales stay in f32: Q4_K uses y += d*S(sc*q*x) - dmin*S(m*Sx)
//    per super-block (Sx = per-sub-block sum of x, multiplied on a k8 MMA);
//    Q8_0 uses y += d*S(q*x) per 32-element block.
//
// The activations are first packed once per call into B fragments in k-step
// order (x_pack_* kernels, a few KB); every CTA copies the part it needs into
// shared memory.  The k-index <-> element permutation of A and B is the same,
// so the sum is the reference's dot product in a different association order.
#include <algorithm>

#include "lc_internal.cuh"

namespace {

constexpr int kWarps = 4;

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t u4_get(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// (scale, scale) f16x2 for a 6-bit integer, exact.
__device__ __forceinline__ __half2 h2_from_u6(uint32_t s) {
    uint32_t v = (s | 0x6400u) * 0x00010001u;
    return __hsub2(lc_u32_as_h2(v), __half2(__float2half_rn(1024.f), __float2half_rn(1024.f)));
}

// ---------------------------------------------------------------------------
// Activation packing.  Table entry (uint2 = B regs {b0b1, b2b3}) for
// [block-step][n-tile][lane]; lanes = 8 when m == 1 (only columns 0/1 used).

// Q4_K: 17 k-steps per 256-element super-block: 16 main steps
// js = h*8 + wi*2 + half, plus the min step (js = 16) carrying Sx.
__global__ void x_pack_q4k(const float *__restrict__ x, uint2 *__restrict__ tab, int m, int k, int nt_count,
                           int lanes, int total) {
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    int lane = idx % lanes;
    int r = idx / lanes;
    int nt = r % nt_count;
    r /= nt_count;
    int js = r % 17;
    int sb = r / 17;
    int g = lane >> 2, t = lane & 3;
    int tok = nt * 4 + (g >> 1), part = g & 1;
    uint2 v = make_uint2(0u, 0u);
    if (tok < m) {
        const float *xr = x + (size_t)tok * k + (size_t)sb * 256;
        if (js < 16) {
            int h = js >> 3, wi = (js >> 1) & 3, half = js & 1;
            int jb = 16 * (t + 4 * h) + 4 * wi;
            auto el = [&](int j) { return 64 * (j >> 5) + (j & 31) + 32 * half; };
            v.x = lc_pack_h2(lc_split_part(xr[el(jb + 0)], part), lc_split_part(xr[el(jb + 2)], part));
            v.y = lc_pack_h2(lc_split_part(xr[el(jb + 1)], part), lc_split_part(xr[el(jb + 3)], part));
        } else {
            float s0 = 0.f, s1 = 0.f;
            for (int e = 0; e < 32; e++) {
                s0 += xr[32 * (2 * t) + e];
                s1 += xr[32 * (2 * t + 1) + e];
            }
            v.x = lc_pack_h2(lc_split_part(s0, part), lc_split_part(s1, part));
        }
    }
    tab[idx] = v;
}

// Q8_0: 2 k-steps per 32-element block; thread t of step ks covers elements
// 16*ks + 4t + {0..3}: b0b1 = (e0, e2), b2b3 = (e1, e3).
__global__ void x_pack_q8(const float *__restrict__ x, uint2 *__restrict__ tab, int m, int k, int nt_count,
                          int lanes, int total) {
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    int lane = idx % lanes;
    int r = idx / lanes;
    int nt = r % nt_count;
    r /= nt_count;
    int ks = r & 1;
    int b = r >> 1;
    int g = lane >> 2, t = lane & 3;
    int tok = nt * 4 + (g >> 1), part = g & 1;
    uint2 v = make_uint2(0u, 0u);
    if (tok < m) {
        const float *xr = x + (size_t)tok * k + (size_t)b * 32 + 16 * ks + 4 * t;
        v.x = lc_pack_h2(lc_split_part(xr[0], part), lc_split_part(xr[2], part));
        v.y = lc_pack_h2(lc_split_part(xr[1], part), lc_split_part(xr[3], part));
    }
    tab[idx] = v;
}

// Copy `n16` 16-byte units of the packed table into shared memory.
__device__ __forceinline__ void copy_tab(uint4 *dst, const uint4 *src, int n16) {
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
}

// Cross-warp reduction of the per-thread results and the store.
template <int NT>
__device__ __forceinline__ void reduce_store(float (&acc)[NT][4], float *red, float *c, int m, int n, int row0,
                                             int atomic_out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        red[((warp * NT + nt) * 32 + lane) * 2 + 0] = acc[nt][0] + acc[nt][1];
        red[((warp * NT + nt) * 32 + lane) * 2 + 1] = acc[nt][2] + acc[nt][3];
    }
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float y0 = 0.f, y1 = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
            y0 += red[((w * NT + nt) * 32 + lane) * 2 + 0];
            y1 += red[((w * NT + nt) * 32 + lane) * 2 + 1];
        }
        int tok = nt * 4 + t;
        if (tok < m) {
            int r0 = row0 + g, r1 = row0 + g + 8;
            float *cr = c + (size_t)tok * n;
            if (atomic_out) {
                if (r0 < n) atomicAdd(cr + r0, y0);
                if (r1 < n) atomicAdd(cr + r1, y1);
            } else {
                if (r0 < n) cr[r0] = y0;
                if (r1 < n) cr[r1] = y1;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Q4_K.  Grid: x = 16-row tiles, y = K chunks of sb_per_chunk super-blocks.
// Warp w of the CTA handles super-blocks w, w+kWarps, ... of the chunk.
template <int NT, int LANES>
__global__ void __launch_bounds__(kWarps * 32) q4k_mma_kernel(const uint2 *__restrict__ tab_g,
                                                              const uint8_t *__restrict__ w, float *__restrict__ c,
                                                              int m, int k, int n, int sb_per_chunk, int half_mode,
                                                              int atomic_out) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int kStep = NT * LANES;  // uint2 entries per k-step
    const int nsb = k >> 8;
    const int sb0 = blockIdx.y * sb_per_chunk;
    const int nloc = min(sb_per_chunk, nsb - sb0);
    uint2 *tab = reinterpret_cast<uint2 *>(smem);
    float *red = reinterpret_cast<float *>(smem + (size_t)sb_per_chunk * 17 * kStep * 8);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int row0 = blockIdx.x * 16;
    const int rg = row0 + g, rg8 = row0 + g + 8;
    const bool vg = rg < n, vg8 = rg8 < n;
    const size_t rowbytes = (size_t)nsb * 144;
    const uint8_t *wg = w + (size_t)(vg ? rg : 0) * rowbytes;
    const uint8_t *wg8 = w + (size_t)(vg8 ? rg8 : 0) * rowbytes;

    copy_tab(reinterpret_cast<uint4 *>(tab), reinterpret_cast<const uint4 *>(tab_g + (size_t)sb0 * 17 * kStep),
             nloc * 17 * kStep / 2);
    __syncthreads();

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    const int p0 = t >> 1;
    const __half2 kNeg1024 = __half2(__float2half_rn(-1024.f), __float2half_rn(-1024.f));
    const __half2 kSixteenth = __half2(__float2half_rn(0.0625f), __float2half_rn(0.0625f));
    const __half2 kNeg64 = __half2(__float2half_rn(-64.f), __float2half_rn(-64.f));
    const __half2 k1024 = __half2(__float2half_rn(1024.f), __float2half_rn(1024.f));

    for (int sbl = warp; sbl < nloc; sbl += kWarps) {
        const size_t off = (size_t)(sb0 + sbl) * 144;
        uint4 H0 = make_uint4(0, 0, 0, 0), H1 = H0, Q0a = H0, Q0b = H0, Q1a = H0, Q1b = H0;
        if (vg) {
            H0 = ldg_stream(wg + off);
            Q0a = ldg_stream(wg + off + 16 + 16 * t);
            Q0b = ldg_stream(wg + off + 16 + 16 * (t + 4));
        }
        if (vg8) {
            H1 = ldg_stream(wg8 + off);
            Q1a = ldg_stream(wg8 + off + 16 + 16 * t);
            Q1b = ldg_stream(wg8 + off + 16 + 16 * (t + 4));
        }
        const float dg = lc_half_to_f32(H0.x & 0xFFFFu, half_mode), dmg = lc_half_to_f32(H0.x >> 16, half_mode);
        const float dg8 = lc_half_to_f32(H1.x & 0xFFFFu, half_mode), dmg8 = lc_half_to_f32(H1.x >> 16, half_mode);

        // Scales of this thread's sub-blocks (get_scale_min_k4, proj_q4k.comp:113-125):
        // lo0 = 2p0, hi0 = 2p0+1 (j < 4); lo1 = 2p0+4, hi1 = 2p0+5 (j >= 4).
        __half2 mul[2][4], add[2][4];  // [row g / g+8][lo0, hi0, lo1, hi1]
        uint32_t mpk[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint4 H = r ? H1 : H0;
            const uint32_t yy = H.y >> (16 * p0), ww = H.w >> (16 * p0);
            const uint32_t s_lo0 = yy & 63u, s_hi0 = (yy >> 8) & 63u;
            const uint32_t s_lo1 = (ww & 15u) | ((yy >> 2) & 0x30u);
            const uint32_t s_hi1 = ((ww >> 8) & 15u) | ((yy >> 10) & 0x30u);
            __half2 h;
            h = h2_from_u6(s_lo0);
            mul[r][0] = h;
            add[r][0] = __hmul2(h, kNeg1024);
            h = h2_from_u6(s_hi0);
            mul[r][1] = __hmul2(h, kSixteenth);
            add[r][1] = __hmul2(h, kNeg64);
            h = h2_from_u6(s_lo1);
            mul[r][2] = h;
            add[r][2] = __hmul2(h, kNeg1024);
            h = h2_from_u6(s_hi1);
            mul[r][3] = __hmul2(h, kSixteenth);
            add[r][3] = __hmul2(h, kNeg64);
            // mins of sub-blocks 2t and 2t+1 for the min step
            uint32_t m0, m1;
            if (t < 2) {
                const uint32_t zz = H.z >> (16 * t);
                m0 = zz & 63u;
                m1 = (zz >> 8) & 63u;
            } else {
                const uint32_t zz = H.z >> (16 * (t - 2)), wz = H.w >> (16 * (t - 2));
                m0 = ((wz >> 4) & 15u) | ((zz >> 2) & 0x30u);
                m1 = ((wz >> 12) & 15u) | ((zz >> 10) & 0x30u);
            }
            mpk[r] = lc_h2_as_u32(__hsub2(lc_u32_as_h2((m0 | 0x6400u) | ((m1 | 0x6400u) << 16)), k1024));
        }

        float cm[NT][4], cmin[NT][4];
#pragma unroll
        for (int i = 0; i < NT; i++)
            cm[i][0] = cm[i][1] = cm[i][2] = cm[i][3] = cmin[i][0] = cmin[i][1] = cmin[i][2] = cmin[i][3] = 0.f;

        const uint2 *tb = tab + (size_t)sbl * 17 * kStep;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 qg = h ? Q0b : Q0a;
            const uint4 qg8 = h ? Q1b : Q1a;
#pragma unroll
            for (int wi = 0; wi < 4; wi++) {
                const uint32_t xg = u4_get(qg, wi), xg8 = u4_get(qg8, wi);
                const uint32_t xgs = xg >> 8, xg8s = xg8 >> 8;
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    const int si = 2 * h + half;  // lo0, hi0, lo1, hi1
                    const uint32_t mask = half ? 0x00F000F0u : 0x000F000Fu;
                    const uint32_t a0 = lc_h2_as_u32(
                        __hfma2(lc_u32_as_h2((xg & mask) | 0x64006400u), mul[0][si], add[0][si]));
                    const uint32_t a1 = lc_h2_as_u32(
                        __hfma2(lc_u32_as_h2((xg8 & mask) | 0x64006400u), mul[1][si], add[1][si]));
                    const uint32_t a2 = lc_h2_as_u32(
                        __hfma2(lc_u32_as_h2((xgs & mask) | 0x64006400u), mul[0][si], add[0][si]));
                    const uint32_t a3 = lc_h2_as_u32(
                        __hfma2(lc_u32_as_h2((xg8s & mask) | 0x64006400u), mul[1][si], add[1][si]));
                    const int js = h * 8 + wi * 2 + half;
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        uint2 b = make_uint2(0u, 0u);
                        if (LANES == 32 || lane < LANES) b = tb[js * kStep + nt * LANES + lane];
                        lc_mma16816(cm[nt], a0, a1, a2, a3, b.x, b.y);
                    }
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            uint2 b = make_uint2(0u, 0u);
            if (LANES == 32 || lane < LANES) b = tb[16 * kStep + nt * LANES + lane];
            lc_mma1688(cmin[nt], mpk[0], mpk[1], b.x);
            acc[nt][0] += dg * cm[nt][0] - dmg * cmin[nt][0];
            acc[nt][1] += dg * cm[nt][1] - dmg * cmin[nt][1];
            acc[nt][2] += dg8 * cm[nt][2] - dmg8 * cmin[nt][2];
            acc[nt][3] += dg8 * cm[nt][3] - dmg8 * cmin[nt][3];
        }
    }
    reduce_store<NT>(acc, red, c, m, n, row0, atomic_out);
}

// ---------------------------------------------------------------------------
// Q8_0.  Rows are processed in block pairs (68 B = 17 aligned words):
// words 0..8 hold d_A and q_A (q_A[4t..4t+3] = funnel(word t, word t+1) >> 16),
// words 8..16 hold d_B (high half of word 8) and q_B (words 9..16).
__device__ __forceinline__ void q8_quads(uint32_t u, uint32_t &lo, uint32_t &hi) {
    // u: four int8 -> (e0, e2) and (e1, e3) as exact f16 pairs.
    const uint32_t b = u ^ 0x80808080u;
    const __half2 k1152 = __half2(__float2half_rn(1152.f), __float2half_rn(1152.f));
    lo = lc_h2_as_u32(__hsub2(lc_u32_as_h2(__byte_perm(b, 0x64646464u, 0x4240)), k1152));
    hi = lc_h2_as_u32(__hsub2(lc_u32_as_h2(__byte_perm(b, 0x64646464u, 0x4341)), k1152));
}

template <int NT, int LANES>
__global__ void __launch_bounds__(kWarps * 32) q8_mma_kernel(const uint2 *__restrict__ tab_g,
                                                             const uint8_t *__restrict__ w, float *__restrict__ c,
                                                             int m, int k, int n, int pairs_per_chunk,
                                                             int half_mode, int atomic_out) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int kStep = NT * LANES;
    const int npairs = k >> 6;
    const int p0 = blockIdx.y * pairs_per_chunk;
    const int nloc = min(pairs_per_chunk, npairs - p0);
    uint2 *tab = reinterpret_cast<uint2 *>(smem);
    float *red = reinterpret_cast<float *>(smem + (size_t)pairs_per_chunk * 4 * kStep * 8);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int row0 = blockIdx.x * 16;
    const int rg = row0 + g, rg8 = row0 + g + 8;
    const bool vg = rg < n, vg8 = rg8 < n;
    const size_t rowbytes = (size_t)npairs * 68;
    const uint8_t *wr[2] = {w + (size_t)(vg ? rg : 0) * rowbytes, w + (size_t)(vg8 ? rg8 : 0) * rowbytes};
    const bool vr[2] = {vg, vg8};

    copy_tab(reinterpret_cast<uint4 *>(tab), reinterpret_cast<const uint4 *>(tab_g + (size_t)p0 * 4 * kStep),
             nloc * 4 * kStep / 2);
    __syncthreads();

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (int pl = warp; pl < nloc; pl += kWarps) {
        const size_t off = (size_t)(p0 + pl) * 68;
        uint32_t wd[2][8];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint8_t *b = wr[r] + off;
            if (vr[r]) {
                wd[r][0] = ldg_u32(b + 4 * t);
                wd[r][1] = ldg_u32(b + 4 * (t + 1));
                wd[r][2] = ldg_u32(b + 4 * (t + 4));
                wd[r][3] = ldg_u32(b + 4 * (t + 5));
                wd[r][4] = ldg_u32(b + 4 * (t + 9));
                wd[r][5] = ldg_u32(b + 4 * (t + 13));
                wd[r][6] = ldg_u32(b);
                wd[r][7] = ldg_u32(b + 32);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) wd[r][i] = 0u;
            }
        }
        const float dA0 = lc_half_to_f32(wd[0][6] & 0xFFFFu, half_mode);
        const float dB0 = lc_half_to_f32(wd[0][7] >> 16, half_mode);
        const float dA1 = lc_half_to_f32(wd[1][6] & 0xFFFFu, half_mode);
        const float dB1 = lc_half_to_f32(wd[1][7] >> 16, half_mode);
        const uint2 *tb = tab + (size_t)pl * 4 * kStep;
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
            float cm[NT][4];
#pragma unroll
            for (int i = 0; i < NT; i++) cm[i][0] = cm[i][1] = cm[i][2] = cm[i][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 2; ks++) {
                uint32_t q0, q1;
                if (blk == 0) {
                    q0 = __funnelshift_r(wd[0][2 * ks], wd[0][2 * ks + 1], 16);
                    q1 = __funnelshift_r(wd[1][2 * ks], wd[1][2 * ks + 1], 16);
                } else {
                    q0 = wd[0][4 + ks];
                    q1 = wd[1][4 + ks];
                }
                uint32_t a0, a2, a1, a3;
                q8_quads(q0, a0, a2);
                q8_quads(q1, a1, a3);
                const int js = blk * 2 + ks;
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    uint2 b = make_uint2(0u, 0u);
                    if (LANES == 32 || lane < LANES) b = tb[js * kStep + nt * LANES + lane];
                    lc_mma16816(cm[nt], a0, a1, a2, a3, b.x, b.y);
                }
            }
            const float d0 = blk ? dB0 : dA0, d1 = blk ? dB1 : dA1;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                acc[nt][0] += d0 * cm[nt][0];
                acc[nt][1] += d0 * cm[nt][1];
                acc[nt][2] += d1 * cm[nt][2];
                acc[nt][3] += d1 * cm[nt][3];
            }
        }
    }
    reduce_store<NT>(acc, red, c, m, n, row0, atomic_out);
}

// ---------------------------------------------------------------------------
// Element-wise fallback for shapes the tiled kernels do not take (Q8_0 rows
// that are not 4-byte aligned).  One warp per (row, token); decodes every
// element with the shader formula.
__global__ void q8_rowwise_kernel(const float *__restrict__ x, const uint8_t *__restrict__ w,
                                  float *__restrict__ c, int m, int k, int n, int half_mode) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int tok = blockIdx.y, lane = threadIdx.x & 31;
    if (row >= n) return;
    const float *xr = x + (size_t)tok * k;
    float acc = 0.f;
    for (int b = lane; b < (k >> 5); b += 32) {
        const uint8_t *blk = w + ((size_t)row * (k >> 5) + b) * 34;
        const float d = lc_half_to_f32(blk[0] | (blk[1] << 8), half_mode);
        float s = 0.f;
        for (int e = 0; e < 32; e++) s += xr[b * 32 + e] * (float)(int8_t)blk[2 + e];
        acc += d * s;
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) c[(size_t)tok * n + row] = acc;
}

// ---------------------------------------------------------------------------
// f32 projection (kernels/proj.comp).  row_major = 0: one warp per output row
// (rows of w contiguous).  row_major = 1: one thread per output (coalesced
// across outputs).
__global__ void f32_rows_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ c,
                                int k, int n, int vec4) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int tok = blockIdx.y, lane = threadIdx.x & 31;
    if (row >= n) return;
    const float *xr = x + (size_t)tok * k;
    const float *wr = w + (size_t)row * k;
    float acc = 0.f;
    if (vec4) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const float4 *w4 = reinterpret_cast<const float4 *>(wr);
        for (int j = lane; j < (k >> 2); j += 32) {
            float4 a = x4[j], b = __ldg(w4 + j);
            acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
        }
    } else {
        for (int j = lane; j < k; j += 32) acc += xr[j] * __ldg(wr + j);
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) c[(size_t)tok * n + row] = acc;
}

__global__ void f32_cols_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ c,
                                int k, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int tok = blockIdx.y;
    if (i >= n) return;
    const float *xr = x + (size_t)tok * k;
    float acc = 0.f;
    for (int j = 0; j < k; j++) acc += xr[j] * __ldg(w + (size_t)j * n + i);
    c[(size_t)tok * n + i] = acc;
}

// ---------------------------------------------------------------------------
template <typename K>
int set_smem(K kernel, size_t bytes) {
    if (bytes > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return lc_fail(LC_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    return LC_OK;
}

constexpr size_t kTabSmemBudget = 100 * 1024;

template <int NT, int LANES>
int launch_q4k(lc_ctx *ctx, const uint2 *tab, const uint8_t *w, float *c, int m, int k, int n) {
    const int nsb = k >> 8;
    const size_t per_sb = (size_t)17 * NT * LANES * 8;
    int spc = (int)std::min<size_t>((size_t)nsb, std::max<size_t>(1, kTabSmemBudget / per_sb));
    const int kch = (nsb + spc - 1) / spc;
    spc = (nsb + kch - 1) / kch;
    const size_t smem = (size_t)spc * per_sb + (size_t)kWarps * NT * 32 * 2 * 4;
    int s = set_smem(q4k_mma_kernel<NT, LANES>, smem);
    if (s) return s;
    if (kch > 1) LC_CUDA(cudaMemsetAsync(c, 0, (size_t)m * n * 4, ctx->stream));
    dim3 grid((n + 15) / 16, kch);
    q4k_mma_kernel<NT, LANES><<<grid, kWarps * 32, smem, ctx->stream>>>(tab, w, c, m, k, n, spc, ctx->half_mode,
                                                                         kch > 1);
    return LC_OK;
}

template <int NT, int LANES>
int launch_q8(lc_ctx *ctx, const uint2 *tab, const uint8_t *w, float *c, int m, int k, int n) {
    const int npairs = k >> 6;
    const size_t per_pair = (size_t)4 * NT * LANES * 8;
    int ppc = (int)std::min<size_t>((size_t)npairs, std::max<size_t>(1, kTabSmemBudget / per_pair));
    const int kch = (npairs + ppc - 1) / ppc;
    ppc = (npairs + kch - 1) / kch;
    const size_t smem = (size_t)ppc * per_pair + (size_t)kWarps * NT * 32 * 2 * 4;
    int s = set_smem(q8_mma_kernel<NT, LANES>, smem);
    if (s) return s;
    if (kch > 1) LC_CUDA(cudaMemsetAsync(c, 0, (size_t)m * n * 4, ctx->stream));
    dim3 grid((n + 15) / 16, kch);
    q8_mma_kernel<NT, LANES><<<grid, kWarps * 32, smem, ctx->stream>>>(tab, w, c, m, k, n, ppc, ctx->half_mode,
                                                                        kch > 1);
    return LC_OK;
}

}  // namespace

namespace lc {

// One launch group handles up to 16 tokens (NT = 4 n-tiles).
int proj_q4k(lc_ctx *ctx, const float *x, const void *wv, float *c, uint32_t m, uint32_t k, uint32_t n,
             uint32_t expert_offset) {
    LC_REQUIRE(k % 256 == 0, LC_ERR_UNSUPPORTED, "proj_q4k: k=%u is not a multiple of 256", k);
    LC_REQUIRE(expert_offset % 256 == 0, LC_ERR_UNSUPPORTED, "proj_q4k: expert_offset=%u not a multiple of 256",
               expert_offset);
    LC_REQUIRE(((uintptr_t)wv & 15) == 0, LC_ERR_INVALID, "proj_q4k: weight pointer not 16-byte aligned");
    const uint8_t *w = (const uint8_t *)wv + (size_t)(expert_offset / 256) * 144;
    const int nsb = k / 256;
    for (uint32_t t0 = 0; t0 < m; t0 += 16) {
        const int mm = (int)std::min<uint32_t>(16, m - t0);
        const int nt = (mm + 3) / 4;
        const int lanes = mm == 1 ? 8 : 32;
        const int total = nsb * 17 * nt * lanes;
        uint2 *tab = (uint2 *)lc_scratch(ctx, LC_SCRATCH_PACK, (size_t)total * 8);
        if (!tab) return LC_ERR_OOM;
        x_pack_q4k<<<(total + 255) / 256, 256, 0, ctx->stream>>>(x + (size_t)t0 * k, tab, mm, k, nt, lanes, total);
        float *cc = c + (size_t)t0 * n;
        int s;
        if (mm == 1)
            s = launch_q4k<1, 8>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 1)
            s = launch_q4k<1, 32>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 2)
            s = launch_q4k<2, 32>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 3)
            s = launch_q4k<3, 32>(ctx, tab, w, cc, mm, k, n);
        else
            s = launch_q4k<4, 32>(ctx, tab, w, cc, mm, k, n);
        if (s) return s;
    }
    return LC_OK;
}

int proj_q8_0(lc_ctx *ctx, const float *x, const void *wv, float *c, uint32_t m, uint32_t k, uint32_t n) {
    LC_REQUIRE(k % 32 == 0, LC_ERR_UNSUPPORTED, "proj_q8_0: k=%u is not a multiple of 32", k);
    const uint8_t *w = (const uint8_t *)wv;
    if (k % 64 != 0 || ((uintptr_t)wv & 3) != 0) {
        dim3 grid((n + 7) / 8, m);
        q8_rowwise_kernel<<<grid, 256, 0, ctx->stream>>>(x, w, c, (int)m, (int)k, (int)n, ctx->half_mode);
        return LC_OK;
    }
    const int nblk = k / 32;
    for (uint32_t t0 = 0; t0 < m; t0 += 16) {
        const int mm = (int)std::min<uint32_t>(16, m - t0);
        const int nt = (mm + 3) / 4;
        const int lanes = mm == 1 ? 8 : 32;
        const int total = nblk * 2 * nt * lanes;
        uint2 *tab = (uint2 *)lc_scratch(ctx, LC_SCRATCH_PACK, (size_t)total * 8);
        if (!tab) return LC_ERR_OOM;
        x_pack_q8<<<(total + 255) / 256, 256, 0, ctx->stream>>>(x + (size_t)t0 * k, tab, mm, k, nt, lanes, total);
        float *cc = c + (size_t)t0 * n;
        int s;
        if (mm == 1)
            s = launch_q8<1, 8>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 1)
            s = launch_q8<1, 32>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 2)
            s = launch_q8<2, 32>(ctx, tab, w, cc, mm, k, n);
        else if (nt == 3)
            s = launch_q8<3, 32>(ctx, tab, w, cc, mm, k, n);
        else
            s = launch_q8<4, 32>(ctx, tab, w, cc, mm, k, n);
        if (s) return s;
    }
    return LC_OK;
}

int proj_f32(lc_ctx *ctx, const float *x, const float *w, float *c, uint32_t m, uint32_t k, uint32_t n,
             uint32_t row_major) {
    if (row_major) {
        dim3 grid((n + 255) / 256, m);
        f32_cols_kernel<<<grid, 256, 0, ctx->stream>>>(x, w, c, (int)k, (int)n);
    } else {
        const int vec4 = (k % 4 == 0) && (((uintptr_t)x | (uintptr_t)w) & 15) == 0;
        dim3 grid((n + 7) / 8, m);
        f32_rows_kernel<<<grid, 256, 0, ctx->stream>>>(x, w, c, (int)k, (int)n, vec4);
    }
    return LC_OK;
}

}  // namespace lc

// ---------------------------------------------------------------------------
// C ABI

static int proj_common(lc_ctx *ctx, int dtype, const float *x, const void *w, float *c, uint32_t m, uint32_t k,
                       uint32_t n, uint32_t expert_offset, const char *what) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "%s: null ctx", what);
    if (m == 0 || n == 0) return LC_OK;
    LC_REQUIRE(x && w && c, LC_ERR_INVALID, "%s: null pointer", what);
    LC_REQUIRE(k > 0, LC_ERR_INVALID, "%s: k must be > 0", what);
    LC_REQUIRE((uint64_t)n * k < (1ull << 40), LC_ERR_INVALID, "%s: n*k too large", what);
    int s = lc_use_device(ctx);
    if (s) return s;
    switch (dtype) {
    case LC_Q4_K: s = lc::proj_q4k(ctx, x, w, c, m, k, n, expert_offset); break;
    case LC_Q8_0: s = lc::proj_q8_0(ctx, x, w, c, m, k, n); break;
    case LC_F32: s = lc::proj_f32(ctx, x, (const float *)w, c, m, k, n, 0); break;
    default: return lc_fail(LC_ERR_UNSUPPORTED, "%s: dtype %d not supported (F32, Q8_0, Q4_K)", what, dtype);
    }
    if (s) return s;
    return lc_after_launch(ctx, what);
}

extern "C" int lc_proj_f32(lc_ctx *ctx, const float *x, const float *w, float *c, uint32_t k, uint32_t n,
                           uint32_t row_major) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_proj_f32: null ctx");
    if (n == 0) return LC_OK;
    LC_REQUIRE(x && w && c, LC_ERR_INVALID, "lc_proj_f32: null pointer");
    int s = lc_use_device(ctx);
    if (s) return s;
    s = lc::proj_f32(ctx, x, w, c, 1, k, n, row_major);
    if (s) return s;
    return lc_after_launch(ctx, "lc_proj_f32");
}

extern "C" int lc_proj_q8_0(lc_ctx *ctx, const float *x, const void *w, float *c, uint32_t k, uint32_t n) {
    return proj_common(ctx, LC_Q8_0, x, w, c, 1, k, n, 0, "lc_proj_q8_0");
}

extern "C" int lc_proj_q4k(lc_ctx *ctx, const float *x, const void *w, float *c, uint32_t k, uint32_t n,
                           uint32_t expert_offset) {
    return proj_common(ctx, LC_Q4_K, x, w, c, 1, k, n, expert_offset, "lc_proj_q4k");
}

extern "C" int lc_proj_quant(lc_ctx *ctx, int dtype, const float *x, const void *w, float *c, uint32_t k,
                             uint32_t n, uint32_t expert_offset) {
    return proj_common(ctx, dtype, x, w, c, 1, k, n, dtype == LC_Q4_K ? expert_offset : 0, "lc_proj_quant");
}

extern "C" int lc_proj_m(lc_ctx *ctx, int dtype, const float *x, const void *w, float *c, uint32_t m, uint32_t k,
                         uint32_t n, uint32_t expert_offset) {
    return proj_common(ctx, dtype, x, w, c, m, k, n, dtype == LC_Q4_K ? expert_offset : 0, "lc_proj_m");
}
