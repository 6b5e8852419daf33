// lc_proj.cu -- fused GGUF dequant + projection (GEMV / small-M GEMM).
//
// Reference: kernels/proj_q4k.comp:60-92, kernels/proj_q8_0.comp:47-67 and
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
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "lc_internal.cuh"
#include "lc_sm100.cuh"

namespace cg = cooperative_groups;

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
// Activation packing for the tiled kernels.  Table entry (uint2 = B regs
// {b0b1, b2b3}) for [block-step][n-tile][lane]; column 2t'+p of n-tile nt is
// token nt*4 + t' (p = f16 hi / lo).  One CTA per token slot (NT*4 of them)
// finds the token's power-of-two scale (act_scale), records 2^-e in
// inv_scale[token], and writes the 8 lanes of every k-step that carry it
// (zeros for the padding slots past m).

__device__ __forceinline__ float block_max_abs(const float *__restrict__ xr, int k) {
    __shared__ float sh[32];
    float v = 0.f;
    for (int i = threadIdx.x; i < k; i += blockDim.x) v = fmaxf(v, fabsf(xr[i]));
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.f;
    if (threadIdx.x < 32)
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) sh[0] = v;
    __syncthreads();
    return sh[0];
}

// Q4_K: 17 k-steps per 256-element super-block: 16 main steps
// js = h*8 + wi*2 + half, plus the min step (js = 16) carrying Sx.
__global__ void x_pack_q4k(const float *__restrict__ x, uint2 *__restrict__ tab, float *__restrict__ inv_scale, int m,
                           int k, int nt_count) {
    const int tk = blockIdx.x, nt = tk >> 2, tl = tk & 3;
    const bool live = tk < m;
    const float *xr = x + (size_t)(live ? tk : 0) * k;
    float s = 0.f, inv = 0.f;
    if (live) {
        act_scale(block_max_abs(xr, k), s, inv);
        if (threadIdx.x == 0) inv_scale[tk] = inv;
    }
    const int nsb = k >> 8;
    for (int e = threadIdx.x; e < nsb * 17 * 8; e += blockDim.x) {
        const int t = e & 3, part = (e >> 2) & 1;
        const int js = (e >> 3) % 17, sb = (e >> 3) / 17;
        const int lane = 4 * (2 * tl + part) + t;
        uint2 v = make_uint2(0u, 0u);
        if (live) {
            const float *xb = xr + (size_t)sb * 256;
            if (js < 16) {
                const int h = js >> 3, wi = (js >> 1) & 3, half = js & 1;
                const int jb = 16 * (t + 4 * h) + 4 * wi;
                auto el = [&](int j) { return 64 * (j >> 5) + (j & 31) + 32 * half; };
                v.x = lc_pack_h2(lc_split_part(xb[el(jb + 0)] * s, part), lc_split_part(xb[el(jb + 2)] * s, part));
                v.y = lc_pack_h2(lc_split_part(xb[el(jb + 1)] * s, part), lc_split_part(xb[el(jb + 3)] * s, part));
            } else {
                float s0 = 0.f, s1 = 0.f;
                for (int i = 0; i < 32; i++) {
                    s0 += xb[32 * (2 * t) + i];
                    s1 += xb[32 * (2 * t + 1) + i];
                }
                // Sx / 32 keeps the scaled 32-element sums inside the f16 range;
                // q4k_unit multiplies dmin by 32 to compensate (both exact)
                v.x = lc_pack_h2(lc_split_part(s0 * s * 0.03125f, part), lc_split_part(s1 * s * 0.03125f, part));
            }
        }
        tab[((size_t)(sb * 17 + js) * nt_count + nt) * 32 + lane] = v;
    }
}

// Q8_0: 2 k-steps per 32-element block; thread t of step ks covers elements
// 16*ks + 4t + {0..3}: b0b1 = (e0, e2), b2b3 = (e1, e3).
__global__ void x_pack_q8(const float *__restrict__ x, uint2 *__restrict__ tab, float *__restrict__ inv_scale, int m,
                          int k, int nt_count) {
    const int tk = blockIdx.x, nt = tk >> 2, tl = tk & 3;
    const bool live = tk < m;
    const float *xr = x + (size_t)(live ? tk : 0) * k;
    float s = 0.f, inv = 0.f;
    if (live) {
        act_scale(block_max_abs(xr, k), s, inv);
        if (threadIdx.x == 0) inv_scale[tk] = inv;
    }
    const int nb = k >> 5;
    for (int e = threadIdx.x; e < nb * 2 * 8; e += blockDim.x) {
        const int t = e & 3, part = (e >> 2) & 1;
        const int ks = (e >> 3) & 1, b = e >> 4;
        const int lane = 4 * (2 * tl + part) + t;
        uint2 v = make_uint2(0u, 0u);
        if (live) {
            const float *xb = xr + (size_t)b * 32 + 16 * ks + 4 * t;
            v.x = lc_pack_h2(lc_split_part(xb[0] * s, part), lc_split_part(xb[2] * s, part));
            v.y = lc_pack_h2(lc_split_part(xb[1] * s, part), lc_split_part(xb[3] * s, part));
        }
        tab[((size_t)(b * 2 + ks) * nt_count + nt) * 32 + lane] = v;
    }
}

// Copy `n16` 16-byte units of the packed table into shared memory.
__device__ __forceinline__ void copy_tab(uint4 *dst, const uint4 *src, int n16) {
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
}

// Cross-warp reduction of the per-thread results and the store.
template <int NT>
__device__ __forceinline__ void reduce_store(float (&acc)[NT][4], float *red, float *c, int m, int n, int row0,
                                             int atomic_out, const float *__restrict__ inv_scale) {
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
            const float inv = inv_scale[tok];
            y0 *= inv;
            y1 *= inv;
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
// Q4_K.
//
// The raw bytes of one 256-element super-block for rows g and g+8 of a
// 16-row tile: headers (d, dmin, 12 scale bytes) and the thread's two 16-byte
// chunks of nibbles (chunks t and t+4 of the 128).
struct Q4Unit {
    uint4 H0, H1, Q0a, Q0b, Q1a, Q1b;
    __device__ __forceinline__ void load(const uint8_t *b0, const uint8_t *b1, int t) {
        H0 = H1 = Q0a = Q0b = Q1a = Q1b = make_uint4(0, 0, 0, 0);
        if (b0) {
            H0 = ldg_stream(b0);
            Q0a = ldg_stream(b0 + 16 + 16 * t);
            Q0b = ldg_stream(b0 + 16 + 16 * (t + 4));
        }
        if (b1) {
            H1 = ldg_stream(b1);
            Q1a = ldg_stream(b1 + 16 + 16 * t);
            Q1b = ldg_stream(b1 + 16 + 16 * (t + 4));
        }
    }
};

// One super-block of one 16-row tile on the tensor cores:
// acc += d * S(sc*q*x) - dmin * S(m*Sx) for rows g, g+8 (c0,c1 / c2,c3).
// tb points at the super-block's 17 k-steps of packed activations
// (NT n-tiles x LANES lanes each).
template <int NT, int LANES>
__device__ __forceinline__ void q4k_unit(const Q4Unit &U, const uint2 *tb, int lane, int half_mode,
                                         float (&acc)[NT][4]) {
    constexpr int kStep = NT * LANES;
    const int t = lane & 3;
    const int p0 = t >> 1;
    const __half2 kNeg1024 = __half2(__float2half_rn(-1024.f), __float2half_rn(-1024.f));
    const __half2 kSixteenth = __half2(__float2half_rn(0.0625f), __float2half_rn(0.0625f));
    const __half2 kNeg64 = __half2(__float2half_rn(-64.f), __float2half_rn(-64.f));
    const __half2 k1024 = __half2(__float2half_rn(1024.f), __float2half_rn(1024.f));
    const float dg = lc_half_to_f32(U.H0.x & 0xFFFFu, half_mode), dmg = lc_half_to_f32(U.H0.x >> 16, half_mode);
    const float dg8 = lc_half_to_f32(U.H1.x & 0xFFFFu, half_mode), dmg8 = lc_half_to_f32(U.H1.x >> 16, half_mode);

    // Scales of this thread's sub-blocks (get_scale_min_k4, proj_q4k.comp:46-58):
    // lo0 = 2p0, hi0 = 2p0+1 (j < 4); lo1 = 2p0+4, hi1 = 2p0+5 (j >= 4).
    __half2 mul[2][4], add[2][4];  // [row g / g+8][lo0, hi0, lo1, hi1]
    uint32_t mpk[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint4 H = r ? U.H1 : U.H0;
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

    // two independent accumulation chains (h = 0 / h = 1) for MMA-level ILP
    float cmh[2][NT][4], cmin[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) cmh[0][i][j] = cmh[1][i][j] = cmin[i][j] = 0.f;

#pragma unroll
    for (int wi = 0; wi < 4; wi++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t xg = u4_get(h ? U.Q0b : U.Q0a, wi), xg8 = u4_get(h ? U.Q1b : U.Q1a, wi);
            const uint32_t xgs = xg >> 8, xg8s = xg8 >> 8;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int si = 2 * h + half;  // lo0, hi0, lo1, hi1
                const uint32_t mask = half ? 0x00F000F0u : 0x000F000Fu;
                const uint32_t a0 =
                    lc_h2_as_u32(__hfma2(lc_u32_as_h2((xg & mask) | 0x64006400u), mul[0][si], add[0][si]));
                const uint32_t a1 =
                    lc_h2_as_u32(__hfma2(lc_u32_as_h2((xg8 & mask) | 0x64006400u), mul[1][si], add[1][si]));
                const uint32_t a2 =
                    lc_h2_as_u32(__hfma2(lc_u32_as_h2((xgs & mask) | 0x64006400u), mul[0][si], add[0][si]));
                const uint32_t a3 =
                    lc_h2_as_u32(__hfma2(lc_u32_as_h2((xg8s & mask) | 0x64006400u), mul[1][si], add[1][si]));
                const int js = h * 8 + wi * 2 + half;
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    uint2 b = make_uint2(0u, 0u);
                    if (LANES == 32 || lane < LANES) b = tb[js * kStep + nt * LANES + lane];
                    lc_mma16816(cmh[h][nt], a0, a1, a2, a3, b.x, b.y);
                }
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        uint2 b = make_uint2(0u, 0u);
        if (LANES == 32 || lane < LANES) b = tb[16 * kStep + nt * LANES + lane];
        lc_mma1688(cmin[nt], mpk[0], mpk[1], b.x);
        // the table carries Sx / 32 (see x_pack_q4k)
        acc[nt][0] += dg * (cmh[0][nt][0] + cmh[1][nt][0]) - 32.f * dmg * cmin[nt][0];
        acc[nt][1] += dg * (cmh[0][nt][1] + cmh[1][nt][1]) - 32.f * dmg * cmin[nt][1];
        acc[nt][2] += dg8 * (cmh[0][nt][2] + cmh[1][nt][2]) - 32.f * dmg8 * cmin[nt][2];
        acc[nt][3] += dg8 * (cmh[0][nt][3] + cmh[1][nt][3]) - 32.f * dmg8 * cmin[nt][3];
    }
}

// Tiled form (any m up to 16 per launch, packed table in global memory).
// Grid: x = 16-row tiles, y = K chunks of sb_per_chunk super-blocks.
// Warp w of the CTA handles super-blocks w, w+kWarps, ... of the chunk.
template <int NT, int LANES>
__global__ void __launch_bounds__(kWarps * 32) q4k_mma_kernel(const uint2 *__restrict__ tab_g,
                                                              const uint8_t *__restrict__ w, float *__restrict__ c,
                                                              int m, int k, int n, int sb_per_chunk, int half_mode,
                                                              int atomic_out, const float *__restrict__ inv_scale) {
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

    for (int sbl = warp; sbl < nloc; sbl += kWarps) {
        const size_t off = (size_t)(sb0 + sbl) * 144;
        Q4Unit U;
        U.load(vg ? wg + off : nullptr, vg8 ? wg8 + off : nullptr, t);
        q4k_unit<NT, LANES>(U, tab + (size_t)sbl * 17 * kStep, lane, half_mode, acc);
    }
    reduce_store<NT>(acc, red, c, m, n, row0, atomic_out, inv_scale);
}

// ---------------------------------------------------------------------------
// Persistent stream-K form for m <= 4 (one n-tile).  One CTA per SM builds
// the packed activation table for the whole K in shared memory, then its
// warps walk equal shares of the flattened (16-row tile, super-block) unit
// space, prefetching the next unit's bytes while the tensor cores work on the
// current one.  A tile whose super-blocks are split between warps is summed
// in `fix_acc` with atomics; the warp that completes the tile's count writes
// the row and leaves fix_acc / fix_cnt zero again for the next call.
constexpr int kSkWarps = 16;

struct Fixup {
    float *acc;       // [tiles][16 rows][4 tokens]
    unsigned *cnt;    // [tiles]
};

// ---------------------------------------------------------------------------
// Integer tensor-core path (m <= 4 tokens).
//
// A is the raw weight integers: Q4_K nibbles become u8 with one mask (low
// nibbles) or a shift and a mask (high nibbles); Q8_0 bytes are used as s8
// unchanged.  B is the activation as a 16-bit integer split into two s8
// digits, x ~= (256*hi + lo) * inv, with one power-free scale per 32-element
// sub-block (inv = max|x| / 32639), so an outlier only coarsens its own
// sub-block.  mma.m16n8k32 (u8 x s8 or s8 x s8 -> s32) sums exactly; k = 32 is
// one sub-block, so the per-sub-block f16 scales are applied once per (row,
// sub-block) in f32.  As in the f16 path, each thread owns B columns
// (2t, 2t+1) = (hi, lo digit) of its own k positions, so the accumulator
// columns a thread holds are the sums over its own sub-block.

__device__ __forceinline__ void lc_imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory layout of the integer stream-K kernels for M tokens and k:
//   [0, 4Mk)          staged x (f32); reused for the B table once digits exist
//   [4Mk, 6Mk)        digits: int8 [M][2][k] (hi, lo)
//   [6Mk, 6Mk + Mk/4) per sub-block (Sx, inv): float2 [M][k/32]
__host__ __device__ __forceinline__ size_t ski_smem_bytes(int m, int k) {
    return (size_t)m * k * 6 + (size_t)m * (k / 32) * 8;
}

// Prologue: stage x, then per 32-element sub-block (one warp each): Sx, scale,
// digits.  Ends with a barrier.
__device__ __forceinline__ void ski_prologue(const float *__restrict__ x, int m, int k, float *xs, int8_t *dig,
                                             float2 *sbi) {
    const bool vec = (((uintptr_t)x) & 15) == 0;
    const int n4 = (m * k) >> 2;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v;
        if (vec) {
            v = __ldg(reinterpret_cast<const float4 *>(x) + i);
        } else {
            v.x = __ldg(x + 4 * i);
            v.y = __ldg(x + 4 * i + 1);
            v.z = __ldg(x + 4 * i + 2);
            v.w = __ldg(x + 4 * i + 3);
        }
        reinterpret_cast<float4 *>(xs)[i] = v;
    }
    __syncthreads();
    // One thread per 32-element sub-block; element e is read at (e + s) mod 32
    // so the 32 threads of a warp hit 32 different banks.
    const int nsub = k >> 5;
    for (int i = threadIdx.x; i < m * nsub; i += blockDim.x) {
        const float *xr = xs + (size_t)i * 32;  // token rows are contiguous: sub-block i of [m*nsub]
        float mx = 0.f, sum = 0.f;
#pragma unroll 8
        for (int e = 0; e < 32; e++) {
            const float v = xr[(e + i) & 31];
            mx = fmaxf(mx, fabsf(v));
            sum += v;
        }
        const bool fin = mx < INFINITY;  // false for inf / nan
        const float scale = (mx > 0.f && fin) ? 32639.f / mx : 0.f;
        const float inv = mx > 0.f ? (fin ? mx * (1.f / 32639.f) : __int_as_float(0x7FC00000)) : 0.f;
        const int tok = i / nsub, s = i - tok * nsub;
        int8_t *dh = dig + ((size_t)tok * 2 + 0) * k + 32 * s;
        int8_t *dl = dig + ((size_t)tok * 2 + 1) * k + 32 * s;
#pragma unroll 8
        for (int e = 0; e < 32; e++) {
            const int ee = (e + i) & 31;
            const int xi = __float2int_rn(xr[ee] * scale);
            const int hi = (xi + 128) >> 8;
            dh[ee] = (int8_t)hi;
            dl[ee] = (int8_t)(xi - (hi << 8));
        }
        sbi[i] = make_float2(sum, inv);
    }
    __syncthreads();
}

// int32 -> f32 without the conversion unit, exact for |v| < 2^22:
// the bits of 1.5 * 2^23 + v, minus 1.5 * 2^23.  Each digit's MMA sum stays
// far below that (Q4_K: 32 * 15 * 128 < 2^16; Q8_0: 32 * 128 * 128 = 2^19),
// so the hi and lo sums are converted separately and combined in f32.
__device__ __forceinline__ float i2f_small(int v) {
    return __int_as_float(v + 0x4B400000) - 12582912.f;
}

__device__ __forceinline__ void lc_imma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void lc_imma_u8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void lc_imma_s8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t dig4(const int8_t *dig, size_t idx) {
    return *reinterpret_cast<const uint32_t *>(dig + idx);
}

// Write (or accumulate) rows g, g+8 of `tile` for the finished part
// [sb_a, sb_b); y holds this thread's partial over its own sub-blocks.
template <int M>
__device__ __forceinline__ void skm_flush(float (&y)[M][2], int tile, int sb_a, int sb_b, int S, int n,
                                          float *__restrict__ out, Fixup fx, int lane) {
    const int g = lane >> 2, t = lane & 3;
    float v0 = 0.f, v1 = 0.f;  // token t's totals after the group reduction
#pragma unroll
    for (int j = 0; j < M; j++) {
        float a = y[j][0], b = y[j][1];
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        if (j == t) v0 = a, v1 = b;
        y[j][0] = y[j][1] = 0.f;
    }
    const bool vt = t < M;
    const int r0 = tile * 16 + g, r1 = r0 + 8;
    if (sb_a == 0 && sb_b == S) {
        if (vt) {
            if (r0 < n) out[(size_t)t * n + r0] = v0;
            if (r1 < n) out[(size_t)t * n + r1] = v1;
        }
        return;
    }
    float *fa = fx.acc + (size_t)tile * 64;
    if (vt) {
        atomicAdd(fa + g * 4 + t, v0);
        atomicAdd(fa + (g + 8) * 4 + t, v1);
    }
    __threadfence();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) {
        const unsigned add = (unsigned)(sb_b - sb_a);
        last = (atomicAdd(fx.cnt + tile, add) + add == (unsigned)S);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    if (vt) {
        const float a = atomicExch(fa + g * 4 + t, 0.f);
        const float b = atomicExch(fa + (g + 8) * 4 + t, 0.f);
        if (r0 < n) out[(size_t)t * n + r0] = a;
        if (r1 < n) out[(size_t)t * n + r1] = b;
    }
    if (lane == 0) atomicExch(fx.cnt + tile, 0u);
}

// ---------------------------------------------------------------------------
// Q4_K GEMV for m <= 4 tokens, weights streamed by TMA.
//
// The weight matrix is a 2D tensor of n rows x (k/256 * 18) u64 words; one
// TMA box is 16 rows x 18 words = one super-block of a 16-row tile (a "unit",
// 2304 B), written to shared memory with a 144-byte row stride.
//
// Work split: CTAs run in clusters of kTmaCluster (one CTA per SM).  Each
// cluster owns a contiguous range of whole 16-row tiles (balanced to one
// tile); the cluster's units, flattened tile-major, are cut into one
// contiguous range per CTA and per consumer warp.  A producer warp fills
// every consumer's ring (R units) at kernel start, so the consumers do not
// block on the TMA queue while they digitise x; after that each consumer
// refills its own ring, one copy per unit consumed.  A consumer accumulates
// the units of one tile in registers and, when the tile changes, adds the
// partial into its CTA's shared-memory accumulator of that tile (f32
// atomics).  After a cluster barrier, each tile's owner CTA sums the
// cluster's accumulators of the tile over distributed shared memory and
// stores the rows.  No split tile crosses a cluster, so nothing goes through
// global memory but the outputs.  (There is no cluster barrier before the
// main loop: its release semantics would wait for the weight copies just
// issued.)
//
// Activations: one scale per (token, super-block): x ~= xi * inv with
// xi = rint(x * 32639 / max|x|) in 16 bits, split into s8 digits
// xi = 256 * hi + lo.  The MMAs (u8 nibbles x s8 digits -> s32) give each
// thread the per-sub-block sums of its own two sub-blocks (2t: low nibbles,
// 2t+1: high nibbles masked in place, i.e. 16x); the 6-bit scales and mins
// are applied in integers:
//   y += d*inv/16 * (256 * A_hi + A_lo) - dmin*inv * B,
//   A_digit = 16*sc_2t*C_2t + sc_2t+1*C16_2t+1,  B = m_2t*X_2t + m_2t+1*X_2t+1,
// with X_s the integer sum of xi over sub-block s.  All integer terms stay
// below 2^31 (|C| <= 32*15*128, sc, m <= 63, |X| <= 32*32639).
constexpr int kTmaUnit = 16 * 144;

struct TmaLayout {
    size_t ring, tab, xs, invs, zero, tacc, bars, total;
};

// Shared memory for NW consumer warps, R stages each, m tokens, k, and at
// most `tl` tiles per cluster:
//   ring  [NW][R][16 rows][144 B]     (128-byte aligned TMA destinations)
//   tab   uint2 [S][2 halves][2 MMA pairs][m][8 lanes][2]  digit fragments
//                                          (see the prologue)
//   xs    int   [m][S][8]                 X of each sub-block
//   invs  float2 [m][S]                   (inv/16, -inv)
//   zero  uint2 [8][m][8]                 B fragment of lanes without one
//   tacc  float [tl][16][m]               this CTA's partial sums of the cluster's tiles
//   bars  uint64 [NW][R]
__host__ __device__ __forceinline__ TmaLayout q4t_layout(int nw, int m, int k, int R, int tl, int unit = kTmaUnit) {
    TmaLayout L;
    const size_t S = (size_t)k / 256;
    L.ring = 0;
    L.tab = L.ring + (size_t)nw * R * unit;
    L.xs = L.tab + S * 64 * m * 8;
    L.invs = L.xs + (size_t)m * S * 32;
    L.zero = (L.invs + (size_t)m * S * 8 + 15) & ~(size_t)15;
    L.tacc = L.zero + (size_t)64 * m * 8;
    L.bars = (L.tacc + (size_t)tl * 16 * m * 4 + 7) & ~(size_t)7;
    L.total = L.bars + (size_t)nw * R * 8 + 128;  // + slack to 128-align the base
    return L;
}

// Add a warp's partial of one tile (rows g, g+8 per thread, summed over the
// thread's sub-blocks; each a (main, min) pair) into this CTA's accumulator
// `ta` of the tile, and clear the partial.
template <int M>
__device__ __forceinline__ void q4t_tile_add(float2 (&acc)[M][2], float *ta, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < M; j++) {
        float a = acc[j][0].x + acc[j][0].y, b = acc[j][1].x + acc[j][1].y;
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        b += __shfl_xor_sync(0xffffffffu, b, 1);
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        if (t == j) {
            atomicAdd(ta + g * M + j, a);
            atomicAdd(ta + (g + 8) * M + j, b);
        }
        acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);
    }
}

// Prologue: one warp per item (token j, super-block sb).  Lane l converts
// elements 8l..8l+7 of the super-block, which are exactly the 8 k positions of
// table entry (MMA half*4 + i, owner t) with t = l/8, half = (l/4)&1, i = l&3;
// it writes that entry's hi (e = 2t) and lo (e = 2t+1) digit words and, with
// its 3 neighbours, the integer sum of sub-block l/4 = 2t + half.  The loads
// are split from the conversion so a warp can issue its first items' loads
// before anything else.
constexpr int kXPre = 4;  // items per warp whose x loads are issued early

__device__ __forceinline__ void q4t_xload(const float *__restrict__ x, int k, int S, int it, float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    const int j = it / S, sb = it - j * S;
    const float *xp = x + (size_t)j * k + (size_t)sb * 256 + 8 * lane;
    if ((((uintptr_t)x) & 15) == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(xp));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(xp) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __ldg(xp + e);
    }
}

template <int M, bool Q8 = false>
__device__ __forceinline__ void q4t_digitize(const float (&v)[8], int S, int it, uint2 *tab, int *xs, float2 *invs) {
    const int lane = threadIdx.x & 31;
    const int j = it / S, sb = it - j * S;
    float mx = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) mx = fmaxf(mx, fabsf(v[e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const bool fin = mx < INFINITY;  // false for inf / nan
    const float scale = (mx > 0.f && fin) ? 32639.f / mx : 0.f;
    const float inv = mx > 0.f ? (fin ? mx * (1.f / 32639.f) : __int_as_float(0x7FC00000)) : 0.f;
    uint32_t h[2] = {0u, 0u}, l[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int xi = __float2int_rn(v[e] * scale);
        const int hi = (xi + 128) >> 8;
        const int lo = xi - (hi << 8);
        sum += xi;
        h[e >> 2] |= (uint32_t)(hi & 0xFF) << (8 * (e & 3));
        l[e >> 2] |= (uint32_t)(lo & 0xFF) << (8 * (e & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    // entry (sb, half, MMA i, token j, e) at uint2 index
    // ((((sb*2 + half)*2 + i/2)*M + j)*8 + e)*2 + i%2: MMAs i and i+1 of a
    // lane are one 16-byte load.  Q4_K: owner t = l/8, half (low / high
    // nibbles) = (l/4)&1.  Q8_0: elements 8l.. are block l/4, so the owner is
    // t = (l/4)&3 and the half (blocks 0-3 / 4-7) is l/16.
    const int t = Q8 ? (lane >> 2) & 3 : lane >> 3, half = Q8 ? lane >> 4 : (lane >> 2) & 1, i = lane & 3;
    uint2 *ent = tab + ((((size_t)(sb * 2 + half) * 2 + (i >> 1)) * M + j) * 8 + 2 * t) * 2 + (i & 1);
    ent[0] = make_uint2(h[0], h[1]);
    ent[2] = make_uint2(l[0], l[1]);
    // xs[(j*S + sb)*8 + 2t + half]: the pair (X_2t, X_2t+1) of owner t is one int2
    if ((lane & 3) == 0) xs[((size_t)j * S + sb) * 8 + (lane >> 2)] = sum;
    if (lane == 0) invs[(size_t)j * S + sb] = make_float2(inv * 0.0625f, -inv);
}

// Lane constants of the scale / min byte extraction (get_scale_min_k4,
// proj_q4k.comp:46-58) for sub-blocks 2t, 2t+1: t < 2 takes the 6-bit
// q[2t], q[2t+1] and q[2t+4], q[2t+5]; t >= 2 combines the low / high nibbles
// of q[2t+4], q[2t+5] with the top two bits of q[2t-4], q[2t-3] (scales) or
// q[2t], q[2t+1] (mins).
struct Q4ScaleSel {
    uint32_t perm, mlo, mhi;
    bool lo;  // t < 2
    __device__ __forceinline__ Q4ScaleSel(int t) {
        perm = (t & 1) ? 0x7632u : 0x5410u;  // bytes 2u, 2u+1 of row 0, then of row 1
        lo = t < 2;
        mlo = lo ? 0x3F3F3F3Fu : 0x0F0F0F0Fu;
        mhi = lo ? 0u : 0x30303030u;
    }
    // (sc, m) of both rows: bytes (row0 2t, row0 2t+1, row1 2t, row1 2t+1)
    __device__ __forceinline__ void get(const uint4 &H0, const uint4 &H1, uint32_t &sc4, uint32_t &mn4) const {
        const uint32_t py = __byte_perm(H0.y, H1.y, perm);
        const uint32_t pz = __byte_perm(H0.z, H1.z, perm);
        const uint32_t pw = __byte_perm(H0.w, H1.w, perm);
        sc4 = ((lo ? py : pw) & mlo) | ((py >> 2) & mhi);
        mn4 = ((lo ? pz : pw >> 4) & mlo) | ((pz >> 2) & mhi);
    }
};

// One unit from shared memory: rows g, g+8 of the stage at `st`.  tbl4: this
// lane's B fragments of the super-block (MMAs 2p, 2p+1 at tbl4[((half*2+p)*M
// + j)*8]).  For m <= 2 only the lanes that own a fragment (`own`) load it
// into bf and the others keep bf at zero; for m > 2 those persistent zero
// fragments would cost too many registers, so every lane loads, the
// non-owners from the zero block `zb`.  xs2 / iv2: (X_2t, X_2t+1) and
// (inv/16, -inv) of token 0, tokens S*4 int2 / S float2 apart.  y[j][r]
// accumulates the (main, min) terms of row g + 8r, summed at the end.
template <int M>
__device__ __forceinline__ void q4t_unit(const uint8_t *st, const uint4 *tbl4, const uint4 *zb, bool own,
                                         uint4 (&bf)[2][2][M], const int2 *xs2, const float2 *iv2, int S,
                                         uint32_t ref_mask, int g, int t, const Q4ScaleSel &sel, float2 (&y)[M][2]) {
    const uint8_t *r0 = st + g * 144, *r1 = st + (g + 8) * 144;
    const uint4 H0 = lds128(r0), H1 = lds128(r1);
    const uint4 A0 = lds128(r0 + 16 + 32 * t), B0 = lds128(r0 + 32 + 32 * t);
    const uint4 A1 = lds128(r1 + 16 + 32 * t), B1 = lds128(r1 + 32 + 32 * t);
#pragma unroll
    for (int half = 0; half < 2; half++)
#pragma unroll
        for (int p = 0; p < 2; p++)
#pragma unroll
            for (int j = 0; j < M; j++) {
                const int o = ((half * 2 + p) * M + j) * 8;
                if constexpr (M <= 2)
                    lds128_if(own, bf[half][p][j], tbl4 + o);
                else
                    bf[half][p][j] = lds128(own ? tbl4 + o : zb + o);
            }
    int c[2][M][4];
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint32_t mask = half ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
#pragma unroll
        for (int p = 0; p < 2; p++) {
            const uint4 &Pg = p ? B0 : A0;
            const uint4 &Pg8 = p ? B1 : A1;
#pragma unroll
            for (int j = 0; j < M; j++) {
                const uint4 &b = bf[half][p][j];
                if (p == 0)
                    lc_imma_u8s8_z(c[half][j], Pg.x & mask, Pg8.x & mask, Pg.y & mask, Pg8.y & mask, b.x, b.y);
                else
                    lc_imma_u8s8(c[half][j], Pg.x & mask, Pg8.x & mask, Pg.y & mask, Pg8.y & mask, b.x, b.y);
                lc_imma_u8s8(c[half][j], Pg.z & mask, Pg8.z & mask, Pg.w & mask, Pg8.w & mask, b.z, b.w);
            }
        }
    }
    uint32_t sc4, mn4;
    sel.get(H0, H1, sc4, mn4);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const float2 dd = scales2_f32(r ? H1.x : H0.x, ref_mask);  // (d, dmin)
        const uint32_t scr = sc4 >> (16 * r), mnr = mn4 >> (16 * r);
        const int sc0x16 = (int)((scr << 4) & 0xFF0u), sc1 = (int)((scr >> 8) & 0xFFu);
        const int mn0 = (int)(mnr & 0xFFu), mn1 = (int)((mnr >> 8) & 0xFFu);
#pragma unroll
        for (int j = 0; j < M; j++) {
            const int2 X = xs2[(size_t)j * S * 4];
            const float2 iv = iv2[(size_t)j * S];
            const int a_hi = sc0x16 * c[0][j][2 * r] + sc1 * c[1][j][2 * r];
            const int a_lo = sc0x16 * c[0][j][2 * r + 1] + sc1 * c[1][j][2 * r + 1];
            const int bm = mn0 * X.x + mn1 * X.y;
            const float a = fmaf(__int2float_rn(a_hi), 256.f, __int2float_rn(a_lo));
            // (main, min) += (d*inv/16, -dmin*inv) * (a, bm)
            y[j][r] = ffma2(fmul2(dd, iv), make_float2(a, __int2float_rn(bm)), y[j][r]);
        }
    }
}

// Weight formats of the TMA GEMV: one unit is 16 rows x 256 elements.
struct FmtQ4K {
    static constexpr int kUnit = 16 * 144;  // one super-block per row
    static constexpr int kBoxX = 18;        // u64 words per unit row
    static constexpr bool kQ8 = false;
};
struct FmtQ8_0 {
    static constexpr int kUnit = 16 * 272;  // eight 34-byte blocks per row
    static constexpr int kBoxX = 136;       // u16 words per unit row
    static constexpr bool kQ8 = true;
};

// One Q8_0 unit (rows g, g+8; blocks 0..7 of the 272-byte unit rows).  Thread t
// owns blocks t and 4+t: its k slots in MMA (h, i) are elements 8i..8i+7 of
// block 4h+t, so after the four MMAs of a half its accumulator columns hold the
// whole block's digit sums, and the block's f16 scale d is applied once per
// (row, block): y += d * inv * (256 * S_hi + S_lo).  The q bytes of block b
// start at byte 34b + 2 of the row (2 bytes off word alignment for even b):
// nine aligned words and a funnel shift give them.
template <int M>
__device__ __forceinline__ void q8t_unit(const uint8_t *st, const uint4 *tbl4, const uint4 *zb, bool own,
                                         uint4 (&bf)[2][2][M], const float2 *iv2, int S, uint32_t ref_mask, int g,
                                         int t, float2 (&y)[M][2]) {
#pragma unroll
    for (int half = 0; half < 2; half++)
#pragma unroll
        for (int p = 0; p < 2; p++)
#pragma unroll
            for (int j = 0; j < M; j++) {
                const int o = ((half * 2 + p) * M + j) * 8;
                if constexpr (M <= 2)
                    lds128_if(own, bf[half][p][j], tbl4 + o);
                else
                    bf[half][p][j] = lds128(own ? tbl4 + o : zb + o);
            }
    const int qsh = (t & 1) ? 0 : 16;        // bit shift of block t's q bytes
    const int qw = (34 * t + 2) >> 2;        // first word of block t's q bytes
    int c[2][M][4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t q[2][8];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(st + (g + 8 * r) * 272) + 34 * h + qw;
            uint32_t W[9];
#pragma unroll
            for (int i = 0; i < 8; i++) W[i] = lds32(w + i);
            W[8] = qsh ? lds32(w + 8) : 0u;  // odd t: aligned, the ninth word is not needed
#pragma unroll
            for (int i = 0; i < 8; i++) q[r][i] = __funnelshift_r(W[i], W[i + 1], qsh);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int j = 0; j < M; j++) {
                const uint4 &b = bf[h][i >> 1][j];
                const uint32_t b0 = (i & 1) ? b.z : b.x, b1 = (i & 1) ? b.w : b.y;
                if (i == 0)
                    lc_imma_s8s8_z(c[h][j], q[0][2 * i], q[1][2 * i], q[0][2 * i + 1], q[1][2 * i + 1], b0, b1);
                else
                    lc_imma_s8s8(c[h][j], q[0][2 * i], q[1][2 * i], q[0][2 * i + 1], q[1][2 * i + 1], b0, b1);
            }
        }
    }
    // d of blocks t and 4+t: the half at byte 34t (word 34t/4, high half for
    // odd t) and at byte 136 + 34t
    const int dw = (34 * t) >> 2;
    const uint32_t dperm = (t & 1) ? 0x7632u : 0x5410u;
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(st + (g + 8 * r) * 272);
        const float2 dd = scales2_f32(__byte_perm(lds32(w + dw), lds32(w + 34 + dw), dperm), ref_mask);
#pragma unroll
        for (int j = 0; j < M; j++) {
            const float inv = -iv2[(size_t)j * S].y;
            const float s0 = fmaf(i2f_small(c[0][j][2 * r]), 256.f, i2f_small(c[0][j][2 * r + 1]));
            const float s1 = fmaf(i2f_small(c[1][j][2 * r]), 256.f, i2f_small(c[1][j][2 * r + 1]));
            y[j][r] = ffma2(fmul2(dd, make_float2(inv, inv)), make_float2(s0, s1), y[j][r]);
        }
    }
}

// NW consumer warps + one producer warp (warp NW) per CTA.
template <class F, int M, int NW, int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__((NW + 1) * 32, 1)
    tma_gemv_kernel(const __grid_constant__ CUtensorMap tm, const float *__restrict__ x, float *__restrict__ y, int k,
                    int n, int half_mode, int R, int tl, unsigned *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // The same offset on every CTA (the dynamic window starts at the same
    // shared address), so a partner's accumulator is at our own offset.
    unsigned char *smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    cg::cluster_group cluster = cg::this_cluster();
    const int S = k >> 8;
    constexpr int kUnit = F::kUnit;
    const TmaLayout L = q4t_layout(NW, M, k, R, tl, kUnit);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    uint2 *tab = reinterpret_cast<uint2 *>(smem + L.tab);
    int *xs = reinterpret_cast<int *>(smem + L.xs);
    float2 *invs = reinterpret_cast<float2 *>(smem + L.invs);
    uint2 *zbuf = reinterpret_cast<uint2 *>(smem + L.zero);
    float *tacc = reinterpret_cast<float *>(smem + L.tacc);
    uint64_t *bars_all = reinterpret_cast<uint64_t *>(smem + L.bars);

    // cluster -> whole tiles; CTA -> contiguous units; warp -> contiguous
    // units.  32-bit arithmetic (the host keeps T*C and T*S*NW below 2^31);
    // CL and NW are compile-time divisors.
    const int rank = (int)cluster.block_rank();
    const int C = gridDim.x / CL, cid = blockIdx.x / CL;
    const int T = (n + 15) >> 4;
    const int tc0 = T * cid / C, tc1 = T * (cid + 1) / C;
    const int uc0 = tc0 * S, ucn = (tc1 - tc0) * S;
    const int U0 = uc0 + ucn * rank / CL, nU = uc0 + ucn * (rank + 1) / CL - U0;
    const int wq = warp < NW ? warp : 0;
    const int w0 = U0 + nU * wq / NW;
    const int my_units = warp < NW ? U0 + nU * (wq + 1) / NW - w0 : 0;
    const uint64_t pol = l2_evict_first_policy();

    float xv[kXPre][8];
    if (warp < NW) {
        // x loads of this warp's first prologue items go out first
#pragma unroll
        for (int p = 0; p < kXPre; p++)
            if (warp + p * NW < M * S) q4t_xload(x, k, S, warp + p * NW, xv[p]);
        if (lane < R) mbar_init(bars_all + warp * R + lane, 1);
        mbar_init_fence();
    } else if (lane == 0) {
        prefetch_tensormap(&tm);
    }
    __syncthreads();  // barriers initialised

    if (warp == NW) {
        // producer: the first R units of every consumer, consumer w on lane w
        if (lane < NW) {
            const int a = U0 + nU * lane / NW, cnt = U0 + nU * (lane + 1) / NW - a;
            int tile = a / S, sb = a - (a / S) * S;
            uint8_t *ring = smem + L.ring + (size_t)lane * R * kUnit;
            for (int q = 0; q < R && q < cnt; q++) {
                mbar_expect_tx(bars_all + lane * R + q, kUnit);
                tma_load_2d(ring + (size_t)q * kUnit, &tm, sb * F::kBoxX, tile * 16, bars_all + lane * R + q, pol);
                if (++sb == S) sb = 0, ++tile;
            }
        }
    } else {
        for (int i = threadIdx.x; i < 64 * M; i += NW * 32) zbuf[i] = make_uint2(0u, 0u);
        for (int i = threadIdx.x; i < tl * 16 * M; i += NW * 32) tacc[i] = 0.f;
#pragma unroll
        for (int p = 0; p < kXPre; p++)
            if (warp + p * NW < M * S) q4t_digitize<M, F::kQ8>(xv[p], S, warp + p * NW, tab, xs, invs);
        for (int it = warp + kXPre * NW; it < M * S; it += NW) {
            float v[8];
            q4t_xload(x, k, S, it, v);
            q4t_digitize<M, F::kQ8>(v, S, it, tab, xs, invs);
        }
        named_barrier_sync(NW * 32);  // consumers only: the table is complete
    }

    uint8_t *ring = smem + L.ring + (size_t)wq * R * kUnit;
    uint64_t *bars = bars_all + wq * R;
    // consumer refills continue after the producer's first R units
    int issued = min(R, my_units), istage = issued == R ? 0 : issued;
    int itile = (w0 + issued) / S, isb = (w0 + issued) - ((w0 + issued) / S) * S;
    auto issue = [&]() {
        tma_unit_lane0(lane, ring + (size_t)istage * kUnit, &tm, isb * F::kBoxX, itile * 16, bars + istage, pol,
                       kUnit);
        if (++istage == R) istage = 0;
        if (++isb == S) isb = 0, ++itile;
        ++issued;
    };

    const bool own = (g >> 1) == t;
    const uint32_t ref_mask = half_mode == LC_HALF_REF ? 0x04000400u : 0u;
    const int2 *xs2 = reinterpret_cast<const int2 *>(xs) + t;
    const Q4ScaleSel sel(t);
    // B fragments: own lanes load their entry of the table; the others keep zeros
    const uint4 *tab4 = reinterpret_cast<const uint4 *>(tab) + g;
    const uint4 *zb4 = reinterpret_cast<const uint4 *>(zbuf);
    uint4 bf[2][2][M];
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int p = 0; p < 2; p++)
#pragma unroll
            for (int j = 0; j < M; j++) bf[h][p][j] = make_uint4(0u, 0u, 0u, 0u);
    float2 acc[M][2];
#pragma unroll
    for (int j = 0; j < M; j++) acc[j][0] = acc[j][1] = make_float2(0.f, 0.f);
    int tile = w0 / S, sb = w0 - (w0 / S) * S, s = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int q = 0; q < my_units; q++) {
        // all lanes wait on the same barrier; the vote keeps the outcome warp-uniform
        if (!__all_sync(0xffffffffu, mbar_wait(bars + s, phase))) {
            ok = false;
            break;
        }
        if constexpr (F::kQ8)
            q8t_unit<M>(ring + (size_t)s * kUnit, tab4 + (size_t)sb * 32 * M, zb4, own, bf, invs + sb, S, ref_mask,
                        g, t, acc);
        else
            q4t_unit<M>(ring + (size_t)s * kUnit, tab4 + (size_t)sb * 32 * M, zb4, own, bf, xs2 + (size_t)sb * 4,
                        invs + sb, S, ref_mask, g, t, sel, acc);
        // the stage's bytes are in registers and consumed (the MMAs and the
        // epilogue above depend on them): hand the stage to the next copy
        __syncwarp();
        if (issued < my_units) issue();
        if (++s == R) s = 0, phase ^= 1u;
        if (++sb == S || q == my_units - 1) {
            q4t_tile_add<M>(acc, tacc + (size_t)(tile - tc0) * 16 * M, lane);
            if (sb == S) sb = 0, ++tile;
        }
    }
    if (!ok) {
        // A wait gave up: record it, then let this warp's copies in flight
        // land (bounded) before the CTA's shared memory is released.
        if (lane == 0) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        for (int st = 0; st < R; st++) {
            const int last = issued - 1 - ((issued - 1 - st) % R + R) % R;  // newest unit issued to stage st
            if (last >= 0) mbar_wait(bars + st, (uint32_t)(last / R) & 1u);
        }
    }
    // every CTA's partials are complete; each tile's owner sums the cluster's
    // copies (distributed shared memory) and stores the rows
    cluster.sync();
    {
        const float *part[CL];
#pragma unroll
        for (int c = 0; c < CL; c++) part[c] = cluster.map_shared_rank(tacc, c);
        const int ntile = tc1 - tc0, nown = ntile > rank ? (ntile - rank + CL - 1) / CL : 0;
        for (int idx = threadIdx.x; idx < nown * 16 * M; idx += blockDim.x) {
            const int q = idx / (16 * M), e = idx - q * 16 * M;
            const int lt = rank + q * CL, r = e / M, j = e - r * M, row = (tc0 + lt) * 16 + r;
            float v = 0.f;
#pragma unroll
            for (int c = 0; c < CL; c++) v += part[c][(size_t)lt * 16 * M + e];
            if (row < n) y[(size_t)j * n + row] = v;
        }
    }
    // partners' shared memory stays alive until every owner has read it
    cluster.sync();
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

// The words of one block pair that thread (g, t) needs for rows g and g+8.
struct Q8Unit {
    uint32_t wd[2][8];
    __device__ __forceinline__ void load(const uint8_t *b0, const uint8_t *b1, int t) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint8_t *b = r ? b1 : b0;
            if (b) {
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
    }
};

// One block pair (two 32-element blocks) of a 16-row tile: acc += d * S(q*x)
// per block.  tb points at the pair's 4 k-steps of packed activations.
template <int NT, int LANES>
__device__ __forceinline__ void q8_unit(const Q8Unit &U, const uint2 *tb, int lane, int half_mode,
                                        float (&acc)[NT][4]) {
    constexpr int kStep = NT * LANES;
    const float dA0 = lc_half_to_f32(U.wd[0][6] & 0xFFFFu, half_mode);
    const float dB0 = lc_half_to_f32(U.wd[0][7] >> 16, half_mode);
    const float dA1 = lc_half_to_f32(U.wd[1][6] & 0xFFFFu, half_mode);
    const float dB1 = lc_half_to_f32(U.wd[1][7] >> 16, half_mode);
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
        float cm[NT][4];
#pragma unroll
        for (int i = 0; i < NT; i++) cm[i][0] = cm[i][1] = cm[i][2] = cm[i][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ks++) {
            uint32_t q0, q1;
            if (blk == 0) {
                q0 = __funnelshift_r(U.wd[0][2 * ks], U.wd[0][2 * ks + 1], 16);
                q1 = __funnelshift_r(U.wd[1][2 * ks], U.wd[1][2 * ks + 1], 16);
            } else {
                q0 = U.wd[0][4 + ks];
                q1 = U.wd[1][4 + ks];
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

template <int NT, int LANES>
__global__ void __launch_bounds__(kWarps * 32) q8_mma_kernel(const uint2 *__restrict__ tab_g,
                                                             const uint8_t *__restrict__ w, float *__restrict__ c,
                                                             int m, int k, int n, int pairs_per_chunk,
                                                             int half_mode, int atomic_out,
                                                             const float *__restrict__ inv_scale) {
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
    const size_t rowbytes = (size_t)npairs * 68;

    copy_tab(reinterpret_cast<uint4 *>(tab), reinterpret_cast<const uint4 *>(tab_g + (size_t)p0 * 4 * kStep),
             nloc * 4 * kStep / 2);
    __syncthreads();

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (int pl = warp; pl < nloc; pl += kWarps) {
        const size_t off = (size_t)(p0 + pl) * 68;
        Q8Unit U;
        U.load(rg < n ? w + (size_t)rg * rowbytes + off : nullptr, rg8 < n ? w + (size_t)rg8 * rowbytes + off : nullptr,
               t);
        q8_unit<NT, LANES>(U, tab + (size_t)pl * 4 * kStep, lane, half_mode, acc);
    }
    reduce_store<NT>(acc, red, c, m, n, row0, atomic_out, inv_scale);
}

// The words of one Q8_0 block pair (68 B) that thread (g, t) needs for rows g
// and g+8: q_A[8t..8t+7] (pair bytes 2+8t.., words 2t..2t+2), q_B[8t..8t+7]
// (words 9+2t, 10+2t), d_A (word 0 low half), d_B (word 8 high half).
struct Q8UnitI {
    uint32_t w[2][7];
    __device__ __forceinline__ void load(const uint8_t *b0, const uint8_t *b1, int t) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint8_t *b = r ? b1 : b0;
            if (b) {
                w[r][0] = ldg_u32(b + 8 * t);
                w[r][1] = ldg_u32(b + 8 * t + 4);
                w[r][2] = ldg_u32(b + 8 * t + 8);
                w[r][3] = ldg_u32(b + 36 + 8 * t);
                w[r][4] = ldg_u32(b + 40 + 8 * t);
                w[r][5] = ldg_u32(b);
                w[r][6] = ldg_u32(b + 32);
            } else {
#pragma unroll
                for (int i = 0; i < 7; i++) w[r][i] = 0u;
            }
        }
    }
};

// One Q8_0 block pair of a 16-row tile, integer MMAs (one k = 32 MMA per
// block and token).  sb4: float4 (Sx, inv of block 2p, Sx, inv of block 2p+1).
template <int M>
__device__ __forceinline__ void q8_unit_int(const Q8UnitI &U, const uint2 *tbl, const float4 *sb4, int sb4_stride,
                                            uint32_t ref_mask, float (&y)[M][2]) {
    int c[2][M][4];
#pragma unroll
    for (int blk = 0; blk < 2; blk++) {
        uint32_t a0, a1, a2, a3;
        if (blk == 0) {
            a0 = __funnelshift_r(U.w[0][0], U.w[0][1], 16);
            a2 = __funnelshift_r(U.w[0][1], U.w[0][2], 16);
            a1 = __funnelshift_r(U.w[1][0], U.w[1][1], 16);
            a3 = __funnelshift_r(U.w[1][1], U.w[1][2], 16);
        } else {
            a0 = U.w[0][3];
            a2 = U.w[0][4];
            a1 = U.w[1][3];
            a3 = U.w[1][4];
        }
#pragma unroll
        for (int j = 0; j < M; j++) {
            const uint2 b = tbl[(blk * M + j) * 8];
            lc_imma_s8s8_z(c[blk][j], a0, a1, a2, a3, b.x, b.y);
        }
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
        // d_A: low half of word 0; d_B: high half of word 8
        const float2 dd = scales2_f32(__byte_perm(U.w[r][5], U.w[r][6], 0x7610), ref_mask);
#pragma unroll
        for (int j = 0; j < M; j++) {
            const float4 f = sb4[j * sb4_stride];
            const float sA = fmaf(i2f_small(c[0][j][2 * r]), 256.f, i2f_small(c[0][j][2 * r + 1]));
            const float sB = fmaf(i2f_small(c[1][j][2 * r]), 256.f, i2f_small(c[1][j][2 * r + 1]));
            y[j][r] = fmaf(dd.y * f.w, sB, fmaf(dd.x * f.y, sA, y[j][r]));
        }
    }
}

// Persistent stream-K Q8_0 projection for M <= 4 tokens (one CTA per SM, x
// digitised into shared memory, warps on equal shares of the flattened units);
// units are (16-row tile, block pair).
template <int M>
__global__ void __launch_bounds__(kSkWarps * 32, 1) q8_sk_kernel(const float *__restrict__ x,
                                                                 const uint8_t *__restrict__ w,
                                                                 float *__restrict__ y, int k, int n,
                                                                 int half_mode, Fixup fx) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int S = k >> 6;  // block pairs per row
    float *xs = reinterpret_cast<float *>(smem);
    uint2 *tab = reinterpret_cast<uint2 *>(smem);  // replaces xs: [S][2][M][8]
    int8_t *dig = reinterpret_cast<int8_t *>(smem + (size_t)M * k * 4);
    float2 *sbi = reinterpret_cast<float2 *>(smem + (size_t)M * k * 6);
    __shared__ __align__(16) uint2 zbuf[2 * M * 8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const size_t rowbytes = (size_t)S * 68;
    const int T = (n + 15) >> 4;
    const long long TS = (long long)T * S;
    const long long Wt = (long long)gridDim.x * kSkWarps;
    const long long wid = (long long)blockIdx.x * kSkWarps + warp;
    const long long u0 = TS * wid / Wt;
    const int n_units = (int)(TS * (wid + 1) / Wt - u0);
    int tile = (int)(u0 / S), sub = (int)(u0 % S);

    int pt = tile, ps = sub, loaded = 0;
    auto load_next = [&](Q8UnitI &U) {
        if (loaded >= n_units) return;
        const int rg = pt * 16 + g, rg8 = rg + 8;
        U.load(rg < n ? w + (size_t)rg * rowbytes + (size_t)ps * 68 : nullptr,
               rg8 < n ? w + (size_t)rg8 * rowbytes + (size_t)ps * 68 : nullptr, t);
        if (++ps == S) ps = 0, ++pt;
        ++loaded;
    };
    Q8UnitI A, B, C;  // three units in flight per warp
    load_next(A);
    load_next(B);
    load_next(C);

    for (int i = threadIdx.x; i < 2 * M * 8; i += blockDim.x) zbuf[i] = make_uint2(0u, 0u);
    ski_prologue(x, M, k, xs, dig, sbi);
    // Table entry (pair p, block blk, token j, e = 2*owner + digit): the
    // owner's 8 k positions are elements 64p + 32blk + 8owner + 0..7.
    for (int idx = threadIdx.x; idx < S * 2 * M * 8; idx += blockDim.x) {
        const int e = idx & 7;
        const int j = (idx >> 3) % M;
        const int blk = (idx / (8 * M)) & 1;
        const int p = idx / (16 * M);
        const int to = e >> 1, dg = e & 1;
        const size_t base = ((size_t)j * 2 + dg) * k + (size_t)p * 64 + 32 * blk + 8 * to;
        tab[idx] = make_uint2(dig4(dig, base), dig4(dig, base + 4));
    }
    __syncthreads();

    const bool own = (g >> 1) == t;
    const int sb4_stride = k >> 6;
    float acc[M][2];
#pragma unroll
    for (int j = 0; j < M; j++) acc[j][0] = acc[j][1] = 0.f;
    const uint32_t ref_mask = half_mode == LC_HALF_REF ? 0x04000400u : 0u;
    int seg0 = sub, done = 0;
    auto step = [&](Q8UnitI &U) {
        const uint2 *tbl = own ? tab + (size_t)sub * 16 * M + g : zbuf;
        q8_unit_int<M>(U, tbl, reinterpret_cast<const float4 *>(sbi) + sub, sb4_stride, ref_mask, acc);
        load_next(U);
        ++done;
        if (sub == S - 1 || done == n_units) {
            skm_flush<M>(acc, tile, seg0, sub + 1, S, n, y, fx, lane);
            seg0 = 0;
        }
        if (++sub == S) sub = 0, ++tile;
    };
    while (done < n_units) {
        step(A);
        if (done == n_units) break;
        step(B);
        if (done == n_units) break;
        step(C);
    }
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
    if (bytes > 48 * 1024) return lc_set_smem_attr((const void *)kernel, bytes);
    return LC_OK;
}

constexpr size_t kTabSmemBudget = 100 * 1024;

template <int NT, int LANES>
int launch_q4k(lc_ctx *ctx, const uint2 *tab, const float *inv_scale, const uint8_t *w, float *c, int m, int k, int n) {
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
                                                                         kch > 1, inv_scale);
    return LC_OK;
}

// TMA tensor maps are encoded with the driver's cuTensorMapEncodeTiled,
// resolved once through the runtime (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out) {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_tiled = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    });
    LC_REQUIRE(g_encode_tiled, LC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    *out = g_encode_tiled;
    return LC_OK;
}

// Quantized weights [n rows] as a 2D tensor whose box is one unit: 16 rows x
// 256 elements (Q4_K: one 144-byte super-block = 18 u64 words; Q8_0: eight
// 34-byte blocks = 136 u16 words).  Rows past n read as zero.
template <class F>
int tma_tensor_map(CUtensorMap *tm, const void *w, uint32_t k, uint32_t n) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    int s = tensor_map_encoder(&enc);
    if (s) return s;
    const cuuint64_t S = k / 256;
    cuuint64_t dims[2] = {S * F::kBoxX, (cuuint64_t)n};
    cuuint64_t strides[1] = {S * (F::kUnit / 16)};
    cuuint32_t box[2] = {(cuuint32_t)F::kBoxX, 16};
    cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType dt = F::kQ8 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT64;
    const CUresult r = enc(tm, dt, 2, const_cast<void *>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    LC_REQUIRE(r == CUDA_SUCCESS, LC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for k=%u n=%u", (int)r, k, n);
    return LC_OK;
}

// Consumer warps per CTA (+ 1 producer warp = 512 threads, <= 128 registers).
// More warps (20 at <= 96 registers for one token) measured slower.
__host__ __device__ constexpr int q4t_warps(int) { return 15; }
// Clusters of 2: more of them are co-resident than clusters of 4 (which left 16 of the
// 148 SMs idle), at a slightly coarser split of the tiles (9.6 against 10.2 us per Q4_K
// 4096->14336 launch at m = 1).
constexpr int kTmaCluster = 2;
// Units in flight per consumer warp.  Two measured fastest on B200 (Q4_K 4096->14336
// at m = 1: 10.2 us with 2, 10.5 with 3, 12.2 with 4, 13.3 with 6 per launch): the
// 15 warps x 2 units already keep ~69 KB per SM in flight, and deeper rings only
// lengthen the producer's start-up fill.
constexpr int kTmaMaxStages = 2;

// Launch geometry of the TMA GEMV: clusters, ring depth, tiles per cluster.
struct TmaPlan {
    int grid = 0, R = 0, tl = 0;
    size_t smem = 0;
};

template <class F, int M>
int tma_max_clusters(size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({dev, smem});
    if (it != cache.end()) return it->second;
    constexpr int NW = q4t_warps(M);
    int s = set_smem(tma_gemv_kernel<F, M, NW, kTmaCluster>, smem);
    if (s) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kTmaCluster * 64, 1, 1);
    cfg.blockDim = dim3((NW + 1) * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, tma_gemv_kernel<F, M, NW, kTmaCluster>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        nc = 0;
    }
    cache[{dev, smem}] = nc;
    return nc;
}

template <class F>
int tma_max_clusters_m(int m, size_t smem) {
    switch (m) {
    case 1: return tma_max_clusters<F, 1>(smem);
    case 2: return tma_max_clusters<F, 2>(smem);
    case 3: return tma_max_clusters<F, 3>(smem);
    default: return tma_max_clusters<F, 4>(smem);
    }
}

// R = 0 when the shapes do not fit (the caller falls back).
template <class F>
TmaPlan tma_plan(const lc_ctx *ctx, int m, int k, int n) {
    TmaPlan p;
    const int T = (n + 15) / 16;
    const int nw = q4t_warps(m);
    // the kernel's 32-bit range arithmetic
    if ((long long)T * (k / 256) * nw >= (1ll << 31) || (long long)T * ctx->num_sms >= (1ll << 31)) return p;
    const int c_sms = std::max(1, ctx->num_sms / kTmaCluster);
    for (int R = kTmaMaxStages; R >= 2; R--) {
        const int C0 = std::min(T, c_sms);
        const int tl = (T + C0 - 1) / C0;
        const size_t b = q4t_layout(nw, m, k, R, tl, F::kUnit).total;
        if (b > ctx->smem_optin) continue;
        // only as many clusters as can be resident at once (one wave)
        const int nc = tma_max_clusters_m<F>(m, b);
        if (nc <= 0) return p;
        const int C = std::min(C0, nc);
        p.tl = (T + C - 1) / C;
        p.smem = q4t_layout(nw, m, k, R, p.tl, F::kUnit).total;
        p.grid = C * kTmaCluster;
        p.R = R;
        return p;
    }
    return p;
}
TmaPlan q4k_tma_plan(const lc_ctx *ctx, int m, int k, int n) { return tma_plan<FmtQ4K>(ctx, m, k, n); }

template <class F, int M>
int launch_tma_m(lc_ctx *ctx, const TmaPlan &p, const CUtensorMap &tm, const float *x, float *c, uint32_t k,
                 uint32_t n) {
    constexpr int NW = q4t_warps(M);
    int s = set_smem(tma_gemv_kernel<F, M, NW, kTmaCluster>, p.smem);
    if (s) return s;
    tma_gemv_kernel<F, M, NW, kTmaCluster><<<p.grid, (NW + 1) * 32, p.smem, ctx->stream>>>(
        tm, x, c, (int)k, (int)n, ctx->half_mode, p.R, p.tl, ctx->dev_status);
    return LC_OK;
}

// The TMA GEMV for m = 1..4 tokens.
template <class F>
int launch_tma(lc_ctx *ctx, const TmaPlan &p, uint32_t m, const float *x, const uint8_t *w, float *c, uint32_t k,
               uint32_t n) {
    CUtensorMap tm;
    int s = tma_tensor_map<F>(&tm, w, k, n);
    if (s) return s;
    switch (m) {
    case 1: return launch_tma_m<F, 1>(ctx, p, tm, x, c, k, n);
    case 2: return launch_tma_m<F, 2>(ctx, p, tm, x, c, k, n);
    case 3: return launch_tma_m<F, 3>(ctx, p, tm, x, c, k, n);
    default: return launch_tma_m<F, 4>(ctx, p, tm, x, c, k, n);
    }
}
int launch_q4k_tma(lc_ctx *ctx, const TmaPlan &p, uint32_t m, const float *x, const uint8_t *w, float *c, uint32_t k,
                   uint32_t n) {
    return launch_tma<FmtQ4K>(ctx, p, m, x, w, c, k, n);
}

template <int M>
int launch_q8_sk(lc_ctx *ctx, int grid, size_t smem, const float *x, const uint8_t *w, float *c, uint32_t k,
                 uint32_t n, Fixup fx) {
    int s = set_smem(q8_sk_kernel<M>, smem);
    if (s) return s;
    q8_sk_kernel<M><<<grid, kSkWarps * 32, smem, ctx->stream>>>(x, w, c, (int)k, (int)n, ctx->half_mode, fx);
    return LC_OK;
}

template <int NT, int LANES>
int launch_q8(lc_ctx *ctx, const uint2 *tab, const float *inv_scale, const uint8_t *w, float *c, int m, int k, int n) {
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
                                                                        kch > 1, inv_scale);
    return LC_OK;
}

}  // namespace

namespace lc {

int proj_q4k_tiled(lc_ctx *ctx, const float *x, const uint8_t *w, float *c, uint32_t m, uint32_t k, uint32_t n,
                   void *pack);
size_t q4k_pack_bytes(uint32_t m_group, uint32_t k);

// One launch group handles up to 16 tokens (NT = 4 n-tiles).
int proj_q4k(lc_ctx *ctx, const float *x, const void *wv, float *c, uint32_t m, uint32_t k, uint32_t n,
             uint32_t expert_offset) {
    LC_REQUIRE(k % 256 == 0, LC_ERR_UNSUPPORTED, "proj_q4k: k=%u is not a multiple of 256", k);
    LC_REQUIRE(expert_offset % 256 == 0, LC_ERR_UNSUPPORTED, "proj_q4k: expert_offset=%u not a multiple of 256",
               expert_offset);
    LC_REQUIRE(((uintptr_t)wv & 15) == 0, LC_ERR_INVALID, "proj_q4k: weight pointer not 16-byte aligned");
    const uint8_t *w = (const uint8_t *)wv + (size_t)(expert_offset / 256) * 144;
    // 1-2 tokens: the f32-activation row GEMV (lc_gemv.cu); 3-8: the int8 tcgen05
    // GEMV; 9-32: the f16 tcgen05 GEMM; more: the lm_head tiles
    if (m <= 2 && gemv_rows_covers(ctx, LC_Q4_K, m, k)) {
        PackSrc src;
        src.x = x;
        ProjOut o;
        o.w = w;
        o.y = c;
        o.n = n;
        const int s = gemv_rows(ctx, LC_Q4_K, src, &o, 1, m, k);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (ctx->gemm_tc && (int)m >= ctx->gemv_i8_min && (int)m <= ctx->gemv_i8_max) {
        const int s = gemv_i8(ctx, LC_Q4_K, x, w, c, m, k, n);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (m <= 4) {
        const TmaPlan p = q4k_tma_plan(ctx, (int)m, (int)k, (int)n);
        if (p.R) return launch_q4k_tma(ctx, p, m, x, w, c, k, n);
    } else if (ctx->gemm_tc) {
        const int s = m <= 32 ? gemm_dq(ctx, LC_Q4_K, x, w, c, m, k, n) : gemm_large(ctx, LC_Q4_K, x, w, c, m, k, n);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    return proj_q4k_tiled(ctx, x, w, c, m, k, n, nullptr);
}

size_t q4k_pack_bytes(uint32_t m_group, uint32_t k) {
    const size_t nt = (m_group + 3) / 4;
    return (size_t)(k / 256) * 17 * nt * 32 * 8 + 16 * 4;
}

// Groups of up to 16 tokens through x_pack_q4k + q4k_mma_kernel.  The packed
// activations go to `pack` (at least q4k_pack_bytes(min(m, 16), k) bytes)
// or, when it is null, to the context's scratch pool.
int proj_q4k_tiled(lc_ctx *ctx, const float *x, const uint8_t *w, float *c, uint32_t m, uint32_t k, uint32_t n,
                   void *pack) {
    const int nsb = k / 256;
    for (uint32_t t0 = 0; t0 < m; t0 += 16) {
        const int mm = (int)std::min<uint32_t>(16, m - t0);
        const int nt = (mm + 3) / 4;
        const size_t tab_bytes = (size_t)nsb * 17 * nt * 32 * 8;
        uint2 *tab = (uint2 *)(pack ? pack : lc_scratch(ctx, LC_SCRATCH_PACK, tab_bytes + 16 * 4));
        if (!tab) return LC_ERR_OOM;
        float *inv = (float *)((char *)tab + tab_bytes);
        x_pack_q4k<<<nt * 4, 256, 0, ctx->stream>>>(x + (size_t)t0 * k, tab, inv, mm, (int)k, nt);
        float *cc = c + (size_t)t0 * n;
        int s;
        if (nt == 1)
            s = launch_q4k<1, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else if (nt == 2)
            s = launch_q4k<2, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else if (nt == 3)
            s = launch_q4k<3, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else
            s = launch_q4k<4, 32>(ctx, tab, inv, w, cc, mm, k, n);
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
    if (m == 1 && gemv_rows_covers(ctx, LC_Q8_0, m, k)) {  // as proj_q4k
        PackSrc src;
        src.x = x;
        ProjOut o;
        o.w = w;
        o.y = c;
        o.n = n;
        const int s = gemv_rows(ctx, LC_Q8_0, src, &o, 1, m, k);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (ctx->gemm_tc && (int)m >= ctx->gemv_i8_min && (int)m <= ctx->gemv_i8_max) {  // as proj_q4k
        const int s = gemv_i8(ctx, LC_Q8_0, x, w, c, m, k, n);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (m <= 4 && k % 256 == 0 && ((uintptr_t)wv & 15) == 0) {
        const TmaPlan p = tma_plan<FmtQ8_0>(ctx, (int)m, (int)k, (int)n);
        if (p.R) return launch_tma<FmtQ8_0>(ctx, p, m, x, w, c, k, n);
    } else if (m > 4 && ctx->gemm_tc) {
        const int s = m <= 32 ? gemm_dq(ctx, LC_Q8_0, x, w, c, m, k, n) : gemm_large(ctx, LC_Q8_0, x, w, c, m, k, n);
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (m <= 4) {
        const int S = (int)(k / 64);
        const size_t smem = ski_smem_bytes((int)m, (int)k);
        if (smem + 8192 <= ctx->smem_optin) {  // + static shared (zero block)
            const int T = (int)((n + 15) / 16);
            Fixup fx;
            fx.acc = (float *)lc_scratch_zeroed(ctx, LC_SCRATCH_FIXUP, (size_t)T * 64 * 4 + (size_t)T * 4 + 256);
            if (!fx.acc) return LC_ERR_OOM;
            fx.cnt = (unsigned *)(fx.acc + (size_t)T * 64);
            const long long units = (long long)T * S;
            const int grid = (int)std::max<long long>(1, std::min<long long>(ctx->num_sms, (units + 31) / 32));
            switch (m) {
            case 1: return launch_q8_sk<1>(ctx, grid, smem, x, w, c, k, n, fx);
            case 2: return launch_q8_sk<2>(ctx, grid, smem, x, w, c, k, n, fx);
            case 3: return launch_q8_sk<3>(ctx, grid, smem, x, w, c, k, n, fx);
            default: return launch_q8_sk<4>(ctx, grid, smem, x, w, c, k, n, fx);
            }
        }
    }
    for (uint32_t t0 = 0; t0 < m; t0 += 16) {
        const int mm = (int)std::min<uint32_t>(16, m - t0);
        const int nt = (mm + 3) / 4;
        const size_t tab_bytes = (size_t)nblk * 2 * nt * 32 * 8;
        uint2 *tab = (uint2 *)lc_scratch(ctx, LC_SCRATCH_PACK, tab_bytes + 16 * 4);
        if (!tab) return LC_ERR_OOM;
        float *inv = (float *)((char *)tab + tab_bytes);
        x_pack_q8<<<nt * 4, 256, 0, ctx->stream>>>(x + (size_t)t0 * k, tab, inv, mm, (int)k, nt);
        float *cc = c + (size_t)t0 * n;
        int s;
        if (nt == 1)
            s = launch_q8<1, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else if (nt == 2)
            s = launch_q8<2, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else if (nt == 3)
            s = launch_q8<3, 32>(ctx, tab, inv, w, cc, mm, k, n);
        else
            s = launch_q8<4, 32>(ctx, tab, inv, w, cc, mm, k, n);
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

// ---------------------------------------------------------------------------
// Q4_K projection that allocates no device memory.
//
// lc_proj_q4k / lc_proj_m put the packed activations of their tiled path
// (m > 4 tokens) in the context's scratch pool, which grows with cudaMalloc the
// first time a larger shape arrives.  Some callers cannot allocate on the call
// path: a serving loop whose memory planner has already handed all of HBM to
// weights and the K/V cache (a cudaMalloc there fails or fragments that plan),
// or a latency-bound decode loop that must not pay cudaMalloc's implicit
// device-wide synchronisation, which stalls every other stream on the GPU.
// This entry point takes that scratch from a fixed static device array
// instead; for m <= 2 it runs the f32-activation row GEMV and for m = 3, 4 the
// cluster GEMV, neither of which needs scratch.
//
// Limits: m in 1..16 tokens; for m = 3, 4 the activation table of m * k must
// fit in shared memory; for m > 4 the packed activations of m * k must fit in
// the array (k <= 15360 at m = 16).  Nothing in the array needs to start at
// zero: each call writes the part it reads.  Calls that overlap on the GPU (two
// streams, or two contexts on one device) share the array and race; callers
// serialise them.
//
// The array's device address is resolved once per context, at lc_init, with
// the context's device current (lc_static_pack_resolve); host code never uses
// the symbol itself, which on the host names a host-side stand-in.

constexpr size_t kStaticPackBytes = (size_t)1 << 20;

static __device__ __align__(256) unsigned char g_static_pack[kStaticPackBytes];

int lc_static_pack_resolve(lc_ctx *ctx) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_pack);
    LC_REQUIRE(e == cudaSuccess && p, LC_ERR_CUDA, "static scratch: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
    ctx->static_pack = p;
    return LC_OK;
}

extern "C" int lc_proj_q4k_static(lc_ctx *ctx, const float *x, const void *wv, float *c, uint32_t m, uint32_t k,
                                  uint32_t n, uint32_t expert_offset) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_proj_q4k_static: null ctx");
    if (m == 0 || n == 0) return LC_OK;
    LC_REQUIRE(x && wv && c, LC_ERR_INVALID, "lc_proj_q4k_static: null pointer");
    LC_REQUIRE(m <= 16, LC_ERR_UNSUPPORTED, "lc_proj_q4k_static: m=%u tokens, at most 16", m);
    LC_REQUIRE(k > 0 && k % 256 == 0, LC_ERR_UNSUPPORTED, "lc_proj_q4k_static: k=%u is not a positive multiple of 256",
               k);
    LC_REQUIRE(expert_offset % 256 == 0, LC_ERR_UNSUPPORTED,
               "lc_proj_q4k_static: expert_offset=%u not a multiple of 256", expert_offset);
    LC_REQUIRE(((uintptr_t)wv & 15) == 0, LC_ERR_INVALID, "lc_proj_q4k_static: weight pointer not 16-byte aligned");
    LC_REQUIRE(ctx->static_pack, LC_ERR_INVALID, "lc_proj_q4k_static: context has no static scratch address");
    int s = lc_use_device(ctx);
    if (s) return s;
    const uint8_t *w = (const uint8_t *)wv + (size_t)(expert_offset / 256) * 144;
    s = LC_ERR_UNSUPPORTED;
    if (m <= 2 && lc::gemv_rows_covers(ctx, LC_Q4_K, m, k)) {
        lc::PackSrc src;
        src.x = x;
        lc::ProjOut o;
        o.w = w, o.y = c, o.n = n;
        s = lc::gemv_rows(ctx, LC_Q4_K, src, &o, 1, m, k);
    }
    if (s != LC_ERR_UNSUPPORTED) {
        // the row GEMV ran (or failed)
    } else if (m <= 4) {
        const TmaPlan p = q4k_tma_plan(ctx, (int)m, (int)k, (int)n);
        LC_REQUIRE(p.R, LC_ERR_UNSUPPORTED,
                   "lc_proj_q4k_static: m*k=%u*%u activations exceed shared memory (%zu of %zu bytes)", m, k,
                   q4t_layout(q4t_warps((int)m), (int)m, (int)k, 2, 1).total, ctx->smem_optin);
        s = launch_q4k_tma(ctx, p, m, x, w, c, k, n);
    } else {
        const size_t need = lc::q4k_pack_bytes(m, k);
        LC_REQUIRE(need <= kStaticPackBytes, LC_ERR_UNSUPPORTED,
                   "lc_proj_q4k_static: packed activations of m*k=%u*%u need %zu bytes, the static scratch has %zu", m,
                   k, need, kStaticPackBytes);
        s = lc::proj_q4k_tiled(ctx, x, w, c, m, k, n, ctx->static_pack);
    }
    if (s) return s;
    return lc_after_launch(ctx, "lc_proj_q4k_static");
}

int lc_tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out) { return tensor_map_encoder(out); }
