// lc_gemm.cu -- quantized-weight GEMM on the 5th-generation tensor cores
// (tcgen05 / TMEM) for blocks of tokens: y[t, i] = sum_j x[t, j] * W[i, j]
// with W in raw GGUF Q4_K or Q8_0 blocks (kernels/proj_q4k.comp:60-92,
// kernels/proj_q8_0.comp:47-67 applied to every row of x).
//
// One CTA per SM, warp-specialised:
//   warp 0      producer: TMA copies of raw weight units (128 rows x 256
//               elements) and of the tokens' f16 activations (+ their Q4_K
//               sub-block sums);
//   warps 1-8   converters: one weight row per thread (the row is the TMEM
//               lane the warp may access), warps 1-4 the first half of a unit,
//               warps 5-8 the second; they dequantise to f16 in registers and
//               store it into tensor memory with tcgen05.st;
//   warps 9-10  issue tcgen05.mma for the even / odd units (kind::f16,
//               A = weights from TMEM, M = 128 rows, B = tokens from shared
//               memory, N = 2 NT, K = 16) with f32 accumulation in TMEM; two
//               issuers overlap one unit's barrier waits and commits with the
//               other's MMAs; warp 9 also allocates the tensor memory;
//   warps 11-14 epilogue: tcgen05.ld of each unit's accumulators, scales, and
//               at the end of a tile's run f32 atomic adds into y (zeroed by
//               the packing kernel).
// Units (128-row tile, super-block) are flattened tile-major and cut into one
// contiguous range per CTA.
//
// With only 2 NT token columns per MMA, an A operand in shared memory would
// cost 4 KB of shared-memory reads per MMA plus the converters' writes:
// shared-memory bandwidth, not the tensor cores, would bound the kernel.
// Tensor memory takes that traffic instead: three A unit slots of 128
// columns (two when the accumulators need more room), then the accumulator
// buffers.  The converters of unit j + slots wait only for the MMAs of unit
// j, so the slots set how far conversion runs ahead of the tensor cores.
//
// Q4_K keeps the weights exact on the tensor cores: A holds the integers
// sc_j * q, so each unit's product P = sum sc_j q x and min term
// M = sum_j m_j Sx_j (Sx_j the sub-block sums of x, one extra K = 16 MMA with
// both operands in shared memory) land in their own TMEM columns, and the
// epilogue accumulates d P - dmin M in f32.  Q8_0 weights become f16(d q) (one
// rounding).
//
// Activations: x [m, k] f32 times a power of two per (token, super-block)
// (exact) becomes x16 [2 NT, k] f16: rows 0..NT-1 the f16 value, rows
// NT..2NT-1 the f16 of the remainder (rows past m zero), so the UMMA sees x to
// ~22 bits; the epilogue adds the two columns of a token and multiplies by the
// inverse scale.  Within each super-block k is in the order the converters
// produce (a fixed permutation; the dot product is the same).
//
// Every mbarrier wait is bounded; on expiry the kernel records
// LC_DEV_WAIT_TIMEOUT in the context's status word, stops issuing work, lets
// the tensor-core work in flight finish (bounded) and frees the TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "lc_internal.cuh"
#include "lc_sm100.cuh"

namespace {

constexpr int kRows = 128;  // weight rows per tile (UMMA M)
constexpr int kConvWarps = 8;
constexpr int kMmaWarp = 1 + kConvWarps;  // first of the two MMA warps (even / odd units)
constexpr int kMmaWarps = 2;
constexpr int kGemmWarps = kMmaWarp + kMmaWarps + 4;  // + 4 epilogue warps
constexpr int kTmemCols = 512;
constexpr int kASlots = 2;      // TMEM A slots of one unit (K = 256)
constexpr int kACols = 128;     // 256 f16 per lane; half h at column 64 h
constexpr int kAccBase = kASlots * kACols;
constexpr int kMinBytes = kRows * 32;  // Q4_K min-term operand: 128 rows x 16 f16

// ---- formats ----------------------------------------------------------------

struct GQ4K {
    static constexpr int kRowBytes = 144;  // one super-block per row and unit
    static constexpr int kBoxX = 18;       // u64 words
    static constexpr bool kQ8 = false;
};
struct GQ8_0 {
    static constexpr int kRowBytes = 272;  // eight 34-byte blocks
    static constexpr int kBoxX = 136;      // u16 words
    static constexpr bool kQ8 = true;
};

// f16 bits of two halves with the reference rule for subnormals (exponent
// field set to 1) when ref_mask is 0x04000400 (kernels/proj_q8_0.comp:27-45).
__device__ __forceinline__ uint32_t fix_sub_h2(uint32_t h2, uint32_t ref_mask) {
    const uint32_t man = h2 & 0x03FF03FFu, ex = h2 & 0x7C007C00u;
    const uint32_t m_nz = (man + 0x03FF03FFu) & 0x04000400u;
    const uint32_t e_nz = ((ex + 0x7C007C00u) & 0x80008000u) >> 5;
    return h2 | (m_nz & ~e_nz & ref_mask);
}

__device__ __forceinline__ __half2 u2h2(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }
__device__ __forceinline__ uint32_t h22u(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

// k order within a super-block.  Position chunk c (8 positions, 4 TMEM
// columns) holds elements
//   Q4_K: qs word c (G = c/8, p = 4(c%8)): 64G + [p, p+2, p+1, p+3, 32+p, 34+p, 33+p, 35+p]
//   Q8_0: block b = c/4, words 2i, 2i+1 (i = c%4): 32b + 8i + [0, 2, 1, 3, 4, 6, 5, 7]
// i.e. two runs of four consecutive elements e0..e0+3 and e1..e1+3, each in
// the order [0, 2, 1, 3] (what the byte-pair extraction yields).

// Q4_K: half g (sub-blocks 4g..4g+3) of one row of a unit -> 64 TMEM columns
// at taddr.  The values are the exact integers sc_j * q (at most 63 * 15): each
// pair comes from one HFMA2 of the nibble pair biased into f16 (1024 + q, or
// 1024 + 16 q for the high nibbles) with sc (sc / 16) and the bias term, which
// is exact because the fused result is an integer below 2048.  d and dmin are
// applied in f32 by the epilogue.
template <int g>
__device__ __forceinline__ void conv_q4k_half(const uint8_t *raw, const uint32_t (&sc)[8], uint32_t taddr) {
    // All 64 qs bytes of the half are loaded before the first tcgen05.st:
    // the stores are volatile asm with a memory clobber, so loads written
    // between them could not be hoisted and each round would pay the full
    // shared-memory latency.
    uint4 Qa[4];
#pragma unroll
    for (int i = 0; i < 4; i++) Qa[i] = lds128(raw + 16 + 64 * g + 16 * i);
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
        const int G = 2 * g + gg;  // qs group: sub-blocks 2G (low), 2G+1 (high nibbles)
        const __half2 slo = __float2half2_rn((float)sc[2 * G]), clo = __float2half2_rn(-1024.f * (float)sc[2 * G]);
        const __half2 shi = __float2half2_rn((float)sc[2 * G + 1] * 0.0625f),
                      chi = __float2half2_rn(-64.f * (float)sc[2 * G + 1]);
#pragma unroll
        for (int w4 = 0; w4 < 2; w4++) {
            const uint4 Q = Qa[2 * gg + w4];
            const uint32_t qw[4] = {Q.x, Q.y, Q.z, Q.w};
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t W = qw[i], W8 = W >> 8;
                o[4 * i + 0] = h22u(__hfma2(u2h2((W & 0x000F000Fu) | 0x64006400u), slo, clo));
                o[4 * i + 1] = h22u(__hfma2(u2h2((W8 & 0x000F000Fu) | 0x64006400u), slo, clo));
                o[4 * i + 2] = h22u(__hfma2(u2h2((W & 0x00F000F0u) | 0x64006400u), shi, chi));
                o[4 * i + 3] = h22u(__hfma2(u2h2((W8 & 0x00F000F0u) | 0x64006400u), shi, chi));
            }
            tmem_st16(taddr + 32 * gg + 16 * w4, o);  // chunks 8gg + 4w4 .. +3
        }
    }
}

// The eight 6-bit (sc, m) pairs of a Q4_K super-block from its 12 scale bytes
// (get_scale_min_k4, kernels/proj_q4k.comp:46-58).
__device__ __forceinline__ void q4k_scale_mins(const uint4 &H, uint32_t (&sc)[8], uint32_t (&mn)[8]) {
    const uint32_t q[3] = {H.y, H.z, H.w};
    auto qb = [&](int j) { return (q[j >> 2] >> (8 * (j & 3))) & 0xFFu; };
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            sc[j] = qb(j) & 63u;
            mn[j] = qb(j + 4) & 63u;
        } else {
            sc[j] = (qb(j + 4) & 0xFu) | ((qb(j - 4) >> 6) << 4);
            mn[j] = (qb(j + 4) >> 4) | ((qb(j) >> 6) << 4);
        }
    }
}

// Q8_0: half h (blocks 4h..4h+3) of one row -> 64 TMEM columns of f16(d * q)
// (one rounding per weight).  Block b's q bytes start at byte 34b + 2 (two
// bytes off word alignment for even b), its f16 d at byte 34b.
template <int h>
__device__ __forceinline__ void conv_q8_half(const uint8_t *raw, uint32_t ref_mask, uint32_t taddr) {
    // The half's blocks span row bytes 136h .. 136h + 135; the 9 aligned
    // 16-byte chunks from byte 128h cover them and are all loaded before the
    // first tcgen05.st (see conv_q4k_half).  Word i of Wd is row word 32h + i.
    uint32_t Wd[36];
#pragma unroll
    for (int i = 0; i < 9; i++) {
        const uint4 v = lds128(raw + 128 * h + 16 * i);
        Wd[4 * i] = v.x, Wd[4 * i + 1] = v.y, Wd[4 * i + 2] = v.z, Wd[4 * i + 3] = v.w;
    }
    const __half2 k1152 = __float2half2_rn(1152.f);
#pragma unroll
    for (int bb = 0; bb < 4; bb++) {
        const int b = 4 * h + bb;
        const int wq = (17 * b + 1) / 2 - 32 * h, sh = (b & 1) ? 0 : 16;
        const uint32_t dw = Wd[((b & 1) ? (17 * (b - 1)) / 2 + 8 : (17 * b) / 2) - 32 * h];
        const uint32_t dbits = fix_sub_h2((b & 1) ? (dw >> 16) : (dw & 0xFFFFu), ref_mask) & 0xFFFFu;
        const __half2 d2 = u2h2(dbits | (dbits << 16));
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t t[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int wi = wq + 2 * i + u;
                t[u] = __funnelshift_r(Wd[wi], (sh && wi + 1 < 36) ? Wd[wi + 1] : 0u, sh);
            }
            o[4 * i + 0] = h22u(__hmul2(__hsub2(u2h2((t[0] & 0x00FF00FFu) ^ 0x64806480u), k1152), d2));
            o[4 * i + 1] = h22u(__hmul2(__hsub2(u2h2(((t[0] >> 8) & 0x00FF00FFu) ^ 0x64806480u), k1152), d2));
            o[4 * i + 2] = h22u(__hmul2(__hsub2(u2h2((t[1] & 0x00FF00FFu) ^ 0x64806480u), k1152), d2));
            o[4 * i + 3] = h22u(__hmul2(__hsub2(u2h2(((t[1] >> 8) & 0x00FF00FFu) ^ 0x64806480u), k1152), d2));
        }
        tmem_st16(taddr + 16 * bb, o);  // chunks 4bb .. 4bb+3
    }
}

// Byte offset of element (row, kk) of a 16-wide K-major operand in the
// no-swizzle core-matrix layout (8 rows x 16 bytes per core matrix, the two
// K groups 128 bytes apart, 8-row groups 256 bytes apart).
__host__ __device__ __forceinline__ uint32_t core16_off(int row, int kk) {
    return (uint32_t)((row >> 3) * 256 + (kk >> 3) * 128 + (row & 7) * 16 + (kk & 7) * 2);
}

// Outputs the packing kernel zeroes for the GEMM's atomic adds.
struct ZeroList {
    float *p[lc::kGroupMax];
    long long n[lc::kGroupMax];
    int cnt;
};

// Activation packing, one warp per (token slot t, super-block sb), grid
// (S, NT / 8) x 256 threads: lane c converts position chunk c.
//   x16[t] / x16[NT + t]: hi / lo f16 of x * s, s = 2^e per (t, sb) putting
//                         max |x * s| in [2^13, 2^14);
//   inv[sb * NT + t]:     1 / s (0 for rows past m);
//   sx16 (Q4_K):          per super-block a 2 NT x 16 K-major operand in the
//                         core-matrix layout: columns 0..7 the sub-block sums
//                         of x * s / 32 (hi in row t, lo in row NT + t),
//                         columns 8..15 zero.
// x is the projection input, or (OP) the SwiGLU product / the softplus head
// gate of two inputs, formed here with the element-wise kernels' own functions,
// or x RMS-normalised with the weight x2 (x16_pack_norm_kernel, one CTA per
// token slot: the norm costs no launch of its own).  The CTAs also zero the
// outputs in `zl`.
// The packing of one (super-block sb, token slot t) by one warp (lane c);
// rms is the row's norm factor for LC_PACK_RMSNORM.
template <int OP>
__device__ __forceinline__ void pack_warp(const float *__restrict__ x, const float *__restrict__ x2, int head_dim,
                                          float rms, int m, int k, int q8, int nt, __half *__restrict__ x16,
                                          uint8_t *__restrict__ sx16, float *__restrict__ inv, int sb, int t, int c) {
    int e0, e1;
    if (q8) {
        e0 = 32 * (c >> 2) + 8 * (c & 3);
        e1 = e0 + 4;
    } else {
        e0 = 64 * (c >> 3) + 4 * (c & 7);
        e1 = e0 + 32;
    }
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (t < m) {
        const float *xr = x + (size_t)t * k + (size_t)sb * 256;
        a = *reinterpret_cast<const float4 *>(xr + e0);
        b = *reinterpret_cast<const float4 *>(xr + e1);
        if constexpr (OP == lc::LC_PACK_SWIGLU) {
            const float *ur = x2 + (size_t)t * k + (size_t)sb * 256;
            const float4 ua = *reinterpret_cast<const float4 *>(ur + e0), ub = *reinterpret_cast<const float4 *>(ur + e1);
            a = make_float4(lc_swiglu(a.x, ua.x), lc_swiglu(a.y, ua.y), lc_swiglu(a.z, ua.z), lc_swiglu(a.w, ua.w));
            b = make_float4(lc_swiglu(b.x, ub.x), lc_swiglu(b.y, ub.y), lc_swiglu(b.z, ub.z), lc_swiglu(b.w, ub.w));
        } else if constexpr (OP == lc::LC_PACK_HEADGATE) {
            // a 4-run lies inside one head (head_dim % 4 == 0)
            const float *gr = x2 + (size_t)t * (k / head_dim);
            const float ga = lc_softplus_f(gr[(sb * 256 + e0) / head_dim]);
            const float gb = lc_softplus_f(gr[(sb * 256 + e1) / head_dim]);
            a = make_float4(a.x * ga, a.y * ga, a.z * ga, a.w * ga);
            b = make_float4(b.x * gb, b.y * gb, b.z * gb, b.w * gb);
        } else if constexpr (OP == lc::LC_PACK_RMSNORM) {
            // rmsnorm.comp: (x * w) * rms, rms of the whole row from the caller
            const float *wr = x2 + (size_t)sb * 256;
            const float4 wa = *reinterpret_cast<const float4 *>(wr + e0), wb = *reinterpret_cast<const float4 *>(wr + e1);
            a = make_float4(a.x * wa.x * rms, a.y * wa.y * rms, a.z * wa.z * rms, a.w * wa.w * rms);
            b = make_float4(b.x * wb.x * rms, b.y * wb.y * rms, b.z * wb.z * rms, b.w * wb.w * rms);
        }
    }
    float mx = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                     fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s, iv;
    act_scale(mx, s, iv);
    if (c == 0) inv[sb * nt + t] = t < m ? iv : 0.f;
    const float v[8] = {a.x * s, a.z * s, a.y * s, a.w * s, b.x * s, b.z * s, b.y * s, b.w * s};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        const float2 hf = __half22float2(h);
        hi[i] = h22u(h);
        lo[i] = h22u(__floats2half2_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y));
    }
    const size_t pos = (size_t)sb * 256 + 8 * c;
    *reinterpret_cast<uint4 *>(x16 + (size_t)t * k + pos) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(x16 + (size_t)(t + nt) * k + pos) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    if (q8) return;
    // sub-block 2G (the a runs) and 2G+1 (the b runs) of lanes 8G..8G+7
    float s0 = (a.x + a.y) + (a.z + a.w), s1 = (b.x + b.y) + (b.z + b.w);
#pragma unroll
    for (int o = 4; o; o >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    const int kk = c & 15, src = 8 * ((kk & 7) >> 1);
    const float g0 = __shfl_sync(0xffffffffu, s0, src), g1 = __shfl_sync(0xffffffffu, s1, src);
    if (c < 16) {
        const float sum = kk < 8 ? ((kk & 1) ? g1 : g0) * (s * 0.03125f) : 0.f;
        const __half h = __float2half_rn(sum);
        uint8_t *blk = sx16 + (size_t)sb * (2 * nt * 32);
        *reinterpret_cast<__half *>(blk + core16_off(t, kk)) = h;
        *reinterpret_cast<__half *>(blk + core16_off(t + nt, kk)) = __float2half_rn(sum - __half2float(h));
    }
}

// 16-byte stores from the first 16-byte boundary, single floats before and after it.
__device__ __forceinline__ void zero_outputs(const ZeroList *Z, long long tid0, long long nthreads) {
    for (int z = 0; z < Z->cnt; z++) {
        float *p = Z->p[z];
        const long long n = Z->n[z];
        const long long head = min(n, (long long)(((16u - ((uint32_t)(uintptr_t)p & 15u)) & 15u) >> 2));
        const long long n4 = (n - head) >> 2;
        if (tid0 < head) p[tid0] = 0.f;
        float4 *q = reinterpret_cast<float4 *>(p + head);
        for (long long i = tid0; i < n4; i += nthreads) q[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (long long i = head + 4 * n4 + tid0; i < n; i += nthreads) p[i] = 0.f;
    }
}

template <int OP>
__global__ void x16_pack_kernel(const float *__restrict__ x, const float *__restrict__ x2, int head_dim, int m, int k,
                                int q8, int nt, __half *__restrict__ x16, uint8_t *__restrict__ sx16,
                                float *__restrict__ inv, const __grid_constant__ ZeroList zl) {
    griddep_launch_dependents();  // the GEMM may start streaming its weights now
    const long long nthreads = (long long)gridDim.x * gridDim.y * blockDim.x;
    zero_outputs(&zl, ((long long)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x, nthreads);
    pack_warp<OP>(x, x2, head_dim, 0.f, m, k, q8, nt, x16, sx16, inv, blockIdx.x, blockIdx.y * 8 + (threadIdx.x >> 5),
                  threadIdx.x & 31);
}

// LC_PACK_RMSNORM: grid (token slots, super-block groups of 8).  A CTA forms
// its token slot's sum of squares over the row (rmsnorm.comp: rsqrt(sum / k +
// eps); the super-block groups of a token repeat it), then its 8 warps pack
// their super-blocks with (x * w) * rms.
__global__ void x16_pack_norm_kernel(const float *__restrict__ x, const float *__restrict__ w, float eps, int m, int k,
                                     int q8, int nt, __half *__restrict__ x16, uint8_t *__restrict__ sx16,
                                     float *__restrict__ inv, const __grid_constant__ ZeroList zl) {
    griddep_launch_dependents();
    __shared__ float red[33];
    zero_outputs(&zl, ((long long)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x,
                 (long long)gridDim.x * gridDim.y * blockDim.x);
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float ss = 0.f;
    if (t < m) {
        const float4 *xr4 = reinterpret_cast<const float4 *>(x + (size_t)t * k);
        for (int i = threadIdx.x; i < (k >> 2); i += blockDim.x) {
            const float4 v = xr4[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nw ? red[lane] : 0.f;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[32] = v;
    }
    __syncthreads();
    const float rms = rsqrtf(red[32] / (float)k + eps);
    const int sb = blockIdx.y * nw + warp;
    if (sb < (k >> 8)) pack_warp<lc::LC_PACK_RMSNORM>(x, w, 0, rms, m, k, q8, nt, x16, sx16, inv, sb, t, lane);
}

struct GemmLayout {
    size_t amin = 0, x = 0, raw = 0, sc = 0, bars = 0, tslot = 0, total = 0;
    int XS = 0, RS = 0, ND = 0, xstage = 0, bufcols = 0, AS = 0, acc = 0;
};

// Shared memory: Q4_K min-term operands (one per TMEM A stage), activation
// stages (+ the sub-block sums for Q4_K), raw weight stages, per-unit
// (d, dmin) slots (Q4_K), barriers.  Every stage size is a multiple of 1024
// bytes.  TMEM: AS A slots of 128 columns, then ND accumulator buffers of
// `bufcols` columns from column `acc`.
template <class F, int NT>
__host__ __device__ constexpr GemmLayout gemm_layout() {
    GemmLayout L{};
    L.XS = NT >= 32 ? 3 : 4;
    L.RS = F::kQ8 ? (NT >= 32 ? 3 : 4) : (NT >= 32 ? 5 : 6);
    L.bufcols = F::kQ8 ? 2 * NT : 4 * NT;  // hi / lo columns (+ the Q4_K min term)
    L.AS = (kTmemCols - 3 * kACols) / L.bufcols >= 2 ? 3 : 2;
    L.acc = L.AS * kACols;
    L.ND = (kTmemCols - L.acc) / L.bufcols < 4 ? (kTmemCols - L.acc) / L.bufcols : 4;
    L.xstage = 2 * NT * 512 + (F::kQ8 ? 0 : 2 * NT * 32);  // both halves of a unit
    L.amin = 0;
    L.x = L.amin + (F::kQ8 ? 0 : (size_t)L.AS * kMinBytes);
    L.raw = L.x + (size_t)L.XS * L.xstage;
    L.sc = L.raw + (size_t)L.RS * kRows * F::kRowBytes;
    L.bars = L.sc + (F::kQ8 ? 0 : (size_t)L.ND * kRows * 8);
    L.tslot = L.bars + (size_t)(2 * L.RS + 2 * L.AS + 2 * L.XS + 3 * L.ND + 1) * 8;
    L.total = L.tslot + 16 + 1024;  // + slack to 1024-align the base
    return L;
}

// Up to kGroupMax weight matrices sharing one activation block: matrix i owns
// the global row tiles [tile_end[i - 1], tile_end[i]).
struct DqGroup {
    CUtensorMap tmw[lc::kGroupMax];
    float *y[lc::kGroupMax];
    int n[lc::kGroupMax];
    int tile_end[lc::kGroupMax];
    int ng;
};

// The matrix of global row tile `tile` and the tile's index inside it.
__device__ __forceinline__ int group_of(const DqGroup *G, int tile, int &ltile) {
    int gi = 0;
    while (gi + 1 < G->ng && tile >= G->tile_end[gi]) gi++;
    ltile = tile - (gi ? G->tile_end[gi - 1] : 0);
    return gi;
}

// Warps of the dq GEMM.  For NT = 16 the converters are two sets of eight that
// take alternate units, so one set's tensor-memory stores and barrier waits
// overlap the other's conversion; NT = 32 keeps one set (its epilogue needs
// the registers).
template <int NT>
struct DqWarps {
    static constexpr int kSets = NT <= 16 ? 2 : 1;
    static constexpr int kConv = kConvWarps * kSets;
    static constexpr int kMma = 1 + kConv;  // first of the two MMA warps
    static constexpr int kAll = kMma + kMmaWarps + 4;
};

template <class F, int NT>
__global__ void __launch_bounds__(DqWarps<NT>::kAll * 32, 1)
    dq_gemm_kernel(const __grid_constant__ DqGroup grp, const __grid_constant__ CUtensorMap tmx,
                   const uint8_t *__restrict__ sx16, const float *__restrict__ inv, int m, int k, int half_mode,
                   unsigned *__restrict__ status) {
    const DqGroup *G = &grp;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr GemmLayout L = gemm_layout<F, NT>();
    constexpr bool Q4 = !F::kQ8;
    constexpr int NB = 2 * NT;  // UMMA N: hi and lo rows of the tokens
    constexpr int kXTiles = NB * 512;  // activations of one unit: two halves of two 64-column boxes
    constexpr int kRawStage = kRows * F::kRowBytes;
    constexpr int ND = L.ND, AS = L.AS;
    using W = DqWarps<NT>;
    uint8_t *amin_ring = smem + L.amin, *x_ring = smem + L.x, *raw_ring = smem + L.raw;
    float2 *dslot = reinterpret_cast<float2 *>(smem + L.sc);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *raw_full = bars, *raw_empty = raw_full + L.RS;
    uint64_t *a_full = raw_empty + L.RS, *a_empty = a_full + AS;
    uint64_t *x_full = a_empty + AS, *x_empty = x_full + L.XS;
    uint64_t *d_full = x_empty + L.XS, *d_empty = d_full + ND, *s_full = d_empty + ND, *drain = s_full + ND;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + L.tslot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = k >> 8, T = G->tile_end[G->ng - 1];
    const long long TS = (long long)T * S;
    const int U0 = (int)(TS * blockIdx.x / gridDim.x), U1 = (int)(TS * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < L.RS; i++) mbar_init(raw_full + i, 1), mbar_init(raw_empty + i, kConvWarps);
        for (int i = 0; i < AS; i++) mbar_init(a_full + i, kConvWarps), mbar_init(a_empty + i, 1);
        for (int i = 0; i < L.XS; i++) mbar_init(x_full + i, 1), mbar_init(x_empty + i, 1);
        for (int i = 0; i < ND; i++) mbar_init(d_full + i, 1), mbar_init(d_empty + i, 4), mbar_init(s_full + i, 4);
        mbar_init(drain, kMmaWarps);
        mbar_init_fence();
    }
    if (warp == W::kMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    bool ok = true;
    auto fail = [&]() {
        ok = false;
        atomicOr(status, LC_DEV_WAIT_TIMEOUT);
    };

    if (warp == 0) {
        if (lane == 0) {  // producer
            const uint64_t pol = l2_evict_first_policy();  // weights: read once
            uint64_t xpol;                                  // activations: read by every CTA
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(xpol));
            for (int u = U0; u < U1 && ok; u++) {
                const int j = u - U0, tile = u / S, sb = u - tile * S;
                const int rs = j % L.RS;
                int ltile;
                const int gi = group_of(G, tile, ltile);
                if (!mbar_wait(raw_empty + rs, ((j / L.RS) & 1) ^ 1)) { fail(); break; }
                mbar_expect_tx(raw_full + rs, kRawStage);
                tma_load_2d(raw_ring + (size_t)rs * kRawStage, &G->tmw[gi], sb * F::kBoxX, ltile * kRows, raw_full + rs,
                            pol);
                if (j == 0) griddep_wait();  // activations come from the packing kernel
                const int xs = j % L.XS;
                if (!mbar_wait(x_empty + xs, ((j / L.XS) & 1) ^ 1)) { fail(); break; }
                uint8_t *xst = x_ring + (size_t)xs * L.xstage;
                mbar_expect_tx(x_full + xs, kXTiles + (Q4 ? NB * 32 : 0));
#pragma unroll
                for (int kc = 0; kc < 4; kc++)  // half kc / 2, 64-column box kc % 2
                    tma_load_2d(xst + kc * NB * 128, &tmx, sb * 256 + kc * 64, 0, x_full + xs, xpol);
                if (Q4) bulk_load(xst + kXTiles, sx16 + (size_t)sb * NB * 32, NB * 32, x_full + xs, xpol);
            }
        }
    } else if (warp <= W::kConv) {  // converters: group g of set `set` converts half g of row r
        const int set = (warp - 1) >> 3, g = ((warp - 1) >> 2) & 1, quad = warp & 3, r = 32 * quad + lane;
        const uint32_t tlane = tbase + ((uint32_t)(32 * quad) << 16);
        const uint32_t ref_mask = half_mode == LC_HALF_REF ? 0x04000400u : 0u;
        if (Q4 && g == 0 && set == 0)  // columns 8..15 of the min-term operands stay zero
            for (int i = 0; i < AS; i++)
                *reinterpret_cast<uint4 *>(amin_ring + i * kMinBytes + core16_off(r, 8)) = make_uint4(0u, 0u, 0u, 0u);
        for (int u = U0 + set; u < U1 && ok; u += W::kSets) {  // set s takes units s, s + kSets, ...
            const int j = u - U0, rs = j % L.RS;
            if (!mbar_wait(raw_full + rs, (j / L.RS) & 1)) { fail(); break; }
            const uint8_t *raw = raw_ring + (size_t)rs * kRawStage + (size_t)r * F::kRowBytes;
            const int as = j % AS;
            if (!mbar_wait(a_empty + as, ((j / AS) & 1) ^ 1)) { fail(); break; }
            tc_fence_after();
            const uint32_t ta = tlane + as * kACols + g * 64;
            if constexpr (Q4) {
                const uint4 H = lds128(raw);
                uint32_t sc[8], mn[8];
                q4k_scale_mins(H, sc, mn);
                if (g == 0)
                    conv_q4k_half<0>(raw, sc, ta);
                else
                    conv_q4k_half<1>(raw, sc, ta);
                if (g == 0) {
                    // min-term operand: m_j (exact in f16) in columns 0..7 of row r
                    uint4 o;
                    o.x = h22u(__floats2half2_rn((float)mn[0], (float)mn[1]));
                    o.y = h22u(__floats2half2_rn((float)mn[2], (float)mn[3]));
                    o.z = h22u(__floats2half2_rn((float)mn[4], (float)mn[5]));
                    o.w = h22u(__floats2half2_rn((float)mn[6], (float)mn[7]));
                    *reinterpret_cast<uint4 *>(amin_ring + as * kMinBytes + core16_off(r, 0)) = o;
                    fence_proxy_async_smem();  // generic-proxy writes -> the tensor cores' reads
                    // (d, 32 dmin) of the unit for the epilogue, once its slot is free
                    const int db = j % ND;
                    if (!mbar_wait(d_empty + db, ((j / ND) & 1) ^ 1)) { fail(); break; }
                    const float2 dd = scales2_f32(H.x, ref_mask);
                    dslot[db * kRows + r] = make_float2(dd.x, 32.f * dd.y);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_full + db);
                }
            } else {
                if (g == 0)
                    conv_q8_half<0>(raw, ref_mask, ta);
                else
                    conv_q8_half<1>(raw, ref_mask, ta);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_full + as);
                mbar_arrive(raw_empty + rs);
            }
        }
    } else if (warp < W::kMma + kMmaWarps) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(kRows, NB);
            // Descriptors of x stage 0 and of the min-term operand stage 0; the
            // start-address field is the low 14 bits (address / 16, below
            // 2^14 for any shared-memory address), so stage and K offsets are
            // plain additions.
            const uint64_t xdesc0 = umma_desc_sw128(smem_addr(x_ring));
            const uint64_t mdesc0 = umma_desc_core16(smem_addr(amin_ring));
            const uint64_t sdesc0 = umma_desc_core16(smem_addr(x_ring) + kXTiles);  // sub-block sums, x stage 0
            // One synchronisation point per unit: the accumulator buffer, the
            // unit's A slot (both converter groups) and its activations, one
            // fence, 16 (+1) MMAs, three commits.
            for (int u = U0 + (warp - W::kMma); u < U1 && ok; u += kMmaWarps) {
                const int j = u - U0, db = j % ND, as = j % AS, xs = j % L.XS;
                if (!mbar_wait(d_empty + db, ((j / ND) & 1) ^ 1) || !mbar_wait(a_full + as, (j / AS) & 1) ||
                    !mbar_wait(x_full + xs, (j / L.XS) & 1)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t dcol = tbase + L.acc + db * L.bufcols;
                const uint64_t xd = xdesc0 + (uint64_t)((xs * L.xstage) >> 4);
                const uint32_t ta = tbase + as * kACols;
#pragma unroll
                for (int kk = 0; kk < 16; kk++)  // half kk / 8 at column 64 (kk / 8) + 8 (kk % 8)
                    umma_f16_ts(dcol, ta + 8 * kk, xd + (uint64_t)(((kk >> 2) * (NB * 128) + (kk & 3) * 32) >> 4), idesc,
                                kk ? 1u : 0u);
                if (Q4)  // min term: sum_j m_j * (sub-block sum of x) / 32
                    umma_f16_ss(dcol + NB, mdesc0 + (uint64_t)((as * kMinBytes) >> 4),
                                sdesc0 + (uint64_t)((xs * L.xstage) >> 4), idesc, 0u);
                umma_commit(a_empty + as);
                umma_commit(x_empty + xs);
                umma_commit(d_full + db);
            }
            // everything issued has completed before the TMEM is freed
            umma_commit(drain);
            if (!mbar_wait(drain, 0)) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        }
    } else {  // epilogue: TMEM lanes 32q..32q+31 = tile rows
        griddep_wait();  // scales and the zeroed y come from the packing kernel
        const int q = warp & 3;
        const uint32_t lanes = (uint32_t)(32 * q) << 16;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        for (int u = U0; u < U1 && ok; u++) {
            const int j = u - U0, db = j % ND, tile = u / S, sb = u - tile * S;
            const uint32_t par = (j / ND) & 1;
            if (!mbar_wait(d_full + db, par)) { fail(); break; }
            tc_fence_after();
            const uint32_t col = tbase + lanes + L.acc + db * L.bufcols;
            float2 dd = make_float2(1.f, 0.f);
            if constexpr (Q4) {
                if (!mbar_wait(s_full + db, par)) { fail(); break; }
                dd = dslot[db * kRows + 32 * q + lane];
            }
            if constexpr (NT == 16) {
                // the accumulators into registers (hi and lo summed), the
                // buffer released to the next MMAs, then the arithmetic
                float pr[16], mn[16], h[16], l[16];
                tmem_ld16(col, h);
                tmem_ld16(col + NT, l);
                tmem_ld_wait();
                tmem_regs_ready(h), tmem_regs_ready(l);
#pragma unroll
                for (int i = 0; i < 16; i++) pr[i] = h[i] + l[i];
                if constexpr (Q4) {
                    tmem_ld16(col + NB, h);
                    tmem_ld16(col + NB + NT, l);
                    tmem_ld_wait();
                    tmem_regs_ready(h), tmem_regs_ready(l);
#pragma unroll
                    for (int i = 0; i < 16; i++) mn[i] = h[i] + l[i];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(d_empty + db);
                float iv16[16];
#pragma unroll
                for (int t = 0; t < 16; t += 4) {
                    const float4 f = __ldg(reinterpret_cast<const float4 *>(inv + sb * NT + t));
                    iv16[t] = f.x, iv16[t + 1] = f.y, iv16[t + 2] = f.z, iv16[t + 3] = f.w;
                }
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    if constexpr (Q4)
                        acc[i] += iv16[i] * (dd.x * pr[i] - dd.y * mn[i]);
                    else
                        acc[i] += iv16[i] * pr[i];
                }
            } else {
                // Per 16 tokens: the hi and lo columns (and the Q4_K min term's)
                // summed, scaled into the row's partial sums.
    #pragma unroll
                for (int c = 0; c < NT / 16; c++) {
                    float iv[16], pr[16], mn[16], h[16], l[16];
    #pragma unroll
                    for (int t = 0; t < 16; t += 4) {
                        const float4 f = __ldg(reinterpret_cast<const float4 *>(inv + sb * NT + 16 * c + t));
                        iv[t] = f.x, iv[t + 1] = f.y, iv[t + 2] = f.z, iv[t + 3] = f.w;
                    }
                    tmem_ld16(col + 16 * c, h);
                    tmem_ld16(col + NT + 16 * c, l);
                    tmem_ld_wait();
                    tmem_regs_ready(h), tmem_regs_ready(l);
    #pragma unroll
                    for (int i = 0; i < 16; i++) pr[i] = h[i] + l[i];
                    if constexpr (Q4) {
                        tmem_ld16(col + NB + 16 * c, h);
                        tmem_ld16(col + NB + NT + 16 * c, l);
                        tmem_ld_wait();
                        tmem_regs_ready(h), tmem_regs_ready(l);
    #pragma unroll
                        for (int i = 0; i < 16; i++) mn[i] = h[i] + l[i];
                    }
    #pragma unroll
                    for (int i = 0; i < 16; i++) {
                        if constexpr (Q4)
                            acc[16 * c + i] += iv[i] * (dd.x * pr[i] - dd.y * mn[i]);
                        else
                            acc[16 * c + i] += iv[i] * pr[i];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(d_empty + db);
            }
            if (u == U1 - 1 || sb == S - 1) {  // end of this CTA's run over the tile
                int ltile;
                const int gi = group_of(G, tile, ltile);
                const int n = G->n[gi], row = ltile * kRows + 32 * q + lane;
                float *y = G->y[gi];
                if (row < n)
#pragma unroll
                    for (int t = 0; t < NT; t++)
                        if (t < m) atomicAdd(y + (size_t)t * n + row, acc[t]);
#pragma unroll
                for (int t = 0; t < NT; t++) acc[t] = 0.f;
            }
        }
    }
    __syncthreads();
    if (warp == W::kMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- the int8 GEMV: 3..16 tokens ---------------------------------------------
//
// kernels/proj_q4k.comp:60-92 and proj_q8_0.comp:47-67 for up to 16 rows of x on
// the tensor cores' 8-bit path (tcgen05.mma kind::i8, K = 32): one MMA covers
// exactly one 32-element Q4_K sub-block / Q8_0 block of 128 weight rows, so the
// weights go to TMEM as their raw integers (Q4_K nibbles as u8, Q8_0 bytes as s8;
// a mask and a shift per 8 weights) and each block's scale is applied by the
// epilogue to that block's own accumulator columns.  The activations are
// X = round(x * s) (|X| <= 16256, s per (token, super-block)) in two s8 digits,
// X = 128 hi + lo, hi in B row t and lo in B row NR/2 + t (N = NR = 16 for up
// to 8 tokens, 32 for up to 16); the sums are exact integers until the
// epilogue's f32 scaling.  Q4_K's min term uses the integer sub-block sums of X.
// Accumulators are per half unit (4 blocks x NR columns); TMEM holds
// 512 / NR... : NR = 16: four A unit slots + four half-unit buffers, NR = 32:
// two A slots + three half-unit buffers.

constexpr int kG8ACols = 64;          // one unit of 8-bit weights: 256 per lane
constexpr int kG8NU = 2;              // per-unit scale slots

template <int NR>
struct G8Cfg {
    static constexpr int kXStage = NR * 256;                   // one unit's digits
    static constexpr int kASlots = NR == 16 ? 4 : 2;
    static constexpr int kHCols = 4 * NR;                      // one half-unit buffer
    static constexpr int kNH = (kTmemCols - kASlots * kG8ACols) / kHCols;  // half-unit buffers
    static constexpr int kDBase = kASlots * kG8ACols;
};

// Activation digits, one CTA per super-block, warp t = token slot t (0..T-1,
// T = blockDim / 32 = NR / 2):
//   x8 [NR][k] s8: row t the hi digit, row T + t the lo digit (zero past m);
//   inv[sb * T + t] = 1 / s; sx[(sb * 8 + j) * T + t] = the integer sum of X over
//   sub-block j (Q4_K).  The CTAs also zero y [m, n].
__global__ void x8_pack_kernel(const float *__restrict__ x, int m, int k, int8_t *__restrict__ x8,
                               float *__restrict__ inv, int *__restrict__ sx, float *__restrict__ y, long long ny) {
    const int T = blockDim.x >> 5;
    griddep_launch_dependents();  // the GEMV may start streaming its weights now
    const long long nthreads = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < ny; i += nthreads) y[i] = 0.f;
    const int sb = blockIdx.x, t = threadIdx.x >> 5, c = threadIdx.x & 31;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (t < m) {
        const float4 a = *reinterpret_cast<const float4 *>(x + (size_t)t * k + (size_t)sb * 256 + 8 * c);
        const float4 b = *reinterpret_cast<const float4 *>(x + (size_t)t * k + (size_t)sb * 256 + 8 * c + 4);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    }
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float s = mx > 0.f && mx < INFINITY ? 16256.f / mx : 0.f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int X = __float2int_rn(v[i] * s);  // |X| <= 16256
        const int hi = (X + 64) >> 7, lo = X - 128 * hi;
        sum += X;
        hw[i >> 2] |= (uint32_t)(hi & 0xFF) << (8 * (i & 3));
        lw[i >> 2] |= (uint32_t)(lo & 0xFF) << (8 * (i & 3));
    }
    *reinterpret_cast<uint2 *>(x8 + (size_t)t * k + (size_t)sb * 256 + 8 * c) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2 *>(x8 + (size_t)(T + t) * k + (size_t)sb * 256 + 8 * c) = make_uint2(lw[0], lw[1]);
    if (c == 0) inv[sb * T + t] = s > 0.f ? 1.f / s : 0.f;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (sx && (c & 3) == 0) sx[(sb * 8 + (c >> 2)) * T + t] = sum;
}

struct G8Layout {
    size_t x = 0, raw = 0, sc = 0, bars = 0, tslot = 0, total = 0;
    int XS = 0, RS = 0;
};

template <class F, int NR>
__host__ __device__ constexpr G8Layout g8_layout() {
    using C = G8Cfg<NR>;
    G8Layout L{};
    L.XS = NR == 16 ? 8 : 6;
    L.RS = F::kQ8 ? (NR == 16 ? 5 : 4) : (NR == 16 ? 9 : 8);
    L.x = 0;
    L.raw = (size_t)L.XS * C::kXStage;
    L.sc = L.raw + (size_t)L.RS * kRows * F::kRowBytes;
    L.bars = L.sc + (size_t)kG8NU * kRows * 64;
    L.tslot = L.bars + (size_t)(2 * L.RS + 2 * C::kASlots + 2 * L.XS + 2 * C::kNH + 2 * kG8NU + 1) * 8;
    L.total = L.tslot + 16 + 1024;
    return L;
}

// Instruction descriptor of kind::i8: D s32, A u8 (a_signed = 0) or s8, B s8, K-major.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n, bool a_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_i8_ts(uint32_t dtmem, uint32_t atmem, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.u32 p, 0, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dtmem),
        "r"(atmem), "l"(bdesc), "r"(idesc)
        : "memory");
}

// N consecutive 32-bit TMEM columns of this thread's lane (s32), N = 4, 8 or 16.
template <int N>
__device__ __forceinline__ void tmem_ld_s32(uint32_t taddr, int (&v)[N]) {
    if constexpr (N == 16)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(taddr));
    else if constexpr (N == 4)
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\n"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(taddr));
    else
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                       "=r"(v[7])
                     : "r"(taddr));
}

template <int N>
__device__ __forceinline__ void tmem_regs_ready_i(int (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; i++) asm volatile("" : "+r"(v[i])::"memory");
}

// One converter thread's half of a unit for the int8 GEMV: blocks 4g..4g+3 of its
// row as raw integers into TMEM at ta (block b at column 8b), and their f32 scales
// (Q4_K: d sc_j and dmin m_j; Q8_0: d).
template <class F, int g>
__device__ __forceinline__ void g8_convert(const uint8_t *raw, uint32_t ta, uint32_t ref_mask, float (&scl)[4],
                                           float (&mns)[4]) {
    if constexpr (!F::kQ8) {
        // qs groups G = 2g, 2g+1: low nibbles = sub-block 2G, high = 2G+1
        uint4 Qa[4];
#pragma unroll
        for (int i = 0; i < 4; i++) Qa[i] = lds128(raw + 16 + 64 * g + 16 * i);
        const uint4 H = lds128(raw);
#pragma unroll
        for (int gg = 0; gg < 2; gg++) {
            const uint4 A = Qa[2 * gg], B = Qa[2 * gg + 1];
            const uint32_t qw[8] = {A.x, A.y, A.z, A.w, B.x, B.y, B.z, B.w};
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                o[i] = qw[i] & 0x0F0F0F0Fu;
                o[8 + i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
            }
            tmem_st16(ta + 16 * gg, o);
        }
        uint32_t sc[8], mn[8];
        q4k_scale_mins(H, sc, mn);
        const float2 dd = scales2_f32(H.x, ref_mask);
#pragma unroll
        for (int i = 0; i < 4; i++) scl[i] = dd.x * (float)sc[4 * g + i], mns[i] = dd.y * (float)mn[4 * g + i];
    } else {
        // blocks 4g..4g+3 span row bytes 136g .. 136g + 135 (see conv_q8_half)
        uint32_t Wd[36];
#pragma unroll
        for (int i = 0; i < 9; i++) {
            const uint4 v = lds128(raw + 128 * g + 16 * i);
            Wd[4 * i] = v.x, Wd[4 * i + 1] = v.y, Wd[4 * i + 2] = v.z, Wd[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int half = 0; half < 2; half++) {
            uint32_t o[16];
#pragma unroll
            for (int bh = 0; bh < 2; bh++) {
                const int bb = 2 * half + bh, b = 4 * g + bb;
                const int wq = (17 * b + 1) / 2 - 32 * g, sh = (b & 1) ? 0 : 16;
                const uint32_t dw = Wd[((b & 1) ? (17 * (b - 1)) / 2 + 8 : (17 * b) / 2) - 32 * g];
                const uint32_t dbits = fix_sub_h2((b & 1) ? (dw >> 16) : (dw & 0xFFFFu), ref_mask) & 0xFFFFu;
                scl[bb] = __half2float(__ushort_as_half((unsigned short)dbits));
                mns[bb] = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int wi = wq + i;
                    o[8 * bh + i] = __funnelshift_r(Wd[wi], (sh && wi + 1 < 36) ? Wd[wi + 1] : 0u, sh);
                }
            }
            tmem_st16(ta + 16 * half, o);
        }
    }
}

template <class F, int MT>
__global__ void __launch_bounds__(kGemmWarps * 32, 1)
    gemv_i8_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                   const float *__restrict__ inv, const int *__restrict__ sx, float *__restrict__ y, int m, int k,
                   int n, int half_mode, unsigned *__restrict__ status) {
    constexpr int NR = MT <= 8 ? 16 : 32, T = NR / 2;  // B rows, token slots
    using C = G8Cfg<NR>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr G8Layout L = g8_layout<F, NR>();
    constexpr bool Q4 = !F::kQ8;
    constexpr int kRawStage = kRows * F::kRowBytes;
    uint8_t *x_ring = smem + L.x, *raw_ring = smem + L.raw;
    float *dslot = reinterpret_cast<float *>(smem + L.sc);  // [NU][128 rows][16]: 8 block scales (+ 8 mins)
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *raw_full = bars, *raw_empty = raw_full + L.RS;
    uint64_t *a_full = raw_empty + L.RS, *a_empty = a_full + C::kASlots;
    uint64_t *x_full = a_empty + C::kASlots, *x_empty = x_full + L.XS;
    uint64_t *d_full = x_empty + L.XS, *d_empty = d_full + C::kNH;  // half-unit accumulator buffers
    uint64_t *s_full = d_empty + C::kNH, *s_empty = s_full + kG8NU, *drain = s_empty + kG8NU;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + L.tslot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = k >> 8, Tt = (n + kRows - 1) / kRows;
    const long long TS = (long long)Tt * S;
    const int U0 = (int)(TS * blockIdx.x / gridDim.x), U1 = (int)(TS * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < L.RS; i++) mbar_init(raw_full + i, 1), mbar_init(raw_empty + i, kConvWarps);
        for (int i = 0; i < C::kASlots; i++) mbar_init(a_full + i, kConvWarps), mbar_init(a_empty + i, 1);
        for (int i = 0; i < L.XS; i++) mbar_init(x_full + i, 1), mbar_init(x_empty + i, 1);
        for (int i = 0; i < C::kNH; i++) mbar_init(d_full + i, 1), mbar_init(d_empty + i, 4);
        for (int i = 0; i < kG8NU; i++) mbar_init(s_full + i, kConvWarps), mbar_init(s_empty + i, 4);
        mbar_init(drain, kMmaWarps);
        mbar_init_fence();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    bool ok = true;
    auto fail = [&]() {
        ok = false;
        atomicOr(status, LC_DEV_WAIT_TIMEOUT);
    };

    if (warp == 0) {
        if (lane == 0) {  // producer: raw weight units and the unit's activation digits
            const uint64_t pol = l2_evict_first_policy();
            uint64_t xpol;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(xpol));
            for (int u = U0; u < U1 && ok; u++) {
                const int j = u - U0, tile = u / S, sb = u - tile * S;
                const int rs = j % L.RS, xs = j % L.XS;
                if (!mbar_wait(raw_empty + rs, ((j / L.RS) & 1) ^ 1)) { fail(); break; }
                mbar_expect_tx(raw_full + rs, kRawStage);
                tma_load_2d(raw_ring + (size_t)rs * kRawStage, &tmw, sb * F::kBoxX, tile * kRows, raw_full + rs, pol);
                if (j == 0) griddep_wait();  // the digits come from the packing kernel
                if (!mbar_wait(x_empty + xs, ((j / L.XS) & 1) ^ 1)) { fail(); break; }
                mbar_expect_tx(x_full + xs, C::kXStage);
#pragma unroll
                for (int c = 0; c < 2; c++)
                    tma_load_2d(x_ring + (size_t)xs * C::kXStage + c * (NR * 128), &tmx, sb * 256 + c * 128, 0,
                                x_full + xs, xpol);
            }
        }
    } else if (warp <= kConvWarps) {  // converters: group g = blocks 4g..4g+3 of row r
        const int g = (warp - 1) >> 2, quad = warp & 3, r = 32 * quad + lane;
        const uint32_t tlane = tbase + ((uint32_t)(32 * quad) << 16);
        const uint32_t ref_mask = half_mode == LC_HALF_REF ? 0x04000400u : 0u;
        for (int u = U0; u < U1 && ok; u++) {
            const int j = u - U0, rs = j % L.RS, as = j % C::kASlots, su = j % kG8NU;
            if (!mbar_wait(raw_full + rs, (j / L.RS) & 1) || !mbar_wait(a_empty + as, ((j / C::kASlots) & 1) ^ 1)) {
                fail();
                break;
            }
            tc_fence_after();
            const uint8_t *raw = raw_ring + (size_t)rs * kRawStage + (size_t)r * F::kRowBytes;
            const uint32_t ta = tlane + as * kG8ACols + 32 * g;  // block b at columns 8b
            float scl[4], mns[4];
            if (g == 0)
                g8_convert<F, 0>(raw, ta, ref_mask, scl, mns);
            else
                g8_convert<F, 1>(raw, ta, ref_mask, scl, mns);
            // the unit's block scales for the epilogue, once its slot is free
            if (!mbar_wait(s_empty + su, ((j / kG8NU) & 1) ^ 1)) { fail(); break; }
            float4 *ds = reinterpret_cast<float4 *>(dslot + ((size_t)su * kRows + r) * 16);
            ds[g] = make_float4(scl[0], scl[1], scl[2], scl[3]);
            if (Q4) ds[2 + g] = make_float4(mns[0], mns[1], mns[2], mns[3]);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(a_full + as);
                mbar_arrive(raw_empty + rs);
                mbar_arrive(s_full + su);
            }
        }
    } else if (warp < kMmaWarp + kMmaWarps) {
        if (lane == 0) {  // MMA issuers: even / odd units, one MMA per 32-element block
            constexpr uint32_t idesc = umma_idesc_i8(kRows, NR, F::kQ8);
            const uint64_t xdesc0 = umma_desc_sw128(smem_addr(x_ring));
            for (int u = U0 + (warp - kMmaWarp); u < U1 && ok; u += kMmaWarps) {
                const int j = u - U0, as = j % C::kASlots, xs = j % L.XS;
                if (!mbar_wait(a_full + as, (j / C::kASlots) & 1) || !mbar_wait(x_full + xs, (j / L.XS) & 1)) {
                    fail();
                    break;
                }
                const uint64_t xd = xdesc0 + (uint64_t)((xs * C::kXStage) >> 4);
                const uint32_t ta = tbase + as * kG8ACols;
                for (int h = 0; h < 2 && ok; h++) {  // half-unit buffer hj = 2j + h
                    const int hj = 2 * j + h, hb = hj % C::kNH;
                    if (!mbar_wait(d_empty + hb, ((hj / C::kNH) & 1) ^ 1)) { fail(); break; }
                    tc_fence_after();
                    const uint32_t dcol = tbase + C::kDBase + hb * C::kHCols;
#pragma unroll
                    for (int bb = 0; bb < 4; bb++) {  // block b = 4h + bb: K bytes 32b of the unit
                        const int b = 4 * h + bb;
                        umma_i8_ts(dcol + NR * bb, ta + 8 * b,
                                   xd + (uint64_t)(((b >> 2) * (NR * 128) + (b & 3) * 32) >> 4), idesc);
                    }
                    umma_commit(d_full + hb);
                }
                if (!ok) break;
                umma_commit(a_empty + as);
                umma_commit(x_empty + xs);
            }
            umma_commit(drain);
            if (!mbar_wait(drain, 0)) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        }
    } else {  // epilogue: TMEM lanes 32q..32q+31 = tile rows
        griddep_wait();  // scales, sums and the zeroed y come from the packing kernel
        const int q = warp & 3;
        const uint32_t lanes = (uint32_t)(32 * q) << 16;
        constexpr int NL = MT <= 4 ? 4 : MT <= 8 ? 8 : 16;  // columns read per digit
        float acc[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) acc[t] = 0.f;
        for (int u = U0; u < U1 && ok; u++) {
            const int j = u - U0, su = j % kG8NU, tile = u / S, sb = u - tile * S;
            float iv[MT];
#pragma unroll
            for (int t = 0; t < MT; t++) iv[t] = __ldg(inv + sb * T + t);
            if (!mbar_wait(s_full + su, (j / kG8NU) & 1)) { fail(); break; }
            const float4 *ds = reinterpret_cast<const float4 *>(dslot + ((size_t)su * kRows + 32 * q + lane) * 16);
            const float4 s0 = ds[0], s1 = ds[1];
            const float scl[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            float mns[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if constexpr (Q4) {
                const float4 m0 = ds[2], m1 = ds[3];
                mns[0] = m0.x, mns[1] = m0.y, mns[2] = m0.z, mns[3] = m0.w;
                mns[4] = m1.x, mns[5] = m1.y, mns[6] = m1.z, mns[7] = m1.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + su);
            float au[MT];
#pragma unroll
            for (int t = 0; t < MT; t++) au[t] = 0.f;
            for (int h = 0; h < 2 && ok; h++) {
                const int hj = 2 * j + h, hb = hj % C::kNH;
                if (!mbar_wait(d_full + hb, (hj / C::kNH) & 1)) { fail(); break; }
                tc_fence_after();
                const uint32_t col = tbase + lanes + C::kDBase + hb * C::kHCols;
#pragma unroll
                for (int bb = 0; bb < 4; bb++) {
                    int hi[NL], lo[NL];
                    tmem_ld_s32<NL>(col + NR * bb, hi);
                    tmem_ld_s32<NL>(col + NR * bb + T, lo);
                    tmem_ld_wait();
                    tmem_regs_ready_i(hi), tmem_regs_ready_i(lo);
#pragma unroll
                    for (int t = 0; t < MT; t++) au[t] += scl[4 * h + bb] * (float)(128 * hi[t] + lo[t]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(d_empty + hb);
            }
            if (!ok) break;
            if constexpr (Q4) {
#pragma unroll
                for (int jb = 0; jb < 8; jb++)
#pragma unroll
                    for (int t = 0; t < MT; t++) au[t] -= mns[jb] * (float)__ldg(sx + (sb * 8 + jb) * T + t);
            }
#pragma unroll
            for (int t = 0; t < MT; t++) acc[t] += iv[t] * au[t];
            if (u == U1 - 1 || sb == S - 1) {
                const int row = tile * kRows + 32 * q + lane;
                if (row < n)
#pragma unroll
                    for (int t = 0; t < MT; t++)
                        if (t < m) atomicAdd(y + (size_t)t * n + row, acc[t]);
#pragma unroll
                for (int t = 0; t < MT; t++) acc[t] = 0.f;
            }
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- lm_head: logits of 128-token tiles fused with argmax -------------------
//
// TargetModel::project_normalized_hidden (src/target.rs:580-605) for many
// hidden rows at once, followed by the argmax of src/lib.rs:456-464.  A tile is
// 128 vocab rows x 256 tokens (N = 256: every MMA at the tensor cores' full
// rate).  The activations are one f16 per element after a per-token power of
// two (no hi / lo split: the logits only feed an argmax, and the split would
// double both the MMAs and the activation reads from L2, which bound the
// kernel: each weight tile re-reads its token tile).  Weights are f16 in TMEM
// (Q8_0: f16(d q); Q4_K: the exact integer sc q, then one HFMA2 with d and
// f16(-dmin m)); the accumulator holds the whole K loop (activation scale per
// token).  Persistent CTAs walk the tiles token-tile fastest, so the CTAs that
// share a weight tile run together and read it from L2.  The epilogue writes
// the logits (optional) and reduces each token's best (logit, row) over the
// warp's 32 rows with redux.sync / ballot, then one atomicMax per warp and
// token on the order-preserving int64 key.

constexpr int kLmTok = 256;           // tokens per tile
constexpr int kLmN = kLmTok;          // UMMA N
constexpr int kLmChunk = kLmN * 128;  // one 64-column activation chunk, 32 KB
constexpr int kLmXS = 4;              // activation chunks in flight: the stream that bounds the kernel
constexpr int kLmWarps = 15;          // weight producer, 8 converters, MMA, 4 epilogue, activation producer
constexpr int kLmMma = 9;
constexpr int kLmXProd = 14;
constexpr unsigned long long kKeyMin = 0x8000000000000000ull;

// Element of position e (0..7) of position chunk c within a super-block (the
// order listed above conv_q4k_half).
__host__ __device__ __forceinline__ int chunk_elem(bool q8, int c, int e) {
    const int base = q8 ? 32 * (c >> 2) + 8 * (c & 3) : 64 * (c >> 3) + 4 * (c & 7);
    return base + (e >> 2) * (q8 ? 4 : 32) + (((e & 1) << 1) | ((e >> 1) & 1));
}

// Q4_K for the lm_head: half g of one row -> 64 TMEM columns of
// f16(d * (sc q) - f16(dmin m)) (sc q exact, one fused rounding).
template <int g>
__device__ __forceinline__ void conv_q4k_half_w(const uint8_t *raw, const uint32_t (&sc)[8], const uint32_t (&mn)[8],
                                                float d, float dmin, uint32_t taddr) {
    uint4 Qa[4];
#pragma unroll
    for (int i = 0; i < 4; i++) Qa[i] = lds128(raw + 16 + 64 * g + 16 * i);
    const __half2 d2 = __float2half2_rn(d);  // d is an f16 value: exact
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {
        const int G = 2 * g + gg;
        const __half2 slo = __float2half2_rn((float)sc[2 * G]), clo = __float2half2_rn(-1024.f * (float)sc[2 * G]);
        const __half2 shi = __float2half2_rn((float)sc[2 * G + 1] * 0.0625f),
                      chi = __float2half2_rn(-64.f * (float)sc[2 * G + 1]);
        const __half2 mlo = __float2half2_rn(-dmin * (float)mn[2 * G]), mhi = __float2half2_rn(-dmin * (float)mn[2 * G + 1]);
#pragma unroll
        for (int w4 = 0; w4 < 2; w4++) {
            const uint4 Q = Qa[2 * gg + w4];
            const uint32_t qw[4] = {Q.x, Q.y, Q.z, Q.w};
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t W = qw[i], W8 = W >> 8;
                o[4 * i + 0] = h22u(__hfma2(__hfma2(u2h2((W & 0x000F000Fu) | 0x64006400u), slo, clo), d2, mlo));
                o[4 * i + 1] = h22u(__hfma2(__hfma2(u2h2((W8 & 0x000F000Fu) | 0x64006400u), slo, clo), d2, mlo));
                o[4 * i + 2] = h22u(__hfma2(__hfma2(u2h2((W & 0x00F000F0u) | 0x64006400u), shi, chi), d2, mhi));
                o[4 * i + 3] = h22u(__hfma2(__hfma2(u2h2((W8 & 0x00F000F0u) | 0x64006400u), shi, chi), d2, mhi));
            }
            tmem_st16(taddr + 32 * gg + 16 * w4, o);
        }
    }
}

// lm_head activation packing, one CTA per token slot (m rounded up to 256):
// x16 [TT * 256][k] f16 (row t: token t) in the converters' k order, x scaled
// by a power of two per token; inv[t] its inverse (0 past m); keys[t] (t < m)
// reset to the smallest key.
__global__ void lmh_pack_kernel(const float *__restrict__ x, int m, int k, int q8, __half *__restrict__ x16,
                                float *__restrict__ inv, unsigned long long *__restrict__ keys) {
    const int t = blockIdx.x;
    __shared__ float red[32];
    float mx = 0.f;
    if (t < m)
        for (int i = threadIdx.x; i < k; i += blockDim.x) mx = fmaxf(mx, fabsf(x[(size_t)t * k + i]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    float s, iv;
    act_scale(red[0], s, iv);
    if (threadIdx.x == 0) {
        inv[t] = t < m ? iv : 0.f;
        if (keys && t < m) keys[t] = kKeyMin;
    }
    __half *xr16 = x16 + (size_t)t * k;
    for (int q = threadIdx.x; q < k / 8; q += blockDim.x) {  // position chunk c of super-block sb
        const int sb = q >> 5, c = q & 31;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (t < m) {
            const float *xr = x + (size_t)t * k + (size_t)sb * 256;
            a = *reinterpret_cast<const float4 *>(xr + chunk_elem(q8 != 0, c, 0));
            b = *reinterpret_cast<const float4 *>(xr + chunk_elem(q8 != 0, c, 4));
        }
        const float v[8] = {a.x * s, a.z * s, a.y * s, a.w * s, b.x * s, b.z * s, b.y * s, b.w * s};
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; i++) h[i] = h22u(__floats2half2_rn(v[2 * i], v[2 * i + 1]));
        *reinterpret_cast<uint4 *>(xr16 + (size_t)q * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

struct LmhLayout {
    size_t x = 0, raw = 0, bars = 0, tslot = 0, total = 0;
    int RS = 0;
};

template <class F>
__host__ __device__ constexpr LmhLayout lmh_layout() {
    LmhLayout L{};
    L.RS = F::kQ8 ? 2 : 3;  // raw weight units (34 / 18 KB) in flight
    L.x = 0;
    L.raw = (size_t)kLmXS * kLmChunk;
    L.bars = L.raw + (size_t)L.RS * kRows * F::kRowBytes;
    L.tslot = L.bars + (size_t)(2 * L.RS + 2 * kASlots + 2 * kLmXS + 2 + 1) * 8;
    L.total = L.tslot + 16 + 1024;
    return L;
}

template <class F>
__global__ void __launch_bounds__(kLmWarps * 32, 1)
    lmh_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
               const float *__restrict__ inv, int m, int k, int n, uint32_t row_offset,
               unsigned long long *__restrict__ keys, float *__restrict__ logits, int half_mode,
               unsigned *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr LmhLayout L = lmh_layout<F>();
    constexpr int kLmRS = L.RS;
    constexpr int kRawStage = kRows * F::kRowBytes;
    uint8_t *x_ring = smem + L.x, *raw_ring = smem + L.raw;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *raw_full = bars, *raw_empty = raw_full + kLmRS;
    uint64_t *a_full = raw_empty + kLmRS, *a_empty = a_full + kASlots;
    uint64_t *x_full = a_empty + kASlots, *x_empty = x_full + kLmXS;
    uint64_t *d_full = x_empty + kLmXS, *d_empty = d_full + 1, *drain = d_empty + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + L.tslot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = k >> 8, RT = (n + kRows - 1) / kRows, TT = (m + kLmTok - 1) / kLmTok;
    const int ntiles = RT * TT;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kLmRS; i++) mbar_init(raw_full + i, 1), mbar_init(raw_empty + i, kConvWarps);
        for (int i = 0; i < kASlots; i++) mbar_init(a_full + i, kConvWarps), mbar_init(a_empty + i, 1);
        for (int i = 0; i < kLmXS; i++) mbar_init(x_full + i, 1), mbar_init(x_empty + i, 1);
        mbar_init(d_full, 1), mbar_init(d_empty, 4), mbar_init(drain, 1);
        mbar_init_fence();
    }
    if (warp == kLmMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot, dacc = tbase + kAccBase;
    bool ok = true;
    auto fail = [&]() {
        ok = false;
        atomicOr(status, LC_DEV_WAIT_TIMEOUT);
    };

    if (warp == 0) {
        if (lane == 0) {  // weight producer
            const uint64_t pol = l2_evict_first_policy();
            int j = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int rt = tile / TT;
                for (int sb = 0; sb < S && ok; sb++, j++) {
                    const int rs = j % kLmRS;
                    if (!mbar_wait(raw_empty + rs, ((j / kLmRS) & 1) ^ 1)) { fail(); break; }
                    mbar_expect_tx(raw_full + rs, kRawStage);
                    tma_load_2d(raw_ring + (size_t)rs * kRawStage, &tmw, sb * F::kBoxX, rt * kRows, raw_full + rs, pol);
                }
            }
        }
    } else if (warp == kLmXProd) {
        if (lane == 0) {  // activation producer: 64-column chunks of the tile's tokens
            uint64_t xpol;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(xpol));
            int xc = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int tt = tile % TT;
                for (int kc = 0; kc < 4 * S && ok; kc++, xc++) {
                    const int xs = xc % kLmXS;
                    if (!mbar_wait(x_empty + xs, ((xc / kLmXS) & 1) ^ 1)) { fail(); break; }
                    mbar_expect_tx(x_full + xs, kLmChunk);
                    tma_load_2d(x_ring + (size_t)xs * kLmChunk, &tmx, kc * 64, tt * kLmN, x_full + xs, xpol);
                }
            }
        }
    } else if (warp <= kConvWarps) {  // converters: group g converts half g of row r
        const int g = (warp - 1) >> 2, quad = warp & 3, r = 32 * quad + lane;
        const uint32_t tlane = tbase + ((uint32_t)(32 * quad) << 16);
        const uint32_t ref_mask = half_mode == LC_HALF_REF ? 0x04000400u : 0u;
        int j = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            for (int sb = 0; sb < S; sb++, j++) {
                const int rs = j % kLmRS, as = j % kASlots;
                if (!mbar_wait(raw_full + rs, (j / kLmRS) & 1) || !mbar_wait(a_empty + as, ((j / kASlots) & 1) ^ 1)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint8_t *raw = raw_ring + (size_t)rs * kRawStage + (size_t)r * F::kRowBytes;
                const uint32_t ta = tlane + as * kACols + g * 64;
                if constexpr (F::kQ8) {
                    if (g == 0)
                        conv_q8_half<0>(raw, ref_mask, ta);
                    else
                        conv_q8_half<1>(raw, ref_mask, ta);
                } else {
                    const uint4 H = lds128(raw);
                    uint32_t sc[8], mn[8];
                    q4k_scale_mins(H, sc, mn);
                    const float2 dd = scales2_f32(H.x, ref_mask);
                    if (g == 0)
                        conv_q4k_half_w<0>(raw, sc, mn, dd.x, dd.y, ta);
                    else
                        conv_q4k_half_w<1>(raw, sc, mn, dd.x, dd.y, ta);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(a_full + as);
                    mbar_arrive(raw_empty + rs);
                }
            }
        }
    } else if (warp == kLmMma) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(kRows, kLmN);
            const uint64_t xdesc0 = umma_desc_sw128(smem_addr(x_ring));
            int j = 0, xc = 0, tc = 0;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, tc++) {
                if (!mbar_wait(d_empty, (tc & 1) ^ 1)) { fail(); break; }
                tc_fence_after();
                for (int sb = 0; sb < S && ok; sb++, j++) {
                    const int as = j % kASlots;
                    if (!mbar_wait(a_full + as, (j / kASlots) & 1)) { fail(); break; }
                    // A was written by other threads' tcgen05.st: fence after that
                    // synchronisation.  The activation chunks arrive by TMA and are
                    // read by the MMA through the same async proxy, ordered by
                    // their mbarrier alone.
                    tc_fence_after();
                    for (int kc = 0; kc < 4; kc++, xc++) {
                        const int xs = xc % kLmXS;
                        if (!mbar_wait(x_full + xs, (xc / kLmXS) & 1)) { fail(); break; }
                        const uint64_t xd = xdesc0 + (uint64_t)((xs * kLmChunk) >> 4);
                        const uint32_t ta = tbase + as * kACols + kc * 32;
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_f16_ts(dacc, ta + 8 * kk, xd + (uint64_t)(2 * kk), idesc, (sb | kc | kk) ? 1u : 0u);
                        umma_commit(x_empty + xs);
                    }
                    umma_commit(a_empty + as);
                }
                if (!ok) break;
                umma_commit(d_full);
            }
            umma_commit(drain);
            if (!mbar_wait(drain, 0)) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        }
    } else {  // epilogue: TMEM lanes 32q..32q+31 = tile rows
        const int q = warp & 3;
        const uint32_t lanes = (uint32_t)(32 * q) << 16;
        int tc = 0;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, tc++) {
            const int rt = tile / TT, tt = tile - rt * TT;
            if (!mbar_wait(d_full, tc & 1)) { fail(); break; }
            tc_fence_after();
            const int row = rt * kRows + 32 * q + lane;
            const bool valid = row < n;
#pragma unroll 1
            for (int c = 0; c < kLmTok / 16; c++) {
                float ph[16], iv[16];
                const int t0 = tt * kLmTok + 16 * c;
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                    const float4 f = __ldg(reinterpret_cast<const float4 *>(inv + t0 + i));
                    iv[i] = f.x, iv[i + 1] = f.y, iv[i + 2] = f.z, iv[i + 3] = f.w;
                }
                tmem_ld16(dacc + lanes + 16 * c, ph);
                tmem_ld_wait();
                tmem_regs_ready(ph);
                // All 16 tokens' warp maxima first (independent redux / ballot
                // pairs), then lane i builds token i's key from the warp-uniform
                // maximum and winning lane: one predicated atomic per lane.
                uint32_t my_o = 0u, my_win = 0u;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int t = t0 + i;
                    const float v = ph[i] * iv[i];
                    if (logits && valid && t < m) logits[(size_t)t * n + row] = v;
                    if (!keys) continue;  // a plain projection: y = logits, no argmax
                    const uint32_t b = __float_as_uint(v);
                    const uint32_t o = valid ? ((b & 0x80000000u) ? ~b : (b | 0x80000000u)) : 0u;
                    const uint32_t mo = __reduce_max_sync(0xffffffffu, o);
                    const uint32_t win = __ballot_sync(0xffffffffu, valid && o == mo);
                    if (lane == i) my_o = mo, my_win = win;
                }
                const int t = t0 + lane;
                if (keys && lane < 16 && t < m && my_win) {
                    const uint32_t wrow = (uint32_t)(rt * kRows + 32 * q + 31 - __clz(my_win));
                    const unsigned long long key =
                        (((unsigned long long)my_o << 32) | (row_offset + wrow)) ^ kKeyMin;  // lc_make_key
                    atomicMax(reinterpret_cast<long long *>(keys) + t, (long long)key);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty);
        }
    }
    __syncthreads();
    if (warp == kLmMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- host -------------------------------------------------------------------

template <class F>
int weight_map_rows128(CUtensorMap *tm, const void *w, uint32_t k, uint32_t n) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    int s = lc_tensor_map_encoder(&enc);
    if (s) return s;
    const cuuint64_t S = k / 256;
    cuuint64_t dims[2] = {S * F::kBoxX, (cuuint64_t)n};
    cuuint64_t strides[1] = {S * F::kRowBytes};
    cuuint32_t box[2] = {(cuuint32_t)F::kBoxX, (cuuint32_t)kRows};
    cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType dt = F::kQ8 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT64;
    const CUresult r = enc(tm, dt, 2, const_cast<void *>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    LC_REQUIRE(r == CUDA_SUCCESS, LC_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
    return LC_OK;
}

// f16 activation rows [rows][k], boxes of 64 columns x box_rows rows, 128-byte swizzle.
int x16_map(CUtensorMap *tm, const void *x16, uint32_t k, int rows, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    int s = lc_tensor_map_encoder(&enc);
    if (s) return s;
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(x16), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    LC_REQUIRE(r == CUDA_SUCCESS, LC_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", (int)r);
    return LC_OK;
}

template <class F, int NT>
int launch_dq_gemm(lc_ctx *ctx, const lc::PackSrc &src, const lc::ProjOut *outs, int ng, uint32_t m, uint32_t k) {
    constexpr GemmLayout L = gemm_layout<F, NT>();
    LC_REQUIRE(L.total <= ctx->smem_optin, LC_ERR_UNSUPPORTED, "dq_gemm: %zu bytes of shared memory needed", L.total);
    const uint32_t S = k / 256;
    const size_t x16_bytes = (size_t)2 * NT * k * 2;
    const size_t sx_bytes = F::kQ8 ? 0 : (size_t)S * 2 * NT * 32;  // multiple of 16
    const size_t inv_bytes = (size_t)S * NT * 4;
    uint8_t *scr = (uint8_t *)lc_scratch(ctx, LC_SCRATCH_PACK, x16_bytes + sx_bytes + inv_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    __half *x16 = reinterpret_cast<__half *>(scr);
    uint8_t *sx16 = scr + x16_bytes;
    float *inv = reinterpret_cast<float *>(scr + x16_bytes + sx_bytes);
    DqGroup grp = {};
    ZeroList zl = {};
    int tiles = 0;
    for (int i = 0; i < ng; i++) {
        int s = weight_map_rows128<F>(&grp.tmw[i], outs[i].w, k, outs[i].n);
        if (s) return s;
        grp.y[i] = outs[i].y;
        grp.n[i] = (int)outs[i].n;
        tiles += (int)((outs[i].n + kRows - 1) / kRows);
        grp.tile_end[i] = tiles;
        if (!outs[i].accumulate) {
            zl.p[zl.cnt] = outs[i].y;
            zl.n[zl.cnt++] = (long long)m * outs[i].n;
        }
    }
    grp.ng = ng;
    CUtensorMap tmx;
    int s = x16_map(&tmx, x16, k, 2 * NT, 2 * NT);
    if (s) return s;
    const dim3 pgrid(S, NT / 8);
    const int q8 = F::kQ8 ? 1 : 0;
    if (src.op == lc::LC_PACK_SWIGLU)
        x16_pack_kernel<lc::LC_PACK_SWIGLU><<<pgrid, 256, 0, ctx->stream>>>(src.x, src.x2, 0, (int)m, (int)k, q8, NT,
                                                                           x16, sx16, inv, zl);
    else if (src.op == lc::LC_PACK_HEADGATE)
        x16_pack_kernel<lc::LC_PACK_HEADGATE><<<pgrid, 256, 0, ctx->stream>>>(src.x, src.x2, src.head_dim, (int)m,
                                                                             (int)k, q8, NT, x16, sx16, inv, zl);
    else if (src.op == lc::LC_PACK_RMSNORM)
        x16_pack_norm_kernel<<<dim3(NT, (S + 7) / 8), 256, 0, ctx->stream>>>(src.x, src.x2, src.eps, (int)m, (int)k,
                                                                            q8, NT, x16, sx16, inv, zl);
    else
        x16_pack_kernel<lc::LC_PACK_PLAIN><<<pgrid, 256, 0, ctx->stream>>>(src.x, nullptr, 0, (int)m, (int)k, q8, NT,
                                                                          x16, sx16, inv, zl);
    s = lc_set_smem_attr((const void *)dq_gemm_kernel<F, NT>, L.total);
    constexpr int kThreads = DqWarps<NT>::kAll * 32;
    if (s) return s;
    const long long TS = (long long)tiles * S;
    const int grid = (int)std::max<long long>(1, std::min<long long>(ctx->num_sms, TS));
    // a programmatic dependent of the packing kernel: weights stream while the
    // activations are packed
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LC_CUDA(cudaLaunchKernelEx(&cfg, dq_gemm_kernel<F, NT>, grp, tmx, (const uint8_t *)sx16, (const float *)inv, (int)m,
                               (int)k, ctx->half_mode, ctx->dev_status));
    return LC_OK;
}

// s8 activation digits [nr][k], boxes of 128 columns x nr rows, 128-byte swizzle.
int x8_map(CUtensorMap *tm, const void *x8, uint32_t k, int nr) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    int s = lc_tensor_map_encoder(&enc);
    if (s) return s;
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)nr};
    cuuint64_t strides[1] = {(cuuint64_t)k};
    cuuint32_t box[2] = {128, (cuuint32_t)nr};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(x8), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    LC_REQUIRE(r == CUDA_SUCCESS, LC_ERR_CUDA, "cuTensorMapEncodeTiled (activation digits) failed (%d)", (int)r);
    return LC_OK;
}

template <class F, int MT>
int launch_gemv_i8(lc_ctx *ctx, const float *x, const uint8_t *w, float *y, uint32_t m, uint32_t k, uint32_t n) {
    constexpr int NR = MT <= 8 ? 16 : 32, T = NR / 2;
    constexpr G8Layout L = g8_layout<F, NR>();
    LC_REQUIRE(L.total <= ctx->smem_optin, LC_ERR_UNSUPPORTED, "gemv_i8: %zu bytes of shared memory needed", L.total);
    const uint32_t S = k / 256;
    const size_t x8_bytes = (size_t)NR * k, inv_bytes = (size_t)S * T * 4;
    const size_t sx_bytes = F::kQ8 ? 0 : (size_t)S * 8 * T * 4;
    uint8_t *scr = (uint8_t *)lc_scratch(ctx, LC_SCRATCH_PACK, x8_bytes + inv_bytes + sx_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    int8_t *x8 = reinterpret_cast<int8_t *>(scr);
    float *inv = reinterpret_cast<float *>(scr + x8_bytes);
    int *sx = F::kQ8 ? nullptr : reinterpret_cast<int *>(scr + x8_bytes + inv_bytes);
    CUtensorMap tmw, tmx;
    int s = weight_map_rows128<F>(&tmw, w, k, n);
    if (s) return s;
    s = x8_map(&tmx, x8, k, NR);
    if (s) return s;
    x8_pack_kernel<<<S, 32 * T, 0, ctx->stream>>>(x, (int)m, (int)k, x8, inv, sx, y, (long long)m * n);
    s = lc_set_smem_attr((const void *)gemv_i8_kernel<F, MT>, L.total);
    if (s) return s;
    const long long TS = (long long)((n + kRows - 1) / kRows) * S;
    const int grid = (int)std::max<long long>(1, std::min<long long>(ctx->num_sms, TS));
    // launched as a programmatic dependent of the packing kernel: weights stream
    // while the activations are digitised
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmWarps * 32);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LC_CUDA(cudaLaunchKernelEx(&cfg, gemv_i8_kernel<F, MT>, tmw, tmx, (const float *)inv, (const int *)sx, y, (int)m,
                               (int)k, (int)n, ctx->half_mode, ctx->dev_status));
    return LC_OK;
}

template <class F>
int launch_lmh(lc_ctx *ctx, const float *x, const uint8_t *w, uint32_t m, uint32_t k, uint32_t n,
               uint32_t row_offset, uint64_t *keys, float *logits) {
    constexpr LmhLayout L = lmh_layout<F>();
    LC_REQUIRE(L.total <= ctx->smem_optin, LC_ERR_UNSUPPORTED, "lm_head: %zu bytes of shared memory needed", L.total);
    const uint32_t TT = (m + kLmTok - 1) / kLmTok, RT = (n + kRows - 1) / kRows;
    const size_t x16_bytes = (size_t)TT * kLmN * k * 2, inv_bytes = (size_t)TT * kLmTok * 4;
    uint8_t *scr = (uint8_t *)lc_scratch(ctx, LC_SCRATCH_PACK, x16_bytes + inv_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    __half *x16 = reinterpret_cast<__half *>(scr);
    float *inv = reinterpret_cast<float *>(scr + x16_bytes);
    CUtensorMap tmw, tmx;
    int s = weight_map_rows128<F>(&tmw, w, k, n);
    if (s) return s;
    s = x16_map(&tmx, x16, k, (int)(TT * kLmN), kLmN);
    if (s) return s;
    lmh_pack_kernel<<<TT * kLmTok, 256, 0, ctx->stream>>>(x, (int)m, (int)k, F::kQ8 ? 1 : 0, x16, inv,
                                                           reinterpret_cast<unsigned long long *>(keys));
    s = lc_set_smem_attr((const void *)lmh_kernel<F>, L.total);
    if (s) return s;
    const long long tiles = (long long)RT * TT;
    const int grid = (int)std::max<long long>(1, std::min<long long>(ctx->num_sms, tiles));
    lmh_kernel<F><<<grid, kLmWarps * 32, L.total, ctx->stream>>>(tmw, tmx, inv, (int)m, (int)k, (int)n, row_offset,
                                                                 reinterpret_cast<unsigned long long *>(keys), logits,
                                                                 ctx->half_mode, ctx->dev_status);
    return LC_OK;
}

}  // namespace

namespace lc {

// Quantized GEMM on tcgen05 for 5..32 tokens; LC_ERR_UNSUPPORTED when the
// shape is not covered (the caller falls back).
int gemm_dq(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n) {
    PackSrc src;
    src.x = x;
    ProjOut out;
    out.w = w;
    out.y = y;
    out.n = n;
    return gemm_dq_group(ctx, dtype, src, &out, 1, m, k);
}

int gemm_dq_group(lc_ctx *ctx, int dtype, const PackSrc &src, const ProjOut *outs, int ng, uint32_t m, uint32_t k) {
    if (m == 0 || m > 32 || ng < 1 || ng > kGroupMax || k % 256 != 0 || ((uintptr_t)src.x & 15) != 0 ||
        (long long)k * 32 >= (1ll << 31))
        return LC_ERR_UNSUPPORTED;
    if ((src.op == LC_PACK_SWIGLU || src.op == LC_PACK_RMSNORM) && ((uintptr_t)src.x2 & 15) != 0)
        return LC_ERR_UNSUPPORTED;
    if (src.op == LC_PACK_HEADGATE && (src.head_dim <= 0 || src.head_dim % 4 != 0 || k % src.head_dim != 0))
        return LC_ERR_UNSUPPORTED;
    long long tiles = 0;
    for (int i = 0; i < ng; i++) {
        if (((uintptr_t)outs[i].w & 15) != 0 || outs[i].n == 0) return LC_ERR_UNSUPPORTED;
        tiles += (outs[i].n + kRows - 1) / kRows;
    }
    if (tiles * (k / 256) >= (1ll << 31)) return LC_ERR_UNSUPPORTED;
    if (dtype == LC_Q4_K)
        return m <= 16 ? launch_dq_gemm<GQ4K, 16>(ctx, src, outs, ng, m, k)
                       : launch_dq_gemm<GQ4K, 32>(ctx, src, outs, ng, m, k);
    if (dtype == LC_Q8_0)
        return m <= 16 ? launch_dq_gemm<GQ8_0, 16>(ctx, src, outs, ng, m, k)
                       : launch_dq_gemm<GQ8_0, 32>(ctx, src, outs, ng, m, k);
    return LC_ERR_UNSUPPORTED;
}

bool routes_to_gemm_dq(const lc_ctx *ctx, uint32_t m) {
    return ctx->gemm_tc && m > 4 && m <= 32 && !((int)m >= ctx->gemv_i8_min && (int)m <= ctx->gemv_i8_max);
}

// lm_head logits + argmax on tcgen05 for a vocab shard (rows [0, n) of w,
// global index row_offset + row); LC_ERR_UNSUPPORTED when the shape is not
// covered.  keys[t] is reset and then receives the shard's best key.
int lm_head_tc(lc_ctx *ctx, int dtype, const float *x, const void *w, uint32_t m, uint32_t k, uint32_t n,
               uint32_t row_offset, uint64_t *keys, float *logits) {
    if (m == 0 || n == 0 || k % 256 != 0 || ((uintptr_t)w & 15) != 0 || ((uintptr_t)x & 15) != 0 ||
        (long long)k * 32 >= (1ll << 31))
        return LC_ERR_UNSUPPORTED;
    const uint8_t *wb = (const uint8_t *)w;
    if (dtype == LC_Q8_0) return launch_lmh<GQ8_0>(ctx, x, wb, m, k, n, row_offset, keys, logits);
    if (dtype == LC_Q4_K) return launch_lmh<GQ4K>(ctx, x, wb, m, k, n, row_offset, keys, logits);
    return LC_ERR_UNSUPPORTED;
}

// ctx->gemv_i8_min..ctx->gemv_i8_max-token projections (at most 16) on the
// 8-bit tensor-core path (by default 3..8: 1 and 2 tokens stream faster through
// the TMA GEMV of lc_proj.cu); LC_ERR_UNSUPPORTED when the shape is not
// covered (the caller falls back).
int gemv_i8(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n) {
    if ((int)m < ctx->gemv_i8_min || (int)m > ctx->gemv_i8_max || m > 16 || k % 256 != 0 ||
        ((uintptr_t)w & 15) != 0 || ((uintptr_t)x & 15) != 0 || (long long)k * 32 >= (1ll << 31))
        return LC_ERR_UNSUPPORTED;
    const uint8_t *wb = (const uint8_t *)w;
    if (dtype == LC_Q4_K)
        return m == 1   ? launch_gemv_i8<GQ4K, 1>(ctx, x, wb, y, m, k, n)
               : m == 2 ? launch_gemv_i8<GQ4K, 2>(ctx, x, wb, y, m, k, n)
               : m <= 4 ? launch_gemv_i8<GQ4K, 4>(ctx, x, wb, y, m, k, n)
               : m <= 8 ? launch_gemv_i8<GQ4K, 8>(ctx, x, wb, y, m, k, n)
                        : launch_gemv_i8<GQ4K, 16>(ctx, x, wb, y, m, k, n);
    if (dtype == LC_Q8_0)
        return m == 1   ? launch_gemv_i8<GQ8_0, 1>(ctx, x, wb, y, m, k, n)
               : m == 2 ? launch_gemv_i8<GQ8_0, 2>(ctx, x, wb, y, m, k, n)
               : m <= 4 ? launch_gemv_i8<GQ8_0, 4>(ctx, x, wb, y, m, k, n)
               : m <= 8 ? launch_gemv_i8<GQ8_0, 8>(ctx, x, wb, y, m, k, n)
                        : launch_gemv_i8<GQ8_0, 16>(ctx, x, wb, y, m, k, n);
    return LC_ERR_UNSUPPORTED;
}

// Projections of more than 32 rows (the context prefill) through the lm_head
// tiles with the argmax off: y [m, n] = x . W^T.  LC_ERR_UNSUPPORTED when the
// shape is not covered.
int gemm_large(lc_ctx *ctx, int dtype, const float *x, const void *w, float *y, uint32_t m, uint32_t k, uint32_t n) {
    return lm_head_tc(ctx, dtype, x, w, m, k, n, 0, nullptr, y);
}

}  // namespace lc
