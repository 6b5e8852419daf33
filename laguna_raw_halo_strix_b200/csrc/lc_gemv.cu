// lc_gemv.cu -- GGUF Q4_K / Q8_0 matrix-vector products for one and two tokens
// with the activations kept in f32 (the decode GEMV).
//
// Reference: kernels/proj_q4k.comp:60-92 and kernels/proj_q8_0.comp:47-67
// compute c[i] = sum_j x[j] * w(i, j), one output row per invocation, with the
// weight decoded to f32 (Q4_K: w = d*sc*q - dmin*m, proj_q4k.comp:87; Q8_0:
// w = d*q, proj_q8_0.comp:53-64) and a serial f32 accumulation.
//
// Here every weight byte streams once from HBM and the activations stay in
// registers, in f32, for the whole kernel:
//
//  * One CTA per SM owns a contiguous range of rows.  Its warps form row
//    groups of one warp per k-slice (2048 elements for one token, 1024 for
//    two); row group r takes rows r, r + rg, ... of the range.  A warp copies
//    its slice of each row (1152 bytes of Q4_K) into a ring of `depth` row
//    buffers in shared memory with 16-byte cp.async, 32 lanes on 512
//    contiguous bytes per instruction: whole cache lines, the fewest memory
//    requests per byte (an SM's outstanding requests, not its bytes, bound its
//    share of HBM).  Lanes then read the bytes of their own k positions.
//  * The activations: the first warp of each k-slice loads them, forms the
//    lanes' pre-scaled pairs (below) once, and leaves them in a shared table
//    that every warp of the slice reads into registers.
//  * Sums are grouped per 32-element sub-block, which carries one scale:
//    Q4_K  y += d * sc * S(q * x) - dmin * m * S(x)
//    Q8_0  y += d * (S((q + 128) * x) - 128 * S(x))
//    -- the reference's products regrouped, in f32 FMAs throughout.  Lane
//    partials of four rows are reduced with warp shuffles; after a named
//    barrier per row group its first warp adds the k-slices in a fixed order
//    and writes y (the result does not depend on timing).
//
// Integer weight -> f32 without the conversion unit: a nibble (or a biased
// byte) masked in place at bit s of a 32-bit word, read as a float, is the
// subnormal q * 2^(s-149) -- exact, and FMA takes subnormal operands at full
// rate (no flush-to-zero anywhere in this file).  Each lane pre-scales its
// activations once by 2^(E - s), E a power of two that puts the lane's largest
// |x| just below 2^101, so every product
//     q * 2^(s-149) * x * 2^(E-s) = q * x * 2^(E-149)
// is a normal float: the FMA rounds it exactly as f32 rounds q * x, and the
// sums are the f32 sums of q * x times a power of two that the row epilogue
// takes out again (f = 2^(149-E)).  One AND per weight and one packed f32x2 FMA
// per two weights (two tokens: per four weight-token products).  Activations
// above 2^105 in magnitude overflow the pre-scale (inf); no real activation
// comes near.
#include <algorithm>
#include <cstdlib>

#include "lc_internal.cuh"
#include "lc_sm100.cuh"

namespace {

constexpr int kGvMaxWarps = 16;  // warps per CTA

// Launch arguments (a __grid_constant__ parameter block).  Up to lc::kGroupMax
// matrices of one format and one k share the activations: their rows form one
// row space, matrix g holding rows [rows_end[g-1], rows_end[g]).
struct GvArgs {
    const uint8_t *w[lc::kGroupMax];
    float *y[lc::kGroupMax];
    int rows_end[lc::kGroupMax];
    int ng;
    const float *x;   // [M][k]
    const float *x2;  // when set, the activation is silu(x) * x2 (kernels/activation.comp)
    int k, row_bytes;
    int ks, rg;  // k-slices (warps per row group), row groups
    int part_rows;  // rows of a CTA's range the partial-sum array holds (>= every range)
    int pairs;      // two matrices of n rows interleaved (row 2i of matrix 0, 2i + 1 of matrix 1):
                    // y[0] [M][n] receives SiLU(matrix 0 row) * (matrix 1 row), activation.comp
    int half_mode;
    unsigned *status;
};

// Shared memory: the ring [warps][depth][slice bytes], the activations xs
// [M][kpad] (f32, SiLU-gated for the SwiGLU form, 4 floats of padding after
// every 64 so the lanes' 16-byte reads of their runs fall in distinct banks),
// partial sums part [part_rows][ks][M] floats (one per row of the CTA's range
// and k-slice, summed once at the end).
__host__ __device__ __forceinline__ int gv_kpad(int k) { return k + (k >> 4); }
struct GvLayout {
    size_t ring, xs, part, total;
};
__host__ __device__ __forceinline__ GvLayout gv_layout(int warps, int depth, int slice_bytes, int k, int part_rows,
                                                       int ks, int m) {
    GvLayout L;
    L.ring = 0;
    L.xs = (size_t)warps * depth * slice_bytes;
    L.part = L.xs + (size_t)m * gv_kpad(k) * 4;  // k rounded up to whole k-slices by the caller
    L.total = L.part + (size_t)part_rows * ks * m * 4 + 128;  // + slack to 128-align the base
    return L;
}

// Virtual row r of the launch -> matrix g and the row within it.
__device__ __forceinline__ void gv_row(const GvArgs &a, int r, int &g, int &i) {
    if (a.pairs) {
        g = r & 1;
        i = r >> 1;
        return;
    }
    g = 0;
    while (g < a.ng - 1 && r >= a.rows_end[g]) g++;
    i = r - (g ? a.rows_end[g - 1] : 0);
}

__device__ __forceinline__ uint64_t fma2b(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul2b(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add2b(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float sum2f(uint64_t v) {
    return __uint_as_float((uint32_t)v) + __uint_as_float((uint32_t)(v >> 32));
}

// Byte k (0..3) of w as a float, exact: the bits of 2^23 + byte minus 2^23.
__device__ __forceinline__ float byte_f(uint32_t w, uint32_t k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | k)) - 8388608.0f;
}

// The lane's exponent E from the largest |x| it holds: max|x| * 2^E < 2^101;
// E = 22 at the least keeps f = 2^(149-E) a float.
__device__ __forceinline__ int lane_exp(float mx) {
    const int eb = (int)(__float_as_uint(mx) >> 23);  // biased exponent, mx >= 0 (inf: 255)
    return max(227 - eb, 22);
}
__device__ __forceinline__ float lane_f(int E) { return __uint_as_float((uint32_t)(276 - E) << 23); }

// N activations of a run [e0, e0 + N) inside one 64-element block, from the
// padded shared copy of a token's row.
template <int N>
__device__ __forceinline__ void load_pad(const float *xs, int e0, float (&v)[N]) {
    const float *p = xs + e0 + ((e0 >> 6) << 2);
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        const float4 a = *reinterpret_cast<const float4 *>(p + i);
        v[i] = a.x, v[i + 1] = a.y, v[i + 2] = a.z, v[i + 3] = a.w;
    }
}

// ---------------------------------------------------------------------------
// Q4_K lane.  A 144-byte super-block: d, dmin (f16) at 0, twelve 6-bit scale /
// min bytes at 4, 128 nibble bytes at 16; nibble byte c of 32-byte group g
// holds element 64g + c (low nibble, sub-block 2g) and 64g + 32 + c (high
// nibble, sub-block 2g + 1) (proj_q4k.comp:77-82).  One token: a lane owns
// group g of its super-block (32 bytes, 64 weights, 4 lanes per super-block,
// 8 super-blocks per warp); two tokens: half of a group (16 bytes, 8 lanes per
// super-block, 4 per warp).
//
// Words are taken in pairs (w0, w1) as one 64-bit value W: the eight nibble
// positions of a byte lane are masked in place from W (bits 0..19) or from
// T = W >> 12 (bits 8..19), each mask giving two subnormal floats, and one
// f32x2 FMA multiplies them by the pre-scaled activations of the two elements
// (c and c + 4) they stand for.
//   pos  0: lo b0 (W, s 0)   1: hi b0 (W, 4)    2: lo b1 (W, 8)   3: hi b1 (W, 12)
//        4: lo b2 (W, 16)    5: hi b2 (T, 8)    6: lo b3 (T, 12)  7: hi b3 (T, 16)
__host__ __device__ constexpr int q4_pos_shift(int pos) { return pos < 5 ? 4 * pos : 4 * pos - 12; }

template <int M>
struct Q4Lane {
    static constexpr int NP = M == 1 ? 4 : 2;  // word pairs per lane
    static constexpr int SPW = M == 1 ? 8 : 4;  // super-blocks per warp slice
    static constexpr int SLICE = SPW * 144;           // bytes of a row per warp slice
    static constexpr int DEPTH = 8;                   // rows in flight per warp (a power of two)
    uint64_t xp[M][NP][8];                      // pre-scaled activation pairs
    float sx[M][2];                             // S(x) over the lane's low / high elements
    float f[M];                                 // 2^(149 - E)
    int hdr, qs;                                // byte offsets in the warp's slice of a row
    int e0;                                     // first low-nibble element of the lane
    uint32_t cm, am, sa, bsel;                  // scale / min byte extraction
    bool on;

    static constexpr int NE = 8 * NP;  // elements per nibble half
    using Raw = float[M][2][NE];         // the lane's activations as loaded

    // Lane geometry: which bytes of a row the lane reads.
    __device__ __forceinline__ void geom(const GvArgs &a, int slice, int lane) {
        const int S = a.k >> 8;
        const int sbl = M == 1 ? lane >> 2 : lane >> 3;
        const int g = M == 1 ? lane & 3 : (lane >> 1) & 3;
        const int half = M == 1 ? 0 : lane & 1;
        const int sb = slice * SPW + sbl;
        on = sb < S;
        hdr = sbl * 144;
        qs = hdr + 16 + 32 * g + 16 * half;
        e0 = sb * 256 + 64 * g + 16 * half;
        // get_scale_min_k4 (proj_q4k.comp:46-58) for sub-blocks 2g, 2g+1 from
        // the header words y = q[0..3], z = q[4..7], w = q[8..11]:
        //   g < 2:  sc = y & 63,                    m = z & 63
        //   g >= 2: sc = (w & 15) | ((y >> 2) & 48), m = ((w >> 4) & 15) | ((z >> 2) & 48)
        // at bytes 2(g&1), 2(g&1)+1 of the word
        const bool lo = g < 2;
        cm = lo ? 0u : 0x0F0F0F0Fu;
        am = lo ? 0x3F3F3F3Fu : 0x30303030u;
        sa = lo ? 0u : 2u;
        bsel = 2u * (uint32_t)(g & 1);
    }

    // The lane's activations (the SwiGLU form reads both inputs).
    __device__ __forceinline__ void load(const float *xs, int kpad, Raw &v) const {
#pragma unroll
        for (int j = 0; j < M; j++) {
            if (on) {
                load_pad<NE>(xs + (size_t)j * kpad, e0, v[j][0]);
                load_pad<NE>(xs + (size_t)j * kpad, e0 + 32, v[j][1]);
            } else {
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int i = 0; i < NE; i++) v[j][h][i] = 0.f;
            }
        }
    }

    // One token: the first warp of each k-slice publishes its lanes' pre-scaled
    // pairs, sums and f as a table the slice's other warps load, written over
    // the slice's own 8704 bytes of xs: [p][pos][lane] pairs, then [lane]
    // (sx0, sx1, f).
    static constexpr bool SHARE = M == 1;
    static constexpr int SLICE_ELEMS = M == 1 ? 2048 : 1024;
    __device__ __forceinline__ void store_table(unsigned char *t, int lane) const {
        uint64_t *tp = reinterpret_cast<uint64_t *>(t);
        float4 *ta = reinterpret_cast<float4 *>(t + M * NP * 8 * 32 * 8);
#pragma unroll
        for (int j = 0; j < M; j++) {
#pragma unroll
            for (int p = 0; p < NP; p++)
#pragma unroll
                for (int pos = 0; pos < 8; pos++) tp[((j * NP + p) * 8 + pos) * 32 + lane] = xp[j][p][pos];
            ta[j * 32 + lane] = make_float4(sx[j][0], sx[j][1], f[j], 0.f);
        }
    }
    __device__ __forceinline__ void load_table(const unsigned char *t, int lane) {
        const uint64_t *tp = reinterpret_cast<const uint64_t *>(t);
        const float4 *ta = reinterpret_cast<const float4 *>(t + M * NP * 8 * 32 * 8);
#pragma unroll
        for (int j = 0; j < M; j++) {
#pragma unroll
            for (int p = 0; p < NP; p++)
#pragma unroll
                for (int pos = 0; pos < 8; pos++) xp[j][p][pos] = tp[((j * NP + p) * 8 + pos) * 32 + lane];
            const float4 v = ta[j * 32 + lane];
            sx[j][0] = v.x, sx[j][1] = v.y, f[j] = v.z;
        }
    }

    struct Bytes {
        uint4 hd, q[NP / 2];
    };
    __device__ __forceinline__ void fetch(const uint8_t *slot, Bytes &b) const {
        b.hd = lds128(slot + hdr);
#pragma unroll
        for (int i = 0; i < NP / 2; i++) b.q[i] = lds128(slot + qs + 16 * i);
    }

    // Sums, exponent and pre-scaled pairs from the loaded activations.
    __device__ __forceinline__ void prep(const Raw &v) {
#pragma unroll
        for (int j = 0; j < M; j++) {
            float mx = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int i = 0; i < NE; i++) {
                mx = fmaxf(mx, fmaxf(fabsf(v[j][0][i]), fabsf(v[j][1][i])));
                s0 += v[j][0][i];
                s1 += v[j][1][i];
            }
            sx[j][0] = s0;
            sx[j][1] = s1;
            const int E = lane_exp(mx);
            f[j] = lane_f(E);
            // one scale pair per nibble shift s in {0, 4, 8, 12, 16}
            uint64_t sc[5][2];
#pragma unroll
            for (int i = 0; i < 5; i++) {
                const int e = E - 4 * i, e1 = min(e, 127);
                const float f1 = __uint_as_float((uint32_t)(e1 + 127) << 23);
                const float f2 = __uint_as_float((uint32_t)(e - e1 + 127) << 23);
                sc[i][0] = pack2f(f1, f1);
                sc[i][1] = pack2f(f2, f2);
            }
#pragma unroll
            for (int p = 0; p < NP; p++)
#pragma unroll
                for (int pos = 0; pos < 8; pos++) {
                    const int b = pos >> 1, h = pos & 1, c = 8 * p + b, si = q4_pos_shift(pos) >> 2;
                    xp[j][p][pos] = mul2b(mul2b(pack2f(v[j][h][c], v[j][h][c + 4]), sc[si][0]), sc[si][1]);
                }
        }
    }

    // Partial dot products of one row for M tokens.
    __device__ __forceinline__ void row(const Bytes &b, uint32_t ref_mask, float (&out)[M]) const {
        uint32_t q[2 * NP];
#pragma unroll
        for (int i = 0; i < NP / 2; i++)
            q[4 * i] = b.q[i].x, q[4 * i + 1] = b.q[i].y, q[4 * i + 2] = b.q[i].z, q[4 * i + 3] = b.q[i].w;
        uint64_t acc[M][4];
#pragma unroll
        for (int j = 0; j < M; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0ull;
#pragma unroll
        for (int p = 0; p < NP; p++) {
            const uint64_t W = (uint64_t)q[2 * p] | ((uint64_t)q[2 * p + 1] << 32);
            const uint64_t T = W >> 12;
            uint64_t v[8];
            v[0] = W & 0x0000000F0000000Full;
            v[1] = W & 0x000000F0000000F0ull;
            v[2] = W & 0x00000F0000000F00ull;
            v[3] = W & 0x0000F0000000F000ull;
            v[4] = W & 0x000F0000000F0000ull;
            v[5] = T & 0x00000F0000000F00ull;
            v[6] = T & 0x0000F0000000F000ull;
            v[7] = T & 0x000F0000000F0000ull;
#pragma unroll
            for (int j = 0; j < M; j++)
#pragma unroll
                for (int pos = 0; pos < 8; pos++) {
                    // low nibbles (even pos) -> acc 0 / 2, high -> 1 / 3, alternating by pair
                    const int ai = (pos & 1) + 2 * ((pos >> 2) & 1);
                    acc[j][ai] = fma2b(v[pos], xp[j][p][pos], acc[j][ai]);
                }
        }
        const float2 dd = scales2_f32(b.hd.x, ref_mask);  // (d, dmin)
        const uint32_t scw = (b.hd.w & cm) | ((b.hd.y >> sa) & am);
        const uint32_t mnw = ((b.hd.w >> 4) & cm) | ((b.hd.z >> sa) & am);
        const float sc0 = byte_f(scw, bsel), sc1 = byte_f(scw, bsel + 1);
        const float m0 = byte_f(mnw, bsel), m1 = byte_f(mnw, bsel + 1);
#pragma unroll
        for (int j = 0; j < M; j++) {
            const float alo = sum2f(add2b(acc[j][0], acc[j][2]));
            const float ahi = sum2f(add2b(acc[j][1], acc[j][3]));
            const float t = fmaf(sc1, ahi, sc0 * alo);
            const float s = fmaf(m1, sx[j][1], m0 * sx[j][0]);
            out[j] = on ? fmaf(dd.x * f[j], t, -(dd.y * s)) : 0.f;
        }
    }
};

// ---------------------------------------------------------------------------
// Q8_0 lane (one token): two 34-byte blocks (f16 d, 32 int8), 68 bytes at
// 68 * lane of the warp's 2176-byte slice, read as 17 aligned words.  Block A's
// q bytes start at byte 2, block B's d sits in the high half of word 8 and its
// q bytes fill words 9..16.  Bytes are biased to q + 128 (0..255) with one XOR
// inside the mask, masked in place at bit 0 or 8 (bytes 2, 3 from the word
// shifted down by 16), and read as subnormals.
struct Q8Lane {
    static constexpr int SLICE = 64 * 34;                  // 64 blocks per warp slice
    static constexpr int DEPTH = 4;                        // rows in flight per warp (a power of two)
    float xp[64];  // pre-scaled activations: block A elements 0..31, block B 32..63
    float sx[2];   // S(x) over block A, block B
    float f;
    int off;       // byte offset of the lane's blocks in the warp's slice of a row
    int e0;        // first element of the lane
    bool on;

    using Raw = float[64];

    __device__ __forceinline__ void geom(const GvArgs &a, int slice, int lane) {
        const int nblk = a.k >> 5;
        const int blk = 64 * slice + 2 * lane;
        on = blk < nblk;
        off = 68 * lane;
        e0 = 32 * blk;
    }

    // As the one-token Q4_K lane: the slice's table over its 8704 bytes of xs,
    // [i][lane] activations, then [lane] (sx0, sx1, f).
    static constexpr bool SHARE = true;
    static constexpr int SLICE_ELEMS = 2048;
    __device__ __forceinline__ void store_table(unsigned char *t, int lane) const {
        float *tp = reinterpret_cast<float *>(t);
#pragma unroll
        for (int i = 0; i < 64; i++) tp[i * 32 + lane] = xp[i];
        reinterpret_cast<float4 *>(t + 64 * 32 * 4)[lane] = make_float4(sx[0], sx[1], f, 0.f);
    }
    __device__ __forceinline__ void load_table(const unsigned char *t, int lane) {
        const float *tp = reinterpret_cast<const float *>(t);
#pragma unroll
        for (int i = 0; i < 64; i++) xp[i] = tp[i * 32 + lane];
        const float4 v = reinterpret_cast<const float4 *>(t + 64 * 32 * 4)[lane];
        sx[0] = v.x, sx[1] = v.y, f = v.z;
    }

    __device__ __forceinline__ void load(const float *xs, int kpad, Raw &v) const {
        (void)kpad;
        if (on) {
            load_pad<64>(xs, e0, v);
        } else {
#pragma unroll
            for (int i = 0; i < 64; i++) v[i] = 0.f;
        }
    }


    struct Bytes {
        uint32_t w[17];
    };
    __device__ __forceinline__ void fetch(const uint8_t *slot, Bytes &b) const {
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(slot + off);
#pragma unroll
        for (int i = 0; i < 17; i++) b.w[i] = lds32(wp + i);
    }

    __device__ __forceinline__ void prep(const Raw &v) {
        float mx = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            mx = fmaxf(mx, fmaxf(fabsf(v[i]), fabsf(v[32 + i])));
            s0 += v[i];
            s1 += v[32 + i];
        }
        sx[0] = s0;
        sx[1] = s1;
        const int E = lane_exp(mx);
        f = lane_f(E);
        float sc[2][2];  // 2^(E - s) for s = 0, 8 as two factors
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int e = E - 8 * i, e1 = min(e, 127);
            sc[i][0] = __uint_as_float((uint32_t)(e1 + 127) << 23);
            sc[i][1] = __uint_as_float((uint32_t)(e - e1 + 127) << 23);
        }
#pragma unroll
        for (int i = 0; i < 64; i++) {
            // byte position of the element in the lane's 68 bytes: A at 2 + i, B at 36 + (i - 32)
            const int bp = i < 32 ? 2 + i : 4 + i;
            xp[i] = (v[i] * sc[bp & 1][0]) * sc[bp & 1][1];
        }
    }

    __device__ __forceinline__ void row(const Bytes &b, uint32_t ref_mask, float (&out)[1]) const {
        const uint32_t *W = b.w;
        // block A in acc[0], acc[1]; block B in acc[2], acc[3]
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 64; i++) {
            const int bp = i < 32 ? 2 + i : 4 + i;
            const uint32_t w = W[bp >> 2];
            const uint32_t src = (bp & 2) ? (w >> 16) : w;
            const uint32_t vb = (bp & 1) ? ((src ^ 0x8000u) & 0xFF00u) : ((src ^ 0x80u) & 0xFFu);
            const int ai = (i >> 5) * 2 + (i & 1);
            acc[ai] = fmaf(__uint_as_float(vb), xp[i], acc[ai]);
        }
        const float2 dd = scales2_f32(__byte_perm(W[0], W[8], 0x7610u), ref_mask);  // (d_A, d_B)
        const float ta = fmaf(acc[0] + acc[1], f, -128.f * sx[0]);
        const float tb = fmaf(acc[2] + acc[3], f, -128.f * sx[1]);
        out[0] = on ? fmaf(dd.x, ta, dd.y * tb) : 0.f;
    }
};


// ---------------------------------------------------------------------------
// Warp-cooperative copy of the warp's slice of a row (nb <= NB bytes, a
// multiple of 16) into `slot`: lane l copies 16-byte chunks l, l + 32, ...
// (a fixed number of predicated copies: no loop).
template <int NB>
__device__ __forceinline__ void gv_copy_slice(const uint8_t *src, uint8_t *slot, int nb, int lane) {
#pragma unroll
    for (int c = 0; c < (NB + 511) / 512; c++) {
        const int off = lane * 16 + c * 512;
        if (off < nb) cp_async16_l2(slot + off, src + off);
    }
}

template <class L, int M>
__global__ void __launch_bounds__(kGvMaxWarps * 32, 1) gemv_rows_kernel(const __grid_constant__ GvArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int slice = warp % a.ks, rgi = warp / a.ks;
    L ln;
    ln.geom(a, slice, lane);
    constexpr int D = L::DEPTH;
    const int kpad = gv_kpad(a.k);
    const GvLayout Lo = gv_layout(nwarps, D, L::SLICE, a.ks * L::SLICE_ELEMS, a.part_rows, a.ks, M);
    unsigned char *ring = smem + Lo.ring + (size_t)warp * D * L::SLICE;
    float *xs = reinterpret_cast<float *>(smem + Lo.xs);
    float *part = reinterpret_cast<float *>(smem + Lo.part);
    // The activations: every thread loads kXB float4 of x (and of x2) per
    // phase, the first phase before any weight request (requests leave an SM
    // in order), and stores them, SiLU-gated for the SwiGLU form, into xs.
    constexpr int kXB = 8;
    const int n4 = M * a.k / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(a.x), *x24 = reinterpret_cast<const float4 *>(a.x2);
    float4 xa[kXB], xb[kXB];
    auto x_load = [&](int start) {
#pragma unroll
        for (int b = 0; b < kXB; b++) {
            const int idx = start + b * (int)blockDim.x;
            if (idx < n4) {
                xa[b] = __ldg(x4 + idx);
                if (x24) xb[b] = __ldg(x24 + idx);
            }
        }
    };
    auto x_store = [&](int start) {
#pragma unroll
        for (int b = 0; b < kXB; b++) {
            const int idx = start + b * (int)blockDim.x;
            if (idx < n4) {
                float4 v = xa[b];
                if (x24) {
                    v.x = lc_swiglu(v.x, xb[b].x), v.y = lc_swiglu(v.y, xb[b].y);
                    v.z = lc_swiglu(v.z, xb[b].z), v.w = lc_swiglu(v.w, xb[b].w);
                }
                const int e = idx * 4, j = e / a.k, ee = e - j * a.k;
                *reinterpret_cast<float4 *>(xs + (size_t)j * kpad + ee + ((ee >> 6) << 2)) = v;
            }
        }
    };
    x_load((int)threadIdx.x);
    const int total = a.rows_end[a.ng - 1];
    // (interleaved pairs stay in one CTA: even range bounds)
    const int pmask = a.pairs ? ~1 : ~0;
    const int r0 = (int)((long long)total * blockIdx.x / gridDim.x) & pmask;
    const int r1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x) & pmask;
    const int nmy = r1 - r0 > rgi ? (r1 - r0 - rgi + a.rg - 1) / a.rg : 0;  // rows r0 + rgi + i * rg
    // this warp's bytes of a row: the slice (the last one may be shorter)
    const int sbytes = min(L::SLICE, a.row_bytes - slice * L::SLICE);
    // source of the warp's slice of its i-th row: a fixed stride when the
    // warp's rows lie in one matrix -- one matrix, or interleaved pairs with an
    // even number of row groups (r0 is even, so the warp keeps one parity)
    const bool fixed = a.ng == 1 || (a.pairs && (a.rg & 1) == 0);
    const int rw = r0 + rgi;
    const size_t rstride = (size_t)(a.ng == 1 ? a.rg : a.rg >> 1) * a.row_bytes;
    const uint8_t *src0 = (a.ng == 1 ? a.w[0] + (size_t)rw * a.row_bytes
                                     : a.w[rw & 1] + (size_t)(rw >> 1) * a.row_bytes) +
                          (size_t)slice * L::SLICE;
    auto slice_ptr = [&](int i) {
        if (fixed) return src0 + (size_t)i * rstride;
        int g, ri;
        gv_row(a, r0 + rgi + i * a.rg, g, ri);
        return a.w[g] + (size_t)ri * a.row_bytes + (size_t)slice * L::SLICE;
    };
    // rows 0 .. D-1 in flight, one cp.async group per row: group r holds row r
#pragma unroll
    for (int d = 0; d < D; d++) {
        if (d < nmy) gv_copy_slice<L::SLICE>(slice_ptr(d), ring + d * L::SLICE, sbytes, lane);
        cp_async_commit();
    }
    x_store((int)threadIdx.x);
    for (int start = (int)threadIdx.x + kXB * (int)blockDim.x; start < n4; start += kXB * (int)blockDim.x) {
        x_load(start);
        x_store(start);
    }
    __syncthreads();
    if constexpr (L::SHARE) {
        // the first warp of each slice forms the pre-scaled activations and
        // publishes them over the slice's own part of xs (it alone reads that
        // part: its lanes' runs lie inside the slice); the other warps load them
        unsigned char *tab = reinterpret_cast<unsigned char *>(xs) + (size_t)slice * gv_kpad(L::SLICE_ELEMS) * 4;
        if (rgi == 0) {
            typename L::Raw raw;
            ln.load(xs, kpad, raw);
            __syncwarp();
            ln.prep(raw);
            ln.store_table(tab, lane);
        }
        __syncthreads();
        if (rgi != 0) ln.load_table(tab, lane);
    } else {
        // every warp forms its lanes' pre-scaled activations from xs
        typename L::Raw raw;
        ln.load(xs, kpad, raw);
        ln.prep(raw);
    }

    const uint32_t ref_mask = a.half_mode == LC_HALF_REF ? 0x04000400u : 0u;
    // One row at a time: a loop body of one row keeps the kernel's hot code
    // small (four rows per iteration with a shared reduction ran slower, most
    // of all for Q8_0).
    for (int i = 0; i < nmy; i++) {
        // Row i has landed for this lane once at most D - 2 newer groups are
        // pending (groups 0..i+D-2 were committed before this point); the warp
        // barrier makes every lane's copies visible and also means every lane
        // is done with row i - 1.
        cp_async_wait<D - 2>();
        __syncwarp();
        // refill row i - 1's buffer with row i - 1 + D
        if (i > 0 && i - 1 + D < nmy)
            gv_copy_slice<L::SLICE>(slice_ptr(i - 1 + D), ring + ((unsigned)(i - 1) & (D - 1)) * L::SLICE, sbytes, lane);
        if (i > 0) cp_async_commit();
        typename L::Bytes bt;
        ln.fetch(ring + ((unsigned)i & (D - 1)) * L::SLICE, bt);
        float o[M];
        ln.row(bt, ref_mask, o);
#pragma unroll
        for (int j = 0; j < M; j++)
#pragma unroll
            for (int off = 16; off; off >>= 1) o[j] += __shfl_xor_sync(0xffffffffu, o[j], off);
        // this k-slice's sum of the row, by row of the CTA's range; no
        // barrier: the k-slices meet once, after the last row
        if (lane == 0) {
            const int lr = rgi + i * a.rg;
#pragma unroll
            for (int j = 0; j < M; j++) part[((size_t)lr * a.ks + slice) * M + j] = o[j];
        }
    }
    cp_async_wait_all();
    __syncthreads();
    // every row of the range: its k-slices added in slice order
    const int nrows = r1 - r0;
    if (a.pairs) {  // SiLU(gate) * up of each pair, one output
        const int n = a.rows_end[0];
        for (int t = threadIdx.x; t < (nrows >> 1) * M; t += blockDim.x) {
            const int lp = t / M, j = t - lp * M, lr = 2 * lp;
            float vg = 0.f, vu = 0.f;
            for (int sl = 0; sl < a.ks; sl++) {
                vg += part[((size_t)lr * a.ks + sl) * M + j];
                vu += part[((size_t)(lr + 1) * a.ks + sl) * M + j];
            }
            a.y[0][(size_t)j * n + ((r0 + lr) >> 1)] = lc_swiglu(vg, vu);
        }
        return;
    }
    for (int t = threadIdx.x; t < nrows * M; t += blockDim.x) {
        const int lr = t / M, j = t - lr * M;
        float v = 0.f;
        for (int sl = 0; sl < a.ks; sl++) v += part[((size_t)lr * a.ks + sl) * M + j];
        int g, ri;
        gv_row(a, r0 + lr, g, ri);
        const int nrow = a.rows_end[g] - (g ? a.rows_end[g - 1] : 0);
        a.y[g][(size_t)j * nrow + ri] = v;
    }
}

// ---------------------------------------------------------------------------
// Host side.

struct GvPlan {
    int ks = 0, rg = 0, grid = 0, threads = 0, part_rows = 0;
    size_t smem = 0;
};

// Geometry for k, m tokens and `rows` rows in all;
// ks = 0 when the shape is not covered.
GvPlan gv_plan(const lc_ctx *ctx, int dtype, int m, int k, int rows) {
    GvPlan p;
    const int se = m == 1 ? 2048 : 1024;  // elements per warp slice
    const int ks = (k + se - 1) / se;
    if (ks < 1 || ks > kGvMaxWarps) return p;
    // row groups: as many as fit in 16 warps
    const int rg = std::max(1, kGvMaxWarps / ks);
    const int threads = ks * rg * 32;
    const int slice_bytes = dtype == LC_Q8_0 ? Q8Lane::SLICE : (m == 1 ? Q4Lane<1>::SLICE : Q4Lane<2>::SLICE);
    const int depth = dtype == LC_Q8_0 ? Q8Lane::DEPTH : (m == 1 ? Q4Lane<1>::DEPTH : Q4Lane<2>::DEPTH);
    // one CTA per SM; more (in waves) only when a CTA's row range would need
    // more than 32 KB of partial sums
    int grid = std::max(1, std::min(ctx->num_sms, rows));
    const long long max_rows = std::max(1, (32 << 10) / (ks * m * 4));
    if ((rows + grid - 1) / grid > max_rows) grid = (int)((rows + max_rows - 1) / max_rows);
    const int part_rows = (rows + grid - 1) / grid + 1;
    const size_t need = gv_layout(ks * rg, depth, slice_bytes, ks * se, part_rows, ks, m).total;
    if (need > ctx->smem_optin) return p;
    p.ks = ks, p.rg = rg, p.threads = threads, p.smem = need, p.part_rows = part_rows;
    p.grid = grid;
    return p;
}

template <class L, int M>
int gv_launch(lc_ctx *ctx, const GvPlan &p, GvArgs &a) {
    auto kern = gemv_rows_kernel<L, M>;
    if (p.smem > 48 * 1024) {
        const int s = lc_set_smem_attr((const void *)kern, p.smem);
        if (s) return s;
    }
    a.ks = p.ks, a.rg = p.rg, a.part_rows = p.part_rows;

    kern<<<p.grid, p.threads, p.smem, ctx->stream>>>(a);
    return LC_OK;
}

}  // namespace

namespace lc {

bool gemv_rows_covers(const lc_ctx *ctx, int dtype, uint32_t m, uint32_t k) {
    if (k == 0 || k % 256 != 0) return false;
    if (dtype == LC_Q4_K) return (m == 1 || m == 2) && (k + (m == 1 ? 2047 : 1023)) / (m == 1 ? 2048 : 1024) <= kGvMaxWarps;
    if (dtype == LC_Q8_0) return m == 1 && (k + 2047) / 2048 <= kGvMaxWarps;
    (void)ctx;
    return false;
}

static int gv_run(lc_ctx *ctx, int dtype, const PackSrc &src, uint32_t m, uint32_t k, long long rows, GvArgs &a) {
    if (rows == 0) return LC_OK;
    a.x = src.x;
    a.x2 = src.op == LC_PACK_SWIGLU ? src.x2 : nullptr;
    a.k = (int)k;
    a.row_bytes = dtype == LC_Q4_K ? (int)(k / 256) * 144 : (int)(k / 32) * 34;
    a.half_mode = ctx->half_mode;
    a.status = ctx->dev_status;
    const GvPlan p = gv_plan(ctx, dtype, (int)m, (int)k, (int)rows);
    LC_REQUIRE(p.ks, LC_ERR_UNSUPPORTED, "gemv_rows: rows of %d bytes do not fit shared memory", a.row_bytes);
    if (dtype == LC_Q8_0) return gv_launch<Q8Lane, 1>(ctx, p, a);
    if (m == 1) return gv_launch<Q4Lane<1>, 1>(ctx, p, a);
    return gv_launch<Q4Lane<2>, 2>(ctx, p, a);
}

static int gv_check(lc_ctx *ctx, int dtype, const PackSrc &src, uint32_t m, uint32_t k) {
    LC_REQUIRE(gemv_rows_covers(ctx, dtype, m, k), LC_ERR_UNSUPPORTED, "gemv_rows: dtype %d m=%u k=%u", dtype, m, k);
    LC_REQUIRE(src.op == LC_PACK_PLAIN || src.op == LC_PACK_SWIGLU, LC_ERR_UNSUPPORTED, "gemv_rows: packing op %d",
               src.op);
    LC_REQUIRE(((uintptr_t)src.x & 15) == 0 && ((uintptr_t)src.x2 & 15) == 0, LC_ERR_UNSUPPORTED,
               "gemv_rows: activations not 16-byte aligned");
    return LC_OK;
}

int gemv_rows(lc_ctx *ctx, int dtype, const PackSrc &src, const ProjOut *outs, int ng, uint32_t m, uint32_t k) {
    LC_REQUIRE(ng >= 1 && ng <= kGroupMax, LC_ERR_INVALID, "gemv_rows: %d matrices", ng);
    if (int s = gv_check(ctx, dtype, src, m, k)) return s;
    GvArgs a = {};
    long long rows = 0;
    for (int g = 0; g < ng; g++) {
        LC_REQUIRE(((uintptr_t)outs[g].w & 15) == 0, LC_ERR_UNSUPPORTED, "gemv_rows: weights not 16-byte aligned");
        LC_REQUIRE(!outs[g].accumulate, LC_ERR_UNSUPPORTED, "gemv_rows: accumulating outputs");
        rows += outs[g].n;
        LC_REQUIRE(rows < (1ll << 30), LC_ERR_INVALID, "gemv_rows: too many rows");
        a.w[g] = (const uint8_t *)outs[g].w;
        a.y[g] = outs[g].y;
        a.rows_end[g] = (int)rows;
    }
    a.ng = ng;
    return gv_run(ctx, dtype, src, m, k, rows, a);
}

int gemv_rows_swiglu(lc_ctx *ctx, int dtype, const PackSrc &src, const void *w_gate, const void *w_up, float *h,
                     uint32_t m, uint32_t k, uint32_t n) {
    if (int s = gv_check(ctx, dtype, src, m, k)) return s;
    LC_REQUIRE((((uintptr_t)w_gate | (uintptr_t)w_up) & 15) == 0, LC_ERR_UNSUPPORTED,
               "gemv_rows: weights not 16-byte aligned");
    LC_REQUIRE(2ll * n < (1ll << 30), LC_ERR_INVALID, "gemv_rows: too many rows");
    GvArgs a = {};
    a.w[0] = (const uint8_t *)w_gate, a.w[1] = (const uint8_t *)w_up;
    a.y[0] = a.y[1] = h;
    a.rows_end[0] = (int)n, a.rows_end[1] = (int)(2 * n);
    a.ng = 2;
    a.pairs = 1;
    return gv_run(ctx, dtype, src, m, k, 2ll * n, a);
}

}  // namespace lc

// ---------------------------------------------------------------------------
// C ABI: the FFN block of the DFlash decoder layer (src/dflash.rs:965-968):
// y = down(SiLU(gate(x)) * up(x)) for m rows of x [m, n_embd].  One or two
// tokens run as two launches: gate and up rows interleaved in one GEMV over x,
// each pair's SiLU(gate) * up formed once where its sums meet, then down;
// 5..32 tokens gate and up on the grouped tcgen05 GEMM, SiLU-gate formed while
// down packs; other m the projections and the activation kernel one by one.

extern "C" int lc_ffn(lc_ctx *ctx, int dtype, const float *x, const void *w_gate, const void *w_up,
                      const void *w_down, float *y, uint32_t m, uint32_t n_embd, uint32_t n_ff) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_ffn: null ctx");
    if (m == 0 || n_embd == 0) return LC_OK;
    LC_REQUIRE(x && w_gate && w_up && w_down && y, LC_ERR_INVALID, "lc_ffn: null pointer");
    LC_REQUIRE(n_ff > 0, LC_ERR_INVALID, "lc_ffn: n_ff must be > 0");
    LC_REQUIRE(dtype == LC_Q4_K || dtype == LC_Q8_0, LC_ERR_UNSUPPORTED, "lc_ffn: dtype %d (Q8_0, Q4_K)", dtype);
    LC_REQUIRE((uint64_t)m * n_ff < (1ull << 31), LC_ERR_INVALID, "lc_ffn: m*n_ff too large");
    int s = lc_use_device(ctx);
    if (s) return s;
    float *gu = (float *)lc_scratch(ctx, LC_SCRATCH_FFN, (size_t)2 * m * n_ff * 4 + 256);
    if (!gu) return LC_ERR_OOM;
    float *g = gu, *u = gu + (size_t)m * n_ff;
    auto proj = [&](const float *xx, const void *w, float *c, uint32_t k, uint32_t n) {
        return dtype == LC_Q4_K ? lc::proj_q4k(ctx, xx, w, c, m, k, n, 0) : lc::proj_q8_0(ctx, xx, w, c, m, k, n);
    };
    if (lc::gemv_rows_covers(ctx, dtype, m, n_embd) && lc::gemv_rows_covers(ctx, dtype, m, n_ff)) {
        lc::PackSrc src;
        src.x = x;
        // gate and up rows interleaved in one launch; each pair's SiLU(gate) * up
        // is formed once, at the end of its CTA, into g
        s = lc::gemv_rows_swiglu(ctx, dtype, src, w_gate, w_up, g, m, n_embd, n_ff);
        if (s == LC_OK) {
            lc::PackSrc hs;
            hs.x = g;
            lc::ProjOut d;
            d.w = w_down, d.y = y, d.n = n_embd;
            s = lc::gemv_rows(ctx, dtype, hs, &d, 1, m, n_ff);
            if (s == LC_OK) return lc_after_launch(ctx, "lc_ffn");
            if (s != LC_ERR_UNSUPPORTED) return s;
            // the down projection's activations do not fit the CTA's shared
            // memory: its own projection route
            if ((s = proj(g, w_down, y, n_ff, n_embd))) return s;
            return lc_after_launch(ctx, "lc_ffn");
        }
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if (lc::routes_to_gemm_dq(ctx, m)) {
        // 5..32 tokens: gate and up in one grouped tcgen05 GEMM, SiLU-gate formed
        // while the down projection packs its activations (as the decoder does)
        lc::PackSrc src;
        src.x = x;
        lc::ProjOut o[2];
        o[0].w = w_gate, o[0].y = g, o[0].n = n_ff;
        o[1].w = w_up, o[1].y = u, o[1].n = n_ff;
        s = lc::gemm_dq_group(ctx, dtype, src, o, 2, m, n_embd);
        if (s == LC_OK) {
            lc::PackSrc hs;
            hs.x = g, hs.x2 = u, hs.op = lc::LC_PACK_SWIGLU;
            lc::ProjOut d;
            d.w = w_down, d.y = y, d.n = n_embd;
            s = lc::gemm_dq_group(ctx, dtype, hs, &d, 1, m, n_ff);
            if (s == LC_OK) return lc_after_launch(ctx, "lc_ffn");
        }
        if (s != LC_ERR_UNSUPPORTED) return s;
    }
    if ((s = proj(x, w_gate, g, n_embd, n_ff)) || (s = proj(x, w_up, u, n_embd, n_ff))) return s;
    if ((s = lc_activation(ctx, g, u, g, m * n_ff))) return s;
    if ((s = proj(g, w_down, y, n_ff, n_embd))) return s;
    return lc_after_launch(ctx, "lc_ffn");
}

// ---------------------------------------------------------------------------
// Host-buffer forms: one call per step for a host that holds its inputs and
// outputs in host memory.

namespace {

// Device staging for x [m, k_in] and the result [m, n_out] in the context's
// scratch (256-byte aligned halves).
int host_io(lc_ctx *ctx, size_t x_floats, size_t y_floats, float **xd, float **yd) {
    const size_t xb = (x_floats * 4 + 255) & ~(size_t)255;
    char *p = (char *)lc_scratch(ctx, LC_SCRATCH_HOSTIO, xb + y_floats * 4 + 256);
    if (!p) return LC_ERR_OOM;
    *xd = (float *)p;
    *yd = (float *)(p + xb);
    return LC_OK;
}

}  // namespace

extern "C" int lc_ffn_host(lc_ctx *ctx, int dtype, const float *x_host, const void *w_gate, const void *w_up,
                           const void *w_down, float *y_host, uint32_t m, uint32_t n_embd, uint32_t n_ff) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_ffn_host: null ctx");
    if (m == 0 || n_embd == 0) return LC_OK;
    LC_REQUIRE(x_host && y_host, LC_ERR_INVALID, "lc_ffn_host: null host buffer");
    int s = lc_use_device(ctx);
    if (s) return s;
    float *xd, *yd;
    if ((s = host_io(ctx, (size_t)m * n_embd, (size_t)m * n_embd, &xd, &yd))) return s;
    const size_t bytes = (size_t)m * n_embd * 4;
    LC_CUDA(cudaMemcpyAsync(xd, x_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    if ((s = lc_ffn(ctx, dtype, xd, w_gate, w_up, w_down, yd, m, n_embd, n_ff))) return s;
    LC_CUDA(cudaMemcpyAsync(y_host, yd, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    return lc_after_launch(ctx, "lc_ffn_host");
}

extern "C" int lc_proj_m_host(lc_ctx *ctx, int dtype, const float *x_host, const void *w, float *c_host, uint32_t m,
                              uint32_t k, uint32_t n, uint32_t expert_offset) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_proj_m_host: null ctx");
    if (m == 0 || n == 0) return LC_OK;
    LC_REQUIRE(x_host && c_host, LC_ERR_INVALID, "lc_proj_m_host: null host buffer");
    int s = lc_use_device(ctx);
    if (s) return s;
    float *xd, *yd;
    if ((s = host_io(ctx, (size_t)m * k, (size_t)m * n, &xd, &yd))) return s;
    LC_CUDA(cudaMemcpyAsync(xd, x_host, (size_t)m * k * 4, cudaMemcpyHostToDevice, ctx->stream));
    if ((s = lc_proj_m(ctx, dtype, xd, w, yd, m, k, n, expert_offset))) return s;
    LC_CUDA(cudaMemcpyAsync(c_host, yd, (size_t)m * n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    LC_CUDA(cudaStreamSynchronize(ctx->stream));
    return lc_after_launch(ctx, "lc_proj_m_host");
}
