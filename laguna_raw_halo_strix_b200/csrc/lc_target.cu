// lc_target.cu -- the target (Laguna) model on the device: the C++ counterpart
// of TargetModel (src/target.rs:105-748), the model whose forward pass verifies
// the draft tokens.
//
// The reference runs one token per call and keeps its K/V cache on the host
// (read back, concatenated and re-uploaded every layer, src/target.rs:465-487),
// and routes the MoE layers on the host (router logits read back, sigmoid and
// sort in Rust, one projection launch per selected expert with two more host
// round trips for the hidden-vector rescale, src/target.rs:653-728).  Here:
//   * a block of m tokens runs in one pass: with LC_TARGET_CACHED the rows are
//     consecutive positions whose K/V land in a device cache and attend
//     causally over it (the verify step of speculative decoding); without it
//     every row is forward_token (position 0, attending to itself only);
//   * routing is one kernel per block (sigmoid + bias, a stable top-k, the
//     optional normalisation and scale), expert work is grouped by expert so
//     each selected expert's weights stream from HBM once per block, and the
//     SwiGLU, the L2 rescale and the weighted sum are kernels of their own;
//   * the dense projections reuse the DFlash model's grouped kernels.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "lc_internal.cuh"

using lc::DevTensor;

namespace {

#define LC_TRY(expr)                \
    do {                            \
        int _s = (expr);            \
        if (_s != LC_OK) return _s; \
    } while (0)

constexpr int kTok = 8;            // activation rows of one expert work item
constexpr int kMaxExperts = 1024;  // router width the selection kernels take
constexpr int kRowsCta = 64;       // output rows per CTA of the expert GEMV

struct TLayer {
    DevTensor attn_norm, q_norm, k_norm, q, k, v, o, gate_attn, ffn_norm, gate, up, down;
    DevTensor probs_bias, gate_inp, gate_exps, up_exps, down_exps, gate_shexp, up_shexp, down_shexp;
    bool is_moe = false;
    bool down_kcat = false;  // ffn_down_exps held k-concatenated ([row][expert][k])
    uint32_t n_q_heads = 0;
};

// One expert's share of a block: up to kTok (token, slot) pairs, by pair index
// p = token * n_sel + slot.  Unused entries repeat pair[0].
struct MoeItem {
    int expert;
    int count;
    int pair[kTok];
};

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Out of every query head h: v of kv head h * n_kv / n_q (mha_attn.comp:33).
// With a single key the online softmax of mha_attn.comp:40-62 gives weight 1
// (l = 1, acc = V), so forward_token's attention output is exactly v.
__global__ void gqa_expand_kernel(const float *__restrict__ v, float *__restrict__ out, int m, int n_q, int n_kv,
                                  int hd) {
    const int total = n_q * hd;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m * total; i += gridDim.x * blockDim.x) {
        const int r = i / total, d = i % total, h = d / hd;
        const int kv = h * n_kv / n_q;
        out[i] = v[(size_t)r * n_kv * hd + kv * hd + d % hd];
    }
}

// Router selection of dispatch_moe_ffn (src/target.rs:653-677), one CTA per
// token: probs = 1 / (1 + exp(-logit)) with exp rounded once to f32 (as the
// host's expf), selection = probs + bias, the n_sel largest selections by a
// stable descending order (equal values keep expert order), scores = their
// probs, then / max(sum, 2^-14) (sum in slot order) and * scale.
__global__ void moe_route_kernel(const float *__restrict__ logits, const float *__restrict__ bias, int ne, int n_sel,
                                 int norm, float scale, int32_t *__restrict__ ids, float *__restrict__ scores) {
    extern __shared__ float sh[];
    float *sel = sh, *prob = sh + ne, *sc = sh + 2 * ne;
    const int t = blockIdx.x;
    const float *lg = logits + (size_t)t * ne;
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        const float ex = (float)exp(-(double)lg[e]);
        const float p = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        prob[e] = p;
        sel[e] = __fadd_rn(p, bias[e]);
    }
    for (int r = threadIdx.x; r < n_sel; r += blockDim.x) {
        ids[(size_t)t * n_sel + r] = -1;
        sc[r] = 0.f;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        const float v = sel[e];
        int rank = 0;
        for (int j = 0; j < ne; j++) {
            const float w = sel[j];
            rank += (w > v) || (w == v && j < e);
        }
        if (rank < n_sel) {
            ids[(size_t)t * n_sel + rank] = e;
            sc[rank] = prob[e];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float denom = 1.f;
        if (norm) {
            float sum = 0.f;
            for (int r = 0; r < n_sel; r++) sum = __fadd_rn(sum, sc[r]);
            denom = fmaxf(sum, 6.103515625e-5f);
        }
        for (int r = 0; r < n_sel; r++) {
            float s = sc[r];
            if (norm) s = __fdiv_rn(s, denom);
            if (scale != 0.f && scale != 1.f) s = __fmul_rn(s, scale);
            scores[(size_t)t * n_sel + r] = s;
        }
    }
}

// Group the block's (token, slot) pairs by expert into work items of at most
// kTok pairs, experts in increasing order and pairs in increasing index.  One
// CTA of at least ne threads' worth of loop (ne <= kMaxExperts).
__global__ void moe_items_kernel(const int32_t *__restrict__ ids, int n_pairs, int ne, MoeItem *__restrict__ items,
                                 int *__restrict__ n_items) {
    __shared__ int first[kMaxExperts + 1];
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        int c = 0;
        for (int p = 0; p < n_pairs; p++) c += ids[p] == e;
        first[e] = (c + kTok - 1) / kTok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int e = 0; e < ne; e++) {
            const int c = first[e];
            first[e] = acc;
            acc += c;
        }
        first[ne] = acc;
        *n_items = acc;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < ne; e += blockDim.x) {
        int it = first[e], c = 0;
        for (int p = 0; p < n_pairs; p++) {
            if (ids[p] != e) continue;
            items[it].pair[c++] = p;
            if (c == kTok) {
                items[it].expert = e;
                items[it].count = kTok;
                it++;
                c = 0;
            }
        }
        if (c > 0) {
            items[it].expert = e;
            items[it].count = c;
            for (int j = c; j < kTok; j++) items[it].pair[j] = items[it].pair[0];
        }
    }
}

// The bytes a lane needs for eight consecutive weights w[k0 + 8*lane .. +8]
// of one row, loaded before any is decoded so a warp keeps the loads of several
// rows in flight: Q4_K the block's 16-byte header (d, dmin, the packed
// scales) and the lane's 8 nibble bytes; Q8_0 the scale and 8 bytes; F32 the
// 8 floats.
template <int DT>
struct ExpRaw {
    uint4 a;  // Q4_K header; Q8_0 .x = the f16 scale; F32 floats 0..3
    uint4 b;  // Q4_K nibbles in .x/.y; Q8_0 bytes in .x/.y; F32 floats 4..7
};

template <int DT>
__device__ __forceinline__ void expert_load8(const uint8_t *__restrict__ wr, int k0, int lane, ExpRaw<DT> &r) {
    const int kk = k0 + 8 * lane;
    if constexpr (DT == LC_Q4_K) {
        const uint8_t *blk = wr + (size_t)(k0 / 256) * 144;
        r.a = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint2 q = __ldg(reinterpret_cast<const uint2 *>(blk + 16 + (lane >> 3) * 32 + (lane & 3) * 8));
        r.b = make_uint4(q.x, q.y, 0u, 0u);
    } else if constexpr (DT == LC_Q8_0) {
        const uint8_t *blk = wr + (size_t)(kk / 32) * 34;
        const uint16_t *qs = reinterpret_cast<const uint16_t *>(blk + 2 + (kk & 31));
        r.a = make_uint4(__ldg(reinterpret_cast<const uint16_t *>(blk)), 0u, 0u, 0u);
        const uint32_t q0 = __ldg(qs), q1 = __ldg(qs + 1), q2 = __ldg(qs + 2), q3 = __ldg(qs + 3);
        r.b = make_uint4(q0 | (q1 << 16), q2 | (q3 << 16), 0u, 0u);
    } else {
        r.a = __ldg(reinterpret_cast<const uint4 *>(wr + (size_t)kk * 4));
        r.b = __ldg(reinterpret_cast<const uint4 *>(wr + (size_t)kk * 4 + 16));
    }
}

// The lane's eight quantised values as exact floats, and the scale terms of
// its sub-block / block:  w_i = mul * q_i - sub  (Q4_K: mul = d*sc, sub =
// dmin*m, proj_q4k.comp:72-87; Q8_0: mul = d, sub = 0, proj_q8_0.comp:53-64;
// F32: q_i = w_i, mul = 1).  An integer 0..255 becomes a float exactly through
// the bit pattern of 2^23 + q minus 2^23 (no conversion instruction).
template <int DT>
__device__ __forceinline__ void expert_decode8(const ExpRaw<DT> &r, int lane, int half_mode, float (&q)[8], float &mul,
                                               float &sub) {
    constexpr uint32_t kMagic = 0x4B000000u;  // 2^23
    if constexpr (DT == LC_Q4_K) {
        const float d = lc_half_to_f32(r.a.x & 0xFFFFu, half_mode), dmin = lc_half_to_f32(r.a.x >> 16, half_mode);
        const uint32_t sw[3] = {r.a.y, r.a.z, r.a.w};  // scale bytes 0..11
        auto sb = [&](int i) { return (sw[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
        const int j = lane >> 2;  // sub-block of 32
        uint32_t sc, mn;
        if (j < 4) {
            sc = sb(j) & 63u;
            mn = sb(j + 4) & 63u;
        } else {
            sc = (sb(j + 4) & 15u) | ((sb(j - 4) >> 6) << 4);
            mn = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
        }
        mul = __fmul_rn(d, (float)sc);
        sub = __fmul_rn(dmin, (float)mn);
        const int shift = (lane & 4) ? 4 : 0;
        const uint32_t lo = r.b.x >> shift, hi = r.b.y >> shift;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t nib = ((i < 4 ? lo : hi) >> (8 * (i & 3))) & 15u;
            q[i] = __uint_as_float(kMagic | nib) - 8388608.0f;
        }
    } else if constexpr (DT == LC_Q8_0) {
        mul = lc_half_to_f32(r.a.x, half_mode);
        sub = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t byte = ((i < 4 ? r.b.x : r.b.y) >> (8 * (i & 3))) & 0xFFu;
            q[i] = __uint_as_float(kMagic | (byte ^ 0x80u)) - 8388736.0f;  // (q + 128) - 128
        }
    } else {
        mul = 1.f;
        sub = 0.f;
        q[0] = __uint_as_float(r.a.x), q[1] = __uint_as_float(r.a.y), q[2] = __uint_as_float(r.a.z);
        q[3] = __uint_as_float(r.a.w), q[4] = __uint_as_float(r.b.x), q[5] = __uint_as_float(r.b.y);
        q[6] = __uint_as_float(r.b.z), q[7] = __uint_as_float(r.b.w);
    }
}

// Y[pair][row] = X[pair / act_div] . W_e[row] for the pairs of each work item:
// expert e's matrix is read once for all of its pairs.  A warp takes kExpRows
// rows at a time (their loads in flight together, each activation load
// shared by them).  blockIdx.z picks one of two weight stacks sharing the
// items (gate and up).  expert_fixed >= 0 makes every item read that expert
// (the reference's Q8_0 / F32 expert quirk).
constexpr int kExpRows = 4;
template <int DT>
__global__ void __launch_bounds__(256) expert_gemv_kernel(const uint8_t *__restrict__ w0, const uint8_t *__restrict__ w1,
                                                          size_t expert_stride, size_t row_stride, int expert_fixed,
                                                          int n, int k, const float *__restrict__ X, int act_div,
                                                          const MoeItem *__restrict__ items,
                                                          const int *__restrict__ n_items, float *Y0, float *Y1,
                                                          int half_mode) {
    if ((int)blockIdx.y >= *n_items) return;
    const MoeItem it = items[blockIdx.y];
    const int e = expert_fixed >= 0 ? expert_fixed : it.expert;
    const uint8_t *W = (blockIdx.z ? w1 : w0) + (size_t)e * expert_stride;
    float *Y = blockIdx.z ? Y1 : Y0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *xr[kTok];
#pragma unroll
    for (int t = 0; t < kTok; t++) xr[t] = X + (size_t)(it.pair[t] / act_div) * k;
    const int row0 = (int)blockIdx.x * kRowsCta, row_end = min(n, row0 + kRowsCta);
    // warp w: rows row0 + w + 8 * (r + kExpRows * g), r < kExpRows
    for (int g = 0; g < kRowsCta / (8 * kExpRows); g++) {
        int rows[kExpRows];
        bool live[kExpRows];
        const uint8_t *wr[kExpRows];
#pragma unroll
        for (int r = 0; r < kExpRows; r++) {
            rows[r] = row0 + warp + 8 * (r + kExpRows * g);
            live[r] = rows[r] < row_end;
            wr[r] = W + (size_t)(live[r] ? rows[r] : row0) * row_stride;
        }
        if (!live[0]) break;
        float acc[kExpRows][kTok];
#pragma unroll
        for (int r = 0; r < kExpRows; r++)
#pragma unroll
            for (int t = 0; t < kTok; t++) acc[r][t] = 0.f;
        for (int k0 = 0; k0 < k; k0 += 256) {
            const int kk = k0 + 8 * lane;
            if (kk >= k) break;  // Q8_0 / F32 with k not a multiple of 256: the tail lanes
            ExpRaw<DT> raw[kExpRows];
#pragma unroll
            for (int r = 0; r < kExpRows; r++) expert_load8<DT>(wr[r], k0, lane, raw[r]);
            float q[kExpRows][8], mul[kExpRows], sub[kExpRows];
#pragma unroll
            for (int r = 0; r < kExpRows; r++) expert_decode8<DT>(raw[r], lane, half_mode, q[r], mul[r], sub[r]);
#pragma unroll
            for (int t = 0; t < kTok; t++) {
                if (t >= it.count) break;
                const float4 a = __ldg(reinterpret_cast<const float4 *>(xr[t] + kk));
                const float4 b = __ldg(reinterpret_cast<const float4 *>(xr[t] + kk + 4));
                // S(x) of the lane's eight elements, shared by the rows
                const float sx = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
#pragma unroll
                for (int r = 0; r < kExpRows; r++) {
                    float s = q[r][0] * a.x;
                    s = fmaf(q[r][1], a.y, s), s = fmaf(q[r][2], a.z, s), s = fmaf(q[r][3], a.w, s);
                    s = fmaf(q[r][4], b.x, s), s = fmaf(q[r][5], b.y, s), s = fmaf(q[r][6], b.z, s);
                    s = fmaf(q[r][7], b.w, s);
                    // y += mul * S(q x) - sub * S(x)
                    acc[r][t] = fmaf(mul[r], s, fmaf(-sub[r], sx, acc[r][t]));
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kExpRows; r++)
#pragma unroll
            for (int t = 0; t < kTok; t++) {
                if (t >= it.count) break;
                const float v = warp_sum(acc[r][t]);
                if (lane == 0 && live[r]) Y[(size_t)it.pair[t] * n + rows[r]] = v;
            }
    }
}

// Per (token, slot) pair p: h = SiLU(gate) * up (activation.comp), col_l2 =
// clamp(|h|, 1e-8, 1e30) and hs = h * 32768 / col_l2 (src/target.rs:700-712).
// gate / up rows: g + p * F (the per-expert projections), or, with `dense`, row
// p / n_sel of every expert's outputs side by side, at ids[p] * F.
__global__ void moe_swiglu_l2_kernel(const float *__restrict__ g, const float *__restrict__ u, int F,
                                     const int32_t *__restrict__ ids, int n_sel, int dense, size_t dense_stride,
                                     float *__restrict__ hs, float *__restrict__ col) {
    __shared__ float red[32];
    const int p = blockIdx.x;
    const size_t base = (size_t)p * F;
    const int e = ids[p];
    if (e < 0) {  // an unfilled slot (the combine skips it)
        if (threadIdx.x == 0) col[p] = 1.f;
        return;
    }
    const size_t src = dense ? (size_t)(p / n_sel) * dense_stride + (size_t)e * F : base;
    float sq = 0.f;
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const float h = lc_swiglu(g[src + i], u[src + i]);
        hs[base + i] = h;
        sq = fmaf(h, h, sq);
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = fminf(fmaxf(sqrtf(v), 1e-8f), 1e30f);
    }
    __syncthreads();
    const float c = red[0];
    if (threadIdx.x == 0) col[p] = c;
    for (int i = threadIdx.x; i < F; i += blockDim.x) hs[base + i] = __fdiv_rn(__fmul_rn(hs[base + i], 32768.f), c);
}

// The down-projection stack from expert-major [expert][row][k] to
// k-concatenated [row][expert][k] (row r holds every expert's row r side by
// side), one warp per (expert, row); row_bytes a multiple of 16.
__global__ void kcat_rows_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int n_exp, int rows,
                                 int row_bytes) {
    const int lane = threadIdx.x & 31;
    const long long unit = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (unit >= (long long)n_exp * rows) return;
    const int e = (int)(unit / rows), r = (int)(unit % rows);
    const uint8_t *sp = src + ((size_t)e * rows + r) * row_bytes;
    uint8_t *dp = dst + ((size_t)r * n_exp + e) * row_bytes;
    for (int c = lane * 16; c < row_bytes; c += 512)
        *reinterpret_cast<uint4 *>(dp + c) = *reinterpret_cast<const uint4 *>(sp + c);
}

// The down projection's input for every token and expert at once: H[t][e*F +
// i] = hs[p][i] * s_p for the token's selected experts (zero elsewhere, set
// before), s_p = (col_p / 32768) * score_p when score_p > 0, else 1 -- the
// per-expert output scale of src/target.rs:714-722 moved before the (linear)
// projection.
__global__ void moe_scatter_kernel(const float *__restrict__ hs, const float *__restrict__ col,
                                   const float *__restrict__ scores, const int32_t *__restrict__ ids, int n_sel, int ne,
                                   int F, float *__restrict__ H) {
    const int p = blockIdx.x, e = ids[p];
    if (e < 0) return;
    const float sc = scores[p];
    const float s = sc > 0.f ? __fmul_rn(__fdiv_rn(col[p], 32768.f), sc) : 1.f;
    float *dst = H + (size_t)(p / n_sel) * ne * F + (size_t)e * F;
    for (int i = threadIdx.x; i < F; i += blockDim.x) dst[i] = __fmul_rn(hs[(size_t)p * F + i], s);
}

// y[t] = ((0 + o_0) + o_1) + ... + shared, o_j = down_j * ((col_j / 32768) *
// score_j) when score_j > 0, else down_j as it is (src/target.rs:714-745).
__global__ void moe_combine_kernel(const float *__restrict__ down, const float *__restrict__ col,
                                   const float *__restrict__ scores, const int32_t *__restrict__ ids,
                                   const float *__restrict__ shared, int n_sel, int E, int m, float *__restrict__ y) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m * E; i += gridDim.x * blockDim.x) {
        const int t = i / E, c = i % E;
        float acc = 0.f;
        for (int j = 0; j < n_sel; j++) {
            const int p = t * n_sel + j;
            if (ids[p] < 0) continue;
            float o = down[(size_t)p * E + c];
            const float sc = scores[p];
            if (sc > 0.f) o = __fmul_rn(o, __fmul_rn(__fdiv_rn(col[p], 32768.f), sc));
            acc = __fadd_rn(acc, o);
        }
        y[i] = __fadd_rn(acc, shared[i]);
    }
}

}  // namespace

struct lc_target {
    lc_ctx *ctx = nullptr;
    lc_target_hparams hp{};
    uint32_t flags = 0;
    uint32_t max_ctx = 0, max_block = 0;
    std::vector<TLayer> layers;
    DevTensor tok_embd, output_norm, output;
    float *freq = nullptr, *freq_swa = nullptr;
    float *kcache = nullptr, *vcache = nullptr;  // [layers][max_ctx][n_kv * head_dim]
    uint32_t cache_len = 0;
    uint32_t qd_max = 0, heads_max = 0, n_sel = 0;
    // block workspace (max_block rows)
    float *x = nullptr, *nx = nullptr, *q = nullptr, *attn = nullptr, *gate = nullptr, *tmp = nullptr;
    float *kbuf = nullptr, *vbuf = nullptr, *ffg = nullptr, *ffu = nullptr, *ffh = nullptr;
    // MoE workspace
    float *router = nullptr, *scores = nullptr, *gu = nullptr, *hs = nullptr, *col = nullptr, *dout = nullptr;
    float *gu_dense = nullptr;  // [2][max_block][n_expert * n_ff_exp]: every expert's gate / up outputs
    float *sh_g = nullptr, *sh_u = nullptr, *sh_h = nullptr, *sh_out = nullptr, *moe_y = nullptr;
    int32_t *ids = nullptr;
    int32_t *route_log = nullptr;       // [layer][max_block][n_sel]: the last selection of each layer
    std::vector<uint32_t> route_rows;  // rows of that selection per layer
    int *n_items = nullptr;
    MoeItem *items = nullptr;
    std::vector<void *> allocs;

    ~lc_target() {
        for (void *p : allocs) cudaFree(p);
    }
    size_t kvd() const { return (size_t)hp.n_kv_heads * hp.head_dim; }
    float *kl(uint32_t l) const { return kcache + (size_t)l * max_ctx * kvd(); }
    float *vl(uint32_t l) const { return vcache + (size_t)l * max_ctx * kvd(); }
};

namespace {

int talloc(lc_target *t, size_t bytes, void **out) {
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes ? bytes : 256);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return lc_fail(LC_ERR_OOM, "lc_target: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    t->allocs.push_back(p);
    *out = p;
    return LC_OK;
}

template <typename T>
int talloc_t(lc_target *t, size_t count, T **out) {
    void *p = nullptr;
    LC_TRY(talloc(t, count * sizeof(T), &p));
    *out = (T *)p;
    return LC_OK;
}

// The slots TargetModel::load fills (src/target.rs:158-244): dense FFN tensors
// on dense layers only, router / expert / shared-expert tensors on MoE layers.
DevTensor *target_slot(lc_target *t, const char *name) {
    if (!strcmp(name, "token_embd.weight")) return &t->tok_embd;
    if (!strcmp(name, "output_norm.weight")) return &t->output_norm;
    if (!strcmp(name, "output.weight")) return &t->output;
    unsigned layer;
    int off = 0;
    if (sscanf(name, "blk.%u.%n", &layer, &off) != 1 || off == 0 || layer >= t->layers.size()) return nullptr;
    const char *suf = name + off;
    TLayer &L = t->layers[layer];
    struct {
        const char *s;
        DevTensor *w;
        int kind;  // 0 any layer, 1 dense only, 2 MoE only
    } tab[] = {{"attn_norm.weight", &L.attn_norm, 0},       {"attn_q_norm.weight", &L.q_norm, 0},
               {"attn_k_norm.weight", &L.k_norm, 0},        {"attn_q.weight", &L.q, 0},
               {"attn_k.weight", &L.k, 0},                  {"attn_v.weight", &L.v, 0},
               {"attn_output.weight", &L.o, 0},             {"attn_gate.weight", &L.gate_attn, 0},
               {"ffn_norm.weight", &L.ffn_norm, 0},         {"ffn_gate.weight", &L.gate, 1},
               {"ffn_up.weight", &L.up, 1},                 {"ffn_down.weight", &L.down, 1},
               {"exp_probs_b.bias", &L.probs_bias, 2},      {"ffn_gate_inp.weight", &L.gate_inp, 2},
               {"ffn_gate_exps.weight", &L.gate_exps, 2},   {"ffn_up_exps.weight", &L.up_exps, 2},
               {"ffn_down_exps.weight", &L.down_exps, 2},   {"ffn_gate_shexp.weight", &L.gate_shexp, 2},
               {"ffn_up_shexp.weight", &L.up_shexp, 2},     {"ffn_down_shexp.weight", &L.down_shexp, 2}};
    for (auto &e : tab)
        if (!strcmp(suf, e.s)) {
            if ((e.kind == 1 && L.is_moe) || (e.kind == 2 && !L.is_moe)) return nullptr;
            return e.w;
        }
    return nullptr;
}

const float *need_f32(const DevTensor &w, const char *what, uint64_t n, int *status) {
    if (!w.ptr || w.dtype != LC_F32 || w.n_el < n) {
        *status = lc_fail(LC_ERR_INVALID, "lc_target: missing f32 tensor %s (%llu elements needed)", what,
                          (unsigned long long)n);
        return nullptr;
    }
    return (const float *)w.ptr;
}

int workspace(lc_target *t) {
    const lc_target_hparams &h = t->hp;
    const size_t B = t->max_block, E = h.n_embd, KVD = t->kvd(), QD = t->qd_max, F = h.n_ff;
    LC_TRY(talloc_t(t, (size_t)h.n_layers * t->max_ctx * KVD, &t->kcache));
    LC_TRY(talloc_t(t, (size_t)h.n_layers * t->max_ctx * KVD, &t->vcache));
    LC_TRY(talloc_t(t, B * E, &t->x));
    LC_TRY(talloc_t(t, B * E, &t->nx));
    LC_TRY(talloc_t(t, B * std::max(QD, E), &t->q));
    LC_TRY(talloc_t(t, B * std::max(QD, E), &t->attn));
    LC_TRY(talloc_t(t, B * std::max<size_t>(t->heads_max, 1), &t->gate));
    LC_TRY(talloc_t(t, B * E, &t->tmp));
    LC_TRY(talloc_t(t, B * KVD, &t->kbuf));
    LC_TRY(talloc_t(t, B * KVD, &t->vbuf));
    if (F) {
        LC_TRY(talloc_t(t, B * F, &t->ffg));
        LC_TRY(talloc_t(t, B * F, &t->ffu));
        LC_TRY(talloc_t(t, B * F, &t->ffh));
    }
    if (h.has_moe) {
        const size_t NE = h.n_expert, P = B * t->n_sel, Fe = h.n_ff_exp, S = h.n_ff_shexp;
        LC_TRY(talloc_t(t, B * NE, &t->router));
        LC_TRY(talloc_t(t, std::max<size_t>(P, 1), &t->ids));
        LC_TRY(talloc_t(t, std::max<size_t>((size_t)h.n_layers * P, 1), &t->route_log));
        LC_TRY(talloc_t(t, std::max<size_t>(P, 1), &t->scores));
        LC_TRY(talloc_t(t, std::max<size_t>(P, 1), &t->items));
        LC_TRY(talloc_t(t, 1, &t->n_items));
        LC_TRY(talloc_t(t, 2 * P * Fe, &t->gu));
        LC_TRY(talloc_t(t, 2 * B * NE * Fe, &t->gu_dense));
        LC_TRY(talloc_t(t, P * Fe, &t->hs));
        LC_TRY(talloc_t(t, std::max<size_t>(P, 1), &t->col));
        LC_TRY(talloc_t(t, P * E, &t->dout));
        LC_TRY(talloc_t(t, B * S, &t->sh_g));
        LC_TRY(talloc_t(t, B * S, &t->sh_u));
        LC_TRY(talloc_t(t, B * S, &t->sh_h));
        LC_TRY(talloc_t(t, B * E, &t->sh_out));
        LC_TRY(talloc_t(t, B * E, &t->moe_y));
    }
    // RoPE tables (src/target.rs:349-371)
    std::vector<float> f(std::max<uint32_t>(h.rope_dim, h.rope_dim_swa) / 2 + 1);
    LC_TRY(talloc_t(t, f.size(), &t->freq));
    LC_TRY(talloc_t(t, f.size(), &t->freq_swa));
    lc_rope_freq(f.data(), h.rope_dim, h.rope_base);
    LC_CUDA(cudaMemcpy(t->freq, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
    std::fill(f.begin(), f.end(), 0.f);
    lc_rope_freq(f.data(), h.rope_dim_swa, h.rope_base_swa);
    LC_CUDA(cudaMemcpy(t->freq_swa, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
    return LC_OK;
}

// Bytes of one [rows, k] matrix of an expert stack, and a check that the
// expert GEMV takes the format and k.
int expert_layout(const DevTensor &w, const char *what, uint32_t n_exp, uint32_t rows, uint32_t k, size_t *expert_bytes,
                  size_t *row_bytes) {
    if (!w.ptr) return lc_fail(LC_ERR_INVALID, "lc_target: missing tensor %s", what);
    if (w.n_el < (uint64_t)n_exp * rows * k)
        return lc_fail(LC_ERR_INVALID, "lc_target: %s has %llu elements, need %u x %u x %u", what,
                       (unsigned long long)w.n_el, n_exp, rows, k);
    const uint32_t be = (uint32_t)lc_type_block_elements(w.dtype), bb = (uint32_t)lc_type_block_bytes(w.dtype);
    const uint32_t need = w.dtype == LC_Q4_K ? 256 : w.dtype == LC_Q8_0 ? 32 : 8;
    if ((w.dtype != LC_Q4_K && w.dtype != LC_Q8_0 && w.dtype != LC_F32) || k % need)
        return lc_fail(LC_ERR_UNSUPPORTED, "lc_target: %s: type %d with k = %u (k must be a multiple of %u)", what,
                       w.dtype, k, need);
    *row_bytes = (size_t)k / be * bb;
    *expert_bytes = *row_bytes * rows;
    // the widest load of each format: the Q4_K block header (16 B), the Q8_0
    // scale and quant pairs (2 B), the F32 float4 (16 B)
    const size_t align = w.dtype == LC_Q8_0 ? 2 : 16;
    if ((((uintptr_t)w.ptr) | *expert_bytes | *row_bytes) & (align - 1))
        return lc_fail(LC_ERR_UNSUPPORTED, "lc_target: %s: expert rows must be %zu-byte aligned", what, align);
    return LC_OK;
}

// expert_stride / row_stride: bytes between experts / between the rows of one
// expert (expert-major stacks: one matrix and one row; the k-concatenated down
// stack: one row and n_expert rows).
int launch_expert_gemv(lc_target *t, const DevTensor &wa, const DevTensor *wb, size_t expert_stride, size_t row_stride,
                       uint32_t n, uint32_t k, const float *X, int act_div, float *Ya, float *Yb, uint32_t max_items) {
    lc_ctx *c = t->ctx;
    const bool ref = (t->flags & LC_TARGET_REF_EXPERT_OFFSET) && wa.dtype != LC_Q4_K;
    const dim3 grid((n + kRowsCta - 1) / kRowsCta, max_items, wb ? 2 : 1);
    const uint8_t *pa = (const uint8_t *)wa.ptr, *pb = wb ? (const uint8_t *)wb->ptr : pa;
#define LC_EXPERT_LAUNCH(DT)                                                                                      \
    expert_gemv_kernel<DT><<<grid, 256, 0, c->stream>>>(pa, pb, expert_stride, row_stride, ref ? 0 : -1, (int)n,    \
                                                         (int)k, X, act_div, t->items, t->n_items, Ya, Yb ? Yb : Ya, \
                                                         c->half_mode)
    switch (wa.dtype) {
    case LC_Q4_K: LC_EXPERT_LAUNCH(LC_Q4_K); break;
    case LC_Q8_0: LC_EXPERT_LAUNCH(LC_Q8_0); break;
    default: LC_EXPERT_LAUNCH(LC_F32); break;
    }
#undef LC_EXPERT_LAUNCH
    return lc_after_launch(c, "lc_target: expert projections");
}

int moe_ffn(lc_target *t, uint32_t l, const float *x, uint32_t m, float *y) {
    const lc_target_hparams &h = t->hp;
    TLayer &L = t->layers[l];
    lc_ctx *c = t->ctx;
    const uint32_t E = h.n_embd, NE = h.n_expert, NS = t->n_sel, Fe = h.n_ff_exp, S = h.n_ff_shexp;
    const uint32_t P = m * NS;
    int s = LC_OK;
    const float *bias = need_f32(L.probs_bias, "exp_probs_b.bias", NE, &s);
    if (s) return s;
    size_t gb, gr, ub, ur, db, dr;
    LC_TRY(expert_layout(L.gate_exps, "ffn_gate_exps.weight", NE, Fe, E, &gb, &gr));
    LC_TRY(expert_layout(L.up_exps, "ffn_up_exps.weight", NE, Fe, E, &ub, &ur));
    LC_TRY(expert_layout(L.down_exps, "ffn_down_exps.weight", NE, E, Fe, &db, &dr));
    // router logits and selection (src/target.rs:648-677)
    LC_TRY(lc::proj_w(c, L.gate_inp, "ffn_gate_inp.weight", x, t->router, m, E, NE));
    moe_route_kernel<<<m, 256, (size_t)(2 * NE + NS) * 4, c->stream>>>(t->router, bias, (int)NE, (int)NS,
                                                                       h.expert_weights_norm ? 1 : 0,
                                                                       h.expert_weights_scale, t->ids, t->scores);
    moe_items_kernel<<<1, 1024, 0, c->stream>>>(t->ids, (int)P, (int)NE, t->items, t->n_items);
    LC_CUDA(cudaMemcpyAsync(t->route_log + (size_t)l * t->max_block * NS, t->ids, (size_t)P * 4,
                            cudaMemcpyDeviceToDevice, c->stream));
    t->route_rows[l] = m;
    LC_TRY(lc_after_launch(c, "lc_target: routing"));
    // the selected experts' gate / up (src/target.rs:681-698).  A block whose
    // selections can cover the expert set (m * n_used >= n_expert) and whose
    // rows run the tcgen05 GEMM computes every expert at once: the stacks are
    // one [n_expert * n_ff_exp, n_embd] matrix each, streamed once at tensor-core
    // speed, and the pairs then take their expert's columns.  Smaller blocks
    // (decode) read only the selected experts.
    const bool dense = P >= NE && lc::routes_to_gemm_dq(c, m) && !(t->flags & LC_TARGET_REF_EXPERT_OFFSET) &&
                       L.gate_exps.dtype == L.up_exps.dtype &&
                       (L.gate_exps.dtype == LC_Q4_K || L.gate_exps.dtype == LC_Q8_0);
    float *g, *u;
    size_t dstride = 0;
    if (dense) {
        dstride = (size_t)NE * Fe;
        g = t->gu_dense;
        u = t->gu_dense + (size_t)m * dstride;
        lc::PackSrc src;
        src.x = x;
        lc::ProjOut outs[2] = {{nullptr, g, NE * Fe, false}, {nullptr, u, NE * Fe, false}};
        const DevTensor *ws[2] = {&L.gate_exps, &L.up_exps};
        const char *names[2] = {"ffn_gate_exps.weight", "ffn_up_exps.weight"};
        LC_TRY(lc::proj_w_block(c, t->tmp, src, nullptr, outs, ws, names, 2, m, E));
    } else {
        g = t->gu;
        u = t->gu + (size_t)P * Fe;
        if (L.gate_exps.dtype == L.up_exps.dtype && gb == ub) {
            LC_TRY(launch_expert_gemv(t, L.gate_exps, &L.up_exps, gb, gr, Fe, E, x, (int)NS, g, u, P));
        } else {
            LC_TRY(launch_expert_gemv(t, L.gate_exps, nullptr, gb, gr, Fe, E, x, (int)NS, g, nullptr, P));
            LC_TRY(launch_expert_gemv(t, L.up_exps, nullptr, ub, ur, Fe, E, x, (int)NS, u, nullptr, P));
        }
    }
    moe_swiglu_l2_kernel<<<P, 256, 0, c->stream>>>(g, u, (int)Fe, t->ids, (int)NS, dense ? 1 : 0, dstride, t->hs,
                                                   t->col);
    if (!(dense && L.down_kcat)) {
        const size_t es = L.down_kcat ? dr : db, rs = L.down_kcat ? (size_t)NE * dr : dr;
        LC_TRY(launch_expert_gemv(t, L.down_exps, nullptr, es, rs, E, Fe, t->hs, 1, t->dout, nullptr, P));
    }
    // shared expert (src/target.rs:726-745)
    {
        lc::PackSrc src;
        src.x = x;
        lc::ProjOut outs[2] = {{nullptr, t->sh_g, S, false}, {nullptr, t->sh_u, S, false}};
        const DevTensor *ws[2] = {&L.gate_shexp, &L.up_shexp};
        const char *names[2] = {"ffn_gate_shexp.weight", "ffn_up_shexp.weight"};
        LC_TRY(lc::proj_w_block(c, t->tmp, src, nullptr, outs, ws, names, 2, m, E));
    }
    {
        lc::PackSrc src;
        src.x = t->sh_g;
        src.x2 = t->sh_u;
        src.op = lc::LC_PACK_SWIGLU;
        lc::ProjOut outs[1] = {{nullptr, t->sh_out, E, false}};
        const DevTensor *ws[1] = {&L.down_shexp};
        const char *names[1] = {"ffn_down_shexp.weight"};
        LC_TRY(lc::proj_w_block(c, t->tmp, src, t->sh_h, outs, ws, names, 1, m, S));
    }
    if (dense && L.down_kcat) {
        // every expert's down projection as one GEMM over k = n_expert * n_ff_exp:
        // y = [H_e ...] . [W_e ...]^T sums the selected experts (the rest are zero)
        float *H = t->gu_dense;  // the gate outputs are consumed
        LC_CUDA(cudaMemsetAsync(H, 0, (size_t)m * NE * Fe * 4, c->stream));
        moe_scatter_kernel<<<P, 256, 0, c->stream>>>(t->hs, t->col, t->scores, t->ids, (int)NS, (int)NE, (int)Fe, H);
        LC_TRY(lc::proj_w(c, L.down_exps, "ffn_down_exps.weight", H, t->dout, m, NE * Fe, E));
        return lc_add(c, t->dout, t->sh_out, y, m * E);
    }
    const int threads = 256, blocks = (int)std::min<size_t>(((size_t)m * E + threads - 1) / threads, 4 * 148);
    moe_combine_kernel<<<blocks, threads, 0, c->stream>>>(t->dout, t->col, t->scores, t->ids, t->sh_out, (int)NS,
                                                           (int)E, (int)m, y);
    return lc_after_launch(c, "lc_target: expert sum");
}

}  // namespace

namespace {

// Q4_K / Q8_0 down-projection stacks go k-concatenated at load time, so a
// block that covers the expert set runs all experts' down projections as one
// GEMM; the per-expert kernel reads the same layout with other strides.  The
// reference's expert-offset behaviour needs the original order and keeps it.
int kcat_down_stacks(lc_target *t) {
    const lc_target_hparams &h = t->hp;
    if (!h.has_moe || (t->flags & LC_TARGET_REF_EXPERT_OFFSET) || h.n_ff_exp % 256 != 0) return LC_OK;
    const uint32_t NE = h.n_expert, E = h.n_embd, Fe = h.n_ff_exp;
    void *tmp = nullptr;
    size_t tmp_bytes = 0;
    int s = LC_OK;
    for (TLayer &L : t->layers) {
        DevTensor &w = L.down_exps;
        if (!L.is_moe || !w.ptr || (w.dtype != LC_Q4_K && w.dtype != LC_Q8_0) || w.n_el < (uint64_t)NE * E * Fe)
            continue;
        const size_t row_bytes = (size_t)Fe / lc_type_block_elements(w.dtype) * lc_type_block_bytes(w.dtype);
        const size_t bytes = row_bytes * E * NE;
        if (row_bytes % 16 || ((uintptr_t)w.ptr & 15)) continue;
        if (bytes > tmp_bytes) {
            if (tmp) cudaFree(tmp);
            tmp = nullptr;
            if (cudaMalloc(&tmp, bytes) != cudaSuccess) {
                cudaGetLastError();
                s = lc_fail(LC_ERR_OOM, "lc_target: cudaMalloc(%zu) for the down-projection layout", bytes);
                break;
            }
            tmp_bytes = bytes;
        }
        const long long units = (long long)NE * E;
        kcat_rows_kernel<<<(unsigned)((units + 7) / 8), 256, 0, t->ctx->stream>>>(
            (const uint8_t *)w.ptr, (uint8_t *)tmp, (int)NE, (int)E, (int)row_bytes);
        cudaError_t e = cudaMemcpyAsync(w.ptr, tmp, bytes, cudaMemcpyDeviceToDevice, t->ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(t->ctx->stream);
        if (e != cudaSuccess) {
            s = lc_fail(LC_ERR_CUDA, "lc_target: down-projection layout: %s", cudaGetErrorString(e));
            break;
        }
        L.down_kcat = true;
    }
    if (tmp) cudaFree(tmp);
    return s;
}

}  // namespace

extern "C" int lc_target_load_gguf(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block,
                                   uint32_t flags, lc_target **out) {
    LC_REQUIRE(ctx && path && out, LC_ERR_INVALID, "lc_target_load_gguf: null argument");
    LC_REQUIRE((flags & ~(uint32_t)(LC_LOAD_BF16_NATIVE | LC_TARGET_REF_EXPERT_OFFSET)) == 0, LC_ERR_INVALID,
               "lc_target_load_gguf: unknown flags %#x", flags);
    LC_REQUIRE(max_ctx >= 1 && max_block >= 1, LC_ERR_INVALID, "lc_target_load_gguf: max_ctx/max_block must be >= 1");
    *out = nullptr;
    LC_TRY(lc_use_device(ctx));
    lc_gguf *g;
    LC_TRY(lc_gguf_open(path, &g));
    lc_target *t = new lc_target();
    t->ctx = ctx;
    t->flags = flags;
    t->max_ctx = max_ctx;
    t->max_block = max_block;
    int s = lc_gguf_target_hparams(g, &t->hp);
    const lc_target_hparams &h = t->hp;
    if (!s && !(h.n_layers && h.n_embd && h.n_heads && h.n_kv_heads && h.head_dim))
        s = lc_fail(LC_ERR_INVALID, "lc_target_load_gguf: incomplete hyper-parameters (block_count, embedding_length, "
                                    "head_count, head_count_kv and key_length are required)");
    if (!s && h.has_moe && (h.n_expert == 0 || h.n_expert > (uint32_t)kMaxExperts || h.n_expert_used == 0))
        s = lc_fail(LC_ERR_UNSUPPORTED, "lc_target_load_gguf: %u experts, %u used (1..%d experts)", h.n_expert,
                    h.n_expert_used, kMaxExperts);
    if (!s) {
        t->layers.resize(h.n_layers);
        t->route_rows.assign(h.n_layers, 0);
        for (uint32_t l = 0; l < h.n_layers; l++) t->layers[l].is_moe = h.has_moe && l > 0;  // src/target.rs:140
        t->n_sel = std::min(h.n_expert_used, h.n_expert);
        s = lc::load_tensors(ctx, g, [t](const char *name) { return target_slot(t, name); }, flags & LC_LOAD_BF16_NATIVE,
                             &t->allocs);
    }
    lc_gguf_close(g);
    if (!s) {
        t->heads_max = h.n_heads;
        for (TLayer &L : t->layers) {
            // src/target.rs:224-233: attn_q's output dim / head_dim, else head_count
            L.n_q_heads = L.q.ptr && L.q.n_dims >= 2 ? (uint32_t)(L.q.shape[1] / h.head_dim) : h.n_heads;
            t->heads_max = std::max(t->heads_max, L.n_q_heads);
        }
        t->qd_max = t->heads_max * h.head_dim;
        s = kcat_down_stacks(t);
        if (!s) s = workspace(t);
    }
    if (s) {
        delete t;
        return s;
    }
    *out = t;
    return LC_OK;
}

extern "C" int lc_target_destroy(lc_target *t) {
    if (!t) return LC_OK;
    lc_use_device(t->ctx);
    cudaStreamSynchronize(t->ctx->stream);
    delete t;
    return LC_OK;
}

extern "C" int lc_target_get_hparams(const lc_target *t, lc_target_hparams *out) {
    LC_REQUIRE(t && out, LC_ERR_INVALID, "lc_target_get_hparams: null argument");
    *out = t->hp;
    return LC_OK;
}

extern "C" int lc_target_layer_info(const lc_target *t, uint32_t layer, uint32_t *is_moe, uint32_t *n_q_heads) {
    LC_REQUIRE(t && layer < t->layers.size(), LC_ERR_INVALID, "lc_target_layer_info: bad layer");
    if (is_moe) *is_moe = t->layers[layer].is_moe;
    if (n_q_heads) *n_q_heads = t->layers[layer].n_q_heads;
    return LC_OK;
}

extern "C" int lc_target_weight(const lc_target *t, const char *name, const void **data, int *dtype,
                                uint64_t *bytes) {
    LC_REQUIRE(t && name && data, LC_ERR_INVALID, "lc_target_weight: null argument");
    const DevTensor *w = target_slot(const_cast<lc_target *>(t), name);
    LC_REQUIRE(w && w->ptr, LC_ERR_INVALID, "lc_target_weight: no tensor %s", name);
    *data = w->ptr;
    if (dtype) *dtype = w->dtype;
    if (bytes) *bytes = w->bytes;
    return LC_OK;
}

extern "C" int lc_target_embed(lc_target *t, const uint32_t *tokens, uint32_t m, float *x) {
    LC_REQUIRE(t && tokens && x, LC_ERR_INVALID, "lc_target_embed: null argument");
    LC_TRY(lc_use_device(t->ctx));
    const DevTensor &w = t->tok_embd;
    const uint32_t E = t->hp.n_embd;
    LC_REQUIRE(w.ptr, LC_ERR_INVALID, "lc_target_embed: the model has no token_embd.weight");
    const uint64_t be = lc_type_block_elements(w.dtype), bb = lc_type_block_bytes(w.dtype);
    LC_REQUIRE(E % be == 0, LC_ERR_UNSUPPORTED, "lc_target_embed: n_embd %u is not a whole number of blocks", E);
    // dequant_to_f32's CPU decoder, Q4_K branch included (src/dflash.rs:331-465)
    const int dt = w.dtype == LC_Q4_K ? LC_Q4_K_DFLASH_CPU : w.dtype;
    for (uint32_t r = 0; r < m; r++) {
        LC_REQUIRE(tokens[r] < t->hp.n_vocab, LC_ERR_INVALID, "lc_target_embed: token %u >= vocab %u", tokens[r],
                   t->hp.n_vocab);
        const size_t off = (size_t)tokens[r] * E / be * bb;
        LC_TRY(lc_dequant(t->ctx, dt, (const uint8_t *)w.ptr + off, (size_t)E / be * bb, E, x + (size_t)r * E));
    }
    return LC_OK;
}

extern "C" int lc_target_routing(const lc_target *t, uint32_t layer, int32_t *ids, uint32_t *m) {
    LC_REQUIRE(t && ids && m, LC_ERR_INVALID, "lc_target_routing: null argument");
    LC_REQUIRE(layer < t->layers.size() && t->layers[layer].is_moe, LC_ERR_INVALID,
               "lc_target_routing: layer %u is not a MoE layer", layer);
    *m = t->route_rows[layer];
    if (*m == 0) return LC_OK;
    const lc_ctx *c = t->ctx;
    LC_CUDA(cudaMemcpyAsync(ids, t->route_log + (size_t)layer * t->max_block * t->n_sel, (size_t)*m * t->n_sel * 4,
                            cudaMemcpyDeviceToDevice, c->stream));
    return LC_OK;
}

extern "C" int lc_target_cache_len(const lc_target *t, uint32_t *len) {
    LC_REQUIRE(t && len, LC_ERR_INVALID, "lc_target_cache_len: null argument");
    *len = t->cache_len;
    return LC_OK;
}

extern "C" int lc_target_cache_truncate(lc_target *t, uint32_t len) {
    LC_REQUIRE(t, LC_ERR_INVALID, "lc_target_cache_truncate: null argument");
    t->cache_len = std::min(t->cache_len, len);
    return LC_OK;
}

extern "C" int lc_target_moe_ffn(lc_target *t, uint32_t layer, const float *x, uint32_t m, float *y, int32_t *ids,
                                 float *scores) {
    LC_REQUIRE(t && x && y, LC_ERR_INVALID, "lc_target_moe_ffn: null argument");
    LC_REQUIRE(layer < t->layers.size() && t->layers[layer].is_moe, LC_ERR_INVALID,
               "lc_target_moe_ffn: layer %u is not a MoE layer", layer);
    LC_REQUIRE(m >= 1 && m <= t->max_block, LC_ERR_INVALID, "lc_target_moe_ffn: %u rows not in 1..%u", m, t->max_block);
    LC_TRY(lc_use_device(t->ctx));
    LC_TRY(moe_ffn(t, layer, x, m, y));
    const size_t P = (size_t)m * t->n_sel;
    if (ids) LC_CUDA(cudaMemcpyAsync(ids, t->ids, P * 4, cudaMemcpyDeviceToDevice, t->ctx->stream));
    if (scores) LC_CUDA(cudaMemcpyAsync(scores, t->scores, P * 4, cudaMemcpyDeviceToDevice, t->ctx->stream));
    return lc_after_launch(t->ctx, "lc_target_moe_ffn");
}

extern "C" int lc_target_forward(lc_target *t, const float *x_in, uint32_t m, uint32_t flags,
                                 const uint32_t *capture_layers, uint32_t n_capture, float *captured, float *hidden,
                                 float *logits, uint64_t *keys) {
    LC_REQUIRE(t && x_in, LC_ERR_INVALID, "lc_target_forward: null argument");
    LC_REQUIRE((flags & ~(uint32_t)LC_TARGET_CACHED) == 0, LC_ERR_INVALID, "lc_target_forward: unknown flags %#x",
               flags);
    LC_REQUIRE(m >= 1 && m <= t->max_block, LC_ERR_INVALID, "lc_target_forward: %u tokens not in 1..%u", m,
               t->max_block);
    const bool cached = flags & LC_TARGET_CACHED;
    LC_REQUIRE(!cached || t->cache_len + m <= t->max_ctx, LC_ERR_INVALID,
               "lc_target_forward: cache of %u positions cannot take %u more (max_ctx %u)", t->cache_len, m,
               t->max_ctx);
    LC_TRY(lc_use_device(t->ctx));
    const lc_target_hparams &h = t->hp;
    const uint32_t E = h.n_embd, KV = h.n_kv_heads, hd = h.head_dim, KVD = (uint32_t)t->kvd();
    // one output slot per distinct listed layer <= n_layers, in layer order
    std::vector<int> slot(h.n_layers + 1, -1);
    for (uint32_t i = 0; i < n_capture; i++)
        if (capture_layers && capture_layers[i] <= h.n_layers) slot[capture_layers[i]] = 0;
    uint32_t n_slots = 0;
    for (int &s : slot)
        if (s == 0) s = (int)n_slots++;
    LC_REQUIRE(n_slots == 0 || captured, LC_ERR_INVALID, "lc_target_forward: capture layers given without a buffer");
    lc_ctx *c = t->ctx;
    cudaStream_t st = c->stream;
    auto capture = [&](uint32_t layer) -> int {
        if (slot[layer] < 0) return LC_OK;
        LC_CUDA(cudaMemcpy2DAsync(captured + (size_t)slot[layer] * E, (size_t)n_slots * E * 4, t->x, (size_t)E * 4,
                                  (size_t)E * 4, m, cudaMemcpyDeviceToDevice, st));
        return LC_OK;
    };
    const uint32_t pos0 = cached ? t->cache_len : 0;
    const float scale = 1.0f / sqrtf((float)hd);  // src/target.rs:779
    LC_CUDA(cudaMemcpyAsync(t->x, x_in, (size_t)m * E * 4, cudaMemcpyDeviceToDevice, st));
    for (uint32_t l = 0; l < h.n_layers; l++) {
        LC_TRY(capture(l));
        const TLayer &L = t->layers[l];
        const uint32_t H = L.n_q_heads, QD = H * hd;
        int s = LC_OK;
        const float *an = need_f32(L.attn_norm, "attn_norm.weight", E, &s);
        const float *qn = need_f32(L.q_norm, "attn_q_norm.weight", hd, &s);
        const float *kn = need_f32(L.k_norm, "attn_k_norm.weight", hd, &s);
        const float *fn = need_f32(L.ffn_norm, "ffn_norm.weight", E, &s);
        if (s) return s;
        // src/target.rs:414-438: norm, then q / k / v (and the head gate of
        // :497-503, which reads the same normalised rows) from one block; the
        // norm is formed while the block is packed (t->nx only on the
        // per-projection route)
        float *kd = cached ? t->kl(l) + (size_t)pos0 * KVD : t->kbuf;
        float *vd = cached ? t->vl(l) + (size_t)pos0 * KVD : t->vbuf;
        const bool gated = L.gate_attn.ptr != nullptr;
        {
            lc::PackSrc src;
            src.x = t->x;
            src.x2 = an;
            src.op = lc::LC_PACK_RMSNORM;
            src.eps = h.norm_eps;
            lc::ProjOut outs[4] = {{nullptr, t->q, QD, false}, {nullptr, kd, KVD, false}, {nullptr, vd, KVD, false},
                                   {nullptr, t->gate, H, false}};
            const DevTensor *ws[4] = {&L.q, &L.k, &L.v, &L.gate_attn};
            const char *names[4] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_gate.weight"};
            LC_TRY(lc::proj_w_block(c, t->tmp, src, t->nx, outs, ws, names, gated ? 4 : 3, m, E));
        }
        // :440-463 -- SWA layers rotate with their own dimension and base
        const bool swa = h.swa && (l % 4 != 0);
        LC_TRY(lc::qk_norm_rope_pair(c, t->q, qn, t->q, H, kd, kn, kd, KV, swa ? t->freq_swa : t->freq, m, hd,
                                     swa ? h.rope_dim_swa : h.rope_dim, h.qk_eps, pos0, cached ? 1 : 0));
        if (cached) {
            // :465-487 -- the cache rows [0, pos0 + m) are adjacent on the device
            LC_TRY(lc_mha_attn(c, t->q, t->kl(l), t->vl(l), t->attn, m, H, KV, hd, pos0 + m, scale, pos0, 1));
        } else {
            const int n = (int)(m * QD);
            gqa_expand_kernel<<<std::min((n + 255) / 256, 4 * 148), 256, 0, st>>>(t->vbuf, t->attn, (int)m, (int)H,
                                                                                  (int)KV, (int)hd);
            LC_TRY(lc_after_launch(c, "lc_target_forward: attention"));
        }
        // :495-514 -- attn * softplus(head gate), output projection, residual add
        {
            lc::PackSrc src;
            src.x = t->attn;
            if (gated) {
                src.x2 = t->gate;
                src.op = lc::LC_PACK_HEADGATE;
                src.head_dim = (int)hd;
            }
            lc::ProjOut outs[1] = {{nullptr, t->x, E, true}};
            const DevTensor *ws[1] = {&L.o};
            const char *names[1] = {"attn_output.weight"};
            LC_TRY(lc::proj_w_block(c, t->tmp, src, t->attn, outs, ws, names, 1, m, QD));
        }
        if (L.is_moe) {
            // :520-524
            LC_TRY(lc_rmsnorm(c, fn, t->x, t->nx, m, E, h.norm_eps));
            LC_TRY(moe_ffn(t, l, t->nx, m, t->moe_y));
            LC_TRY(lc_add(c, t->x, t->moe_y, t->x, m * E));
        } else {
            // :526-546
            const uint32_t F = h.n_ff;
            LC_REQUIRE(F > 0, LC_ERR_INVALID, "lc_target_forward: dense layer %u without feed_forward_length", l);
            {  // ffn_norm formed while packing
                lc::PackSrc src;
                src.x = t->x;
                src.x2 = fn;
                src.op = lc::LC_PACK_RMSNORM;
                src.eps = h.norm_eps;
                lc::ProjOut outs[2] = {{nullptr, t->ffg, F, false}, {nullptr, t->ffu, F, false}};
                const DevTensor *ws[2] = {&L.gate, &L.up};
                const char *names[2] = {"ffn_gate.weight", "ffn_up.weight"};
                LC_TRY(lc::proj_w_block(c, t->tmp, src, t->nx, outs, ws, names, 2, m, E));
            }
            {
                lc::PackSrc src;
                src.x = t->ffg;
                src.x2 = t->ffu;
                src.op = lc::LC_PACK_SWIGLU;
                lc::ProjOut outs[1] = {{nullptr, t->x, E, true}};
                const DevTensor *ws[1] = {&L.down};
                const char *names[1] = {"ffn_down.weight"};
                LC_TRY(lc::proj_w_block(c, t->tmp, src, t->ffh, outs, ws, names, 1, m, F));
            }
        }
    }
    LC_TRY(capture(h.n_layers));
    if (cached) t->cache_len += m;
    // :556-575 -- output_norm in place, then the lm_head (or the hidden state itself)
    float *hid = hidden ? hidden : t->nx;
    if (t->output_norm.ptr) {
        int s = LC_OK;
        const float *on = need_f32(t->output_norm, "output_norm.weight", E, &s);
        if (s) return s;
        LC_TRY(lc_rmsnorm(c, on, t->x, hid, m, E, h.norm_eps));
    } else {
        LC_CUDA(cudaMemcpyAsync(hid, t->x, (size_t)m * E * 4, cudaMemcpyDeviceToDevice, st));
    }
    if (logits || keys) {
        const uint32_t V = h.n_vocab;
        if (t->output.ptr) {
            LC_REQUIRE(V > 0 && t->output.n_el >= (uint64_t)V * E, LC_ERR_INVALID,
                       "lc_target_forward: output.weight has %llu elements, need %u x %u",
                       (unsigned long long)t->output.n_el, V, E);
            if (keys)
                LC_TRY(lc_lm_head_argmax(c, t->output.dtype, hid, t->output.ptr, m, E, V, 0, keys, logits));
            else
                LC_TRY(lc_proj_m(c, t->output.dtype, hid, t->output.ptr, logits, m, E, V, 0));
        } else {
            if (logits) LC_CUDA(cudaMemcpyAsync(logits, hid, (size_t)m * E * 4, cudaMemcpyDeviceToDevice, st));
            if (keys) LC_TRY(lc_argmax_rows(c, hid, m, E, 0, keys));
        }
    }
    return lc_after_launch(c, "lc_target_forward");
}
