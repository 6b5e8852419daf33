// lc_attn.cu -- GQA attention of kernels/mha_attn.comp:31-72 for a block of
// query rows.  attn_tc_kernel (tensor cores, 3xTF32) is the default;
// attn_partial_kernel (f32 FMA) runs with LC_GEMM_TC=0.
//
// The reference runs one invocation per (head, dim) and walks all positions
// with an online softmax (m starts at -1e30, causal break at p > q_pos, output
// 0 when no key is visible).  Here every key/value row of one KV head is
// staged in shared memory once and reused by all query heads of the group and
// all query rows (up to 64 query vectors per CTA): the CTA grid is
// (kv head, key split, query chunk) and a second kernel merges the split
// partial softmax states.  Arithmetic is fp32 throughout.
#include <algorithm>

#include "lc_internal.cuh"

namespace {

constexpr int kQV = 64;   // query vectors per CTA
constexpr int kTK = 32;   // keys per tile
constexpr int kHD = 128;  // head_dim handled by this kernel
constexpr int kThreads = 256;
constexpr float kNegInit = -1e30f;
// Padded shared-memory row strides (floats, 16-byte aligned): the 8 query
// vectors (stride 132) and the 4 key rows (stride 132) a warp reads at once fall
// in different banks; probabilities stride 36.
constexpr int kQS = kHD + 4;
constexpr int kKS = kHD + 4;
constexpr int kPS = kTK + 4;

// 16-byte global -> shared copy that bypasses registers (cp.async); src_bytes 0
// writes zeros (keys past the split's end).
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Partials: o[split][row][head][d], ml[split][row][head] = (m, l).
__global__ void __launch_bounds__(kThreads) attn_partial_kernel(const float *__restrict__ q,
                                                                const float *__restrict__ k,
                                                                const float *__restrict__ v, float *__restrict__ o_part,
                                                                float2 *__restrict__ ml_part, int m, int n_q, int n_kv,
                                                                int seq_len, int keys_per_split, float scale,
                                                                uint32_t q_pos0, int causal) {
    extern __shared__ __align__(16) float sm[];
    float *sQ = sm;                     // [kQV][kQS]
    float *sK0 = sQ + kQV * kQS;        // two buffers of [kTK][kKS]
    float *sV0 = sK0 + 2 * kTK * kKS;   // two buffers of [kTK][kHD]
    float *sP = sV0 + 2 * kTK * kHD;    // [kQV][kPS]

    const int hk = blockIdx.x, split = blockIdx.y, chunk = blockIdx.z;
    const int G = n_q / n_kv;
    const int qv_total = m * G;
    const int qv0 = chunk * kQV;
    const int nqv = min(kQV, qv_total - qv0);
    const int tid = threadIdx.x;
    const int p_begin = split * keys_per_split;
    const int p_end = min(seq_len, p_begin + keys_per_split);
    const int ldq = n_q * kHD, ldk = n_kv * kHD;

    // query vector i of this chunk: global qv = qv0 + i -> row r = qv / G, head h = hk*G + qv % G;
    // 32 threads per vector, one float4 each (rows past nqv zero)
    for (int qi = tid >> 5; qi < kQV; qi += kThreads / 32) {
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < nqv) {
            const int gq = qv0 + qi, r = gq / G, h = hk * G + gq % G;
            val = *reinterpret_cast<const float4 *>(q + (size_t)r * ldq + h * kHD + 4 * (tid & 31));
        }
        *reinterpret_cast<float4 *>(sQ + qi * kQS + 4 * (tid & 31)) = val;
    }

    const int my_qv = tid >> 2;     // 0..63
    const int sub = tid & 3;        // 4 threads per query vector
    const bool active = my_qv < nqv;
    int my_row = 0;
    if (active) my_row = (qv0 + my_qv) / G;
    const long long my_pos = (long long)q_pos0 + my_row;

    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0.f;
    float run_m = kNegInit, run_l = 0.f;

    // K / V tiles double-buffered with cp.async: tile t+1 streams in while tile
    // t is computed
    auto load_tile = [&](int t0, int buf) {
        const int nk = min(kTK, p_end - t0);
        float *sK = sK0 + buf * kTK * kKS, *sV = sV0 + buf * kTK * kHD;
        for (int i = tid; i < kTK * (kHD / 4); i += kThreads) {  // 16-byte copies, coalesced
            const int kk = i / (kHD / 4), d4 = i % (kHD / 4);
            const size_t off = (size_t)(t0 + (kk < nk ? kk : 0)) * ldk + hk * kHD + 4 * d4;
            const uint32_t nb = kk < nk ? 16u : 0u;
            cp_async16(sK + kk * kKS + 4 * d4, k + off, nb);
            cp_async16(sV + kk * kHD + 4 * d4, v + off, nb);
        }
        cp_async_commit();
    };
    if (p_begin < p_end) load_tile(p_begin, 0);
    int buf = 0;
    for (int t0 = p_begin; t0 < p_end; t0 += kTK, buf ^= 1) {
        const int nk = min(kTK, p_end - t0);
        if (t0 + kTK < p_end) {
            load_tile(t0 + kTK, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // tile t0 (and the staged queries) visible to every thread
        const float *sK = sK0 + buf * kTK * kKS, *sV = sV0 + buf * kTK * kHD;

        // scores of this thread's query against keys sub + 4i (i = 0..7: the 4
        // sub-threads of a query read adjacent rows, in different banks), 4 dims
        // per step (9 independent 16-byte loads per 32 FMAs)
        float s[8];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i] = 0.f;
        const float *qrow = sQ + my_qv * kQS;
        const float *krow = sK + sub * kKS;
#pragma unroll 4
        for (int d = 0; d < kHD; d += 4) {
            const float4 qd = *reinterpret_cast<const float4 *>(qrow + d);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 kd = *reinterpret_cast<const float4 *>(krow + 4 * i * kKS + d);
                s[i] += qd.x * kd.x + qd.y * kd.y + qd.z * kd.z + qd.w * kd.w;
            }
        }
        float tmax = kNegInit;
        bool vis[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int kk = sub + 4 * i;
            const long long p = t0 + kk;
            vis[i] = active && kk < nk && (!causal || p <= my_pos);
            s[i] *= scale;
            if (vis[i]) tmax = fmaxf(tmax, s[i]);
        }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(run_m, tmax);
        const float corr = expf(run_m - m_new);
        float psum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float p = vis[i] ? expf(s[i] - m_new) : 0.f;
            psum += p;
            sP[my_qv * kPS + sub + 4 * i] = p;
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        run_l = run_l * corr + psum;
        run_m = m_new;
        __syncwarp();
        // acc[4j .. 4j+3] = d of float4 column sub + 4j (the sub-threads read
        // adjacent 16-byte columns of a V row, in different banks)
#pragma unroll
        for (int i = 0; i < 32; i++) acc[i] *= corr;
#pragma unroll 2
        for (int kk = 0; kk < nk; kk++) {
            const float p = sP[my_qv * kPS + kk];
            const float4 *vr = reinterpret_cast<const float4 *>(sV + kk * kHD) + sub;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 vv = vr[4 * j];
                acc[4 * j + 0] += p * vv.x;
                acc[4 * j + 1] += p * vv.y;
                acc[4 * j + 2] += p * vv.z;
                acc[4 * j + 3] += p * vv.w;
            }
        }
        __syncthreads();  // done with this buffer and sP before they are overwritten
    }
    if (!active) return;
    const int gq = qv0 + my_qv, r = gq / G, h = hk * G + gq % G;
    const size_t base = ((size_t)split * m + r) * n_q + h;
    float4 *op = reinterpret_cast<float4 *>(o_part + base * kHD) + sub;
#pragma unroll
    for (int j = 0; j < 8; j++) op[4 * j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
    if (sub == 0) ml_part[base] = make_float2(run_m, run_l);
}

// ---- tensor-core form (head_dim 128) ----------------------------------------
//
// The same partial softmax states as attn_partial_kernel, computed with
// mma.sync m16n8k8 TF32 in the 3xTF32 form (a = a_hi + a_lo, b = b_hi + b_lo,
// a b ~ a_hi b_hi + a_hi b_lo + a_lo b_hi with f32 accumulation: about f32
// accuracy).  One CTA per (KV head, key split, chunk of 64 query vectors), 8
// warps: warp w takes query vectors 16 (w % 4) .. +15 against keys 32 (w / 4)
// .. +31 of every 64-key tile (two warps per scheduler), with its own online
// softmax state; the two key halves are merged in shared memory at the end.
// Per tile S = Q K^T (16 x 32 per warp) in registers, the softmax on its
// fragments, P through shared memory into A-fragment layout, O += P V (16 x 128
// per warp).  K / V tiles double-buffered with cp.async.

constexpr int kTcKeys = 64;              // keys per tile
constexpr int kTcWarps = 8;
constexpr int kTcQS = kHD + 4;           // sQ / sK row stride: fragment loads conflict-free
constexpr int kTcVS = kHD + 8;           // sV row stride (B fragments of P V read down columns)
constexpr int kTcPS = kTcKeys / 2 + 4;   // sP row stride (32 keys per warp)

__device__ __forceinline__ uint32_t tf32_bits(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
    return r;
}
// x ~ hi + lo, both TF32
__device__ __forceinline__ void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_bits(x);
    lo = tf32_bits(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// An A fragment split once into its TF32 hi / lo parts.
struct Tf32Frag {
    uint32_t h[4], l[4];
};
__device__ __forceinline__ Tf32Frag tf32_frag(const float (&a)[4]) {
    Tf32Frag f;
#pragma unroll
    for (int i = 0; i < 4; i++) tf32_split(a[i], f.h[i], f.l[i]);
    return f;
}

// d += a b with b given as f32: three TF32 products (small terms first).
__device__ __forceinline__ void mma_3xtf32(float (&d)[4], const Tf32Frag &a, float b0f, float b1f) {
    uint32_t bh0, bl0, bh1, bl1;
    tf32_split(b0f, bh0, bl0);
    tf32_split(b1f, bh1, bl1);
    mma_tf32(d, a.l, bh0, bh1);
    mma_tf32(d, a.h, bl0, bl1);
    mma_tf32(d, a.h, bh0, bh1);
}

__global__ void __launch_bounds__(kTcWarps * 32, 1)
    attn_tc_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                   float *__restrict__ o_part, float2 *__restrict__ ml_part, int m, int n_q, int n_kv, int seq_len,
                   int keys_per_split, float scale, uint32_t q_pos0, int causal) {
    extern __shared__ __align__(16) float sm[];
    float *sQ = sm;                                // [64][kTcQS]
    float *sK0 = sQ + kQV * kTcQS;                 // 2 x [64][kTcQS]
    float *sV0 = sK0 + 2 * kTcKeys * kTcQS;        // 2 x [64][kTcVS]
    float *sP = sV0 + 2 * kTcKeys * kTcVS;         // [8 warps][16][kTcPS]
    const int hk = blockIdx.x, split = blockIdx.y, chunk = blockIdx.z;
    const int G = n_q / n_kv, qv_total = m * G, qv0 = chunk * kQV;
    const int nqv = min(kQV, qv_total - qv0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int qg = warp & 3, kh = warp >> 2;  // query group, key half
    const int p_begin = split * keys_per_split, p_end = min(seq_len, p_begin + keys_per_split);
    const int ldq = n_q * kHD, ldk = n_kv * kHD;

    // stage the 64 query vectors (rows past nqv zero): 32 threads per vector
    for (int qi = tid >> 5; qi < kQV; qi += kTcWarps) {
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < nqv) {
            const int gq = qv0 + qi, r = gq / G, h = hk * G + gq % G;
            val = *reinterpret_cast<const float4 *>(q + (size_t)r * ldq + h * kHD + 4 * lane);
        }
        *reinterpret_cast<float4 *>(sQ + qi * kTcQS + 4 * lane) = val;
    }
    auto load_tile = [&](int t0, int buf) {
        const int nk = min(kTcKeys, p_end - t0);
        float *sK = sK0 + buf * kTcKeys * kTcQS, *sV = sV0 + buf * kTcKeys * kTcVS;
        for (int i = tid; i < kTcKeys * (kHD / 4); i += kTcWarps * 32) {
            const int kk = i / (kHD / 4), d4 = i % (kHD / 4);
            const size_t off = (size_t)(t0 + (kk < nk ? kk : 0)) * ldk + hk * kHD + 4 * d4;
            const uint32_t nb = kk < nk ? 16u : 0u;
            cp_async16(sK + kk * kTcQS + 4 * d4, k + off, nb);
            cp_async16(sV + kk * kTcVS + 4 * d4, v + off, nb);
        }
        cp_async_commit();
    };

    // this thread's two query rows in the warp's 16: g and g + 8
    const int qa = qg * 16 + g, qb = qa + 8;
    const long long pos_a = (long long)q_pos0 + (qv0 + qa) / G, pos_b = (long long)q_pos0 + (qv0 + qb) / G;
    const bool act_a = qa < nqv, act_b = qb < nqv;
    float o[16][4];  // O[16 rows x 128 dims]: n-tile j = dims 8j..8j+7
#pragma unroll
    for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = kNegInit, m_b = kNegInit, l_a = 0.f, l_b = 0.f;

    if (p_begin < p_end) load_tile(p_begin, 0);
    int buf = 0;
    for (int t0 = p_begin; t0 < p_end; t0 += kTcKeys, buf ^= 1) {
        if (t0 + kTcKeys < p_end) {
            load_tile(t0 + kTcKeys, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *sK = sK0 + buf * kTcKeys * kTcQS, *sV = sV0 + buf * kTcKeys * kTcVS;
        // S = Q K^T: 4 n-tiles of 8 keys (this warp's half), 16 k-steps of 8 dims
        float sc[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
        const float *qw = sQ + (qg * 16) * kTcQS;
        const int key0 = 32 * kh;
#pragma unroll 2
        for (int kk = 0; kk < kHD; kk += 8) {
            const float a[4] = {qw[g * kTcQS + kk + t], qw[(g + 8) * kTcQS + kk + t], qw[g * kTcQS + kk + t + 4],
                                qw[(g + 8) * kTcQS + kk + t + 4]};
            const Tf32Frag af = tf32_frag(a);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float *kr = sK + (key0 + 8 * j + g) * kTcQS + kk;
                mma_3xtf32(sc[j], af, kr[t], kr[t + 4]);
            }
        }
        // online softmax over this tile (rows g, g + 8 of the warp)
        float tmax_a = kNegInit, tmax_b = kNegInit;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int key = t0 + key0 + 8 * j + 2 * t + (c & 1);
                const bool rb = c >= 2;
                const bool vis = (rb ? act_b : act_a) && key < p_end && (!causal || key <= (rb ? pos_b : pos_a));
                sc[j][c] = vis ? sc[j][c] * scale : -INFINITY;
                if (vis) {
                    if (rb) tmax_b = fmaxf(tmax_b, sc[j][c]);
                    else tmax_a = fmaxf(tmax_a, sc[j][c]);
                }
            }
#pragma unroll
        for (int o2 = 1; o2 <= 2; o2 <<= 1) {
            tmax_a = fmaxf(tmax_a, __shfl_xor_sync(0xffffffffu, tmax_a, o2));
            tmax_b = fmaxf(tmax_b, __shfl_xor_sync(0xffffffffu, tmax_b, o2));
        }
        const float mn_a = fmaxf(m_a, tmax_a), mn_b = fmaxf(m_b, tmax_b);
        const float cr_a = expf(m_a - mn_a), cr_b = expf(m_b - mn_b);
        float ps_a = 0.f, ps_b = 0.f;
        float *pw = sP + (warp * 16) * kTcPS;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float p0 = sc[j][0] == -INFINITY ? 0.f : expf(sc[j][0] - mn_a);
            const float p1 = sc[j][1] == -INFINITY ? 0.f : expf(sc[j][1] - mn_a);
            const float p2 = sc[j][2] == -INFINITY ? 0.f : expf(sc[j][2] - mn_b);
            const float p3 = sc[j][3] == -INFINITY ? 0.f : expf(sc[j][3] - mn_b);
            ps_a += p0 + p1;
            ps_b += p2 + p3;
            *reinterpret_cast<float2 *>(pw + g * kTcPS + 8 * j + 2 * t) = make_float2(p0, p1);
            *reinterpret_cast<float2 *>(pw + (g + 8) * kTcPS + 8 * j + 2 * t) = make_float2(p2, p3);
        }
#pragma unroll
        for (int o2 = 1; o2 <= 2; o2 <<= 1) {
            ps_a += __shfl_xor_sync(0xffffffffu, ps_a, o2);
            ps_b += __shfl_xor_sync(0xffffffffu, ps_b, o2);
        }
        l_a = l_a * cr_a + ps_a;
        l_b = l_b * cr_b + ps_b;
        m_a = mn_a;
        m_b = mn_b;
#pragma unroll
        for (int j = 0; j < 16; j++) o[j][0] *= cr_a, o[j][1] *= cr_a, o[j][2] *= cr_b, o[j][3] *= cr_b;
        __syncwarp();
        // O += P V: 16 n-tiles of 8 dims, 4 k-steps of 8 keys (this warp's half)
#pragma unroll 2
        for (int kk = 0; kk < kTcKeys / 2; kk += 8) {
            const float a[4] = {pw[g * kTcPS + kk + t], pw[(g + 8) * kTcPS + kk + t], pw[g * kTcPS + kk + t + 4],
                                pw[(g + 8) * kTcPS + kk + t + 4]};
            const Tf32Frag af = tf32_frag(a);
#pragma unroll
            for (int j = 0; j < 16; j++)
                mma_3xtf32(o[j], af, sV[(key0 + kk + t) * kTcVS + 8 * j + g],
                           sV[(key0 + kk + t + 4) * kTcVS + 8 * j + g]);
        }
        __syncthreads();  // done with this K / V buffer before it is refilled
    }
    // merge the two key halves: warps 4..7 hand (m, l, O) to warps 0..3 through
    // shared memory (the K buffers, free after the loop's final barrier)
    float *xch = sK0 + (size_t)(qg * 32 + lane) * 68;
    if (kh == 1) {
#pragma unroll
        for (int j = 0; j < 16; j++)
            *reinterpret_cast<float4 *>(xch + 4 * j) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
        *reinterpret_cast<float4 *>(xch + 64) = make_float4(m_a, m_b, l_a, l_b);
    }
    __syncthreads();
    if (kh == 1) return;
    {
        const float4 ml = *reinterpret_cast<const float4 *>(xch + 64);
        const float Ma = fmaxf(m_a, ml.x), Mb = fmaxf(m_b, ml.y);
        const float a0 = expf(m_a - Ma), a1 = expf(ml.x - Ma), b0 = expf(m_b - Mb), b1 = expf(ml.y - Mb);
        l_a = l_a * a0 + ml.z * a1;
        l_b = l_b * b0 + ml.w * b1;
        m_a = Ma;
        m_b = Mb;
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const float4 u = *reinterpret_cast<const float4 *>(xch + 4 * j);
            o[j][0] = o[j][0] * a0 + u.x * a1;
            o[j][1] = o[j][1] * a0 + u.y * a1;
            o[j][2] = o[j][2] * b0 + u.z * b1;
            o[j][3] = o[j][3] * b0 + u.w * b1;
        }
    }
    // partial states, as attn_partial_kernel: o_part[split][row][head][d], ml_part = (m, l)
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int qi = half ? qb : qa;
        if (qi >= nqv) continue;
        const int gq = qv0 + qi, r = gq / G, h = hk * G + gq % G;
        const size_t base = ((size_t)split * m + r) * n_q + h;
        float *op = o_part + base * kHD;
#pragma unroll
        for (int j = 0; j < 16; j++)
            *reinterpret_cast<float2 *>(op + 8 * j + 2 * t) = make_float2(o[j][2 * half], o[j][2 * half + 1]);
        if (t == 0) ml_part[base] = half ? make_float2(m_b, l_b) : make_float2(m_a, l_a);
    }
}


// out[r][h][d] = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s  (0 if no key visible),
// merged in one pass with a running maximum so each split's loads are
// independent of the others.
__global__ void attn_combine_kernel(const float *__restrict__ o_part, const float2 *__restrict__ ml_part,
                                    float *__restrict__ out, int m, int n_q, int splits) {
    const int rh = blockIdx.x;  // r * n_q + h
    const int d = threadIdx.x;  // kHD threads
    const size_t stride = (size_t)m * n_q;
    float M = kNegInit, L = 0.f, O = 0.f;
#pragma unroll 8
    for (int s = 0; s < splits; s++) {
        const float2 ml = ml_part[s * stride + rh];
        const float o = o_part[(s * stride + rh) * kHD + d];
        if (ml.y == 0.f) continue;
        const float Mn = fmaxf(M, ml.x);
        const float a = expf(M - Mn), b = expf(ml.x - Mn);
        L = L * a + ml.y * b;
        O = O * a + o * b;
        M = Mn;
    }
    out[(size_t)rh * kHD + d] = L > 0.f ? O / L : 0.f;
}

}  // namespace

extern "C" int lc_mha_attn(lc_ctx *ctx, const float *q, const float *k, const float *v, float *out, uint32_t m,
                           uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t seq_len, float scale,
                           uint32_t q_pos0, uint32_t causal) {
    LC_REQUIRE(ctx, LC_ERR_INVALID, "lc_mha_attn: null ctx");
    int s = lc_use_device(ctx);
    if (s) return s;
    if (m == 0 || n_q_heads == 0) return LC_OK;
    LC_REQUIRE(q && out && (seq_len == 0 || (k && v)), LC_ERR_INVALID, "lc_mha_attn: null pointer");
    LC_REQUIRE((((uintptr_t)q | (uintptr_t)(seq_len ? k : q) | (uintptr_t)(seq_len ? v : q)) & 15) == 0,
               LC_ERR_INVALID, "lc_mha_attn: q, k and v must be 16-byte aligned");
    LC_REQUIRE(head_dim == kHD, LC_ERR_UNSUPPORTED, "lc_mha_attn: head_dim %u (this kernel runs 128)", head_dim);
    LC_REQUIRE(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0, LC_ERR_UNSUPPORTED,
               "lc_mha_attn: n_q_heads %u must be a multiple of n_kv_heads %u", n_q_heads, n_kv_heads);
    const int G = n_q_heads / n_kv_heads;
    const int qv_total = (int)m * G;
    const int chunks = (qv_total + kQV - 1) / kQV;
    // about one CTA per SM (each stages its query vectors once, so a split of
    // several key tiles amortises that), at least one tile of keys per split
    int splits = 1;
    if (seq_len > 0) {
        const int want = std::max(1, ctx->num_sms / std::max(1, (int)n_kv_heads * chunks));
        const int max_splits = (int)((seq_len + kTK - 1) / kTK);
        splits = std::min(want, max_splits);
    }
    // the tensor-core kernel (default) works in tiles of 64 keys, the f32 one in 32
    const bool tc = ctx->gemm_tc != 0;
    const int tile = tc ? kTcKeys : kTK;
    int kps = seq_len > 0 ? (int)((seq_len + splits - 1) / splits) : 1;
    kps = ((kps + tile - 1) / tile) * tile;
    splits = seq_len > 0 ? (int)((seq_len + kps - 1) / kps) : 1;
    const size_t o_bytes = (size_t)splits * m * n_q_heads * kHD * 4;
    const size_t ml_bytes = (size_t)splits * m * n_q_heads * 8;
    char *scr = (char *)lc_scratch(ctx, LC_SCRATCH_ATTN, o_bytes + ml_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    float *o_part = (float *)scr;
    float2 *ml_part = (float2 *)(scr + ((o_bytes + 255) & ~(size_t)255));
    dim3 grid(n_kv_heads, splits, chunks);
    if (tc) {
        const size_t smem =
            (size_t)(kQV * kTcQS + 2 * kTcKeys * kTcQS + 2 * kTcKeys * kTcVS + kTcWarps * 16 * kTcPS) * 4;
        s = lc_set_smem_attr((const void *)attn_tc_kernel, smem);
        if (s) return s;
        attn_tc_kernel<<<grid, kTcWarps * 32, smem, ctx->stream>>>(q, seq_len ? k : q, seq_len ? v : q, o_part,
                                                                   ml_part, (int)m, (int)n_q_heads, (int)n_kv_heads,
                                                                   (int)seq_len, kps, scale, q_pos0, (int)causal);
    } else {
        const size_t smem = (size_t)(kQV * kQS + 2 * kTK * kKS + 2 * kTK * kHD + kQV * kPS) * 4;
        s = lc_set_smem_attr((const void *)attn_partial_kernel, smem);
        if (s) return s;
        attn_partial_kernel<<<grid, kThreads, smem, ctx->stream>>>(q, seq_len ? k : q, seq_len ? v : q, o_part,
                                                                   ml_part, (int)m, (int)n_q_heads, (int)n_kv_heads,
                                                                   (int)seq_len, kps, scale, q_pos0, (int)causal);
    }
    attn_combine_kernel<<<m * n_q_heads, kHD, 0, ctx->stream>>>(o_part, ml_part, out, (int)m, (int)n_q_heads,
                                                                 splits);
    return lc_after_launch(ctx, "lc_mha_attn");
}
