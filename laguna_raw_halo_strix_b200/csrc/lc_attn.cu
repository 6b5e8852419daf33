// lc_attn.cu -- GQA attention of kernels/mha_attn.comp:31-72 for a block of
// query rows.
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
    int kps = seq_len > 0 ? (int)((seq_len + splits - 1) / splits) : 1;
    kps = ((kps + kTK - 1) / kTK) * kTK;
    splits = seq_len > 0 ? (int)((seq_len + kps - 1) / kps) : 1;
    const size_t o_bytes = (size_t)splits * m * n_q_heads * kHD * 4;
    const size_t ml_bytes = (size_t)splits * m * n_q_heads * 8;
    char *scr = (char *)lc_scratch(ctx, LC_SCRATCH_ATTN, o_bytes + ml_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    float *o_part = (float *)scr;
    float2 *ml_part = (float2 *)(scr + ((o_bytes + 255) & ~(size_t)255));
    const size_t smem = (size_t)(kQV * kQS + 2 * kTK * kKS + 2 * kTK * kHD + kQV * kPS) * 4;
    s = lc_set_smem_attr((const void *)attn_partial_kernel, smem);
    if (s) return s;
    dim3 grid(n_kv_heads, splits, chunks);
    attn_partial_kernel<<<grid, kThreads, smem, ctx->stream>>>(q, seq_len ? k : q, seq_len ? v : q, o_part, ml_part,
                                                               (int)m, (int)n_q_heads, (int)n_kv_heads, (int)seq_len,
                                                               kps, scale, q_pos0, (int)causal);
    attn_combine_kernel<<<m * n_q_heads, kHD, 0, ctx->stream>>>(o_part, ml_part, out, (int)m, (int)n_q_heads,
                                                                 splits);
    return lc_after_launch(ctx, "lc_mha_attn");
}
