// lc_attn.cu -- GQA attention of kernels/mha_attn.comp:31-72 for a block of
// query rows.  attn_tc5_kernel (tcgen05, f16 hi / lo operands) is the default;
// attn_partial_kernel (f32 FMA) runs with LC_GEMM_TC=0.
//
// The reference runs one invocation per (head, dim) and walks all positions
// with an online softmax (m starts at -1e30, causal break at p > q_pos, output
// 0 when no key is visible).  Here every key/value row of one KV head is
// staged in shared memory once and reused by all query heads of the group and
// all query rows (up to 64 query vectors per CTA): the CTA grid is
// (kv head, key split, query chunk) and a second kernel merges the split
// partial softmax states.  The f32 kernel computes in fp32 throughout; the
// tcgen05 kernel multiplies f16 hi / lo parts of the fp32 values (about 22
// significant bits) with fp32 accumulation and keeps the softmax in fp32.
#include <algorithm>

#include "lc_internal.cuh"
#include "lc_sm100.cuh"

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

// ---- tcgen05 form (head_dim 128) --------------------------------------------
//
// One CTA per (KV head, 128-key tile, 64 query vectors).  Q, K and V go to
// shared memory as f16 hi / lo planes (x * 2^e = hi + lo, e per query row, per
// key row and per V tile, so no value leaves the f16 range and about 22
// significant bits survive), K-major with the 128-byte swizzle the UMMA
// descriptors read.  V is stored transposed (row = head dim, K = key) so both
// products read K-major operands:
//   S = Q K^T  (M 128, N 128 keys, K 128 dims):  Ql Kh + Qh Kl + Qh Kh
//   O = P V    (M 128, N 128 dims, K 128 keys), P in tensor memory: Pl Vh + Ph Vl + Ph Vh
// The MMAs run M = 128 over the 64 query rows: A rows 64..127 read whatever
// follows the Q rows of a box, and their S / P / O lanes are never used.  A
// query row's softmax runs in the two warps that share its TMEM lane (one per
// 64-key half); the CTA writes the unnormalised (O, m, l) of its key tile for
// attn_combine_kernel.  TMEM columns: S 0..127, P 128..255 (hi 128..191, lo
// 192..255), O 256..383.
constexpr int kAtRows = 64, kAtKeys = 128;
constexpr int kAtThreads = 256;
constexpr uint32_t kAtQBox = 64 * 128;   // 64 rows x 64 f16 (one 128-byte swizzle span)
constexpr uint32_t kAtBox = 128 * 128;   // 128 rows x 64 f16
constexpr uint32_t kAtQh = 0, kAtQl = 2 * kAtQBox;                          // Q: 64 rows x 128 dims
constexpr uint32_t kAtKh = 4 * kAtQBox, kAtKl = kAtKh + 2 * kAtBox;          // K: 128 keys x 128 dims
constexpr uint32_t kAtVh = kAtKl + 2 * kAtBox, kAtVl = kAtVh + 2 * kAtBox;   // V^T: 128 dims x 128 keys
constexpr uint32_t kAtRaw = kAtVl + 2 * kAtBox;                              // raw f32 Q rows (32 KB)
constexpr uint32_t kAtInvQ = kAtRaw + kAtRows * 512, kAtInvK = kAtInvQ + 256, kAtRed = kAtInvK + 512,
                   kAtMisc = kAtRed + 1024;
constexpr uint32_t kAtSmem = kAtMisc + 64 + 1024;  // + slack to 1024-align the base
constexpr uint32_t kAtColS = 0, kAtColP = 128, kAtColO = 256, kAtTmemCols = 512;

// Byte offset of f16 element (row, k) in an operand plane of two boxes of 64
// K-elements (box_bytes apart): rows 128 bytes apart in 8-row groups of 1024
// bytes, 16-byte chunks XOR-ed with the row within its group (the 128-byte
// swizzle of the UMMA descriptor).
__device__ __forceinline__ uint32_t at_off(int row, int k, uint32_t box_bytes) {
    const uint32_t byte = (uint32_t)(k & 63) * 2;
    return (uint32_t)(k >> 6) * box_bytes + (uint32_t)(row >> 3) * 1024 + (uint32_t)(row & 7) * 128 +
           ((((byte >> 4) ^ (uint32_t)(row & 7)) << 4) | (byte & 15));
}

// hi / lo f16 pairs of (a, b): a ~ hi.x + lo.x, b ~ hi.y + lo.y.
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Global load issued where it stands (a volatile asm keeps its place among the
// cp.async staging copies): the V tile's latency overlaps theirs.
__device__ __forceinline__ float ldg_stream(const float *p) {
    float x;
    asm volatile("ld.global.nc.f32 %0, [%1];\n" : "=f"(x) : "l"(p));
    return x;
}

__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t a, uint32_t b) {
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};\n" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t a) {
    asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(addr), "r"(a) : "memory");
}

// Rows [0, nrows) of a raw f32 [rows][128] block in shared memory -> hi / lo
// planes: warp w converts rows w, w + 8, ..., lane l dims 4l..4l+3, eight rows
// per pass.  inv[row] = 1 / scale of the row.
__device__ __forceinline__ void at_rows_to_planes(const unsigned char *raw, int nrows, int warp, int lane,
                                                  uint32_t hi_plane, uint32_t lo_plane, uint32_t box_bytes,
                                                  float *inv) {
#pragma unroll 1
    for (int r0 = warp; r0 < nrows; r0 += 64) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int row = min(r0 + 8 * u, 127);  // rows past nrows: loaded, not used
            x[u] = *reinterpret_cast<const float4 *>(raw + row * 512 + 16 * lane);
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int row = r0 + 8 * u;
            float mx = fmaxf(fmaxf(fabsf(x[u].x), fabsf(x[u].y)), fmaxf(fabsf(x[u].z), fabsf(x[u].w)));
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (row >= nrows) continue;
            float s, iv;
            act_scale(mx, s, iv);
            if (lane == 0) inv[row] = iv;
            uint32_t h0, l0, h1, l1;
            split2(x[u].x * s, x[u].y * s, h0, l0);
            split2(x[u].z * s, x[u].w * s, h1, l1);
            const uint32_t off = at_off(row, 4 * lane, box_bytes);
            st_shared_v2(hi_plane + off, h0, h1);
            st_shared_v2(lo_plane + off, l0, l1);
        }
    }
}

__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc5_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                    float *__restrict__ o_part, float2 *__restrict__ ml_part, int m, int n_q, int n_kv, int seq_len,
                    float scale, uint32_t q_pos0, int causal, unsigned *__restrict__ status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_addr(smem);
    float *inv_q = reinterpret_cast<float *>(smem + kAtInvQ), *inv_k = reinterpret_cast<float *>(smem + kAtInvK);
    float *red_m = reinterpret_cast<float *>(smem + kAtRed), *red_l = red_m + 2 * kAtRows;
    unsigned *vmax = reinterpret_cast<unsigned *>(smem + kAtMisc);
    uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + kAtMisc + 8), *bar_o = bar_s + 1;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + kAtMisc + 24);
    const int hk = blockIdx.x, split = blockIdx.y, chunk = blockIdx.z;
    const int G = n_q / n_kv, qv_total = m * G, qv0 = chunk * kAtRows;
    const int nqv = min(kAtRows, qv_total - qv0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p_begin = split * kAtKeys, p_end = min(seq_len, p_begin + kAtKeys), nk = max(0, p_end - p_begin);
    const int ldq = n_q * 128, ldk = n_kv * 128;

    griddep_launch_dependents();  // the combine kernel may be scheduled now
    if (threadIdx.x == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        *vmax = 0u;
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                     "r"(kAtTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
        tc_fence_before();
    }
    // V rows into registers (loads issued here, in program order): warp w takes
    // key pairs (2p, 2p + 1), p = w + 8 i, lane l dims l + 32 c
    float vv[8][2][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int key = 2 * (warp + 8 * i) + e;
#pragma unroll
            for (int c = 0; c < 4; c++)
                vv[i][e][c] = key < nk ? ldg_stream(v + (size_t)(p_begin + key) * ldk + hk * 128 + lane + 32 * c) : 0.f;
        }
    // raw Q and K rows by cp.async (Q -> the staging space, K -> the V planes'
    // space, converted before V is written there)
#pragma unroll 1
    for (int idx = threadIdx.x; idx < kAtKeys * 32; idx += kAtThreads) {
        const int row = idx >> 5, ch = idx & 31;
        if (row < nqv) {
            const int gq = qv0 + row, r = gq / G, h = hk * G + gq % G;
            cp_async16(smem + kAtRaw + row * 512 + 16 * ch, q + (size_t)r * ldq + h * 128 + 4 * ch, 16u);
        }
        if (row < nk)
            cp_async16(smem + kAtVh + row * 512 + 16 * ch, k + (size_t)(p_begin + row) * ldk + hk * 128 + 4 * ch, 16u);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    // Q and K planes, and the V tile's maximum, in one phase
    at_rows_to_planes(smem + kAtRaw, nqv, warp, lane, sbase + kAtQh, sbase + kAtQl, kAtQBox, inv_q);
    at_rows_to_planes(smem + kAtVh, nk, warp, lane, sbase + kAtKh, sbase + kAtKl, kAtBox, inv_k);
    {
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int e = 0; e < 2; e++)
#pragma unroll
                for (int c = 0; c < 4; c++) mx = fmaxf(mx, fabsf(vv[i][e][c]));
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) atomicMax(vmax, __float_as_uint(mx));  // non-negative floats order as integers
    }
    fence_proxy_async_smem();  // generic-proxy stores -> the tensor cores' reads
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    constexpr uint32_t idesc = umma_idesc_f16(128, 128);
    if (threadIdx.x == 0) {  // S = Q K^T, small products first
        const uint64_t qh = umma_desc_sw128(sbase + kAtQh), ql = umma_desc_sw128(sbase + kAtQl);
        const uint64_t kh = umma_desc_sw128(sbase + kAtKh), kl = umma_desc_sw128(sbase + kAtKl);
        const uint32_t ds = tbase + kAtColS;
#pragma unroll
        for (int t = 0; t < 3; t++) {
            const uint64_t qa = t == 0 ? ql : qh, kb = t == 1 ? kl : kh;
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                const uint64_t qo = ((kk >> 2) * kAtQBox + (kk & 3) * 32) >> 4;
                const uint64_t ko = ((kk >> 2) * kAtBox + (kk & 3) * 32) >> 4;
                umma_f16_ss(ds, qa + qo, kb + ko, idesc, (t | kk) ? 1u : 0u);
            }
        }
        umma_commit(bar_s);
    }
    // V, transposed, into the V planes (their space held raw K, converted
    // above): one scale for the tile, f16x2 of key pairs (2p, 2p + 1) per dim
    float v_iv;
    {
        float s;
        act_scale(__uint_as_float(*vmax), s, v_iv);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int k0 = 2 * (warp + 8 * i);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t hi, lo;
                split2(vv[i][0][c] * s, vv[i][1][c] * s, hi, lo);
                const uint32_t off = at_off(lane + 32 * c, k0, kAtBox);
                st_shared_u32(sbase + kAtVh + off, hi);
                st_shared_u32(sbase + kAtVl + off, lo);
            }
        }
    }
    fence_proxy_async_smem();
    // softmax: warps w and w + 4 (w = 0, 1) share query row 32 w + lane (its TMEM
    // lane) and take keys 64 (warp >> 2) .. +63; the halves exchange maxima and
    // sums through shared memory.  Scores are in log2 units (exp2).
    const bool sw = (warp & 3) < 2;
    const int srow = 32 * (warp & 3) + lane, shalf = warp >> 2;
    const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
    float sv[64];
    float tmax = kNegInit, row_m = kNegInit, row_l = 0.f;
    int klim = 0;
    if (sw) {
        const bool real = srow < nqv;
        const long long pos = (long long)q_pos0 + (qv0 + srow) / G;
        long long lim = real ? nk : 0;  // keys [0, lim) of the tile are visible to the row
        if (causal) lim = min(lim, max(0ll, pos - p_begin + 1));
        klim = (int)lim - 64 * shalf;
        const float fq = inv_q[srow] * (scale * 1.4426950408889634f);  // log2(e)
        if (!mbar_wait(bar_s, 0)) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float t[16];
            tmem_ld16(tbase + lanes + kAtColS + 64 * shalf + 16 * c, t);
#pragma unroll
            for (int j = 0; j < 16; j++) sv[16 * c + j] = t[j];
        }
        tmem_ld_wait();
        tmem_regs_ready(sv);
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
            const float4 ik = *reinterpret_cast<const float4 *>(inv_k + 64 * shalf + j);
            sv[j] *= ik.x * fq, sv[j + 1] *= ik.y * fq, sv[j + 2] *= ik.z * fq, sv[j + 3] *= ik.w * fq;
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (j + u < klim) tmax = fmaxf(tmax, sv[j + u]);
        }
        red_m[kAtRows * shalf + srow] = tmax;
    }
    named_barrier_sync(kAtThreads);
    if (sw) {
        tmax = fmaxf(tmax, red_m[kAtRows * (shalf ^ 1) + srow]);
        float lsum = 0.f;
#pragma unroll
        for (int c = 0; c < 2; c++) {  // 32 keys -> 16 columns of hi and 16 of lo
            uint32_t ph[16], pl[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int k0 = 32 * c + 2 * j;
                const float p0 = k0 < klim ? exp2f(sv[k0] - tmax) : 0.f;
                const float p1 = k0 + 1 < klim ? exp2f(sv[k0 + 1] - tmax) : 0.f;
                lsum += p0 + p1;
                split2(p0, p1, ph[j], pl[j]);
            }
            tmem_st16(tbase + lanes + kAtColP + 32 * shalf + 16 * c, ph);
            tmem_st16(tbase + lanes + kAtColP + 64 + 32 * shalf + 16 * c, pl);
        }
        red_l[kAtRows * shalf + srow] = lsum;
        row_m = tmax == kNegInit ? kNegInit : tmax * 0.6931471805599453f;  // natural-log units
        row_l = lsum;
        tmem_st_wait();
        tc_fence_before();
    }
    __syncthreads();  // V planes and P complete
    tc_fence_after();
    if (threadIdx.x == 0) {  // O = P V
        const uint64_t vh = umma_desc_sw128(sbase + kAtVh), vl = umma_desc_sw128(sbase + kAtVl);
        const uint32_t d_o = tbase + kAtColO, pa = tbase + kAtColP;
#pragma unroll
        for (int t = 0; t < 3; t++) {
            const uint32_t pc = t == 0 ? pa + 64 : pa;
            const uint64_t vb = t == 1 ? vl : vh;
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                const uint64_t vo = ((kk >> 2) * kAtBox + (kk & 3) * 32) >> 4;
                umma_f16_ts(d_o, pc + 8 * kk, vb + vo, idesc, (t | kk) ? 1u : 0u);
            }
        }
        umma_commit(bar_o);
    }
    if (sw) {  // partial states: columns 64 shalf.. of the row's O
        if (!mbar_wait(bar_o, 0)) atomicOr(status, LC_DEV_WAIT_TIMEOUT);
        tc_fence_after();
        float o[64];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float t[16];
            tmem_ld16(tbase + lanes + kAtColO + 64 * shalf + 16 * c, t);
#pragma unroll
            for (int j = 0; j < 16; j++) o[16 * c + j] = t[j];
        }
        tmem_ld_wait();
        tmem_regs_ready(o);
        if (srow < nqv) {
            const int gq = qv0 + srow, r = gq / G, h = hk * G + gq % G;
            const size_t base = ((size_t)split * m + r) * n_q + h;
            float4 *op = reinterpret_cast<float4 *>(o_part + base * 128 + 64 * shalf);
#pragma unroll
            for (int j = 0; j < 16; j++)
                op[j] = make_float4(o[4 * j] * v_iv, o[4 * j + 1] * v_iv, o[4 * j + 2] * v_iv, o[4 * j + 3] * v_iv);
            if (shalf == 0) ml_part[base] = make_float2(row_m, row_l + red_l[kAtRows + srow]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(kAtTmemCols)
                     : "memory");
    }
}

// out[r][h][d] = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s (0 if no key is
// visible), M the largest m_s of the splits that saw a key.  One warp per
// (row, head), lane l owning dims 4l..4l+3; the split states are read
// lane-parallel (split s by lane s % 32) and M and the weights formed with
// shuffles, so every split's loads are independent of the others.  Launched as
// a programmatic dependent of the partial kernel.
constexpr int kCombineFast = 24;  // splits merged from registers (2064 keys: 17 tiles)

__global__ void attn_combine_kernel(const float *__restrict__ o_part, const float2 *__restrict__ ml_part,
                                    float *__restrict__ out, int m, int n_q, int splits) {
    griddep_wait();  // the partial states
    const int rh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (rh >= m * n_q) return;
    const size_t stride = (size_t)m * n_q;
    if (splits <= kCombineFast) {
        // every split's output row requested with the (m, l) states, before
        // the weights they wait for: one round trip to L2 instead of two
        float4 ov[kCombineFast];
#pragma unroll
        for (int j = 0; j < kCombineFast; j++)
            if (j < splits) ov[j] = *reinterpret_cast<const float4 *>(o_part + ((size_t)j * stride + rh) * kHD + 4 * lane);
        const float2 ml = lane < splits ? ml_part[lane * stride + rh] : make_float2(kNegInit, 0.f);
        float M = ml.y != 0.f ? ml.x : kNegInit;
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = (lane < splits && ml.y != 0.f) ? expf(ml.x - M) : 0.f;
        float L = lane < splits ? ml.y * w : 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kCombineFast; j++)
            if (j < splits) {
                const float b = __shfl_sync(0xffffffffu, w, j);
                O.x += ov[j].x * b, O.y += ov[j].y * b, O.z += ov[j].z * b, O.w += ov[j].w * b;
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        *reinterpret_cast<float4 *>(out + (size_t)rh * kHD + 4 * lane) =
            L > 0.f ? make_float4(O.x / L, O.y / L, O.z / L, O.w / L) : make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    float M = kNegInit;
    for (int s0 = 0; s0 < splits; s0 += 32)
        if (s0 + lane < splits) {
            const float2 ml = ml_part[(s0 + lane) * stride + rh];
            if (ml.y != 0.f) M = fmaxf(M, ml.x);
        }
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += 32) {
        float w = 0.f;
        if (s0 + lane < splits) {
            const float2 ml = ml_part[(s0 + lane) * stride + rh];
            w = ml.y != 0.f ? expf(ml.x - M) : 0.f;
            L += ml.y * w;
        }
        const int ns = min(32, splits - s0);
#pragma unroll 16
        for (int j = 0; j < ns; j++) {
            const float b = __shfl_sync(0xffffffffu, w, j);
            const float4 o = *reinterpret_cast<const float4 *>(o_part + ((s0 + j) * stride + rh) * kHD + 4 * lane);
            O.x += o.x * b, O.y += o.y * b, O.z += o.z * b, O.w += o.w * b;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    *reinterpret_cast<float4 *>(out + (size_t)rh * kHD + 4 * lane) =
        L > 0.f ? make_float4(O.x / L, O.y / L, O.z / L, O.w / L) : make_float4(0.f, 0.f, 0.f, 0.f);
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
    // the tcgen05 kernel (default) takes one tile of 128 keys per CTA; the f32
    // one about one CTA per SM, in tiles of 32 keys
    const bool tc = ctx->gemm_tc != 0;
    int kps = seq_len > 0 ? (int)((seq_len + splits - 1) / splits) : 1;
    kps = tc ? kAtKeys : ((kps + kTK - 1) / kTK) * kTK;
    splits = seq_len > 0 ? (int)((seq_len + kps - 1) / kps) : 1;
    const size_t o_bytes = (size_t)splits * m * n_q_heads * kHD * 4;
    const size_t ml_bytes = (size_t)splits * m * n_q_heads * 8;
    char *scr = (char *)lc_scratch(ctx, LC_SCRATCH_ATTN, o_bytes + ml_bytes + 256);
    if (!scr) return LC_ERR_OOM;
    float *o_part = (float *)scr;
    float2 *ml_part = (float2 *)(scr + ((o_bytes + 255) & ~(size_t)255));
    static_assert(kAtRows == kQV, "both kernels take chunks of the same query vectors");
    dim3 grid(n_kv_heads, splits, chunks);
    if (tc) {
        s = lc_set_smem_attr((const void *)attn_tc5_kernel, kAtSmem);
        if (s) return s;
        attn_tc5_kernel<<<grid, kAtThreads, kAtSmem, ctx->stream>>>(
            q, seq_len ? k : q, seq_len ? v : q, o_part, ml_part, (int)m, (int)n_q_heads, (int)n_kv_heads,
            (int)seq_len, scale, q_pos0, (int)causal, ctx->dev_status);
    } else {
        const size_t smem = (size_t)(kQV * kQS + 2 * kTK * kKS + 2 * kTK * kHD + kQV * kPS) * 4;
        s = lc_set_smem_attr((const void *)attn_partial_kernel, smem);
        if (s) return s;
        attn_partial_kernel<<<grid, kThreads, smem, ctx->stream>>>(q, seq_len ? k : q, seq_len ? v : q, o_part,
                                                                   ml_part, (int)m, (int)n_q_heads, (int)n_kv_heads,
                                                                   (int)seq_len, kps, scale, q_pos0, (int)causal);
    }
    // a programmatic dependent of the partial kernel: its CTAs are resident
    // before the partial states are complete and wait for them on the device
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((m * n_q_heads + 1) / 2);
    cfg.blockDim = dim3(64);
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LC_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_kernel, (const float *)o_part, (const float2 *)ml_part, out, (int)m,
                               (int)n_q_heads, splits));
    return lc_after_launch(ctx, "lc_mha_attn");
}
