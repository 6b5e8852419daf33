/*
 * laguna_oracle.c -- CPU restatement of laguna-raw's quantized projection path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * Nothing in the product library links or calls this file.
 *
 * Compiled with -O3 -ffp-contract=off so every float expression rounds in the
 * order the reference writes it.  Work is split over output rows with OpenMP;
 * each row is computed by one thread in the reference's sequential order, so
 * results do not depend on the thread count.
 */
#include "laguna_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void lco_set_threads(int n) { g_threads = n; }

int lco_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

#define LCO_PARALLEL_FOR _Pragma("omp parallel for schedule(static) num_threads(lco_get_threads())")

static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* kernels/proj_q8_0.comp:27-45 half_to_f32 (identical to proj_q4k.comp
 * fp16_to_f32 and src/dflash.rs:314-329).  Subnormals keep the implicit one. */
float lco_half_to_f32_ref(uint16_t h_bits) {
    uint32_t sign = h_bits & 0x8000u;
    uint32_t e = (h_bits >> 10) & 0x1Fu;
    uint32_t mant = h_bits & 0x3FFu;
    if (e == 0u) {
        if (mant == 0u) return bits_f32(sign << 16);
        return bits_f32((sign << 16) | ((1u - 15u + 127u) << 23) | (mant << 13));
    }
    if (e == 31u) {
        if (mant == 0u) return bits_f32((sign << 16) | 0x7F800000u);
        return bits_f32((sign << 16) | 0x7F800000u | (mant << 13));
    }
    return bits_f32((sign << 16) | ((e - 15u + 127u) << 23) | (mant << 13));
}

/* src/dflash.rs:437-462: sign * 2^(e-15) * (1 + m/1024), subnormals
 * sign * 2^-14 * (m/1024), NaN -> f32::NAN (0x7FC00000). */
float lco_half_to_f32_ieee(uint16_t h_bits) {
    float sign = (h_bits & 0x8000u) ? -1.0f : 1.0f;
    int e = (h_bits >> 10) & 0x1F;
    float mant = (float)(h_bits & 0x3FFu);
    if (e == 0) {
        if (mant == 0.0f) return sign * 0.0f;
        return sign * ldexpf(1.0f, -14) * (mant / 1024.0f);
    }
    if (e == 31) {
        if (mant == 0.0f) return sign * INFINITY;
        return bits_f32(0x7FC00000u);
    }
    return sign * ldexpf(1.0f, e - 15) * (1.0f + mant / 1024.0f);
}

static inline uint16_t rd16(const uint8_t *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}

void lco_dequant_to_f32(const uint8_t *data, size_t nbytes, int dtype,
                        size_t n, float *out) {
    switch (dtype) {
    case LCO_F32: /* src/dflash.rs:333-350 */
        for (size_t i = 0; i < n; i++) {
            size_t off = i * 4;
            if (off + 4 <= nbytes) {
                uint32_t b = (uint32_t)data[off] | ((uint32_t)data[off + 1] << 8) |
                             ((uint32_t)data[off + 2] << 16) | ((uint32_t)data[off + 3] << 24);
                out[i] = bits_f32(b);
            } else {
                out[i] = 0.0f;
            }
        }
        return;
    case LCO_BF16: /* src/dflash.rs:351-378: decoded with the f16 layout */
        for (size_t i = 0; i < n; i++) {
            size_t off = i * 2;
            out[i] = (off + 2 <= nbytes) ? lco_half_to_f32_ref(rd16(data + off)) : 0.0f;
        }
        return;
    case LCO_Q8_0: { /* src/dflash.rs:379-397 */
        for (size_t i = 0; i < n; i++) out[i] = 0.0f;
        size_t nblk = (n + 31) / 32;
        for (size_t b = 0; b < nblk; b++) {
            size_t off = b * 34;
            if (off + 34 > nbytes) break;
            float d = lco_half_to_f32_ref(rd16(data + off));
            size_t start = b * 32, end = start + 32 < n ? start + 32 : n;
            for (size_t i = 0; i < end - start; i++) {
                float q = (float)(int8_t)data[off + 2 + i];
                out[start + i] = q * d;
            }
        }
        return;
    }
    case LCO_Q4_K: { /* src/dflash.rs:398-436 (a bf16 d/k4/signs + 3-bit layout,
                      * not GGUF Q4_K; restated as written) */
        for (size_t i = 0; i < n; i++) out[i] = 0.0f;
        size_t nblk = (n + 255) / 256;
        for (size_t b = 0; b < nblk; b++) {
            size_t base = b * 144;
            if (base + 144 > nbytes) break;
            float d = bits_f32((uint32_t)rd16(data + base) << 16);
            float k4 = bits_f32((uint32_t)rd16(data + base + 2) << 16);
            float signs = bits_f32((uint32_t)rd16(data + base + 4) << 16);
            size_t start = b * 256, end = start + 256 < n ? start + 256 : n;
            for (size_t i = 0; i < end - start; i++) {
                size_t bi = base + 6 + i / 2;
                if (bi >= base + 144) break;
                uint8_t byte = data[bi];
                uint32_t q = (i % 2 == 0) ? ((byte >> 4) & 7u) : (byte & 7u);
                float s = signs < 0.0f ? -1.0f : 1.0f;
                out[start + i] = (float)q * d + s * k4;
            }
        }
        return;
    }
    case LCO_F16: /* src/dflash.rs:437-462 */
        for (size_t i = 0; i < n; i++) {
            size_t off = i * 2;
            out[i] = (off + 2 <= nbytes) ? lco_half_to_f32_ieee(rd16(data + off)) : 0.0f;
        }
        return;
    default: /* src/dflash.rs:463 */
        for (size_t i = 0; i < n; i++) out[i] = 0.0f;
        return;
    }
}

/* proj_q8_0.comp:54-63: blk = lin/32 at 34 B, f16 d then int8 q[lin%32]. */
float lco_q8_0_weight(const uint8_t *w, uint32_t lin) {
    uint32_t blk = lin / 32u, elm = lin % 32u, off = blk * 34u;
    float d = lco_half_to_f32_ref(rd16(w + off));
    int q = (int)(int8_t)w[off + 2u + elm];
    return (float)q * d;
}

/* proj_q4k.comp:46-58 get_scale_min_k4. */
static inline void scale_min_k4(uint32_t j, const uint8_t *q, uint32_t *d, uint32_t *m) {
    uint32_t b0 = q[j];
    uint32_t b4 = q[4u + (j & 3u)];
    uint32_t bp = q[8u + (j & 3u)];
    if (j < 4u) {
        *d = b0 & 63u;
        *m = b4 & 63u;
    } else {
        uint32_t d_hi = q[j - 4u];
        *d = (bp & 15u) | ((d_hi >> 6) << 4);
        *m = (bp >> 4) | ((b4 >> 6) << 4);
    }
}

/* proj_q4k.comp:67-87: 144-B super-block, d/dmin f16 at 0/2, scales at 4,
 * nibbles at 16 + (e/64)*32 + e%32 (low nibble when e%64 < 32). */
float lco_q4k_weight(const uint8_t *w, uint32_t lin) {
    uint32_t blk = lin / 256u, elm = lin % 256u;
    const uint8_t *b = w + (size_t)blk * 144u;
    float d = lco_half_to_f32_ref(rd16(b));
    float dmin = lco_half_to_f32_ref(rd16(b + 2));
    uint32_t sb = elm / 32u, g64 = elm / 64u, w64 = elm % 64u;
    uint8_t qb = b[16u + g64 * 32u + (w64 % 32u)];
    float q = (float)((w64 < 32u) ? (qb & 0xFu) : ((qb >> 4) & 0xFu));
    uint32_t sc, mn;
    scale_min_k4(sb, b + 4, &sc, &mn);
    return d * (float)sc * q - dmin * (float)mn;
}

void lco_dequant_shader(const uint8_t *w, int dtype, size_t n, float *out) {
    LCO_PARALLEL_FOR
    for (size_t i = 0; i < n; i++) {
        if (dtype == LCO_Q8_0)
            out[i] = lco_q8_0_weight(w, (uint32_t)i);
        else if (dtype == LCO_Q4_K)
            out[i] = lco_q4k_weight(w, (uint32_t)i);
        else if (dtype == LCO_F16)
            out[i] = lco_half_to_f32_ref(rd16(w + 2 * i));
        else if (dtype == LCO_F32)
            out[i] = bits_f32((uint32_t)w[4 * i] | ((uint32_t)w[4 * i + 1] << 8) |
                              ((uint32_t)w[4 * i + 2] << 16) | ((uint32_t)w[4 * i + 3] << 24));
        else
            out[i] = 0.0f;
    }
}

/* ------------------------------------------------------------------------ */

void lco_proj_f32(const float *x, const float *w, float *c, uint32_t k,
                  uint32_t n, uint32_t row_major) {
    LCO_PARALLEL_FOR
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float acc = 0.0f;
        for (uint32_t j = 0; j < k; j++) {
            size_t idx = row_major ? (size_t)j * n + (size_t)i : (size_t)j + (size_t)i * k;
            acc += x[j] * w[idx];
        }
        c[i] = acc;
    }
}

void lco_proj_q8_0(const float *x, const uint8_t *w, float *c, uint32_t k,
                   uint32_t n) {
    LCO_PARALLEL_FOR
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float acc = 0.0f;
        for (uint32_t j = 0; j < k; j++) {
            uint32_t lin = (uint32_t)i * k + j;
            acc += x[j] * lco_q8_0_weight(w, lin);
        }
        c[i] = acc;
    }
}

void lco_proj_q4k(const float *x, const uint8_t *w, float *c, uint32_t k,
                  uint32_t n, uint32_t expert_offset) {
    LCO_PARALLEL_FOR
    for (int64_t i = 0; i < (int64_t)n; i++) {
        float acc = 0.0f;
        for (uint32_t j = 0; j < k; j++) {
            uint32_t lin = expert_offset + (uint32_t)i * k + j;
            acc += x[j] * lco_q4k_weight(w, lin);
        }
        c[i] = acc;
    }
}

void lco_proj_f32_m(const float *x, const float *w, float *c, uint32_t m,
                    uint32_t k, uint32_t n, uint32_t row_major) {
    for (uint32_t r = 0; r < m; r++)
        lco_proj_f32(x + (size_t)r * k, w, c + (size_t)r * n, k, n, row_major);
}

void lco_proj_q8_0_m(const float *x, const uint8_t *w, float *c, uint32_t m,
                     uint32_t k, uint32_t n) {
    for (uint32_t r = 0; r < m; r++)
        lco_proj_q8_0(x + (size_t)r * k, w, c + (size_t)r * n, k, n);
}

void lco_proj_q4k_m(const float *x, const uint8_t *w, float *c, uint32_t m,
                    uint32_t k, uint32_t n, uint32_t expert_offset) {
    for (uint32_t r = 0; r < m; r++)
        lco_proj_q4k(x + (size_t)r * k, w, c + (size_t)r * n, k, n, expert_offset);
}

/* ------------------------------------------------------------------------ */

void lco_rmsnorm(const float *x, const float *w, float *y, uint32_t m,
                 uint32_t n, float eps) {
    for (uint32_t r = 0; r < m; r++) {
        const float *xr = x + (size_t)r * n;
        float *yr = y + (size_t)r * n;
        float mean_sq = 0.0f;
        for (uint32_t j = 0; j < n; j++) {
            float v = xr[j];
            mean_sq += v * v;
        }
        mean_sq /= (float)n;
        float rms = 1.0f / sqrtf(mean_sq + eps);
        for (uint32_t i = 0; i < n; i++) yr[i] = xr[i] * w[i] * rms;
    }
}

void lco_qk_norm_rope(const float *x, const float *w, const float *freq,
                      float *y, uint32_t m, uint32_t n_heads,
                      uint32_t head_dim, uint32_t rope_dim, float eps,
                      const uint32_t *pos) {
    uint32_t total = n_heads * head_dim;
    for (uint32_t r = 0; r < m; r++) {
        const float *xr = x + (size_t)r * total;
        float *yr = y + (size_t)r * total;
        uint32_t p = pos[r];
        for (uint32_t i = 0; i < total; i++) {
            uint32_t head = i / head_dim, dim = i % head_dim, base = head * head_dim;
            float mean_sq = 0.0f;
            for (uint32_t d = 0; d < head_dim; d++) mean_sq += xr[base + d] * xr[base + d];
            mean_sq /= (float)head_dim;
            float rms = 1.0f / sqrtf(mean_sq + eps);
            float normed = xr[i] * w[dim] * rms;
            if (dim >= rope_dim) {
                yr[i] = normed;
            } else {
                uint32_t hf = dim % (rope_dim / 2u);
                float angle = freq[hf] * (float)p;
                float cf = cosf(angle), sf = sinf(angle);
                if (dim < rope_dim / 2u) {
                    uint32_t pi = i + head_dim / 2u;
                    float pn = xr[pi] * w[pi % head_dim] * rms;
                    yr[i] = normed * cf - pn * sf;
                } else {
                    uint32_t pi = i - head_dim / 2u;
                    float pn = xr[pi] * w[pi % head_dim] * rms;
                    yr[i] = normed * cf + pn * sf;
                }
            }
        }
    }
}

void lco_activation(const float *gate, const float *up, float *h, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) {
        float g = gate[i];
        float s = g * (1.0f / (1.0f + expf(-g)));
        h[i] = s * up[i];
    }
}

void lco_add(const float *a, const float *b, float *c, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) c[i] = a[i] + b[i];
}

void lco_gate_mul(const float *v, const float *gate, float *out, uint32_t n_hd,
                  uint32_t head_dim) {
    for (uint32_t i = 0; i < n_hd; i++) out[i] = v[i] * gate[i / head_dim];
}

void lco_softplus(const float *g, float *out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = g[i] > 20.0f ? g[i] : logf(1.0f + expf(g[i]));
}

void lco_mha_attn(const float *Q, const float *K, const float *V, float *out,
                  uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim,
                  uint32_t seq_len, float scale, uint32_t q_pos,
                  uint32_t causal) {
    uint32_t total = n_q_heads * head_dim;
    for (uint32_t d = 0; d < total; d++) {
        uint32_t h = d / head_dim, dim = d % head_dim;
        uint32_t kv_h = h * n_kv_heads / n_q_heads;
        uint32_t q_base = h * head_dim;
        float m = -1e30f, l = 0.0f, acc = 0.0f;
        for (uint32_t p = 0; p < seq_len; p++) {
            if (causal != 0u && p > q_pos) break;
            size_t k_base = (size_t)p * n_kv_heads * head_dim + (size_t)kv_h * head_dim;
            float dot = 0.0f;
            for (uint32_t j = 0; j < head_dim; j++) dot += Q[q_base + j] * K[k_base + j];
            float score = dot * scale;
            float m_new = m > score ? m : score;
            float corr = expf(m - m_new);
            float wgt = expf(score - m_new);
            l = l * corr + wgt;
            acc = acc * corr + wgt * V[k_base + dim];
            m = m_new;
        }
        out[d] = (l > 0.0f) ? (acc / l) : 0.0f;
    }
}

void lco_enc_aux_norm(const float *x, const float *w, float *y,
                      uint32_t n_feat, uint32_t n_aux, uint32_t n_tokens,
                      float eps) {
    size_t total = (size_t)n_feat * n_aux * n_tokens;
    for (size_t idx = 0; idx < total; idx++) {
        size_t tok = idx / ((size_t)n_feat * n_aux);
        size_t aux = (idx % ((size_t)n_feat * n_aux)) / n_feat;
        size_t feat = idx % n_feat;
        size_t base = (aux + tok * n_aux) * n_feat;
        float mean_sq = 0.0f;
        for (uint32_t i = 0; i < n_feat; i++) {
            float v = x[base + i];
            mean_sq += v * v;
        }
        mean_sq /= (float)n_feat;
        float rms = 1.0f / sqrtf(mean_sq + eps);
        y[idx] = x[idx] * rms * w[feat + aux * n_feat];
    }
}

void lco_rope_freq(float *freq, uint32_t rope_dim, float base) {
    for (uint32_t i = 0; i < rope_dim / 2; i++)
        freq[i] = 1.0f / powf(base, (2.0f * (float)i) / (float)rope_dim);
}

size_t lco_argmax(const float *logits, size_t n) {
    if (n == 0) return 0;
    size_t best = 0;
    for (size_t i = 1; i < n; i++) {
        /* cmp::max_by(cur, new): keep cur only when cur > new (Greater);
         * Less, Equal and unordered (NaN -> Equal) all take the new one. */
        if (!(logits[best] > logits[i])) best = i;
    }
    return best;
}

void lco_gate_attn(const float *attn, const float *gate, float *out, uint32_t n_heads, uint32_t head_dim) {
    for (uint32_t i = 0; i < n_heads * head_dim; i++) {
        float g = logf(1.0f + expf(gate[i / head_dim]));
        out[i] = attn[i] * g;
    }
}

uint32_t lco_moe_select(const float *logits, const float *bias, uint32_t n_exp, uint32_t n_used, int norm,
                        float scale, int32_t *ids, float *scores) {
    /* sort_by(|a, b| b.0.partial_cmp(&a.0)) is stable: among equal selection
     * values the lower expert comes first.  Picking the best remaining expert
     * n_used times gives the same order. */
    uint32_t n_sel = n_used < n_exp ? n_used : n_exp;
    for (uint32_t s = 0; s < n_sel; s++) {
        int32_t best = -1;
        float best_v = 0.0f;
        for (uint32_t e = 0; e < n_exp; e++) {
            int taken = 0;
            for (uint32_t t = 0; t < s; t++) taken |= ids[t] == (int32_t)e;
            if (taken) continue;
            float p = 1.0f / (1.0f + expf(-logits[e]));
            float v = p + bias[e];
            if (best < 0 || v > best_v) best = (int32_t)e, best_v = v;
        }
        ids[s] = best;
        scores[s] = 1.0f / (1.0f + expf(-logits[best]));
    }
    if (norm) {
        float sum = 0.0f;
        for (uint32_t s = 0; s < n_sel; s++) sum += scores[s];
        float denom = sum > 6.103515625e-5f ? sum : 6.103515625e-5f;
        for (uint32_t s = 0; s < n_sel; s++) scores[s] /= denom;
    }
    if (scale != 0.0f && scale != 1.0f)
        for (uint32_t s = 0; s < n_sel; s++) scores[s] *= scale;
    return n_sel;
}

float lco_moe_l2_scale(const float *h, uint32_t n, float *out) {
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; i++) sum += h[i] * h[i];
    float col = sqrtf(sum);
    if (col < 1e-8f) col = 1e-8f;
    if (col > 1e30f) col = 1e30f;
    for (uint32_t i = 0; i < n; i++) out[i] = h[i] * 32768.0f / col;
    return col;
}

/* keep f32_bits referenced for debug builds */
uint32_t lco__f32_bits(float f) { return f32_bits(f); }
