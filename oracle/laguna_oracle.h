/*
 * laguna_oracle.h -- CPU restatement of laguna-raw's quantized projection path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * library (laguna_raw_halo_strix_b200/csrc) and the timed CPU baseline of
 * bench.py.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it.  The product path never calls into it.
 *
 * Every function restates one piece of the reference (auryn-macmillan/
 * laguna-raw-halo-strix); the citation is given per function as
 * `file:line` within that project.  Floating point follows the reference's
 * written operation order with no FMA contraction (-ffp-contract=off).
 *
 * Parity pinning: the half decoder and the Q8_0 / F32 dequant are pinned by the
 * reference's own unit tests (src/dflash.rs:1334-1365), the block and byte sizes
 * by src/gguf.rs:659-732, proj.comp by src/lib.rs:120-165, rmsnorm by
 * src/lib.rs:167-210.  The shader bodies (proj_q8_0.comp, proj_q4k.comp and the
 * interleaved shaders) are additionally pinned against the reference's GLSL
 * sources compiled for the CPU by oracle/build_ref.py (oracle/_ref/), and through
 * the committed fixtures in tests/golden/.
 */
#ifndef LAGUNA_ORACLE_H
#define LAGUNA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type ids (src/gguf.rs:45-88). */
enum {
    LCO_F32 = 0,
    LCO_F16 = 1,
    LCO_Q8_0 = 8,
    LCO_Q4_K = 12,
    LCO_BF16 = 30,
};

/* --- scalar decoders ---------------------------------------------------- */

/* f16 bits -> f32 exactly as kernels/proj_q8_0.comp:27-45 (= proj_q4k.comp
 * fp16_to_f32 and src/dflash.rs:314-329 bf16_to_f32): subnormal halves decode
 * to sign | 113<<23 | mant<<13, i.e. 2^-14 * (1 + mant/1024). */
float lco_half_to_f32_ref(uint16_t h);
/* IEEE f16 -> f32 as src/dflash.rs:437-462 (the F16 branch). */
float lco_half_to_f32_ieee(uint16_t h);

/* --- dequant ----------------------------------------------------------- */

/* src/dflash.rs:331-465 dequant_to_f32, all branches (F32, BF16 [decoded as
 * f16 with the subnormal quirk], Q8_0, the non-GGUF Q4_K layout of :398-436,
 * F16, anything else -> zeros).  nbytes bounds every read like the Rust code. */
void lco_dequant_to_f32(const uint8_t *data, size_t nbytes, int dtype,
                        size_t n_elements, float *out);

/* Per-element weight decode of the GPU shaders: element `lin` of a Q8_0 tensor
 * (proj_q8_0.comp:54-63) and of a GGUF Q4_K tensor (proj_q4k.comp:67-87). */
float lco_q8_0_weight(const uint8_t *w, uint32_t lin);
float lco_q4k_weight(const uint8_t *w, uint32_t lin);
/* Dequantize n elements starting at element 0 with the shader formulas. */
void lco_dequant_shader(const uint8_t *w, int dtype, size_t n, float *out);

/* --- projections (one output row per invocation, sequential K) ---------- */

/* kernels/proj.comp:23-33.  row_major != 0 reads w[j*n + i]. */
void lco_proj_f32(const float *x, const float *w, float *c, uint32_t k,
                  uint32_t n, uint32_t row_major);
/* kernels/proj_q8_0.comp:47-67. */
void lco_proj_q8_0(const float *x, const uint8_t *w, float *c, uint32_t k,
                   uint32_t n);
/* kernels/proj_q4k.comp:60-92 (lin = expert_offset + i*k + j). */
void lco_proj_q4k(const float *x, const uint8_t *w, float *c, uint32_t k,
                  uint32_t n, uint32_t expert_offset);
/* M-row forms: the single-row shader applied to each of m rows of x
 * (x is [m, k] row-major, c is [m, n]). */
void lco_proj_f32_m(const float *x, const float *w, float *c, uint32_t m,
                    uint32_t k, uint32_t n, uint32_t row_major);
void lco_proj_q8_0_m(const float *x, const uint8_t *w, float *c, uint32_t m,
                     uint32_t k, uint32_t n);
void lco_proj_q4k_m(const float *x, const uint8_t *w, float *c, uint32_t m,
                    uint32_t k, uint32_t n, uint32_t expert_offset);

/* --- interleaved kernels ------------------------------------------------ */

/* kernels/rmsnorm.comp:22-35 (y = x*w*inversesqrt(mean(x^2)+eps)), m rows. */
void lco_rmsnorm(const float *x, const float *w, float *y, uint32_t m,
                 uint32_t n, float eps);
/* kernels/qk_norm_rope.comp:29-67 for m rows; row r uses position pos[r]. */
void lco_qk_norm_rope(const float *x, const float *w, const float *freq,
                      float *y, uint32_t m, uint32_t n_heads,
                      uint32_t head_dim, uint32_t rope_dim, float eps,
                      const uint32_t *pos);
/* kernels/activation.comp:21-29: h = silu(gate) * up. */
void lco_activation(const float *gate, const float *up, float *h, uint32_t n);
/* kernels/add.comp:21-25. */
void lco_add(const float *a, const float *b, float *c, uint32_t n);
/* kernels/gate_mul.comp:24-30: out[i] = v[i] * gate[i / head_dim]. */
void lco_gate_mul(const float *v, const float *gate, float *out, uint32_t n_hd,
                  uint32_t head_dim);
/* host softplus of src/dflash.rs:957: g > 20 ? g : ln(1 + e^g). */
void lco_softplus(const float *g, float *out, uint32_t n);
/* kernels/mha_attn.comp:31-72, one query vector (n_q_heads*head_dim). */
void lco_mha_attn(const float *q, const float *k, const float *v, float *out,
                  uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim,
                  uint32_t seq_len, float scale, uint32_t q_pos,
                  uint32_t causal);
/* kernels/enc_aux_norm.comp:24-43. */
void lco_enc_aux_norm(const float *x, const float *w, float *y,
                      uint32_t n_feat, uint32_t n_aux, uint32_t n_tokens,
                      float eps);
/* RoPE frequency table of src/dflash.rs:901-907: 1 / base^(2i/rope_dim). */
void lco_rope_freq(float *freq, uint32_t rope_dim, float base);
/* src/lib.rs:456-464 argmax: Iterator::max_by with partial_cmp, so the last
 * maximal index wins and a NaN compares Equal. */
size_t lco_argmax(const float *logits, size_t n);

/* ---- target model (src/target.rs) ---- */
/* gate_attn.comp:22-31: out[i] = attn[i] * log(1 + exp(gate[i / head_dim])). */
void lco_gate_attn(const float *attn, const float *gate, float *out, uint32_t n_heads, uint32_t head_dim);
/* Router selection of dispatch_moe_ffn (src/target.rs:653-677): probs =
 * 1 / (1 + exp(-logit)); the min(n_used, n_exp) largest probs + bias by a
 * stable descending sort (equal values keep expert order); scores = their
 * probs, divided by max(sum, 6.103515625e-5) when norm, times scale when scale
 * is neither 0 nor 1.  Returns the number selected. */
uint32_t lco_moe_select(const float *logits, const float *bias, uint32_t n_exp, uint32_t n_used, int norm,
                        float scale, int32_t *ids, float *scores);
/* src/target.rs:700-712: col_l2 = clamp(sqrt(sum h^2), 1e-8, 1e30), the sum
 * taken in order in f32; out[i] = h[i] * 32768 / col_l2.  Returns col_l2. */
float lco_moe_l2_scale(const float *h, uint32_t n, float *out);

/* Number of OpenMP threads the oracle runs with (0 = library default). */
void lco_set_threads(int n);
int lco_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
