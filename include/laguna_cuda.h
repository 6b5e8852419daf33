/*
 * laguna_cuda.h -- C ABI of the B200 (sm_100a) backend for laguna-raw's
 * quantized projection path.
 *
 * This library replaces the reference's Vulkan runtime (src/vulkan.rs) and the
 * shader launches behind its typed dispatch helpers (src/dflash.rs:979-1327,
 * src/target.rs:1086-1162).  Weights stay in their raw GGUF block layout
 * (Q8_0: 34-byte blocks of 32 elements; Q4_K: 144-byte super-blocks of 256)
 * and are decoded inside the kernels.
 *
 * Conventions
 *  - Every function returns an lc_status (0 = LC_OK); none aborts.  On failure
 *    lc_last_error() returns a message (thread-local, valid until the next
 *    call on the same thread).
 *  - Compute entry points take DEVICE pointers (from lc_buf_device_ptr() or
 *    any CUDA allocation on the context's device) and enqueue on the context's
 *    stream.  They return once the work is enqueued, unless lc_set_sync(ctx, 1)
 *    was called, in which case each call waits for its work like the
 *    reference's fenced submit_compute (src/vulkan.rs:326-334).
 *  - Sizes are uint32 like the reference's push constants
 *    (e.g. kernels/proj_q8_0.comp:17-20); byte counts are size_t.
 *  - Quantized weights are row-major: element (i, j) of an n x k projection is
 *    element i*k + j of the GGUF tensor (kernels/proj_q8_0.comp:54,
 *    kernels/proj_q4k.comp:67).  The quantized kernels require k to be a
 *    multiple of the block size (32 for Q8_0, 256 for Q4_K) and the weight
 *    pointer to be 16-byte aligned; other shapes return LC_ERR_UNSUPPORTED.
 *  - f16 scales decode by the reference rule by default: subnormal halves map
 *    to 2^-14 * (1 + m/1024) (kernels/proj_q8_0.comp:27-45).  lc_set_half_mode
 *    selects IEEE decoding instead.
 */
#ifndef LAGUNA_CUDA_H
#define LAGUNA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
typedef enum {
    LC_OK = 0,
    LC_ERR_INVALID = 1,      /* null pointer, size out of range, misaligned */
    LC_ERR_UNSUPPORTED = 2,  /* dtype or shape this backend does not run    */
    LC_ERR_CUDA = 3,         /* a CUDA runtime call failed                  */
    LC_ERR_OOM = 4,          /* device allocation failed                    */
    LC_ERR_TIMEOUT = 5,      /* a bounded device-side wait expired          */
    LC_ERR_IO = 6            /* file could not be read / is not GGUF v3     */
} lc_status;

/* ---- tensor types: GGUF ids (src/gguf.rs:45-88) ------------------------- */
enum {
    LC_F32 = 0,
    LC_F16 = 1,
    LC_Q8_0 = 8,
    LC_Q4_K = 12,
    LC_BF16 = 30,
    /* lc_dequant only: the reference CPU decoder's own "Q4_K" branch
     * (src/dflash.rs:398-436), a bf16 d/k4/signs + 3-bit layout that differs
     * from GGUF Q4_K; provided so test-dequant parity covers every branch. */
    LC_Q4_K_DFLASH_CPU = 1012
};

/* ---- f16 decode modes ---------------------------------------------------- */
enum {
    LC_HALF_REF = 0,  /* reference rule (default) */
    LC_HALF_IEEE = 1  /* IEEE-754 binary16        */
};

typedef struct lc_ctx lc_ctx;
typedef struct lc_buf lc_buf;

/* ---- runtime: replaces VulkanContext (src/vulkan.rs:5-100) -------------- */

/* Message for the last failure on this thread ("" if none). */
const char *lc_last_error(void);
/* Library version string. */
const char *lc_version(void);
/* Number of CUDA devices visible. */
int lc_device_count(int *count);
/* VulkanContext::init (src/vulkan.rs:16-100): open `device`, create a stream. */
int lc_init(int device, lc_ctx **out);
/* Release the context and everything it owns (the reference leaks). */
int lc_destroy(lc_ctx *ctx);
/* Enqueue on an external cudaStream_t (NULL restores the context's own). */
int lc_set_stream(lc_ctx *ctx, void *cuda_stream);
/* The cudaStream_t work is enqueued on. */
void *lc_get_stream(lc_ctx *ctx);
/* Wait for all enqueued work: the fence wait of submit_compute
 * (src/vulkan.rs:326-334). */
int lc_synchronize(lc_ctx *ctx);
/* 1: every compute call waits for completion (reference behaviour); 0: async. */
int lc_set_sync(lc_ctx *ctx, int sync);
/* Wait for the context's stream, then report (and clear) the device status
 * word: LC_ERR_TIMEOUT if a kernel's bounded wait on its own asynchronous
 * copies gave up (the launch's outputs are then invalid), else LC_OK.  Kernels
 * never hang on such a wait; this call is how the host learns of it. */
int lc_device_status(lc_ctx *ctx);
/* Device memory (bytes) the context holds in its grow-only scratch slots;
 * 0 until a call needs scratch.  No counterpart in the reference, whose
 * buffers are all created up front (ForwardBuffers::new, src/dflash.rs:259-285). */
int lc_ctx_scratch_bytes(lc_ctx *ctx, size_t *bytes);
/* LC_HALF_REF (default) or LC_HALF_IEEE for every f16 scale decode. */
int lc_set_half_mode(lc_ctx *ctx, int mode);
/* Device the context runs on. */
int lc_ctx_device(lc_ctx *ctx, int *device);

/* ---- buffers: replace GpuBuffer (src/vulkan.rs:342-452) ------------------ */

/* GpuBuffer::new (src/vulkan.rs:350-398): `bytes` of device memory
 * (256-byte aligned, zero-filled). */
int lc_buf_alloc(lc_ctx *ctx, size_t bytes, lc_buf **out);
/* Free a buffer (the reference's GpuBuffer has no Drop). */
int lc_buf_free(lc_buf *buf);
/* Device pointer of a buffer, for the compute entry points. */
void *lc_buf_device_ptr(const lc_buf *buf);
/* Size in bytes. */
size_t lc_buf_size(const lc_buf *buf);
/* GpuBuffer::upload (src/vulkan.rs:400-430): copy `bytes` host bytes to
 * offset 0.  Synchronous with respect to the context's stream. */
int lc_buf_upload(lc_buf *buf, const void *src, size_t bytes);
/* Upload at a byte offset. */
int lc_buf_upload_at(lc_buf *buf, size_t offset, const void *src, size_t bytes);
/* Read `bytes` from a byte offset into host memory (waits for the stream). */
int lc_buf_read(lc_buf *buf, size_t offset, void *dst, size_t bytes);
/* GpuBuffer::read_f32 (src/vulkan.rs:432-452): read n floats from offset 0. */
int lc_buf_read_f32(lc_buf *buf, float *dst, size_t n);

/* ---- projections --------------------------------------------------------- */

/* dispatch_proj / dispatch_proj_row (src/dflash.rs:1009-1052), kernels/proj.comp:
 * c[i] = sum_j x[j] * w[row_major ? j*n + i : i*k + j]. */
int lc_proj_f32(lc_ctx *ctx, const float *x, const float *w, float *c,
                uint32_t k, uint32_t n, uint32_t row_major);
/* Q8_0 projection, the WeightType::Q8_0 arm of dispatch_proj_quant_expert
 * (src/target.rs:1118-1138) running kernels/proj_q8_0.comp:47-67. */
int lc_proj_q8_0(lc_ctx *ctx, const float *x, const void *w, float *c,
                 uint32_t k, uint32_t n);
/* Q4_K projection, the WeightType::Q4_K arm (src/target.rs:1139-1160) running
 * kernels/proj_q4k.comp:60-92; expert_offset is in elements (multiple of 256). */
int lc_proj_q4k(lc_ctx *ctx, const float *x, const void *w, float *c,
                uint32_t k, uint32_t n, uint32_t expert_offset);
/* dispatch_proj_quant_expert (src/target.rs:1098-1162): dtype switch over
 * LC_F32 / LC_Q8_0 / LC_Q4_K (expert_offset applies to Q4_K only, as in the
 * reference; LC_F32 ignores it). */
int lc_proj_quant(lc_ctx *ctx, int dtype, const float *x, const void *w,
                  float *c, uint32_t k, uint32_t n, uint32_t expert_offset);
/* M-row projection: the same projection applied to each row of x [m, k],
 * writing c [m, n] -- the draft-block (m = 16) and lm_head (m = 1024) forms
 * the reference would reach by m calls of the single-row dispatch. */
int lc_proj_m(lc_ctx *ctx, int dtype, const float *x, const void *w, float *c,
              uint32_t m, uint32_t k, uint32_t n, uint32_t expert_offset);
/* Q4_K projection of m = 1..16 rows of x [m, k] that allocates no device
 * memory, for callers that cannot allocate on the call path: a serving loop
 * whose memory plan has given all of HBM to weights and K/V, or a decode loop
 * that must not pay cudaMalloc's device-wide synchronisation.  Results equal
 * lc_proj_m with LC_Q4_K within the projection tolerance (some m run different
 * kernels).  m <= 4 needs no scratch; for m = 5..16 the packed activations
 * live in a fixed static device array of 1 MiB (k <= 15360 at m = 16),
 * resolved per context at lc_init.  Shapes beyond that, m > 16, or (m = 3, 4)
 * m * k beyond shared memory return LC_ERR_UNSUPPORTED.  Calls that overlap
 * on one GPU share the array and race: serialise them.  A context must not be
 * used across a cudaDeviceReset.  No counterpart in the reference. */
int lc_proj_q4k_static(lc_ctx *ctx, const float *x, const void *w, float *c,
                       uint32_t m, uint32_t k, uint32_t n, uint32_t expert_offset);

/* The FFN block of a DFlash decoder layer (src/dflash.rs:965-968:
 * dispatch_proj gate and up, dispatch_activation, dispatch_proj down) in one
 * call: y [m, n_embd] = down(SiLU(x W_gate^T) * (x W_up^T)) for x [m, n_embd]
 * (device), Q8_0 or Q4_K weights (gate / up: n_ff x n_embd, down: n_embd x
 * n_ff).  The intermediate [2, m, n_ff] lives in the context's scratch.  The
 * residual add stays with the caller. */
int lc_ffn(lc_ctx *ctx, int dtype, const float *x, const void *w_gate, const void *w_up, const void *w_down,
           float *y, uint32_t m, uint32_t n_embd, uint32_t n_ff);

/* Host-buffer forms, the reference's upload -> dispatch -> read_f32 sequence
 * (GpuBuffer::upload src/vulkan.rs:400-430, dispatch_proj* src/dflash.rs:
 * 1009-1090, GpuBuffer::read_f32 src/vulkan.rs:432-452) in one call: x_host is
 * copied into the context's scratch, the computation runs, the result is
 * copied into y_host / c_host, and the call returns once it is there.  Host
 * buffers in page-locked memory make both copies asynchronous DMA.  Weights
 * stay device pointers. */
int lc_ffn_host(lc_ctx *ctx, int dtype, const float *x_host, const void *w_gate, const void *w_up,
                const void *w_down, float *y_host, uint32_t m, uint32_t n_embd, uint32_t n_ff);
int lc_proj_m_host(lc_ctx *ctx, int dtype, const float *x_host, const void *w, float *c_host, uint32_t m, uint32_t k,
                   uint32_t n, uint32_t expert_offset);

/* ---- dequant ------------------------------------------------------------- */

/* dequant_to_f32 (src/dflash.rs:331-465) on the device.  LC_Q8_0 / LC_F16 /
 * LC_BF16 / LC_F32 / LC_Q4_K_DFLASH_CPU follow the CPU decoder branch for
 * branch (reads bounded by src_bytes, missing elements 0); LC_Q4_K decodes
 * GGUF Q4_K with the GPU shader formula of kernels/proj_q4k.comp:72-87.
 * Other dtypes produce zeros like the reference's fallback arm. */
int lc_dequant(lc_ctx *ctx, int dtype, const void *src, size_t src_bytes,
               size_t n, float *out);

/* ---- kernels interleaved with the projections ---------------------------- */

/* dispatch_rmsnorm (src/dflash.rs:979-1007), kernels/rmsnorm.comp, over m rows
 * of n: out = x * w * inversesqrt(mean(x^2) + eps).  out may alias x. */
int lc_rmsnorm(lc_ctx *ctx, const float *w, const float *x, float *out,
               uint32_t m, uint32_t n, float eps);
/* dispatch_qk_norm_rope (src/dflash.rs:1093-1129), kernels/qk_norm_rope.comp,
 * over m rows of n_heads*head_dim; row r is rotated at position pos0 + r.
 * out may alias x. */
int lc_qk_norm_rope(lc_ctx *ctx, const float *x, const float *w,
                    const float *freq, float *out, uint32_t m,
                    uint32_t n_heads, uint32_t head_dim, uint32_t rope_dim,
                    float eps, uint32_t pos0);
/* dispatch_activation (src/dflash.rs:1305-1327): h = silu(gate) * up. */
int lc_activation(lc_ctx *ctx, const float *gate, const float *up, float *h,
                  uint32_t n);
/* dispatch_add (src/dflash.rs:1281-1303): c = a + b. */
int lc_add(lc_ctx *ctx, const float *a, const float *b, float *c, uint32_t n);
/* dispatch_gate_mul (src/dflash.rs:1236-1267): out[i] = v[i] * gate[i/head_dim]
 * for i < n_hd (gate holds n_hd/head_dim values per row). */
int lc_gate_mul(lc_ctx *ctx, const float *v, const float *gate, float *out,
                uint32_t n_hd, uint32_t n_heads, uint32_t head_dim);
/* The host softplus of src/dflash.rs:956-958 moved on-device:
 * out = g > 20 ? g : ln(1 + e^g). */
int lc_softplus(lc_ctx *ctx, const float *g, float *out, uint32_t n);
/* dispatch_enc_aux_norm (src/dflash.rs:1201-1233), kernels/enc_aux_norm.comp. */
int lc_enc_aux_norm(lc_ctx *ctx, const float *x, const float *w, float *y,
                    uint32_t n_feat, uint32_t n_aux, uint32_t n_tokens,
                    float eps);
/* dispatch_mha_attn_seq (src/dflash.rs:1160-1198), kernels/mha_attn.comp, for
 * m query rows q [m, n_q_heads*head_dim] over k, v [seq_len, n_kv_heads*head_dim];
 * query r sits at position q_pos0 + r (key p is visible iff !causal || p <= pos).
 * head_dim 128; q, k and v 16-byte aligned. */
int lc_mha_attn(lc_ctx *ctx, const float *q, const float *k, const float *v,
                float *out, uint32_t m, uint32_t n_q_heads, uint32_t n_kv_heads,
                uint32_t head_dim, uint32_t seq_len, float scale,
                uint32_t q_pos0, uint32_t causal);
/* RoPE frequency table (src/dflash.rs:901-907) on the host:
 * freq[i] = 1 / base^(2i/rope_dim), i < rope_dim/2. */
int lc_rope_freq(float *freq_host, uint32_t rope_dim, float base);

/* ---- lm_head + argmax ----------------------------------------------------- */

/* Order-preserving key of (logit, index), compared as SIGNED int64: the high
 * 32 bits order the f32 value, the low 32 bits hold the index, so the maximum
 * key is the largest logit with ties broken toward the LARGER index -- the
 * rule of src/lib.rs:456-464 (Iterator::max_by keeps the last maximum).  A
 * plain int64 MAX reduction (ncclInt64 / torch.int64) combines shards. */
uint64_t lc_pack_key(float value, uint32_t index);
float lc_key_value(uint64_t key);
uint32_t lc_key_index(uint64_t key);
/* Row-wise argmax of logits [m, n] into keys[m] (device); index = row_offset + j. */
int lc_argmax_rows(lc_ctx *ctx, const float *logits, uint32_t m, uint32_t n,
                   uint32_t row_offset, uint64_t *keys);
/* project_normalized_hidden (src/target.rs:580-605) for m hidden rows fused
 * with argmax (src/lib.rs:456-464): logits = x [m, k] . W[n_local rows]^T for
 * a vocab shard whose first row is global row `row_offset`; keys[r] (device)
 * receives the shard-local best (logit, global index).  `logits` (device,
 * [m, n_local]) may be NULL; when given, the logits are written too. */
int lc_lm_head_argmax(lc_ctx *ctx, int dtype, const float *x, const void *w,
                      uint32_t m, uint32_t k, uint32_t n_local,
                      uint32_t row_offset, uint64_t *keys, float *logits);

/* ---- vocab-sharded lm_head over several GPUs (NCCL owned by the library) -- */

/* The reference projects each hidden row onto the whole vocabulary on one
 * device (project_normalized_hidden, src/target.rs:580-605, then argmax,
 * src/lib.rs:456-464).  Sharded, each rank holds a contiguous range of vocab
 * rows; its shard's keys (lc_lm_head_argmax) are combined by one int64 MAX
 * all-reduce, which yields the reference's argmax over the whole vocabulary.
 * NCCL is loaded at run time (libnccl.so.2); without it these calls return
 * LC_ERR_UNSUPPORTED.  Every wait is bounded by the communicator's timeout:
 * when it expires (a rank never arrived) the communicator is aborted -- its
 * kernels end, the context stays usable -- and LC_ERR_TIMEOUT is returned. */
typedef struct lc_comm lc_comm;
/* A 128-byte id for lc_comm_init, made by one rank and handed to the others
 * out of band (ncclGetUniqueId). */
int lc_comm_unique_id(void *id128);
/* The communicator of rank `rank` of n_ranks on the context's device
 * (ncclCommInitRankConfig, non-blocking, waited on for at most timeout_ms). */
int lc_comm_init(lc_ctx *ctx, const void *id128, int n_ranks, int rank, int timeout_ms, lc_comm **out);
/* Finalise (bounded) and free; an aborted communicator is just freed. */
int lc_comm_destroy(lc_comm *comm);
int lc_comm_rank(const lc_comm *comm, int *rank, int *n_ranks);
/* keys[n] (device, packed by lc_pack_key) <- their maximum over the ranks,
 * enqueued on the context's stream. */
int lc_comm_allreduce_max_keys(lc_ctx *ctx, lc_comm *comm, uint64_t *keys, uint32_t n);
/* Wait for the context's stream, polling the communicator for errors, for at
 * most its timeout: LC_OK, or LC_ERR_TIMEOUT / LC_ERR_CUDA with the
 * communicator aborted. */
int lc_comm_wait(lc_ctx *ctx, lc_comm *comm);
/* This rank's shard of the lm_head (rows row_offset .. row_offset + n_local
 * of the vocabulary) for m hidden rows x [m, k], then the MAX all-reduce:
 * keys[m] (device) end with the global (logit, token) of every row.  Enqueued
 * on the context's stream (lc_comm_wait bounds the wait; a context in sync
 * mode waits here). */
int lc_lm_head_argmax_sharded(lc_ctx *ctx, lc_comm *comm, int dtype, const float *x, const void *w_shard,
                              uint32_t m, uint32_t k, uint32_t n_local, uint32_t row_offset, uint64_t *keys);

/* ---- failure detection ----------------------------------------------------- */

/* Self-check of the device-side bounded waits: one CTA waits on a barrier
 * nobody arrives on, gives up after `spins` polls and records it in the
 * status word, so that lc_device_status(ctx) returns LC_ERR_TIMEOUT and the
 * context stays usable.  No counterpart in the reference, whose waits are
 * unbounded fences (src/vulkan.rs:326-334). */
int lc_check_bounded_wait(lc_ctx *ctx, uint32_t spins);

/* ---- GGUF v3 reader: replaces GGUFReader (src/gguf.rs) ------------------- */

typedef struct lc_gguf lc_gguf;

/* TensorType::block_size / block_elements (src/gguf.rs:88-141) for the
 * supported types (F32, F16, BF16, Q8_0, Q4_K); 0 for others. */
uint64_t lc_type_block_bytes(int dtype);
uint64_t lc_type_block_elements(int dtype);
/* TensorInfo::n_bytes (src/gguf.rs:186-201): ceil(n/elements)*block_bytes. */
uint64_t lc_tensor_bytes(int dtype, uint64_t n_elements);
/* GGUFReader::open (src/gguf.rs:321-400): header, metadata, tensor infos,
 * data offset aligned to general.alignment (default 32). */
int lc_gguf_open(const char *path, lc_gguf **out);
int lc_gguf_close(lc_gguf *g);
uint64_t lc_gguf_tensor_count(const lc_gguf *g);
/* Tensor i: name (valid while g is open), GGUF type id, dims, shape[4]
 * (ne0 first), byte offset relative to the data section, byte size. */
int lc_gguf_tensor_info(const lc_gguf *g, uint64_t i, const char **name, int *dtype, uint32_t *n_dims,
                        uint64_t shape[4], uint64_t *offset, uint64_t *n_bytes);
/* GGUFReader::tensor_by_name (src/gguf.rs:407): index or LC_ERR_INVALID. */
int lc_gguf_find(const lc_gguf *g, const char *name, uint64_t *index);
/* GGUFReader::read_tensor_data (src/gguf.rs:415-421): raw bytes into host memory. */
int lc_gguf_read(lc_gguf *g, uint64_t index, void *dst, uint64_t bytes);
/* The same bytes without a copy: *data points into the reader's read-only
 * mapping of the file (valid until lc_gguf_close), *bytes = n_bytes.  A tensor
 * that lies past the end of the file is LC_ERR_IO, as read_exact's short read
 * is in the reference. */
int lc_gguf_tensor_data(const lc_gguf *g, uint64_t index, const void **data, uint64_t *bytes);
/* Numeric / string metadata by key (any integer or float type). */
int lc_gguf_meta_u64(const lc_gguf *g, const char *key, uint64_t *out);
int lc_gguf_meta_f32(const lc_gguf *g, const char *key, float *out);
int lc_gguf_meta_str(const lc_gguf *g, const char *key, const char **out);

/* ---- DFlash draft model: replaces DFlashModel (src/dflash.rs:6-976) ------- */

typedef struct {
    uint32_t n_layers;    /* block_count */
    uint32_t n_embd;      /* embedding_length */
    uint32_t n_heads;     /* attention.head_count */
    uint32_t n_kv_heads;  /* attention.head_count_kv */
    uint32_t head_dim;    /* attention.key_length */
    uint32_t rope_dim;    /* rope.dimension_count */
    uint32_t n_ff;        /* feed_forward_length */
    uint32_t n_aux;       /* len(target_layers): encoder inputs = n_aux * n_embd */
    float rope_base;      /* rope.freq_base, default 500000 (src/dflash.rs:903) */
    float norm_eps;       /* RMSNorm eps, 1e-5 (src/dflash.rs:987) */
    float qk_eps;         /* QK-norm eps, 1e-6 (src/dflash.rs:1105) */
} lc_dflash_hparams;

typedef struct lc_dflash lc_dflash;

/* Model::from_reader (src/model.rs:29-129) hyper-parameters with the
 * laguna./dflash./bare key aliases of populate_metadata (src/gguf.rs:516-653). */
int lc_gguf_dflash_hparams(const lc_gguf *g, lc_dflash_hparams *out);
/* An empty model with device workspaces for up to max_ctx context rows and
 * max_block block tokens. */
int lc_dflash_create(lc_ctx *ctx, const lc_dflash_hparams *hp, uint32_t max_ctx, uint32_t max_block,
                     lc_dflash **out);
/* Model::upload_tensor_quantized (src/model.rs:174-184): upload one GGUF
 * tensor by name ("blk.N.attn_q.weight", "fc.weight", ...).  Projection
 * weights stay raw (F32 / Q8_0 / Q4_K); F16 / BF16 tensors are decoded to f32
 * on the device with dequant_to_f32's rules. */
int lc_dflash_set_tensor(lc_dflash *m, const char *name, int dtype, const void *host_data, size_t bytes);
/* DFlashModel::load (src/dflash.rs:34-119) from a GGUF file, raw-block upload. */
int lc_dflash_load_gguf(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block, lc_dflash **out);
/* lc_dflash_load_gguf with load flags.  The file is mapped, every tensor the
 * draft path uses goes into one device allocation through pinned staging
 * buffers (host copies of one chunk overlap the DMA of the previous one), with
 * one synchronisation at the end.  LC_LOAD_BF16_NATIVE decodes BF16 tensors
 * as bfloat16 (f32 = bits << 16); without it they follow the reference, which
 * reads BF16 bits with the f16 layout (src/dflash.rs:351-378). */
enum { LC_LOAD_BF16_NATIVE = 1 };
int lc_dflash_load_gguf_ex(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block, uint32_t flags,
                           lc_dflash **out);
int lc_dflash_destroy(lc_dflash *m);
/* The device copy of a loaded tensor (the slots DFlashModel::load fills,
 * src/dflash.rs:60-107): its address, dtype as stored (F16 / BF16 tensors are
 * held as LC_F32) and byte size.  LC_ERR_INVALID for a name the model does
 * not hold. */
int lc_dflash_weight(const lc_dflash *m, const char *name, const void **data, int *dtype, uint64_t *bytes);
int lc_dflash_get_hparams(const lc_dflash *m, lc_dflash_hparams *out);
/* DFlashModel::encode (src/dflash.rs:157-234) for n_ctx rows of target
 * features [n_ctx, n_aux*n_embd] (device) -> enc_out [n_ctx, n_embd] (device). */
int lc_dflash_encode(lc_dflash *m, const float *features, uint32_t n_ctx, float *enc_out);
/* Per-layer context K/V of forward_injected_decode_hidden (src/dflash.rs:933-936)
 * for every encoder row: row p is rotated at position p. */
int lc_dflash_set_context(lc_dflash *m, const float *enc_out, uint32_t n_ctx);
/* The layer loop of forward_injected_decode_hidden (src/dflash.rs:938-975)
 * for a block of m token inputs x [m, n_embd] (device) at positions
 * n_ctx .. n_ctx+m-1, attending causally over [context K/V; block K/V];
 * hidden [m, n_embd] (device) gets the output_norm'ed states.  With n_ctx = 1
 * and m = 1 this is the reference's computation. */
int lc_dflash_decode_block(lc_dflash *m, const float *x, uint32_t m_tokens, float *hidden);
/* forward_injected_decode_hidden (src/dflash.rs:877-976) with host buffers:
 * features [n_aux*n_embd], token_input [n_embd] -> hidden [n_embd]. */
int lc_dflash_forward_injected_decode_hidden(lc_dflash *m, const float *features_host, const float *token_host,
                                             float *hidden_host);
/* forward_from_input (src/dflash.rs:735-851), the legacy single-token decoder
 * behind the `encode` CLI: input [n_embd] (device) -> hidden [n_embd]
 * (device); when logits is not NULL, the fc.weight buffer reinterpreted as
 * [n_vocab, n_embd] rows (src/dflash.rs:839-847) projects the hidden state and
 * n_vocab receives the row count. */
int lc_dflash_forward_from_input(lc_dflash *m, const float *input, float *hidden, float *logits,
                                 uint32_t *n_vocab);
/* forward_token (src/dflash.rs:469-733) behind the `forward` CLI: the input is
 * token_embd read as [n_embd][vocab] (x[i] = emb[i*vocab + token_id],
 * src/dflash.rs:482-485), then forward_from_input's layer loop. */
int lc_dflash_forward_token(lc_dflash *m, uint32_t token_id, float *hidden, float *logits, uint32_t *n_vocab);

/* ---- Target (Laguna) model: TargetModel (src/target.rs:105-748) ---------- */

/* Model::from_reader (src/model.rs:29-129) for the target: dense keys as the
 * DFlash reader, plus the SWA rope and expert sizes (metadata first, then the
 * shapes of ffn_gate_exps / ffn_gate_shexp). */
typedef struct {
    uint32_t n_layers;            /* block_count */
    uint32_t n_embd;              /* embedding_length */
    uint32_t n_ff;                /* feed_forward_length (dense FFN) */
    uint32_t n_heads;             /* attention.head_count (first array element) */
    uint32_t n_kv_heads;          /* attention.head_count_kv (second array element) */
    uint32_t head_dim;            /* attention.key_length (no fallback) */
    uint32_t rope_dim;            /* rope.dimension_count */
    uint32_t rope_dim_swa;        /* rope.dimension_count_swa */
    uint32_t swa;                 /* rope_dim_swa > 0 or attention.sliding_window > 0 (src/target.rs:328) */
    uint32_t n_expert;            /* expert.count, else the last dim of ffn_gate_exps */
    uint32_t n_expert_used;       /* expert.used_count, else 10 when experts exist */
    uint32_t n_ff_exp;            /* expert.feed_forward_length, else from the shapes */
    uint32_t n_ff_shexp;          /* expert.shared_feed_forward_length, else from the shapes */
    uint32_t has_moe;             /* a tensor named *ffn_gate_exps*: layers >= 1 are MoE */
    uint32_t has_shexp;           /* a tensor named *ffn_gate_shexp* */
    uint32_t expert_weights_norm; /* expert_weights_norm (default 0) */
    uint32_t n_vocab;             /* token_embd elements / n_embd (src/target.rs:287-291) */
    float rope_base;              /* rope.freq_base, default 500000 */
    float rope_base_swa;          /* rope.freq_base_swa, default 10000 */
    float expert_weights_scale;   /* expert_weights_scale, default 1 */
    float norm_eps;               /* 1e-5 (src/target.rs:970) */
    float qk_eps;                 /* 1e-6 (src/target.rs:897) */
} lc_target_hparams;

typedef struct lc_target lc_target;

int lc_gguf_target_hparams(const lc_gguf *g, lc_target_hparams *out);
/* The target_layers metadata array (a DFlash draft's capture layers,
 * src/gguf.rs:633-638): its integer elements, the first `cap` into out[];
 * *n receives the count (0 when the key is absent). */
int lc_gguf_target_layers(const lc_gguf *g, int64_t *out, uint32_t cap, uint32_t *n);

/* TargetModel::load (src/target.rs:130-266) on the loader of
 * lc_dflash_load_gguf_ex (mapped file, pinned staging, one allocation; raw
 * F32 / Q8_0 / Q4_K blocks, F16 / BF16 decoded to f32).  Dense layers take
 * ffn_gate/up/down, MoE layers (layer >= 1 of a model with experts) the
 * router, expert and shared-expert tensors.  The K/V cache holds max_ctx
 * positions per layer; a forward takes at most max_block tokens.  Flags:
 * LC_LOAD_BF16_NATIVE, and LC_TARGET_REF_EXPERT_OFFSET, which reproduces the
 * reference's dispatch_proj_quant_expert (src/target.rs:1098-1162), where the
 * expert offset reaches only the Q4_K kernel so every Q8_0 / F32 expert
 * projection reads expert 0; by default every format reads its own expert. */
enum { LC_TARGET_REF_EXPERT_OFFSET = 2 };
int lc_target_load_gguf(lc_ctx *ctx, const char *path, uint32_t max_ctx, uint32_t max_block, uint32_t flags,
                        lc_target **out);
int lc_target_destroy(lc_target *t);
int lc_target_get_hparams(const lc_target *t, lc_target_hparams *out);
/* Layer `layer`: MoE or dense, and its query heads (attn_q rows / head_dim,
 * src/target.rs:225-235). */
int lc_target_layer_info(const lc_target *t, uint32_t layer, uint32_t *is_moe, uint32_t *n_q_heads);
/* The device copy of a loaded tensor, as lc_dflash_weight. */
int lc_target_weight(const lc_target *t, const char *name, const void **data, int *dtype, uint64_t *bytes);
/* x [m, n_embd] (device) <- the token embeddings of tokens[m] (host): row
 * token of token_embd decoded with dequant_to_f32 (target_token_embedding,
 * src/lib.rs:431-454). */
int lc_target_embed(lc_target *t, const uint32_t *tokens, uint32_t m, float *x);
/* forward_token_impl (src/target.rs:314-578) for m token inputs x [m, n_embd]
 * (device).  Without LC_TARGET_CACHED each row is forward_token: position 0,
 * attending to itself only, nothing cached.  With it the rows are the next m
 * positions of one sequence (cache_len .. cache_len + m - 1): their K/V are
 * appended to the cache and each row attends causally over the cache -- one
 * launch sequence for a block of draft tokens, equal to m calls of
 * forward_token_cached.  Outputs (device, each optional):
 *   captured [m, n_capture, n_embd]: the input of each listed layer (index
 *     n_layers = the last layer's output), in increasing layer order;
 *   hidden [m, n_embd]: the output_norm'ed state;
 *   logits [m, n_vocab]: output.weight . hidden (hidden itself without an
 *     output weight, src/target.rs:564-575);
 *   keys [m]: lc_pack_key(max logit, token), the last maximum winning. */
enum { LC_TARGET_CACHED = 1 };
int lc_target_forward(lc_target *t, const float *x, uint32_t m, uint32_t flags, const uint32_t *capture_layers,
                      uint32_t n_capture, float *captured, float *hidden, float *logits, uint64_t *keys);
/* The expert selection of MoE layer `layer` in the most recent forward (or
 * lc_target_moe_ffn) that ran it: ids[m][n_expert_used] (device, enqueued on
 * the context's stream) and m, the rows of that call. */
int lc_target_routing(const lc_target *t, uint32_t layer, int32_t *ids, uint32_t *m);
/* Positions held in the K/V cache (TargetKvCache::len). */
int lc_target_cache_len(const lc_target *t, uint32_t *len);
/* Drop cached positions from len on (rejected draft tokens); len = 0 is
 * TargetKvCache::clear. */
int lc_target_cache_truncate(lc_target *t, uint32_t len);

/* dispatch_moe_ffn (src/target.rs:607-748) on the device for m rows of the
 * normalised input x [m, n_embd]: router logits, sigmoid + bias top-k
 * selection (ties to the lower expert), optional normalisation and scale,
 * the selected experts' SwiGLU FFNs with the reference's per-expert L2
 * rescaling of the hidden vector, their weighted sum and the shared expert.
 * y [m, n_embd] = the FFN output (the residual add stays with the caller).
 * Expert tensors hold n_expert matrices back to back (gate / up: n_ff_exp x
 * n_embd each, down: n_embd x n_ff_exp).  ids / scores [m, n_expert_used]
 * (device, optional) receive the selection.  Uses the target's workspaces. */
int lc_target_moe_ffn(lc_target *t, uint32_t layer, const float *x, uint32_t m, float *y, int32_t *ids,
                      float *scores);

#ifdef __cplusplus
}
#endif
#endif /* LAGUNA_CUDA_H */
