"""Seeded synthetic GGUF blocks and activations with the value distributions of
the benchmark configurations (no model checkpoints are available offline).

Q8_0 block (34 B, 32 elements; src/gguf.rs:97,134): f16 d = |N(0,1)|*0.02/127,
int8 q uniform in [-127, 127].
Q4_K super-block (144 B, 256 elements; src/gguf.rs:101,136): f16 d, dmin =
|N(0,1)|*1e-3; eight 6-bit (scale, min) pairs uniform in 0..63 packed into 12
bytes the way kernels/proj_q4k.comp:46-58 (get_scale_min_k4) unpacks them;
128 bytes of nibbles uniform in 0..15.
"""
from __future__ import annotations

import numpy as np

Q8_0_BLOCK = 34
Q4_K_BLOCK = 144


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """(..., 8) 6-bit scales and mins -> (..., 12) bytes.

    Inverse of get_scale_min_k4: for j < 4 the low 6 bits of byte j / j+4 hold
    sc[j] / m[j]; for j >= 4 byte j+4 holds sc[j] & 15 | (m[j] & 15) << 4 and the
    top two bits of bytes j-4 / j hold sc[j] >> 4 / m[j] >> 4.
    """
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 15) | ((mn[..., 4:8] & 15) << 4)
    return out


def q8_0_blocks(rows: int, k: int, rng: np.random.Generator, d_scale: float = 0.02 / 127) -> np.ndarray:
    """rows x k weights as raw Q8_0 bytes, shape (rows, k/32*34)."""
    assert k % 32 == 0
    nb = rows * (k // 32)
    d = (np.abs(rng.standard_normal(nb)) * d_scale).astype(np.float16)
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
    blk = np.empty((nb, Q8_0_BLOCK), np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = q.view(np.uint8)
    return blk.reshape(rows, (k // 32) * Q8_0_BLOCK)


def q4k_blocks(rows: int, k: int, rng: np.random.Generator, d_scale: float = 1e-3) -> np.ndarray:
    """rows x k weights as raw Q4_K bytes, shape (rows, k/256*144)."""
    assert k % 256 == 0
    nb = rows * (k // 256)
    d = (np.abs(rng.standard_normal(nb)) * d_scale).astype(np.float16)
    dmin = (np.abs(rng.standard_normal(nb)) * d_scale).astype(np.float16)
    sc = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.int32).astype(np.uint8)
    blk = np.empty((nb, Q4_K_BLOCK), np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
    blk[:, 4:16] = pack_scale_min_k4(sc, mn)
    blk[:, 16:] = qs
    return blk.reshape(rows, (k // 256) * Q4_K_BLOCK)


def weight_blocks(dtype: int, rows: int, k: int, rng: np.random.Generator) -> np.ndarray:
    from .lc import F32, Q4_K, Q8_0

    if dtype == Q4_K:
        return q4k_blocks(rows, k, rng)
    if dtype == Q8_0:
        return q8_0_blocks(rows, k, rng)
    if dtype == F32:
        return (rng.standard_normal((rows, k)) * 0.02).astype(np.float32).view(np.uint8)
    raise ValueError(dtype)


def row_bytes(dtype: int, k: int) -> int:
    from .lc import F32, Q4_K, Q8_0

    return {Q4_K: k // 256 * Q4_K_BLOCK, Q8_0: k // 32 * Q8_0_BLOCK, F32: 4 * k}[dtype]


def activations(m: int, k: int, rng: np.random.Generator) -> np.ndarray:
    return rng.standard_normal((m, k)).astype(np.float32)


def dflash_tensors(hp: dict, wtype: int, rng: np.random.Generator, share: bool = False):
    """Seeded synthetic DFlash draft-model tensors, name -> (dtype, array): the
    quantized projections in `wtype` blocks (BASELINE block distributions), the
    norms f32 near 1.  With share=True one array per distinct projection shape
    serves every layer (a timing model: each layer still gets its own device
    copy, so every layer's weights stream from HBM)."""
    from .lc import F32

    E, H, KV, hd, F, A = (hp[k] for k in ("n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "n_aux"))
    QD, KVD = H * hd, KV * hd
    cache = {}

    def W(rows, k):
        if share and (rows, k) in cache:
            return cache[(rows, k)]
        v = (wtype, weight_blocks(wtype, rows, k, rng).reshape(-1))
        if share:
            cache[(rows, k)] = v
        return v

    def N(n):
        return (F32, (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))

    t = {"fc.weight": W(E, A * E), "enc.aux_norm.weight": N(A * E), "enc.output_norm.weight": N(E),
         "output_norm.weight": N(E)}
    for layer in range(hp["n_layers"]):
        p = f"blk.{layer}."
        t.update({p + "attn_norm.weight": N(E), p + "attn_q.weight": W(QD, E), p + "attn_k.weight": W(KVD, E),
                  p + "attn_v.weight": W(KVD, E), p + "attn_output.weight": W(E, QD),
                  p + "attn_q_norm.weight": N(hd), p + "attn_k_norm.weight": N(hd),
                  p + "attn_gate.weight": W(H, E), p + "ffn_norm.weight": N(E), p + "ffn_gate.weight": W(F, E),
                  p + "ffn_up.weight": W(F, E), p + "ffn_down.weight": W(E, F)})
    return t


def q4k_blocks_centered(rows: int, k: int, rng: np.random.Generator, w_scale: float) -> np.ndarray:
    """rows x k Q4_K weights of mean ~0 and std ~w_scale: dmin = d and each
    sub-block's min = 7.5 x its scale, so w = d * sc * (q - 7.5).  Used where a
    stack of random layers must keep its activations finite (the target model)."""
    assert k % 256 == 0
    nb = rows * (k // 256)
    d = (np.abs(rng.standard_normal(nb)) * w_scale / (4.6 * 4.5) + 1e-6).astype(np.float16)
    sc = rng.integers(1, 9, size=(nb, 8))
    blk = np.empty((nb, Q4_K_BLOCK), np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 4:16] = pack_scale_min_k4(sc, np.rint(7.5 * sc))
    blk[:, 16:] = rng.integers(0, 256, size=(nb, 128)).astype(np.uint8)
    return blk.reshape(rows, (k // 256) * Q4_K_BLOCK)


def target_tensors(hp: dict, rng: np.random.Generator, share: bool = True):
    """Seeded synthetic target (Laguna) tensors, name -> (dtype, array, GGUF
    shape): Q4_K projections and expert stacks of std ~0.5/sqrt(k), Q8_0 token
    embeddings and output, f32 norms, router and bias.  Layer 0 is dense, the
    others MoE (when n_expert > 0).  With share=True one array per distinct
    shape serves every layer and expert (a timing model: each still gets its
    own device copy)."""
    from .lc import F32, Q4_K, Q8_0

    E, H, KV, hd, F = (hp[k] for k in ("n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff"))
    NE, Fe, S, V = hp["n_expert"], hp["n_ff_exp"], hp["n_ff_shexp"], hp["n_vocab"]
    QD, KVD = H * hd, KV * hd
    cache = {}

    def W(rows, k, shape):
        key = ("q4", rows, k)
        if not (share and key in cache):
            cache[key] = q4k_blocks_centered(rows, k, rng, 0.5 / np.sqrt(k)).reshape(-1)
        return (Q4_K, cache[key], shape)

    def stack(rows, k, shape):
        one = W(rows, k, None)[1]
        return (Q4_K, np.concatenate([one if share else
                                      q4k_blocks_centered(rows, k, rng, 0.5 / np.sqrt(k)).reshape(-1)
                                      for _ in range(NE)]), shape)

    def N(n):
        return (F32, (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32), (n,))

    def Q8(rows, k):
        return (Q8_0, q8_0_blocks(rows, k, rng, d_scale=0.5 / (58.0 * np.sqrt(k))).reshape(-1), (k, rows))

    t = {"token_embd.weight": Q8(V, E), "output.weight": Q8(V, E), "output_norm.weight": N(E)}
    for layer in range(hp["n_layers"]):
        p = f"blk.{layer}."
        t.update({p + "attn_norm.weight": N(E), p + "ffn_norm.weight": N(E), p + "attn_q_norm.weight": N(hd),
                  p + "attn_k_norm.weight": N(hd), p + "attn_q.weight": W(QD, E, (E, QD)),
                  p + "attn_k.weight": W(KVD, E, (E, KVD)), p + "attn_v.weight": W(KVD, E, (E, KVD)),
                  p + "attn_output.weight": W(E, QD, (QD, E)), p + "attn_gate.weight": W(H, E, (E, H))})
        if NE and layer > 0:
            t.update({p + "ffn_gate_inp.weight": (F32, (rng.standard_normal(NE * E) / np.sqrt(E)).astype(np.float32),
                                                  (E, NE)),
                      p + "exp_probs_b.bias": (F32, (0.02 * rng.permutation(NE)).astype(np.float32), (NE,)),
                      p + "ffn_gate_exps.weight": stack(Fe, E, (E, Fe, NE)),
                      p + "ffn_up_exps.weight": stack(Fe, E, (E, Fe, NE)),
                      p + "ffn_down_exps.weight": stack(E, Fe, (Fe, E, NE)),
                      p + "ffn_gate_shexp.weight": W(S, E, (E, S)), p + "ffn_up_shexp.weight": W(S, E, (E, S)),
                      p + "ffn_down_shexp.weight": W(E, S, (S, E))})
        else:
            t.update({p + "ffn_gate.weight": W(F, E, (E, F)), p + "ffn_up.weight": W(F, E, (E, F)),
                      p + "ffn_down.weight": W(E, F, (F, E))})
    return t


def target_meta(hp: dict) -> dict:
    """GGUF metadata of a synthetic target model (laguna.* keys)."""
    return {"general.architecture": "laguna", "laguna.block_count": hp["n_layers"],
            "laguna.embedding_length": hp["n_embd"], "laguna.feed_forward_length": hp["n_ff"],
            "laguna.attention.head_count": hp["n_heads"], "laguna.attention.head_count_kv": hp["n_kv_heads"],
            "laguna.attention.key_length": hp["head_dim"], "laguna.rope.dimension_count": hp["rope_dim"],
            "laguna.rope.dimension_count_swa": hp["rope_dim_swa"], "expert.count": hp["n_expert"],
            "expert.used_count": hp["n_expert_used"], "expert.feed_forward_length": hp["n_ff_exp"],
            "expert.shared_feed_forward_length": hp["n_ff_shexp"], "laguna.expert_weights_norm": True,
            "laguna.expert_weights_scale": 2.5}
