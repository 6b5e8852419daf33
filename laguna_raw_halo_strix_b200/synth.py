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
