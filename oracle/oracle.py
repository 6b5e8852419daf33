"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two CPU implementations live under oracle/:

* `liblaguna_oracle.so` -- the C restatement of the reference path
  (laguna_oracle.c); always available (built by `make -C oracle`).
* `_ref/libref_shaders.so` -- laguna-raw's own GLSL shader sources compiled for
  the CPU by build_ref.py.  It can only be built where the reference tree is
  present; the built .so travels with the repository snapshot.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
import this module.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liblaguna_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_shaders.so")

F32 = 0
F16 = 1
Q8_0 = 8
Q4_K = 12
BF16 = 30

_fp = C.POINTER(C.c_float)
_u8 = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)


def _p(a, t=_fp):
    return a.ctypes.data_as(t)


def build_oracle() -> str:
    src = os.path.join(HERE, "laguna_oracle.c")
    if not os.path.exists(ORACLE_LIB) or os.path.getmtime(ORACLE_LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return ORACLE_LIB


def reference_tree() -> str:
    """Where the reference source tree is read from: $LAGUNA_REFERENCE, else a
    directory named `reference` beside this repository's root."""
    return os.environ.get("LAGUNA_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build_ref(reference: str | None = None) -> str | None:
    """Build oracle/_ref when the reference tree exists; return its path or None."""
    reference = reference or reference_tree()
    if os.path.exists(REF_LIB):
        return REF_LIB
    if not os.path.isdir(os.path.join(reference, "kernels")):
        return None
    from build_ref import build  # type: ignore  # noqa: E402

    return build(reference)


class Oracle:
    """The C restatement (laguna_oracle.c)."""

    def __init__(self, threads: int = 0):
        self.lib = C.CDLL(build_oracle())
        L = self.lib
        L.lco_half_to_f32_ref.restype = C.c_float
        L.lco_half_to_f32_ref.argtypes = [C.c_uint16]
        L.lco_half_to_f32_ieee.restype = C.c_float
        L.lco_half_to_f32_ieee.argtypes = [C.c_uint16]
        L.lco_dequant_to_f32.argtypes = [_u8, C.c_size_t, C.c_int, C.c_size_t, _fp]
        L.lco_dequant_shader.argtypes = [_u8, C.c_int, C.c_size_t, _fp]
        L.lco_proj_f32_m.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.lco_proj_q8_0_m.argtypes = [_fp, _u8, _fp, C.c_uint32, C.c_uint32, C.c_uint32]
        L.lco_proj_q4k_m.argtypes = [_fp, _u8, _fp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.lco_rmsnorm.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_float]
        L.lco_qk_norm_rope.argtypes = [_fp, _fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_uint32,
                                       C.c_uint32, C.c_float, _u32p]
        L.lco_activation.argtypes = [_fp, _fp, _fp, C.c_uint32]
        L.lco_add.argtypes = [_fp, _fp, _fp, C.c_uint32]
        L.lco_gate_mul.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32]
        L.lco_softplus.argtypes = [_fp, _fp, C.c_uint32]
        L.lco_mha_attn.argtypes = [_fp, _fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_uint32,
                                   C.c_uint32, C.c_float, C.c_uint32, C.c_uint32]
        L.lco_enc_aux_norm.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]
        L.lco_rope_freq.argtypes = [_fp, C.c_uint32, C.c_float]
        L.lco_argmax.restype = C.c_size_t
        L.lco_argmax.argtypes = [_fp, C.c_size_t]
        L.lco_gate_attn.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32]
        L.lco_moe_select.restype = C.c_uint32
        L.lco_moe_select.argtypes = [_fp, _fp, C.c_uint32, C.c_uint32, C.c_int, C.c_float,
                                     C.POINTER(C.c_int32), _fp]
        L.lco_moe_l2_scale.restype = C.c_float
        L.lco_moe_l2_scale.argtypes = [_fp, C.c_uint32, _fp]
        L.lco_set_threads.argtypes = [C.c_int]
        L.lco_get_threads.restype = C.c_int
        if threads:
            L.lco_set_threads(threads)

    # -- scalar / dequant ---------------------------------------------------
    def half_ref(self, h: int) -> float:
        return self.lib.lco_half_to_f32_ref(h)

    def half_ieee(self, h: int) -> float:
        return self.lib.lco_half_to_f32_ieee(h)

    def dequant_to_f32(self, data: bytes | np.ndarray, dtype: int, n: int) -> np.ndarray:
        buf = np.frombuffer(bytes(data), np.uint8).copy() if not isinstance(data, np.ndarray) else \
            np.ascontiguousarray(data, np.uint8)
        if buf.size == 0:
            buf = np.zeros(1, np.uint8)
            nbytes = 0
        else:
            nbytes = buf.size
        out = np.empty(max(n, 1), np.float32)
        self.lib.lco_dequant_to_f32(_p(buf, _u8), nbytes, dtype, n, _p(out))
        return out[:n]

    def dequant_shader(self, w: np.ndarray, dtype: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.lib.lco_dequant_shader(_p(np.ascontiguousarray(w, np.uint8), _u8), dtype, n, _p(out))
        return out

    # -- projections ----------------------------------------------------------
    def proj(self, dtype: int, x: np.ndarray, w: np.ndarray, k: int, n: int,
             expert_offset: int = 0, row_major: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        m = x.size // k
        c = np.empty((m, n), np.float32)
        if dtype == F32:
            self.lib.lco_proj_f32_m(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(c), m, k, n, row_major)
        elif dtype == Q8_0:
            self.lib.lco_proj_q8_0_m(_p(x), _p(np.ascontiguousarray(w, np.uint8), _u8), _p(c), m, k, n)
        elif dtype == Q4_K:
            self.lib.lco_proj_q4k_m(_p(x), _p(np.ascontiguousarray(w, np.uint8), _u8), _p(c), m, k, n,
                                    expert_offset)
        else:
            raise ValueError(f"unsupported dtype {dtype}")
        return c if x.ndim > 1 else c[0]

    # -- interleaved ops ------------------------------------------------------
    def rmsnorm(self, x, w, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        n = w.size
        y = np.empty_like(x)
        self.lib.lco_rmsnorm(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(y), x.size // n, n, eps)
        return y

    def qk_norm_rope(self, x, w, freq, n_heads, head_dim, rope_dim, eps, pos):
        # The shader's pair index leaves the head unless rope_dim is 0 or head_dim.
        if rope_dim not in (0, head_dim):
            raise ValueError("qk_norm_rope: rope_dim must be 0 or head_dim")
        x = np.ascontiguousarray(x, np.float32)
        m = x.size // (n_heads * head_dim)
        pos = np.ascontiguousarray(np.broadcast_to(np.asarray(pos, np.uint32), (m,)), np.uint32)
        y = np.empty_like(x)
        self.lib.lco_qk_norm_rope(_p(x), _p(np.ascontiguousarray(w, np.float32)),
                                  _p(np.ascontiguousarray(freq, np.float32)), _p(y), m, n_heads,
                                  head_dim, rope_dim, eps, _p(pos, _u32p))
        return y

    def activation(self, gate, up):
        g = np.ascontiguousarray(gate, np.float32)
        h = np.empty_like(g)
        self.lib.lco_activation(_p(g), _p(np.ascontiguousarray(up, np.float32)), _p(h), g.size)
        return h

    def add(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        c = np.empty_like(a)
        self.lib.lco_add(_p(a), _p(np.ascontiguousarray(b, np.float32)), _p(c), a.size)
        return c

    def gate_mul(self, v, gate, head_dim):
        v = np.ascontiguousarray(v, np.float32)
        out = np.empty_like(v)
        self.lib.lco_gate_mul(_p(v), _p(np.ascontiguousarray(gate, np.float32)), _p(out), v.size, head_dim)
        return out

    def softplus(self, g):
        g = np.ascontiguousarray(g, np.float32)
        out = np.empty_like(g)
        self.lib.lco_softplus(_p(g), _p(out), g.size)
        return out

    def mha_attn(self, q, k, v, n_q_heads, n_kv_heads, head_dim, seq_len, scale, q_pos, causal=1):
        q = np.ascontiguousarray(q, np.float32)
        out = np.empty(n_q_heads * head_dim, np.float32)
        self.lib.lco_mha_attn(_p(q), _p(np.ascontiguousarray(k, np.float32)),
                              _p(np.ascontiguousarray(v, np.float32)), _p(out), n_q_heads, n_kv_heads,
                              head_dim, seq_len, scale, q_pos, causal)
        return out

    def enc_aux_norm(self, x, w, n_feat, n_aux, n_tokens, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.lco_enc_aux_norm(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(y), n_feat, n_aux,
                                  n_tokens, eps)
        return y

    def rope_freq(self, rope_dim, base=500000.0):
        f = np.empty(rope_dim // 2, np.float32)
        self.lib.lco_rope_freq(_p(f), rope_dim, base)
        return f

    # -- target model --------------------------------------------------------
    def gate_attn(self, attn, gate, n_heads, head_dim):
        a = np.ascontiguousarray(attn, np.float32)
        out = np.empty_like(a)
        self.lib.lco_gate_attn(_p(a), _p(np.ascontiguousarray(gate, np.float32)), _p(out), n_heads, head_dim)
        return out

    def moe_select(self, logits, bias, n_used, norm=False, scale=1.0):
        lg = np.ascontiguousarray(logits, np.float32)
        ids = np.zeros(n_used, np.int32)
        sc = np.zeros(n_used, np.float32)
        n = self.lib.lco_moe_select(_p(lg), _p(np.ascontiguousarray(bias, np.float32)), lg.size, n_used,
                                    int(bool(norm)), scale, ids.ctypes.data_as(C.POINTER(C.c_int32)), _p(sc))
        return ids[:n], sc[:n]

    def moe_l2_scale(self, h):
        h = np.ascontiguousarray(h, np.float32)
        out = np.empty_like(h)
        col = self.lib.lco_moe_l2_scale(_p(h), h.size, _p(out))
        return out, np.float32(col)

    def argmax(self, logits) -> int:
        l = np.ascontiguousarray(logits, np.float32)
        return int(self.lib.lco_argmax(_p(l), l.size))


class RefShaders:
    """laguna-raw's GLSL shaders compiled for the CPU (oracle/_ref)."""

    def __init__(self, path: str | None = None):
        path = path or REF_LIB
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)

    def run(self, name: str, buffers: list[np.ndarray], push: bytes, invocations: int) -> None:
        fn = getattr(self.lib, "ref_" + name)
        fn.argtypes = [C.POINTER(C.c_void_p), C.c_void_p, C.c_uint32]
        arr = (C.c_void_p * len(buffers))(*[b.ctypes.data for b in buffers])
        pb = C.create_string_buffer(push, max(len(push), 4))
        fn(arr, C.cast(pb, C.c_void_p), invocations)

    @staticmethod
    def groups(n: int) -> int:
        """Invocation count of a dispatch of ceil(n/256) workgroups of 256."""
        return ((n + 255) // 256) * 256


def pad4(w: np.ndarray) -> np.ndarray:
    """Byte buffer padded to a whole number of 32-bit words (a `uint[]` binding)."""
    b = np.ascontiguousarray(w, np.uint8).ravel()
    pad = (-b.size) % 4
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.uint8)])
    return b
