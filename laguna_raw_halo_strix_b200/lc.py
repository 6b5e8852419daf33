"""ctypes binding of liblaguna_cuda.so (the C ABI declared in include/laguna_cuda.h).

This module is a thin host-side mirror of the reference's dispatch helpers
(src/dflash.rs:979-1327, src/target.rs:1086-1162): every method enqueues one
library call on the context's stream.  Arguments are device pointers (ints) or
torch CUDA tensors; torch is used only for device memory and streams.

There is no CPU fallback: if the shared library cannot be loaded (or built
with nvcc), importing the functions raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "liblaguna_cuda.so")
CSRC = os.path.join(PKG, "csrc")

LC_OK = 0
LC_ERR_INVALID = 1
LC_ERR_UNSUPPORTED = 2
LC_ERR_CUDA = 3
LC_ERR_OOM = 4
LC_ERR_TIMEOUT = 5
LC_ERR_IO = 6

F32 = 0
F16 = 1
Q8_0 = 8
Q4_K = 12
BF16 = 30
Q4_K_DFLASH_CPU = 1012

HALF_REF = 0
HALF_IEEE = 1

LOAD_BF16_NATIVE = 1  # lc_dflash_load_gguf_ex flag

_STATUS = {0: "LC_OK", 1: "LC_ERR_INVALID", 2: "LC_ERR_UNSUPPORTED", 3: "LC_ERR_CUDA", 4: "LC_ERR_OOM",
           5: "LC_ERR_TIMEOUT", 6: "LC_ERR_IO"}


class LagunaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{_STATUS.get(status, status)}: {msg}")
        self.status = status


_lock = threading.Lock()
_lib = None

_vp = C.c_void_p
_u32 = C.c_uint32
_f = C.c_float
_sz = C.c_size_t
_i = C.c_int

# name -> (restype, argtypes)
SIGNATURES = {
    "lc_last_error": (C.c_char_p, []),
    "lc_version": (C.c_char_p, []),
    "lc_device_count": (_i, [C.POINTER(_i)]),
    "lc_init": (_i, [_i, C.POINTER(_vp)]),
    "lc_destroy": (_i, [_vp]),
    "lc_set_stream": (_i, [_vp, _vp]),
    "lc_get_stream": (_vp, [_vp]),
    "lc_synchronize": (_i, [_vp]),
    "lc_set_sync": (_i, [_vp, _i]),
    "lc_set_half_mode": (_i, [_vp, _i]),
    "lc_ctx_device": (_i, [_vp, C.POINTER(_i)]),
    "lc_ctx_scratch_bytes": (_i, [_vp, C.POINTER(_sz)]),
    "lc_buf_alloc": (_i, [_vp, _sz, C.POINTER(_vp)]),
    "lc_buf_free": (_i, [_vp]),
    "lc_buf_device_ptr": (_vp, [_vp]),
    "lc_buf_size": (_sz, [_vp]),
    "lc_buf_upload": (_i, [_vp, _vp, _sz]),
    "lc_buf_upload_at": (_i, [_vp, _sz, _vp, _sz]),
    "lc_buf_read": (_i, [_vp, _sz, _vp, _sz]),
    "lc_buf_read_f32": (_i, [_vp, C.POINTER(_f), _sz]),
    "lc_proj_f32": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_proj_q8_0": (_i, [_vp, _vp, _vp, _vp, _u32, _u32]),
    "lc_proj_q4k": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_proj_quant": (_i, [_vp, _i, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_device_status": (_i, [_vp]),
    "lc_proj_m": (_i, [_vp, _i, _vp, _vp, _vp, _u32, _u32, _u32, _u32]),
    "lc_proj_q4k_static": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32]),
    "lc_ffn": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_ffn_host": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_proj_m_host": (_i, [_vp, _i, _vp, _vp, _vp, _u32, _u32, _u32, _u32]),
    "lc_comm_unique_id": (_i, [_vp]),
    "lc_comm_init": (_i, [_vp, _vp, _i, _i, _i, C.POINTER(_vp)]),
    "lc_comm_destroy": (_i, [_vp]),
    "lc_comm_rank": (_i, [_vp, C.POINTER(_i), C.POINTER(_i)]),
    "lc_comm_allreduce_max_keys": (_i, [_vp, _vp, _vp, _u32]),
    "lc_comm_wait": (_i, [_vp, _vp]),
    "lc_lm_head_argmax_sharded": (_i, [_vp, _vp, _i, _vp, _vp, _u32, _u32, _u32, _u32, _vp]),
    "lc_check_bounded_wait": (_i, [_vp, _u32]),
    "lc_dequant": (_i, [_vp, _i, _vp, _sz, _sz, _vp]),
    "lc_rmsnorm": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _f]),
    "lc_qk_norm_rope": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _f, _u32]),
    "lc_activation": (_i, [_vp, _vp, _vp, _vp, _u32]),
    "lc_add": (_i, [_vp, _vp, _vp, _vp, _u32]),
    "lc_gate_mul": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "lc_softplus": (_i, [_vp, _vp, _vp, _u32]),
    "lc_enc_aux_norm": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _f]),
    "lc_mha_attn": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f, _u32, _u32]),
    "lc_rope_freq": (_i, [C.POINTER(_f), _u32, _f]),
    "lc_pack_key": (C.c_uint64, [_f, _u32]),
    "lc_key_value": (_f, [C.c_uint64]),
    "lc_key_index": (_u32, [C.c_uint64]),
    "lc_argmax_rows": (_i, [_vp, _vp, _u32, _u32, _u32, _vp]),
    "lc_lm_head_argmax": (_i, [_vp, _i, _vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp]),
    # GGUF reader
    "lc_type_block_bytes": (C.c_uint64, [_i]),
    "lc_type_block_elements": (C.c_uint64, [_i]),
    "lc_tensor_bytes": (C.c_uint64, [_i, C.c_uint64]),
    "lc_gguf_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
    "lc_gguf_close": (_i, [_vp]),
    "lc_gguf_tensor_count": (C.c_uint64, [_vp]),
    "lc_gguf_tensor_info": (_i, [_vp, C.c_uint64, C.POINTER(C.c_char_p), C.POINTER(_i), C.POINTER(_u32),
                                 C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "lc_gguf_find": (_i, [_vp, C.c_char_p, C.POINTER(C.c_uint64)]),
    "lc_gguf_read": (_i, [_vp, C.c_uint64, _vp, C.c_uint64]),
    "lc_gguf_tensor_data": (_i, [_vp, C.c_uint64, C.POINTER(_vp), C.POINTER(C.c_uint64)]),
    "lc_gguf_meta_u64": (_i, [_vp, C.c_char_p, C.POINTER(C.c_uint64)]),
    "lc_gguf_meta_f32": (_i, [_vp, C.c_char_p, C.POINTER(_f)]),
    "lc_gguf_meta_str": (_i, [_vp, C.c_char_p, C.POINTER(C.c_char_p)]),
    "lc_gguf_dflash_hparams": (_i, [_vp, _vp]),
    # DFlash model
    "lc_dflash_create": (_i, [_vp, _vp, _u32, _u32, C.POINTER(_vp)]),
    "lc_dflash_set_tensor": (_i, [_vp, C.c_char_p, _i, _vp, _sz]),
    "lc_dflash_load_gguf": (_i, [_vp, C.c_char_p, _u32, _u32, C.POINTER(_vp)]),
    "lc_dflash_load_gguf_ex": (_i, [_vp, C.c_char_p, _u32, _u32, _u32, C.POINTER(_vp)]),
    "lc_dflash_weight": (_i, [_vp, C.c_char_p, C.POINTER(_vp), C.POINTER(_i), C.POINTER(C.c_uint64)]),
    # target model
    "lc_gguf_target_hparams": (_i, [_vp, _vp]),
    "lc_gguf_target_layers": (_i, [_vp, C.POINTER(C.c_int64), _u32, C.POINTER(_u32)]),
    "lc_target_load_gguf": (_i, [_vp, C.c_char_p, _u32, _u32, _u32, C.POINTER(_vp)]),
    "lc_target_destroy": (_i, [_vp]),
    "lc_target_get_hparams": (_i, [_vp, _vp]),
    "lc_target_layer_info": (_i, [_vp, _u32, C.POINTER(_u32), C.POINTER(_u32)]),
    "lc_target_weight": (_i, [_vp, C.c_char_p, C.POINTER(_vp), C.POINTER(_i), C.POINTER(C.c_uint64)]),
    "lc_target_embed": (_i, [_vp, C.POINTER(_u32), _u32, _vp]),
    "lc_target_forward": (_i, [_vp, _vp, _u32, _u32, C.POINTER(_u32), _u32, _vp, _vp, _vp, _vp]),
    "lc_target_routing": (_i, [_vp, _u32, _vp, C.POINTER(_u32)]),
    "lc_target_cache_len": (_i, [_vp, C.POINTER(_u32)]),
    "lc_target_cache_truncate": (_i, [_vp, _u32]),
    "lc_target_moe_ffn": (_i, [_vp, _u32, _vp, _u32, _vp, _vp, _vp]),
    "lc_dflash_destroy": (_i, [_vp]),
    "lc_dflash_get_hparams": (_i, [_vp, _vp]),
    "lc_dflash_encode": (_i, [_vp, _vp, _u32, _vp]),
    "lc_dflash_set_context": (_i, [_vp, _vp, _u32]),
    "lc_dflash_decode_block": (_i, [_vp, _vp, _u32, _vp]),
    "lc_dflash_forward_injected_decode_hidden": (_i, [_vp, _vp, _vp, _vp]),
    "lc_dflash_forward_from_input": (_i, [_vp, _vp, _vp, _vp, C.POINTER(_u32)]),
    "lc_dflash_forward_token": (_i, [_vp, _u32, _vp, _vp, C.POINTER(_u32)]),
}


class HParams(C.Structure):
    """lc_dflash_hparams (include/laguna_cuda.h)."""

    _fields_ = [("n_layers", _u32), ("n_embd", _u32), ("n_heads", _u32), ("n_kv_heads", _u32),
                ("head_dim", _u32), ("rope_dim", _u32), ("n_ff", _u32), ("n_aux", _u32),
                ("rope_base", _f), ("norm_eps", _f), ("qk_eps", _f)]


class TargetHParams(C.Structure):
    """lc_target_hparams (include/laguna_cuda.h)."""

    _fields_ = [("n_layers", _u32), ("n_embd", _u32), ("n_ff", _u32), ("n_heads", _u32), ("n_kv_heads", _u32),
                ("head_dim", _u32), ("rope_dim", _u32), ("rope_dim_swa", _u32), ("swa", _u32),
                ("n_expert", _u32), ("n_expert_used", _u32), ("n_ff_exp", _u32), ("n_ff_shexp", _u32),
                ("has_moe", _u32), ("has_shexp", _u32), ("expert_weights_norm", _u32), ("n_vocab", _u32),
                ("rope_base", _f), ("rope_base_swa", _f), ("expert_weights_scale", _f), ("norm_eps", _f),
                ("qk_eps", _f)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


TARGET_CACHED = 1  # lc_target_forward flag
TARGET_REF_EXPERT_OFFSET = 2  # lc_target_load_gguf flag


def _sources_newer(lib: str) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    for d in (CSRC, os.path.join(os.path.dirname(PKG), "include")):
        for f in os.listdir(d):
            if f.endswith((".cu", ".cuh", ".h", ".cpp", ".hpp")) and os.path.getmtime(os.path.join(d, f)) > t:
                return True
    return False


def build(force: bool = False) -> str:
    """Compile the CUDA library in-tree (nvcc, sm_100a)."""
    if force or _sources_newer(LIB_PATH):
        subprocess.run(["make", "-s", "-j8", "-C", CSRC], check=True)
    return LIB_PATH


def lib():
    """Load liblaguna_cuda.so (building it with nvcc if it is missing or stale)."""
    global _lib
    with _lock:
        if _lib is None:
            path = build()
            L = C.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return lib().lc_last_error().decode()


def check(status: int, what: str = "") -> None:
    if status != LC_OK:
        raise LagunaError(status, f"{what}: {last_error()}" if what else last_error())


def ptr(t) -> int:
    """Device pointer of a torch tensor / int / None."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return t.data_ptr()


def pack_key(value: float, index: int) -> int:
    return int(lib().lc_pack_key(value, index))


def key_value(key: int) -> float:
    return float(lib().lc_key_value(key & 0xFFFFFFFFFFFFFFFF))


def key_index(key: int) -> int:
    return int(lib().lc_key_index(key & 0xFFFFFFFFFFFFFFFF))


class Context:
    """An lc_ctx: one device, one stream (by default torch's current stream)."""

    def __init__(self, device: int = 0, stream=None, sync: bool = False):
        self.L = lib()
        h = C.c_void_p()
        check(self.L.lc_init(device, C.byref(h)), "lc_init")
        self.h = h
        self.device = device
        if stream is not None:
            self.set_stream(stream)
        if sync:
            check(self.L.lc_set_sync(self.h, 1))

    def close(self):
        if getattr(self, "h", None):
            self.L.lc_destroy(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream) -> None:
        """stream: torch.cuda.Stream, raw cudaStream_t int, or None (the context's
        own stream).  A torch stream whose handle is 0 (torch's default stream) maps
        to cudaStreamLegacy, so the work really runs on that stream: a NULL handle
        would select the context's own stream instead."""
        if stream is None:
            raw = None
        elif hasattr(stream, "cuda_stream"):
            raw = stream.cuda_stream or 0x1  # cudaStreamLegacy
        else:
            raw = stream or None
        check(self.L.lc_set_stream(self.h, raw), "lc_set_stream")

    def synchronize(self) -> None:
        check(self.L.lc_synchronize(self.h), "lc_synchronize")

    def set_half_mode(self, mode: int) -> None:
        check(self.L.lc_set_half_mode(self.h, mode), "lc_set_half_mode")

    # -- projections -----------------------------------------------------------
    def proj_f32(self, x, w, c, k, n, row_major=0):
        check(self.L.lc_proj_f32(self.h, ptr(x), ptr(w), ptr(c), k, n, row_major), "lc_proj_f32")

    def proj_q8_0(self, x, w, c, k, n):
        check(self.L.lc_proj_q8_0(self.h, ptr(x), ptr(w), ptr(c), k, n), "lc_proj_q8_0")

    def proj_q4k(self, x, w, c, k, n, expert_offset=0):
        check(self.L.lc_proj_q4k(self.h, ptr(x), ptr(w), ptr(c), k, n, expert_offset), "lc_proj_q4k")

    def proj_quant(self, dtype, x, w, c, k, n, expert_offset=0):
        check(self.L.lc_proj_quant(self.h, dtype, ptr(x), ptr(w), ptr(c), k, n, expert_offset), "lc_proj_quant")

    def device_status(self):
        check(self.L.lc_device_status(self.h), "lc_device_status")

    def proj_m(self, dtype, x, w, c, m, k, n, expert_offset=0):
        check(self.L.lc_proj_m(self.h, dtype, ptr(x), ptr(w), ptr(c), m, k, n, expert_offset), "lc_proj_m")

    def scratch_bytes(self) -> int:
        v = _sz(0)
        check(self.L.lc_ctx_scratch_bytes(self.h, C.byref(v)), "lc_ctx_scratch_bytes")
        return int(v.value)

    def proj_q4k_static(self, x, w, c, m, k, n, expert_offset=0):
        check(self.L.lc_proj_q4k_static(self.h, ptr(x), ptr(w), ptr(c), m, k, n, expert_offset),
              "lc_proj_q4k_static")

    def ffn(self, dtype, x, w_gate, w_up, w_down, y, m, n_embd, n_ff):
        check(self.L.lc_ffn(self.h, dtype, ptr(x), ptr(w_gate), ptr(w_up), ptr(w_down), ptr(y), m, n_embd, n_ff),
              "lc_ffn")

    def ffn_host(self, dtype, x_host, w_gate, w_up, w_down, y_host, m, n_embd, n_ff):
        """lc_ffn_host: x_host / y_host are host buffers (page-locked for
        asynchronous copies); returns once y_host holds the result."""
        check(self.L.lc_ffn_host(self.h, dtype, ptr(x_host), ptr(w_gate), ptr(w_up), ptr(w_down), ptr(y_host), m,
                                 n_embd, n_ff), "lc_ffn_host")

    def proj_m_host(self, dtype, x_host, w, c_host, m, k, n, expert_offset=0):
        check(self.L.lc_proj_m_host(self.h, dtype, ptr(x_host), ptr(w), ptr(c_host), m, k, n, expert_offset),
              "lc_proj_m_host")

    def dequant(self, dtype, src, src_bytes, n, out):
        check(self.L.lc_dequant(self.h, dtype, ptr(src), src_bytes, n, ptr(out)), "lc_dequant")

    # -- interleaved ops ---------------------------------------------------------
    def rmsnorm(self, w, x, out, m, n, eps=1e-5):
        check(self.L.lc_rmsnorm(self.h, ptr(w), ptr(x), ptr(out), m, n, eps), "lc_rmsnorm")

    def qk_norm_rope(self, x, w, freq, out, m, n_heads, head_dim, rope_dim, eps, pos0):
        check(self.L.lc_qk_norm_rope(self.h, ptr(x), ptr(w), ptr(freq), ptr(out), m, n_heads, head_dim, rope_dim,
                                     eps, pos0), "lc_qk_norm_rope")

    def activation(self, gate, up, h, n):
        check(self.L.lc_activation(self.h, ptr(gate), ptr(up), ptr(h), n), "lc_activation")

    def add(self, a, b, c, n):
        check(self.L.lc_add(self.h, ptr(a), ptr(b), ptr(c), n), "lc_add")

    def gate_mul(self, v, gate, out, n_hd, n_heads, head_dim):
        check(self.L.lc_gate_mul(self.h, ptr(v), ptr(gate), ptr(out), n_hd, n_heads, head_dim), "lc_gate_mul")

    def softplus(self, g, out, n):
        check(self.L.lc_softplus(self.h, ptr(g), ptr(out), n), "lc_softplus")

    def enc_aux_norm(self, x, w, y, n_feat, n_aux, n_tokens, eps=1e-5):
        check(self.L.lc_enc_aux_norm(self.h, ptr(x), ptr(w), ptr(y), n_feat, n_aux, n_tokens, eps),
              "lc_enc_aux_norm")

    def mha_attn(self, q, k, v, out, m, n_q_heads, n_kv_heads, head_dim, seq_len, scale, q_pos0, causal=1):
        check(self.L.lc_mha_attn(self.h, ptr(q), ptr(k), ptr(v), ptr(out), m, n_q_heads, n_kv_heads, head_dim,
                                 seq_len, scale, q_pos0, causal), "lc_mha_attn")

    def argmax_rows(self, logits, m, n, row_offset, keys):
        check(self.L.lc_argmax_rows(self.h, ptr(logits), m, n, row_offset, ptr(keys)), "lc_argmax_rows")

    def check_bounded_wait(self, spins: int = 1024) -> None:
        check(self.L.lc_check_bounded_wait(self.h, spins), "lc_check_bounded_wait")

    def lm_head_argmax(self, dtype, x, w, m, k, n_local, row_offset, keys, logits=None):
        check(self.L.lc_lm_head_argmax(self.h, dtype, ptr(x), ptr(w), m, k, n_local, row_offset, ptr(keys),
                                       ptr(logits)), "lc_lm_head_argmax")


def comm_unique_id() -> bytes:
    """128-byte id for Comm, made by one rank and passed to the others."""
    buf = C.create_string_buffer(128)
    check(lib().lc_comm_unique_id(buf), "lc_comm_unique_id")
    return buf.raw


class Comm:
    """An lc_comm: the library's NCCL communicator over the ranks' contexts."""

    def __init__(self, ctx: Context, unique_id: bytes, n_ranks: int, rank: int, timeout_ms: int = 30000):
        self.ctx, self.L = ctx, lib()
        assert len(unique_id) == 128
        h = C.c_void_p()
        check(self.L.lc_comm_init(ctx.h, C.create_string_buffer(unique_id, 128), n_ranks, rank, timeout_ms,
                                  C.byref(h)), "lc_comm_init")
        self.h = h
        self.rank, self.n_ranks = rank, n_ranks

    def allreduce_max_keys(self, keys, n):
        check(self.L.lc_comm_allreduce_max_keys(self.ctx.h, self.h, ptr(keys), n), "lc_comm_allreduce_max_keys")

    def wait(self):
        check(self.L.lc_comm_wait(self.ctx.h, self.h), "lc_comm_wait")

    def lm_head_argmax(self, dtype, x, w, m, k, n_local, row_offset, keys):
        check(self.L.lc_lm_head_argmax_sharded(self.ctx.h, self.h, dtype, ptr(x), ptr(w), m, k, n_local, row_offset,
                                               ptr(keys)), "lc_lm_head_argmax_sharded")

    def close(self):
        if getattr(self, "h", None):
            status = self.L.lc_comm_destroy(self.h)
            self.h = None
            check(status, "lc_comm_destroy")


def rope_freq(rope_dim: int, base: float = 500000.0):
    import numpy as np

    f = np.empty(max(rope_dim // 2, 1), np.float32)
    check(lib().lc_rope_freq(f.ctypes.data_as(C.POINTER(C.c_float)), rope_dim, base), "lc_rope_freq")
    return f[: rope_dim // 2]
