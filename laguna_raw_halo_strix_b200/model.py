"""Host-side handles for the GGUF reader and the DFlash draft model of the C ABI
(lc_gguf_*, lc_dflash_* in include/laguna_cuda.h).  The model logic itself is
C++ in the library; these classes only marshal arguments."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lc

_TYPE_NAMES = {lc.F32: "F32", lc.F16: "F16", lc.Q8_0: "Q8_0", lc.Q4_K: "Q4_K", lc.BF16: "BF16"}


class Gguf:
    """GGUFReader (src/gguf.rs:321-421) over lc_gguf_*."""

    def __init__(self, path: str):
        self.L = lc.lib()
        h = C.c_void_p()
        lc.check(self.L.lc_gguf_open(path.encode(), C.byref(h)), "lc_gguf_open")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.L.lc_gguf_close(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def tensors(self):
        out = []
        for i in range(self.L.lc_gguf_tensor_count(self.h)):
            name = C.c_char_p()
            dt = C.c_int()
            nd = C.c_uint32()
            shape = (C.c_uint64 * 4)()
            off = C.c_uint64()
            nb = C.c_uint64()
            lc.check(self.L.lc_gguf_tensor_info(self.h, i, C.byref(name), C.byref(dt), C.byref(nd), shape,
                                                C.byref(off), C.byref(nb)), "lc_gguf_tensor_info")
            out.append(dict(name=name.value.decode(), dtype=dt.value, shape=tuple(shape[: nd.value]),
                            offset=off.value, n_bytes=nb.value))
        return out

    def read(self, name: str) -> np.ndarray:
        idx = C.c_uint64()
        lc.check(self.L.lc_gguf_find(self.h, name.encode(), C.byref(idx)), "lc_gguf_find")
        info = self.tensors()[idx.value]
        buf = np.empty(info["n_bytes"], np.uint8)
        lc.check(self.L.lc_gguf_read(self.h, idx.value, buf.ctypes.data, buf.size), "lc_gguf_read")
        return buf

    def view(self, name: str) -> np.ndarray:
        """The tensor's bytes in place, a read-only view of the file mapping
        (lc_gguf_tensor_data); valid while the reader is open."""
        idx = C.c_uint64()
        lc.check(self.L.lc_gguf_find(self.h, name.encode(), C.byref(idx)), "lc_gguf_find")
        p = C.c_void_p()
        n = C.c_uint64()
        lc.check(self.L.lc_gguf_tensor_data(self.h, idx.value, C.byref(p), C.byref(n)), "lc_gguf_tensor_data")
        if n.value == 0:
            a = np.empty(0, np.uint8)
        else:
            a = np.frombuffer((C.c_uint8 * n.value).from_address(p.value), np.uint8)
        a.flags.writeable = False
        return a

    def meta_u64(self, key: str):
        v = C.c_uint64()
        return v.value if self.L.lc_gguf_meta_u64(self.h, key.encode(), C.byref(v)) == lc.LC_OK else None

    def meta_f32(self, key: str):
        v = C.c_float()
        return v.value if self.L.lc_gguf_meta_f32(self.h, key.encode(), C.byref(v)) == lc.LC_OK else None

    def meta_str(self, key: str):
        v = C.c_char_p()
        return v.value.decode() if self.L.lc_gguf_meta_str(self.h, key.encode(), C.byref(v)) == lc.LC_OK else None

    def hparams(self) -> lc.HParams:
        hp = lc.HParams()
        lc.check(self.L.lc_gguf_dflash_hparams(self.h, C.byref(hp)), "lc_gguf_dflash_hparams")
        return hp


def hparams(**kw) -> lc.HParams:
    hp = lc.HParams()
    hp.rope_base, hp.norm_eps, hp.qk_eps = 500000.0, 1e-5, 1e-6
    for k, v in kw.items():
        setattr(hp, k, v)
    return hp


class DFlash:
    """DFlashModel (src/dflash.rs) over lc_dflash_*; buffers are device pointers
    or torch CUDA tensors."""

    def __init__(self, ctx: lc.Context, hp: lc.HParams | None = None, max_ctx: int = 2048, max_block: int = 16,
                 gguf_path: str | None = None, flags: int = 0):
        self.L = lc.lib()
        self.ctx = ctx
        h = C.c_void_p()
        if gguf_path is not None:
            lc.check(self.L.lc_dflash_load_gguf_ex(ctx.h, gguf_path.encode(), max_ctx, max_block, flags,
                                                   C.byref(h)), "lc_dflash_load_gguf_ex")
        else:
            lc.check(self.L.lc_dflash_create(ctx.h, C.byref(hp), max_ctx, max_block, C.byref(h)), "lc_dflash_create")
        self.h = h
        self.hp = lc.HParams()
        lc.check(self.L.lc_dflash_get_hparams(self.h, C.byref(self.hp)))

    def close(self):
        if getattr(self, "h", None):
            self.L.lc_dflash_destroy(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def weight(self, name: str):
        """(device address, dtype as stored, bytes) of a loaded tensor."""
        p = C.c_void_p()
        dt = C.c_int()
        n = C.c_uint64()
        lc.check(self.L.lc_dflash_weight(self.h, name.encode(), C.byref(p), C.byref(dt), C.byref(n)),
                 "lc_dflash_weight")
        return p.value, dt.value, n.value

    def set_tensor(self, name: str, dtype: int, data: np.ndarray):
        a = np.ascontiguousarray(data)
        lc.check(self.L.lc_dflash_set_tensor(self.h, name.encode(), dtype, a.ctypes.data, a.nbytes),
                 f"lc_dflash_set_tensor({name})")

    def encode(self, features, n_ctx: int, enc_out):
        lc.check(self.L.lc_dflash_encode(self.h, lc.ptr(features), n_ctx, lc.ptr(enc_out)), "lc_dflash_encode")

    def set_context(self, enc_out, n_ctx: int):
        lc.check(self.L.lc_dflash_set_context(self.h, lc.ptr(enc_out), n_ctx), "lc_dflash_set_context")

    def decode_block(self, x, m: int, hidden):
        lc.check(self.L.lc_dflash_decode_block(self.h, lc.ptr(x), m, lc.ptr(hidden)), "lc_dflash_decode_block")

    def forward_injected_decode_hidden(self, features: np.ndarray, token: np.ndarray) -> np.ndarray:
        f = np.ascontiguousarray(features, np.float32)
        t = np.ascontiguousarray(token, np.float32)
        out = np.empty(self.hp.n_embd, np.float32)
        lc.check(self.L.lc_dflash_forward_injected_decode_hidden(self.h, f.ctypes.data, t.ctypes.data,
                                                                 out.ctypes.data),
                 "lc_dflash_forward_injected_decode_hidden")
        return out

    def forward_from_input(self, inp, hidden, logits=None) -> int:
        nv = C.c_uint32(0)
        lc.check(self.L.lc_dflash_forward_from_input(self.h, lc.ptr(inp), lc.ptr(hidden), lc.ptr(logits),
                                                     C.byref(nv)), "lc_dflash_forward_from_input")
        return nv.value

    def forward_token(self, token_id: int, hidden, logits=None) -> int:
        nv = C.c_uint32(0)
        lc.check(self.L.lc_dflash_forward_token(self.h, token_id, lc.ptr(hidden), lc.ptr(logits), C.byref(nv)),
                 "lc_dflash_forward_token")
        return nv.value
