"""Host-side handle of the target (Laguna) model of the C ABI (lc_target_* in
include/laguna_cuda.h), TargetModel of src/target.rs.  The model logic is C++
and CUDA in the library; this class marshals arguments.  Device buffers are
torch CUDA tensors or raw device addresses."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import lc


class Target:
    """TargetModel (src/target.rs:105-748) over lc_target_*."""

    def __init__(self, ctx: lc.Context, gguf_path: str, max_ctx: int = 256, max_block: int = 16, flags: int = 0):
        self.L = lc.lib()
        self.ctx = ctx
        self.max_block = max_block
        h = C.c_void_p()
        lc.check(self.L.lc_target_load_gguf(ctx.h, gguf_path.encode(), max_ctx, max_block, flags, C.byref(h)),
                 "lc_target_load_gguf")
        self.h = h
        self.hp = lc.TargetHParams()
        lc.check(self.L.lc_target_get_hparams(self.h, C.byref(self.hp)), "lc_target_get_hparams")

    def close(self):
        if getattr(self, "h", None):
            self.L.lc_target_destroy(self.h)
            self.h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def layer_info(self, layer: int):
        moe, heads = C.c_uint32(), C.c_uint32()
        lc.check(self.L.lc_target_layer_info(self.h, layer, C.byref(moe), C.byref(heads)), "lc_target_layer_info")
        return bool(moe.value), heads.value

    def weight(self, name: str):
        p, dt, n = C.c_void_p(), C.c_int(), C.c_uint64()
        lc.check(self.L.lc_target_weight(self.h, name.encode(), C.byref(p), C.byref(dt), C.byref(n)),
                 "lc_target_weight")
        return p.value, dt.value, n.value

    def embed(self, tokens, x):
        """x [m, n_embd] (device) <- target_token_embedding of each token (src/lib.rs:431-454)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        lc.check(self.L.lc_target_embed(self.h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size, lc.ptr(x)),
                 "lc_target_embed")

    def forward(self, x, m: int, cached: bool = False, capture=(), captured=None, hidden=None, logits=None,
                keys=None):
        cap = np.ascontiguousarray(capture, np.uint32)
        lc.check(self.L.lc_target_forward(self.h, lc.ptr(x), m, lc.TARGET_CACHED if cached else 0,
                                          cap.ctypes.data_as(C.POINTER(C.c_uint32)) if cap.size else None, cap.size,
                                          lc.ptr(captured), lc.ptr(hidden), lc.ptr(logits), lc.ptr(keys)),
                 "lc_target_forward")

    def routing(self, layer: int):
        """(ids [m, n_expert_used] int32 on the device, m) of the last call that ran MoE layer `layer`."""
        import torch

        n_sel = min(self.hp.n_expert_used, self.hp.n_expert)
        ids = torch.empty(self.max_block * n_sel, dtype=torch.int32, device=torch.device("cuda", self.ctx.device))
        m = C.c_uint32()
        lc.check(self.L.lc_target_routing(self.h, layer, lc.ptr(ids), C.byref(m)), "lc_target_routing")
        return ids[: m.value * n_sel].view(m.value, n_sel), m.value

    @property
    def cache_len(self) -> int:
        n = C.c_uint32()
        lc.check(self.L.lc_target_cache_len(self.h, C.byref(n)), "lc_target_cache_len")
        return n.value

    def truncate(self, n: int):
        lc.check(self.L.lc_target_cache_truncate(self.h, n), "lc_target_cache_truncate")

    def moe_ffn(self, layer: int, x, m: int, y, ids=None, scores=None):
        lc.check(self.L.lc_target_moe_ffn(self.h, layer, lc.ptr(x), m, lc.ptr(y), lc.ptr(ids), lc.ptr(scores)),
                 "lc_target_moe_ffn")


def target_hparams(path: str) -> lc.TargetHParams:
    """lc_gguf_target_hparams of a GGUF file (host only, no device)."""
    from .model import Gguf

    g = Gguf(path)
    hp = lc.TargetHParams()
    lc.check(g.L.lc_gguf_target_hparams(g.h, C.byref(hp)), "lc_gguf_target_hparams")
    g.close()
    return hp
