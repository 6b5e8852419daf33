"""CPU restatement of the target (Laguna) model's forward pass -- TEST
INFRASTRUCTURE ONLY, the checker for lc_target_* (never imported by the
product library).

TargetOracle follows TargetModel::forward_token_impl (src/target.rs:314-578)
and dispatch_moe_ffn (src/target.rs:607-748) one token at a time, on the C
restatements of the shaders in laguna_oracle.c (pinned against the reference's
own GLSL by tests/test_oracle.py) and of the host-side router arithmetic
(lco_moe_select, lco_moe_l2_scale).

Deliberate difference from the reference, behind a switch: the reference's
dispatch_proj_quant_expert (src/target.rs:1098-1162) hands the expert offset
only to the Q4_K kernel, so its Q8_0 and F32 expert projections always read
expert 0.  By default this oracle (like the CUDA path) gives every format its
own expert; ref_expert_offset=True reproduces the reference.
"""
from __future__ import annotations

import numpy as np

import oracle as orc

_BLOCK = {orc.F32: (1, 4), orc.Q8_0: (32, 34), orc.Q4_K: (256, 144)}


def n_elements(dtype: int, a: np.ndarray) -> int:
    be, bb = _BLOCK[dtype]
    nbytes = np.asarray(a).nbytes
    return nbytes // bb * be


def expert_slice(dtype: int, a: np.ndarray, e: int, rows: int, k: int) -> np.ndarray:
    """Expert e of a stack of n_expert [rows, k] matrices (the element offset
    e * rows * k of src/target.rs:681-683)."""
    be, bb = _BLOCK[dtype]
    if dtype == orc.F32:
        f = np.ascontiguousarray(a, np.float32).reshape(-1)
        return f[e * rows * k:(e + 1) * rows * k]
    b = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
    per = rows * k // be * bb
    return b[e * per:(e + 1) * per]


class TargetOracle:
    """hp: dict with n_layers, n_embd, n_ff, n_heads, n_kv_heads, head_dim,
    rope_dim, rope_dim_swa, swa, rope_base, rope_base_swa, n_expert,
    n_expert_used, n_ff_exp, n_ff_shexp, has_moe, expert_weights_norm,
    expert_weights_scale, n_vocab; tensors: name -> (dtype, array)."""

    def __init__(self, hp: dict, tensors: dict, o: orc.Oracle | None = None, ref_expert_offset: bool = False):
        self.hp = hp
        self.t = tensors
        self.o = o or orc.Oracle()
        self.ref_expert_offset = ref_expert_offset
        self.freq = self.o.rope_freq(hp["rope_dim"], hp["rope_base"]) if hp["rope_dim"] else np.zeros(1, np.float32)
        rds = hp.get("rope_dim_swa", 0)
        self.freq_swa = self.o.rope_freq(rds, hp.get("rope_base_swa", 10000.0)) if rds else np.zeros(1, np.float32)
        self.clear()

    # -- cache (TargetKvCache, src/target.rs:74-101) --------------------------
    def clear(self):
        self.cache_k = [[] for _ in range(self.hp["n_layers"])]
        self.cache_v = [[] for _ in range(self.hp["n_layers"])]
        self.cache_len = 0

    def truncate(self, n: int):
        for l in range(self.hp["n_layers"]):
            del self.cache_k[l][n:]
            del self.cache_v[l][n:]
        self.cache_len = min(self.cache_len, n)

    # -- helpers ---------------------------------------------------------------
    def _f32(self, name):
        dt, a = self.t[name]
        assert dt == orc.F32, name
        return np.ascontiguousarray(a, np.float32).reshape(-1)

    def _proj(self, name, x, k, n):
        dt, w = self.t[name]
        return self.o.proj(dt, np.atleast_2d(x), w, k, n).reshape(-1)

    def is_moe(self, l):
        return bool(self.hp["has_moe"]) and l > 0  # src/target.rs:140

    def n_q_heads(self, l):
        dt, a = self.t[f"blk.{l}.attn_q.weight"]
        return n_elements(dt, a) // self.hp["n_embd"] // self.hp["head_dim"]  # src/target.rs:224-235

    def embed(self, token: int) -> np.ndarray:
        """target_token_embedding (src/lib.rs:431-454): row `token` of
        dequant_to_f32(token_embd)."""
        dt, a = self.t["token_embd.weight"]
        E = self.hp["n_embd"]
        if dt == orc.F32:
            return np.ascontiguousarray(a, np.float32).reshape(-1)[token * E:(token + 1) * E].copy()
        n = n_elements(dt, a)
        return self.o.dequant_to_f32(np.ascontiguousarray(a).view(np.uint8).reshape(-1), dt, n)[token * E:(token + 1) * E]

    # -- MoE FFN (src/target.rs:607-748) --------------------------------------
    def moe_ffn(self, l, nx):
        h, o = self.hp, self.o
        E, F = h["n_embd"], h["n_ff_exp"]
        p = f"blk.{l}."
        logits = self._proj(p + "ffn_gate_inp.weight", nx, E, h["n_expert"])
        ids, scores = o.moe_select(logits, self._f32(p + "exp_probs_b.bias"), h["n_expert_used"],
                                   h["expert_weights_norm"], h["expert_weights_scale"])
        moe_out = np.zeros(E, np.float32)
        for e, sc in zip(ids, scores):
            def w(name, rows, k):
                dt, a = self.t[p + name]
                ee = 0 if (self.ref_expert_offset and dt != orc.Q4_K) else int(e)
                return dt, expert_slice(dt, a, ee, rows, k)

            dg, wg = w("ffn_gate_exps.weight", F, E)
            du, wu = w("ffn_up_exps.weight", F, E)
            dd, wd = w("ffn_down_exps.weight", E, F)
            g = o.proj(dg, nx[None, :], wg, E, F)[0]
            u = o.proj(du, nx[None, :], wu, E, F)[0]
            hid = o.activation(g, u)
            hs, col = o.moe_l2_scale(hid)
            out = o.proj(dd, hs[None, :], wd, F, E)[0]
            if sc > 0.0:
                out_scale = np.float32(np.float32(col / np.float32(32768.0)) * np.float32(sc))
                out = (out * out_scale).astype(np.float32)
            moe_out = o.add(moe_out, out)
        S = h["n_ff_shexp"]
        g = self._proj(p + "ffn_gate_shexp.weight", nx, E, S)
        u = self._proj(p + "ffn_up_shexp.weight", nx, E, S)
        so = self._proj(p + "ffn_down_shexp.weight", o.activation(g, u), S, E)
        return o.add(moe_out, so), ids, scores

    # -- one token (forward_token_impl) ----------------------------------------
    def forward_token(self, inp, capture=(), cached=False):
        h, o = self.hp, self.o
        E, KV, hd = h["n_embd"], h["n_kv_heads"], h["head_dim"]
        KVD = KV * hd
        scale = float(np.float32(1.0) / np.float32(np.sqrt(np.float32(hd))))
        pos = self.cache_len if cached else 0
        x = np.array(inp, np.float32).reshape(-1)
        captured = []
        for l in range(h["n_layers"]):
            if l in capture:
                captured.append(x.copy())
            p = f"blk.{l}."
            H = self.n_q_heads(l)
            QD = H * hd
            nx = o.rmsnorm(x, self._f32(p + "attn_norm.weight"), 1e-5)
            q = self._proj(p + "attn_q.weight", nx, E, QD)
            k = self._proj(p + "attn_k.weight", nx, E, KVD)
            v = self._proj(p + "attn_v.weight", nx, E, KVD)
            swa_layer = bool(h.get("swa", 0)) and l % 4 != 0  # src/target.rs:440
            rd = h["rope_dim_swa"] if swa_layer else h["rope_dim"]
            fr = self.freq_swa if swa_layer else self.freq
            qn = o.qk_norm_rope(q, self._f32(p + "attn_q_norm.weight"), fr, H, hd, rd, 1e-6, pos)
            kn = o.qk_norm_rope(k, self._f32(p + "attn_k_norm.weight"), fr, KV, hd, rd, 1e-6, pos)
            if cached:
                self.cache_k[l].append(kn.copy())
                self.cache_v[l].append(v.copy())
                n = len(self.cache_k[l])
                attn = o.mha_attn(qn, np.concatenate(self.cache_k[l]), np.concatenate(self.cache_v[l]), H, KV, hd,
                                  n, scale, n - 1, 1)
            else:
                attn = o.mha_attn(qn, kn, v, H, KV, hd, 1, scale, 0, 1)
            if p + "attn_gate.weight" in self.t:
                g = self._proj(p + "attn_gate.weight", nx, E, H)
                attn = o.gate_attn(attn, g, H, hd)
            x = o.add(x, self._proj(p + "attn_output.weight", attn, QD, E))
            nx = o.rmsnorm(x, self._f32(p + "ffn_norm.weight"), 1e-5)
            if self.is_moe(l):
                f, _, _ = self.moe_ffn(l, nx)
            else:
                F = h["n_ff"]
                act = o.activation(self._proj(p + "ffn_gate.weight", nx, E, F), self._proj(p + "ffn_up.weight", nx, E, F))
                f = self._proj(p + "ffn_down.weight", act, F, E)
            x = o.add(x, f)
        if h["n_layers"] in capture:
            captured.append(x.copy())
        if cached:
            self.cache_len += 1
        if "output_norm.weight" in self.t:
            x = o.rmsnorm(x, self._f32("output_norm.weight"), 1e-5)
        hidden = x
        if "output.weight" in self.t:
            logits = self._proj("output.weight", hidden, E, h["n_vocab"])
        else:
            logits = hidden.copy()
        return captured, hidden, logits

    def forward(self, xs, capture=(), cached=False):
        """Rows of xs in order; returns (captured [m, n_cap, E], hidden [m, E],
        logits [m, V])."""
        xs = np.atleast_2d(np.asarray(xs, np.float32))
        caps, hids, logs = [], [], []
        for r in range(xs.shape[0]):
            c, hd, lg = self.forward_token(xs[r], capture, cached)
            caps.append(np.stack(c) if c else np.zeros((0, self.hp["n_embd"]), np.float32))
            hids.append(hd)
            logs.append(lg)
        return np.stack(caps), np.stack(hids), np.stack(logs)


# -- seeded synthetic target models (test fixtures) ------------------------------

def default_hp(**kw) -> dict:
    hp = dict(n_layers=4, n_embd=512, n_ff=768, n_heads=4, n_kv_heads=2, head_dim=128, rope_dim=128,
              rope_dim_swa=128, swa=1, rope_base=500000.0, rope_base_swa=10000.0, n_expert=16, n_expert_used=4,
              n_ff_exp=256, n_ff_shexp=256, has_moe=1, expert_weights_norm=1, expert_weights_scale=2.5,
              n_vocab=1000, q_heads={2: 8}, gate_layers=(0, 2, 3))
    hp.update(kw)
    return hp


def tensor_shape(name: str, hp: dict) -> tuple:
    """GGUF shape (ne0 = input dim first) of each target tensor."""
    E, KV, hd, F = hp["n_embd"], hp["n_kv_heads"], hp["head_dim"], hp["n_ff"]
    NE, Fe, S, V = hp["n_expert"], hp["n_ff_exp"], hp["n_ff_shexp"], hp["n_vocab"]
    if not name.startswith("blk."):
        return {"token_embd.weight": (E, V), "output.weight": (E, V), "output_norm.weight": (E,)}[name]
    l = int(name.split(".")[1])
    H = hp["q_heads"].get(l, hp["n_heads"])
    suf = name.split(".", 2)[2]
    return {"attn_norm.weight": (E,), "ffn_norm.weight": (E,), "attn_q_norm.weight": (hd,),
            "attn_k_norm.weight": (hd,), "attn_q.weight": (E, H * hd), "attn_k.weight": (E, KV * hd),
            "attn_v.weight": (E, KV * hd), "attn_output.weight": (H * hd, E), "attn_gate.weight": (E, H),
            "ffn_gate.weight": (E, F), "ffn_up.weight": (E, F), "ffn_down.weight": (F, E),
            "ffn_gate_inp.weight": (E, NE), "exp_probs_b.bias": (NE,), "ffn_gate_exps.weight": (E, Fe, NE),
            "ffn_up_exps.weight": (E, Fe, NE), "ffn_down_exps.weight": (Fe, E, NE),
            "ffn_gate_shexp.weight": (E, S), "ffn_up_shexp.weight": (E, S), "ffn_down_shexp.weight": (S, E)}[suf]


def make_target(hp: dict, wtype: int, rng: np.random.Generator, expert_type: int | None = None,
                out_type: int = orc.Q8_0, embd_type: int = orc.F32) -> dict:
    """Seeded synthetic target weights: quantized projections (wtype; the
    expert stacks expert_type), f32 norms, router and bias."""
    from laguna_raw_halo_strix_b200 import synth

    E, KV, hd, F = hp["n_embd"], hp["n_kv_heads"], hp["head_dim"], hp["n_ff"]
    NE, Fe, S, V = hp["n_expert"], hp["n_ff_exp"], hp["n_ff_shexp"], hp["n_vocab"]
    et = wtype if expert_type is None else expert_type

    # weights of about 0.5 / sqrt(k) and mean ~0, so the residual stream of a
    # random model stays finite through the layers: Q4_K sub-blocks take
    # dmin = d and min = 7.5 * scale (w = d * sc * (q - 7.5))
    def blocks(dt, rows, k):
        if dt == orc.Q4_K:
            nb = rows * (k // 256)
            d = (np.abs(rng.standard_normal(nb)) * 0.5 / (4.6 * 4.5 * np.sqrt(k)) + 1e-6).astype(np.float16)
            sc = rng.integers(1, 9, size=(nb, 8))
            mn = np.rint(7.5 * sc)
            b = np.empty((nb, 144), np.uint8)
            b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
            b[:, 2:4] = d.view(np.uint8).reshape(nb, 2)
            b[:, 4:16] = synth.pack_scale_min_k4(sc, mn)
            b[:, 16:] = rng.integers(0, 256, size=(nb, 128)).astype(np.uint8)
            return b.reshape(-1)
        return synth.q8_0_blocks(rows, k, rng, d_scale=0.5 / (58.0 * np.sqrt(k))).reshape(-1)

    def W(rows, k, dt=wtype):
        if dt == orc.F32:
            return (orc.F32, (0.5 * rng.standard_normal(rows * k) / np.sqrt(k)).astype(np.float32))
        return (dt, blocks(dt, rows, k))

    def stack(rows, k):
        if et == orc.F32:
            return (orc.F32, (0.5 * rng.standard_normal(NE * rows * k) / np.sqrt(k)).astype(np.float32))
        return (et, np.concatenate([blocks(et, rows, k) for _ in range(NE)]))

    def N(n):
        return (orc.F32, (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))

    t = {"output_norm.weight": N(E), "output.weight": W(V, E, out_type)}
    if embd_type == orc.F32:
        t["token_embd.weight"] = (orc.F32, (0.5 * rng.standard_normal(V * E)).astype(np.float32))
    else:
        t["token_embd.weight"] = W(V, E, embd_type)
    for l in range(hp["n_layers"]):
        p = f"blk.{l}."
        H = hp["q_heads"].get(l, hp["n_heads"])
        t.update({p + "attn_norm.weight": N(E), p + "ffn_norm.weight": N(E), p + "attn_q_norm.weight": N(hd),
                  p + "attn_k_norm.weight": N(hd), p + "attn_q.weight": W(H * hd, E), p + "attn_k.weight": W(KV * hd, E),
                  p + "attn_v.weight": W(KV * hd, E), p + "attn_output.weight": W(E, H * hd)})
        if l in hp["gate_layers"]:
            t[p + "attn_gate.weight"] = W(H, E)
        if hp["has_moe"] and l > 0:
            t.update({p + "ffn_gate_inp.weight": (orc.F32, (rng.standard_normal(NE * E) / np.sqrt(E)).astype(np.float32)),
                      # distinct biases keep the top-k away from near-ties
                      p + "exp_probs_b.bias": (orc.F32, (0.02 * rng.permutation(NE)).astype(np.float32)),
                      p + "ffn_gate_exps.weight": stack(Fe, E), p + "ffn_up_exps.weight": stack(Fe, E),
                      p + "ffn_down_exps.weight": stack(E, Fe),
                      p + "ffn_gate_shexp.weight": W(S, E), p + "ffn_up_shexp.weight": W(S, E),
                      p + "ffn_down_shexp.weight": W(E, S)})
        else:
            t.update({p + "ffn_gate.weight": W(F, E), p + "ffn_up.weight": W(F, E), p + "ffn_down.weight": W(E, F)})
    return t


def gguf_meta(hp: dict) -> dict:
    return {"general.architecture": "laguna", "laguna.block_count": hp["n_layers"],
            "laguna.embedding_length": hp["n_embd"], "laguna.feed_forward_length": hp["n_ff"],
            "laguna.attention.head_count": hp["n_heads"], "laguna.attention.head_count_kv": hp["n_kv_heads"],
            "laguna.attention.key_length": hp["head_dim"], "laguna.rope.dimension_count": hp["rope_dim"],
            "laguna.rope.dimension_count_swa": hp["rope_dim_swa"], "laguna.rope.freq_base": hp["rope_base"],
            "laguna.rope.freq_base_swa": hp["rope_base_swa"], "expert.count": hp["n_expert"],
            "expert.used_count": hp["n_expert_used"], "expert.feed_forward_length": hp["n_ff_exp"],
            "expert.shared_feed_forward_length": hp["n_ff_shexp"],
            "laguna.expert_weights_norm": bool(hp["expert_weights_norm"]),
            "laguna.expert_weights_scale": float(hp["expert_weights_scale"])}


def gguf_tensors(t: dict, hp: dict) -> list:
    return [(name, dt, tensor_shape(name, hp), np.ascontiguousarray(a).view(np.uint8).reshape(-1))
            for name, (dt, a) in t.items()]
