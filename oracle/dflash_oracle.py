"""CPU oracle of the DFlash draft model's op sequence (TEST INFRASTRUCTURE ONLY).

Composes the C restatement's kernels (laguna_oracle.c) in the order of the
reference's DFlashModel:

* encode                          -- src/dflash.rs:157-234
* forward_injected_decode_hidden  -- src/dflash.rs:877-976
* forward_from_input              -- src/dflash.rs:735-851 (legacy decoder)

Projections use the shader formulas of the weight's type (proj.comp,
proj_q8_0.comp, proj_q4k.comp).  The reference has one context vector and one
query token; the block form generalises it with the reference's own rules:
context rows sit at positions 0..n_ctx-1, block token r at n_ctx + r, and the
mha_attn causal rule (key p visible iff p <= q_pos) applies.  With n_ctx = 1
and one token this is exactly the reference's computation.
"""
from __future__ import annotations

import numpy as np

import oracle as orc

LAYER_TENSORS = ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm",
                 "attn_gate", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]


def proj_blas(o: orc.Oracle, dtype: int, x: np.ndarray, w: np.ndarray, k: int, n: int,
              chunk_rows: int = 16384) -> np.ndarray:
    """x [m, k] . W^T for a weight of n rows: W dequantised bit-exactly by the
    shader formula (oracle.dequant_shader, kernels/proj_q4k.comp:87 and
    proj_q8_0.comp:53-64), products summed by BLAS in f32 (blocked sums), in
    row chunks.  It differs from the reference's serial f32 sum by ~1e-6
    relative -- far below the parity tolerances -- and runs the full-size
    configurations in seconds on the host cores."""
    x = np.ascontiguousarray(np.atleast_2d(np.asarray(x, np.float32)))
    out = np.empty((x.shape[0], n), np.float32)
    if dtype == orc.F32:
        wf = np.asarray(w, np.float32).reshape(n, k)
        return (x @ wf.T).astype(np.float32)
    bb = 144 if dtype == orc.Q4_K else 34
    be = 256 if dtype == orc.Q4_K else 32
    raw = np.ascontiguousarray(w).view(np.uint8).ravel()
    rb = k // be * bb
    chunk_rows = max(1, min(chunk_rows, (1 << 26) // k))  # <= 256 MB of f32 weights at a time
    for r0 in range(0, n, chunk_rows):
        r1 = min(n, r0 + chunk_rows)
        wf = o.dequant_shader(raw[r0 * rb:r1 * rb], dtype, (r1 - r0) * k).reshape(r1 - r0, k)
        out[:, r0:r1] = x @ wf.T
    return out


class DFlashOracle:
    def __init__(self, hp: dict, tensors: dict, o: orc.Oracle | None = None, fast_proj: bool = False):
        """hp: n_layers, n_embd, n_heads, n_kv_heads, head_dim, rope_dim, n_ff,
        n_aux, rope_base, norm_eps, qk_eps.  tensors: name -> (dtype, array);
        f32 tensors as float32 arrays, quantized ones as raw uint8 blocks.
        fast_proj: projections through proj_blas (full-size configurations)
        instead of the shader restatement."""
        self.hp = hp
        self.t = tensors
        self.o = o or orc.Oracle()
        self.fast_proj = fast_proj
        self.freq = self.o.rope_freq(hp["rope_dim"], hp["rope_base"])

    def _f32(self, name):
        dt, a = self.t[name]
        assert dt == orc.F32
        return a

    def _proj(self, name, x, k, n):
        dt, w = self.t[name]
        if self.fast_proj:
            return proj_blas(self.o, dt, x, w, k, n)
        return self.o.proj(dt, np.atleast_2d(x), w, k, n).reshape(-1, n)

    def encode(self, feats):
        h = self.hp
        E, A = h["n_embd"], h["n_aux"]
        n_ctx = feats.size // (E * A)
        y = self.o.enc_aux_norm(feats.reshape(-1), self._f32("enc.aux_norm.weight"), E, A, n_ctx, h["norm_eps"])
        e = self._proj("fc.weight", y.reshape(n_ctx, E * A), E * A, E)
        return self.o.rmsnorm(e, self._f32("enc.output_norm.weight"), h["norm_eps"]).reshape(n_ctx, E)

    def context_kv(self, enc):
        h = self.hp
        E, KVD = h["n_embd"], h["n_kv_heads"] * h["head_dim"]
        n_ctx = enc.shape[0]
        kv = []
        for l in range(h["n_layers"]):
            p = f"blk.{l}."
            nx = self.o.rmsnorm(enc, self._f32(p + "attn_norm.weight"), h["norm_eps"])
            k = self._proj(p + "attn_k.weight", nx, E, KVD)
            v = self._proj(p + "attn_v.weight", nx, E, KVD)
            k = self.o.qk_norm_rope(k, self._f32(p + "attn_k_norm.weight"), self.freq, h["n_kv_heads"],
                                    h["head_dim"], h["rope_dim"], h["qk_eps"], np.arange(n_ctx))
            kv.append((k.reshape(n_ctx, KVD), v.reshape(n_ctx, KVD)))
        return kv

    def decode_block(self, x, kv):
        h = self.hp
        E, H, KV, hd, F = h["n_embd"], h["n_heads"], h["n_kv_heads"], h["head_dim"], h["n_ff"]
        QD, KVD = H * hd, KV * hd
        x = np.array(x, np.float32).reshape(-1, E)
        m = x.shape[0]
        n_ctx = kv[0][0].shape[0]
        pos = n_ctx + np.arange(m)
        scale = float(np.float32(1.0) / np.float32(np.sqrt(np.float32(hd))))
        for l in range(h["n_layers"]):
            p = f"blk.{l}."
            nx = self.o.rmsnorm(x, self._f32(p + "attn_norm.weight"), h["norm_eps"])
            q = self._proj(p + "attn_q.weight", nx, E, QD)
            k = self._proj(p + "attn_k.weight", nx, E, KVD)
            v = self._proj(p + "attn_v.weight", nx, E, KVD)
            q = self.o.qk_norm_rope(q, self._f32(p + "attn_q_norm.weight"), self.freq, H, hd, h["rope_dim"],
                                    h["qk_eps"], pos).reshape(m, QD)
            k = self.o.qk_norm_rope(k, self._f32(p + "attn_k_norm.weight"), self.freq, KV, hd, h["rope_dim"],
                                    h["qk_eps"], pos).reshape(m, KVD)
            ks = np.concatenate([kv[l][0], k], 0)
            vs = np.concatenate([kv[l][1], v], 0)
            attn = np.stack([self.o.mha_attn(q[r], ks, vs, H, KV, hd, n_ctx + m, scale, n_ctx + r, 1)
                             for r in range(m)])
            g = self.o.softplus(self._proj(p + "attn_gate.weight", nx, E, H))
            attn = self.o.gate_mul(attn.reshape(-1), g.reshape(-1), hd).reshape(m, QD)
            x = self.o.add(x, self._proj(p + "attn_output.weight", attn, QD, E))
            nx = self.o.rmsnorm(x, self._f32(p + "ffn_norm.weight"), h["norm_eps"])
            act = self.o.activation(self._proj(p + "ffn_gate.weight", nx, E, F),
                                    self._proj(p + "ffn_up.weight", nx, E, F))
            x = self.o.add(x, self._proj(p + "ffn_down.weight", act, F, E))
        return self.o.rmsnorm(x, self._f32("output_norm.weight"), h["norm_eps"])

    def forward_injected_decode_hidden(self, feats, token):
        enc = self.encode(feats)
        return self.decode_block(token, self.context_kv(enc))[0]

    def forward_from_input(self, inp):
        """src/dflash.rs:735-851: q/k are computed there but feed nothing; the
        per-head gate multiplies v repeated to n_heads*head_dim (repeat_v.comp)."""
        h = self.hp
        E, H, KV, hd, F = h["n_embd"], h["n_heads"], h["n_kv_heads"], h["head_dim"], h["n_ff"]
        QD, KVD = H * hd, KV * hd
        x = np.array(inp, np.float32).reshape(1, E)
        for l in range(h["n_layers"]):
            p = f"blk.{l}."
            nx = self.o.rmsnorm(x, self._f32(p + "attn_norm.weight"), h["norm_eps"])
            v = self._proj(p + "attn_v.weight", nx, E, KVD).reshape(-1)
            v_rep = v[np.arange(QD) % KVD]
            g = self.o.softplus(self._proj(p + "attn_gate.weight", nx, E, H).reshape(-1))
            attn = self.o.gate_mul(v_rep, g, hd)
            x = self.o.add(x, self._proj(p + "attn_output.weight", attn, QD, E))
            nx = self.o.rmsnorm(x, self._f32(p + "ffn_norm.weight"), h["norm_eps"])
            act = self.o.activation(self._proj(p + "ffn_gate.weight", nx, E, F),
                                    self._proj(p + "ffn_up.weight", nx, E, F))
            x = self.o.add(x, self._proj(p + "ffn_down.weight", act, F, E))
        return self.o.rmsnorm(x, self._f32("output_norm.weight"), h["norm_eps"])[0]

    def fc_logits(self, hidden):
        """src/dflash.rs:839-847: fc.weight reinterpreted as [n_vocab, n_embd]."""
        dt, w = self.t["fc.weight"]
        E = self.hp["n_embd"]
        nel = (w.size // 144 * 256) if dt == orc.Q4_K else (w.size // 34 * 32) if dt == orc.Q8_0 else w.size
        vocab = nel // E
        return self.o.proj(dt, hidden.reshape(1, E), w, E, vocab)[0]


def make_model(hp: dict, wtype: int, rng: np.random.Generator):
    """Seeded synthetic DFlash weights: quantized projections (wtype), f32 norms."""
    from laguna_raw_halo_strix_b200 import synth

    E, H, KV, hd, F, A = (hp[k] for k in ("n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "n_aux"))
    QD, KVD = H * hd, KV * hd

    def W(rows, k):
        return (wtype, synth.weight_blocks(wtype, rows, k, rng).reshape(-1))

    def N(n):
        return (orc.F32, (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))

    t = {"fc.weight": W(E, A * E), "enc.aux_norm.weight": N(A * E), "enc.output_norm.weight": N(E),
         "output_norm.weight": N(E)}
    for l in range(hp["n_layers"]):
        p = f"blk.{l}."
        t.update({p + "attn_norm.weight": N(E), p + "attn_q.weight": W(QD, E), p + "attn_k.weight": W(KVD, E),
                  p + "attn_v.weight": W(KVD, E), p + "attn_output.weight": W(E, QD),
                  p + "attn_q_norm.weight": N(hd), p + "attn_k_norm.weight": N(hd),
                  p + "attn_gate.weight": W(H, E), p + "ffn_norm.weight": N(E), p + "ffn_gate.weight": W(F, E),
                  p + "ffn_up.weight": W(F, E), p + "ffn_down.weight": W(E, F)})
    return t


def tensor_shape(name: str, hp: dict) -> tuple:
    """GGUF shape (ne0 = input dim first) of each DFlash tensor."""
    E, H, KV, hd, F, A = (hp[k] for k in ("n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "n_aux"))
    suf = name.split(".", 2)[-1] if name.startswith("blk.") else name
    shapes = {"fc.weight": (A * E, E), "enc.aux_norm.weight": (A * E,), "enc.output_norm.weight": (E,),
              "output_norm.weight": (E,), "attn_norm.weight": (E,), "attn_q.weight": (E, H * hd),
              "attn_k.weight": (E, KV * hd), "attn_v.weight": (E, KV * hd), "attn_output.weight": (H * hd, E),
              "attn_q_norm.weight": (hd,), "attn_k_norm.weight": (hd,), "attn_gate.weight": (E, H),
              "ffn_norm.weight": (E,), "ffn_gate.weight": (E, F), "ffn_up.weight": (E, F),
              "ffn_down.weight": (F, E)}
    return shapes[suf]
