"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Every output here comes from laguna-raw's GLSL shaders compiled for the CPU
(oracle/_ref, built by oracle/build_ref.py from the reference tree), run on
seeded synthetic inputs:

  proj_q8_0.npz, proj_q4k.npz, proj_f32.npz  -- kernels/proj*.comp
  dequant_shader.npz   -- the reference's per-element weight decode, read back
                          through proj_q8_0 / proj_q4k with one-hot x (exact:
                          c[i] = 0 + ... + 1*w(i,j) + 0*... )
  ops.npz              -- rmsnorm, qk_norm_rope, activation, add, gate_mul,
                          mha_attn, enc_aux_norm

Run here (where the reference tree exists):  python tests/golden/make_golden.py
The fixtures are small and committed; tests read them without the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from laguna_raw_halo_strix_b200 import synth  # noqa: E402
import oracle as orc  # noqa: E402
from build_ref import build  # noqa: E402


def u32(*v):
    return np.array(v, np.uint32).tobytes()


def f32b(v):
    return np.array([v], np.float32).tobytes()


def main():
    ref = orc.RefShaders(build(orc.reference_tree()))
    G = orc.RefShaders.groups

    # ---- projections --------------------------------------------------------
    rng = np.random.default_rng(1234)
    k, n = 256, 37
    x = synth.activations(1, k, rng)[0]
    w = synth.q8_0_blocks(n, k, rng)
    c = np.zeros(n, np.float32)
    ref.run("proj_q8_0", [x, orc.pad4(w), c], u32(k, n), G(n))
    np.savez_compressed(os.path.join(HERE, "proj_q8_0.npz"), x=x, w=w, c=c, k=k, n=n)

    k, n = 512, 45
    x = synth.activations(1, k, rng)[0]
    w2 = synth.q4k_blocks(2 * n, k, rng)  # two "experts" of n rows
    c0 = np.zeros(n, np.float32)
    c1 = np.zeros(n, np.float32)
    ref.run("proj_q4k", [x, orc.pad4(w2), c0], u32(k, n, 0), G(n))
    ref.run("proj_q4k", [x, orc.pad4(w2), c1], u32(k, n, n * k), G(n))
    np.savez_compressed(os.path.join(HERE, "proj_q4k.npz"), x=x, w=w2, c0=c0, c1=c1, k=k, n=n)

    k, n = 64, 19
    x = synth.activations(1, k, rng)[0]
    wf = (rng.standard_normal((n, k)) * 0.1).astype(np.float32)
    c0 = np.zeros(n, np.float32)
    c1 = np.zeros(n, np.float32)
    ref.run("proj", [x, wf, c0], u32(k, n, 0), G(n))
    ref.run("proj", [x, wf, c1], u32(k, n, 1), G(n))
    np.savez_compressed(os.path.join(HERE, "proj_f32.npz"), x=x, w=wf, c0=c0, c1=c1, k=k, n=n)

    # ---- dequant via one-hot projections -------------------------------------
    n = 4
    wq8 = synth.q8_0_blocks(n, 64, rng)
    wq4 = synth.q4k_blocks(n, 256, rng)
    deq8 = np.zeros((n, 64), np.float32)
    deq4 = np.zeros((n, 256), np.float32)
    for j in range(64):
        e = np.zeros(64, np.float32)
        e[j] = 1.0
        c = np.zeros(n, np.float32)
        ref.run("proj_q8_0", [e, orc.pad4(wq8), c], u32(64, n), G(n))
        deq8[:, j] = c
    for j in range(256):
        e = np.zeros(256, np.float32)
        e[j] = 1.0
        c = np.zeros(n, np.float32)
        ref.run("proj_q4k", [e, orc.pad4(wq4), c], u32(256, n, 0), G(n))
        deq4[:, j] = c
    np.savez_compressed(os.path.join(HERE, "dequant_shader.npz"), wq8=wq8, deq8=deq8, wq4=wq4, deq4=deq4)

    # ---- interleaved ops -------------------------------------------------------
    out = {}
    nn = 4096
    xr = rng.standard_normal(nn).astype(np.float32)
    wr = (1.0 + 0.1 * rng.standard_normal(nn)).astype(np.float32)
    y = np.zeros(nn, np.float32)
    ref.run("rmsnorm", [xr, wr, y], u32(nn) + f32b(1e-5), G(nn))
    out.update(rms_x=xr, rms_w=wr, rms_y=y)

    nh, hd = 4, 128
    xq = rng.standard_normal(nh * hd).astype(np.float32)
    wq = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = orc.Oracle().rope_freq(hd, 500000.0)
    out.update(qk_x=xq, qk_w=wq, qk_freq=freq)
    for pos in (0, 1, 7, 2063):
        yq = np.zeros(nh * hd, np.float32)
        ref.run("qk_norm_rope", [xq, wq, freq, yq], u32(nh, hd, hd) + f32b(1e-6) + u32(pos), G(nh * hd))
        out[f"qk_y_pos{pos}"] = yq

    na = 1000
    g = (3 * rng.standard_normal(na)).astype(np.float32)
    up = rng.standard_normal(na).astype(np.float32)
    h = np.zeros(na, np.float32)
    ref.run("activation", [g, up, h], u32(na), G(na))
    s = np.zeros(na, np.float32)
    ref.run("add", [g, up, s], u32(na), G(na))
    out.update(act_gate=g, act_up=up, act_h=h, add_c=s)

    v = rng.standard_normal(nh * hd).astype(np.float32)
    gate = np.abs(rng.standard_normal(nh)).astype(np.float32)
    gm = np.zeros(nh * hd, np.float32)
    ref.run("gate_mul", [v, gate, gm], u32(nh * hd, nh, hd, 0), G(nh * hd))
    out.update(gm_v=v, gm_gate=gate, gm_out=gm)

    nq, nkv, seq = 8, 2, 5
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kk = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    vv = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    out.update(att_q=q, att_k=kk, att_v=vv, att_scale=scale)
    for q_pos, causal in ((2, 1), (4, 1), (0, 1), (1, 0)):
        o = np.zeros(nq * hd, np.float32)
        ref.run("mha_attn", [q, kk, vv, o], u32(nq, nkv, hd, seq) + f32b(float(scale)) + u32(q_pos, causal),
                G(nq * hd))
        out[f"att_out_p{q_pos}_c{causal}"] = o

    nf, naux, ntok = 512, 5, 3
    xe = rng.standard_normal(nf * naux * ntok).astype(np.float32)
    we = (1.0 + 0.1 * rng.standard_normal(nf * naux)).astype(np.float32)
    ye = np.zeros_like(xe)
    ref.run("enc_aux_norm", [xe, we, ye], u32(nf, naux, ntok) + f32b(1e-5), G(xe.size))
    out.update(enc_x=xe, enc_w=we, enc_y=ye, enc_dims=np.array([nf, naux, ntok]))

    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
