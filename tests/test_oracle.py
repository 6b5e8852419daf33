"""CPU tests: the oracle pinned against the reference's own tests and outputs.

* Known answers from the reference's unit tests and CLI self-tests
  (src/dflash.rs:1334-1381, src/gguf.rs:659-732, src/lib.rs:120-210).
* Golden fixtures produced by the reference's GLSL shaders compiled for the
  CPU (tests/golden/make_golden.py).
* When oracle/_ref is present, random cases against the compiled shaders.
"""
import os

import numpy as np
import pytest

import oracle as orc
from laguna_raw_halo_strix_b200 import synth


# ---- src/dflash.rs unit tests -------------------------------------------------

def test_half_known_answers(oracle):
    # dflash.rs:1334-1344: "BF16" 0x3C00 -> 1.0, 0x3E00 -> 1.5 (f16 bit patterns)
    out = oracle.dequant_to_f32(np.array([0x3C00], np.uint16).tobytes(), orc.BF16, 1)
    assert abs(out[0] - 1.0) < 1e-6
    out = oracle.dequant_to_f32(np.array([0x3E00], np.uint16).tobytes(), orc.BF16, 1)
    assert abs(out[0] - 1.5) < 1e-6


def test_q8_0_known_answer(oracle):
    # dflash.rs:1347-1356: d = 0x3C00, q = 1 -> 1.0
    data = bytearray(34)
    data[0:2] = (0x3C00).to_bytes(2, "little")
    for i in range(32):
        data[2 + i] = 1
    out = oracle.dequant_to_f32(bytes(data), orc.Q8_0, 32)
    assert abs(out[0] - 1.0) < 1e-3
    assert np.all(out == 1.0)


def test_f32_passthrough(oracle):
    # dflash.rs:1359-1365
    vals = (np.arange(16, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    out = oracle.dequant_to_f32(vals.tobytes(), orc.F32, 16)
    assert abs(out[5] - 0.005) < 1e-6
    assert np.array_equal(out, vals)


def test_unsupported_is_zero(oracle):
    # dflash.rs:1368-1373 (Q5_0 = id 6 in the reference's enum order -> zeros)
    out = oracle.dequant_to_f32(bytes(32), 6, 16)
    assert out.shape == (16,) and np.all(out == 0)


def test_half_subnormal_quirk(oracle):
    # proj_q8_0.comp:32-36: subnormal halves keep the implicit one
    assert oracle.half_ref(0x0001) == pytest.approx(2.0 ** -14 * (1 + 1 / 1024), rel=0, abs=0)
    assert oracle.half_ieee(0x0001) == 2.0 ** -24
    assert np.signbit(oracle.half_ref(0x8000)) and oracle.half_ref(0x8000) == 0.0
    assert oracle.half_ref(0x7C00) == np.inf and np.isnan(oracle.half_ref(0x7E00))
    # normals agree with IEEE
    for h in (0x3C00, 0x0400, 0x7BFF, 0xBC00, 0x1234):
        assert oracle.half_ref(h) == oracle.half_ieee(h) == float(np.array([h], np.uint16).view(np.float16)[0])


def test_ieee_half_all_patterns(oracle):
    hs = np.arange(65536, dtype=np.uint32)
    ref = hs.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([oracle.half_ieee(int(h)) for h in hs[::97]], np.float32)
    r = ref[::97]
    nan = np.isnan(r)
    assert np.array_equal(got[~nan], r[~nan]) and np.all(np.isnan(got[nan]))


def test_dequant_bounds(oracle):
    # Reads are bounded by the byte count; elements past the data are 0.
    w = synth.q8_0_blocks(1, 64, np.random.default_rng(3)).ravel()
    full = oracle.dequant_to_f32(w, orc.Q8_0, 64)
    part = oracle.dequant_to_f32(w[:50], orc.Q8_0, 64)
    assert np.array_equal(part[:32], full[:32]) and np.all(part[32:] == 0)
    empty = oracle.dequant_to_f32(b"", orc.F32, 3)
    assert np.all(empty == 0)


# ---- src/gguf.rs unit tests ---------------------------------------------------

def test_block_sizes():
    # gguf.rs:667-693 / :710-732
    assert synth.Q8_0_BLOCK == 34 and synth.Q4_K_BLOCK == 144
    assert synth.row_bytes(8, 1024) == 1088
    assert synth.row_bytes(12, 256) * 30 == 30 * 144
    assert synth.q8_0_blocks(1, 1024, np.random.default_rng(0)).nbytes == 1088
    assert synth.q4k_blocks(30, 256, np.random.default_rng(0)).nbytes == 4320


# ---- src/lib.rs CLI self-tests -------------------------------------------------

def test_matmul_selftest(oracle):
    # lib.rs:120-165: a = 0.1*i (8), b = 0.01*i (24), c[j] = sum_i a[i]*b[j*8+i]
    a = (np.arange(8, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    b = (np.arange(24, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    c = oracle.proj(orc.F32, a, b, 8, 3)
    exp = np.array([sum(a[i] * b[j * 8 + i] for i in range(8)) for j in range(3)], np.float32)
    assert np.abs(c - exp).max() < 1e-4


def test_rmsnorm_selftest(oracle):
    # lib.rs:167-210
    x = ((np.arange(4, dtype=np.float32) + 1) * 0.5).astype(np.float32)
    w = np.array([0.5, 1.0, 1.5, 2.0], np.float32)
    y = oracle.rmsnorm(x, w, 1e-5)
    ms = np.float32((x * x).sum() / 4)
    exp = x * np.float32(1 / np.sqrt(ms + 1e-5)) * w
    assert np.abs(y - exp).max() < 1e-4


def test_argmax_last_max_wins(oracle):
    # lib.rs:456-464: Iterator::max_by keeps the last maximum
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 2
    assert oracle.argmax(np.array([5], np.float32)) == 0
    assert oracle.argmax(np.array([-1, -1, -1], np.float32)) == 2
    # NaN compares Equal, so the scan moves on to it
    assert oracle.argmax(np.array([1, np.nan, 0.5], np.float32)) == 2


# ---- golden fixtures (reference shaders compiled for the CPU) -----------------

def test_golden_proj(oracle, golden):
    g = golden("proj_q8_0")
    c = oracle.proj(orc.Q8_0, g["x"], g["w"], int(g["k"]), int(g["n"]))
    assert np.array_equal(c, g["c"])
    g = golden("proj_q4k")
    k, n = int(g["k"]), int(g["n"])
    assert np.array_equal(oracle.proj(orc.Q4_K, g["x"], g["w"], k, n, expert_offset=0), g["c0"])
    assert np.array_equal(oracle.proj(orc.Q4_K, g["x"], g["w"], k, n, expert_offset=n * k), g["c1"])
    g = golden("proj_f32")
    k, n = int(g["k"]), int(g["n"])
    assert np.array_equal(oracle.proj(orc.F32, g["x"], g["w"], k, n, row_major=0), g["c0"])
    assert np.array_equal(oracle.proj(orc.F32, g["x"], g["w"], k, n, row_major=1), g["c1"])


def test_golden_dequant(oracle, golden):
    g = golden("dequant_shader")
    assert np.array_equal(oracle.dequant_shader(g["wq8"], orc.Q8_0, g["deq8"].size).reshape(g["deq8"].shape),
                          g["deq8"])
    assert np.array_equal(oracle.dequant_shader(g["wq4"], orc.Q4_K, g["deq4"].size).reshape(g["deq4"].shape),
                          g["deq4"])
    # the Rust CPU decoder's Q8_0 branch agrees with the shader decode
    assert np.array_equal(oracle.dequant_to_f32(g["wq8"].ravel(), orc.Q8_0, g["deq8"].size),
                          g["deq8"].ravel())


def test_golden_ops(oracle, golden):
    g = golden("ops")
    assert np.array_equal(oracle.rmsnorm(g["rms_x"], g["rms_w"], 1e-5), g["rms_y"])
    for pos in (0, 1, 7, 2063):
        y = oracle.qk_norm_rope(g["qk_x"], g["qk_w"], g["qk_freq"], 4, 128, 128, 1e-6, pos)
        assert np.array_equal(y, g[f"qk_y_pos{pos}"]), pos
    assert np.array_equal(oracle.activation(g["act_gate"], g["act_up"]), g["act_h"])
    assert np.array_equal(oracle.add(g["act_gate"], g["act_up"]), g["add_c"])
    assert np.array_equal(oracle.gate_mul(g["gm_v"], g["gm_gate"], 128), g["gm_out"])
    for q_pos, causal in ((2, 1), (4, 1), (0, 1), (1, 0)):
        o = oracle.mha_attn(g["att_q"], g["att_k"], g["att_v"], 8, 2, 128, 5, float(g["att_scale"]), q_pos, causal)
        assert np.array_equal(o, g[f"att_out_p{q_pos}_c{causal}"]), (q_pos, causal)
    nf, naux, ntok = (int(v) for v in g["enc_dims"])
    assert np.array_equal(oracle.enc_aux_norm(g["enc_x"], g["enc_w"], nf, naux, ntok, 1e-5), g["enc_y"])


# ---- live comparison with the compiled reference shaders -----------------------

def _ref():
    path = orc.build_ref()
    if path is None:
        pytest.skip("reference tree absent and oracle/_ref not built")
    return orc.RefShaders(path)


@pytest.mark.parametrize("seed", [0, 1])
def test_ref_shaders_random(oracle, seed):
    ref = _ref()
    rng = np.random.default_rng(seed)
    G = orc.RefShaders.groups
    k, n = 768, 29
    x = synth.activations(1, k, rng)[0]
    w = synth.q4k_blocks(n, k, rng)
    c = np.zeros(n, np.float32)
    ref.run("proj_q4k", [x, orc.pad4(w), c], np.array([k, n, 0], np.uint32).tobytes(), G(n))
    assert np.array_equal(oracle.proj(orc.Q4_K, x, w, k, n), c)
    w8 = synth.q8_0_blocks(n, k, rng)
    c8 = np.zeros(n, np.float32)
    ref.run("proj_q8_0", [x, orc.pad4(w8), c8], np.array([k, n], np.uint32).tobytes(), G(n))
    assert np.array_equal(oracle.proj(orc.Q8_0, x, w8, k, n), c8)


def test_synth_scale_packing_roundtrip(oracle):
    # The packing used by the generators is the inverse of get_scale_min_k4:
    # decoded weights of a block with d = 1, dmin = 0, q = 1 equal the scales.
    rng = np.random.default_rng(5)
    sc = rng.integers(0, 64, size=(3, 8))
    mn = rng.integers(0, 64, size=(3, 8))
    blk = np.zeros((3, 144), np.uint8)
    blk[:, 0:2] = np.array([0x3C00], np.uint16).view(np.uint8)  # d = 1
    blk[:, 4:16] = synth.pack_scale_min_k4(sc, mn)
    blk[:, 16:] = 0x11  # q = 1 everywhere
    w = oracle.dequant_shader(blk, orc.Q4_K, 3 * 256).reshape(3, 8, 32)
    assert np.array_equal(w[:, :, 0], sc.astype(np.float32))
    blk[:, 0:2] = 0
    blk[:, 2:4] = np.array([0x3C00], np.uint16).view(np.uint8)  # dmin = 1, d = 0
    w = oracle.dequant_shader(blk, orc.Q4_K, 3 * 256).reshape(3, 8, 32)
    assert np.array_equal(w[:, :, 0], -mn.astype(np.float32))
