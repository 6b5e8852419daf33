"""GPU parity: every kernel of the C ABI against the CPU oracle and the golden
fixtures of the reference shaders.

Tolerances (stated per test):
  * dequant: bit-exact;
  * projections: max|err| <= 1e-3 * ||y||_inf (f32 accumulation, reordered sums);
  * element-wise ops: bit-exact where the reference is exactly rounded
    (add, gate_mul), else 2e-6 relative (exp/log/sin/cos/rsqrt ulp differences).
"""
import numpy as np
import pytest

import oracle as orc
from conftest import check_tol, to_dev
from laguna_raw_halo_strix_b200 import lc, synth

pytestmark = pytest.mark.gpu


def run_proj(ctx, dev, dtype, x, w, m, k, n, eo=0):
    import torch

    xd = to_dev(np.ascontiguousarray(x, np.float32).reshape(m, k), dev)
    wd = to_dev(np.ascontiguousarray(w).view(np.uint8).ravel(), dev)
    cd = torch.full((m, n), float("nan"), device=dev)
    if m == 1 and dtype == lc.Q4_K:
        ctx.proj_q4k(xd, wd, cd, k, n, eo)
    elif m == 1 and dtype == lc.Q8_0:
        ctx.proj_q8_0(xd, wd, cd, k, n)
    elif m == 1 and dtype == lc.F32:
        ctx.proj_f32(xd, wd, cd, k, n, 0)
    else:
        ctx.proj_m(dtype, xd, wd, cd, m, k, n, eo)
    torch.cuda.synchronize()
    return cd.cpu().numpy()


# ---- golden fixtures --------------------------------------------------------------

def test_golden_proj(ctx, dev, golden):
    g = golden("proj_q8_0")
    c = run_proj(ctx, dev, lc.Q8_0, g["x"], g["w"], 1, int(g["k"]), int(g["n"]))
    check_tol(c[0], g["c"], 1e-3, "q8_0 golden")
    g = golden("proj_q4k")
    k, n = int(g["k"]), int(g["n"])
    check_tol(run_proj(ctx, dev, lc.Q4_K, g["x"], g["w"], 1, k, n, 0)[0], g["c0"], 1e-3, "q4k golden e0")
    check_tol(run_proj(ctx, dev, lc.Q4_K, g["x"], g["w"], 1, k, n, n * k)[0], g["c1"], 1e-3, "q4k golden e1")
    g = golden("proj_f32")
    k, n = int(g["k"]), int(g["n"])
    check_tol(run_proj(ctx, dev, lc.F32, g["x"], g["w"], 1, k, n)[0], g["c0"], 1e-5, "f32 golden")


def test_golden_dequant_bitexact(ctx, dev, golden):
    import torch

    g = golden("dequant_shader")
    for key_w, key_d, dt in (("wq8", "deq8", lc.Q8_0), ("wq4", "deq4", lc.Q4_K)):
        w = to_dev(g[key_w].ravel(), dev)
        out = torch.empty(g[key_d].size, device=dev)
        ctx.dequant(dt, w, g[key_w].nbytes, g[key_d].size, out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), g[key_d].ravel().view(np.uint32)), dt


# ---- projections vs oracle at many shapes ------------------------------------------

@pytest.mark.parametrize("m,k,n", [(1, 256, 1), (1, 256, 17), (1, 4096, 300), (2, 512, 33), (3, 1024, 64),
                                   (4, 256, 50), (5, 512, 40), (16, 1024, 129), (17, 256, 20), (1, 14336, 64)])
def test_q4k_vs_oracle(ctx, dev, oracle, m, k, n):
    rng = np.random.default_rng(m * 1000 + n)
    w = synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    c = run_proj(ctx, dev, lc.Q4_K, x, w, m, k, n)
    ref = oracle.proj(orc.Q4_K, x, w, k, n).reshape(m, n)
    for r in range(m):
        check_tol(c[r], ref[r], 1e-3, f"q4k m={m} row {r}")


@pytest.mark.parametrize("m,k,n", [(1, 64, 1), (1, 256, 31), (1, 4096, 300), (2, 128, 33), (4, 4096, 16),
                                   (7, 512, 45), (16, 4096, 130), (1, 96, 10), (3, 32, 5), (2, 14336, 100),
                                   (3, 768, 1000)])
def test_q8_0_vs_oracle(ctx, dev, oracle, m, k, n):
    rng = np.random.default_rng(m * 7 + n)
    w = synth.q8_0_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    c = run_proj(ctx, dev, lc.Q8_0, x, w, m, k, n)
    ref = oracle.proj(orc.Q8_0, x, w, k, n).reshape(m, n)
    for r in range(m):
        check_tol(c[r], ref[r], 1e-3, f"q8_0 m={m} row {r}")


def test_q4k_expert_offset(ctx, dev, oracle):
    rng = np.random.default_rng(11)
    k, n = 512, 24
    w = synth.q4k_blocks(3 * n, k, rng)
    x = synth.activations(1, k, rng)
    for e in range(3):
        c = run_proj(ctx, dev, lc.Q4_K, x, w, 1, k, n, e * n * k)
        check_tol(c[0], oracle.proj(orc.Q4_K, x, w, k, n, expert_offset=e * n * k), 1e-3, f"expert {e}")


def test_f32_proj_both_layouts(ctx, dev, oracle):
    import torch

    rng = np.random.default_rng(2)
    for k, n in ((8, 3), (100, 37), (4096, 70)):
        x = synth.activations(1, k, rng)[0]
        w = (rng.standard_normal(n * k) * 0.1).astype(np.float32)
        for rm in (0, 1):
            cd = torch.empty(n, device=dev)
            ctx.proj_f32(to_dev(x, dev), to_dev(w, dev), cd, k, n, rm)
            torch.cuda.synchronize()
            check_tol(cd.cpu().numpy(), oracle.proj(orc.F32, x, w, k, n, row_major=rm), 1e-5, f"f32 rm={rm}")


def test_matmul_selftest_gpu(ctx, dev):
    # src/lib.rs:120-165 run through the device path
    import torch

    a = (np.arange(8, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    b = (np.arange(24, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    c = torch.empty(3, device=dev)
    ctx.proj_f32(to_dev(a, dev), to_dev(b, dev), c, 8, 3, 0)
    torch.cuda.synchronize()
    exp = np.array([sum(a[i] * b[j * 8 + i] for i in range(8)) for j in range(3)], np.float32)
    assert np.abs(c.cpu().numpy() - exp).max() < 1e-4


def test_half_mode_ieee(ctx, dev, oracle):
    # IEEE decoding differs from the reference rule only on subnormal scales.
    rng = np.random.default_rng(4)
    k, n = 256, 64
    w = synth.q8_0_blocks(n, k, rng)
    x = synth.activations(1, k, rng)
    ref_mode = run_proj(ctx, dev, lc.Q8_0, x, w, 1, k, n)[0]
    ctx.set_half_mode(lc.HALF_IEEE)
    try:
        ieee = run_proj(ctx, dev, lc.Q8_0, x, w, 1, k, n)[0]
    finally:
        ctx.set_half_mode(lc.HALF_REF)
    wf = w.reshape(-1, 34)
    d = wf[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(n, k // 32)
    q = wf[:, 2:].view(np.int8).astype(np.float32).reshape(n, k // 32, 32)
    exp = (q * d[:, :, None]).reshape(n, k) @ x[0].astype(np.float32)
    check_tol(ieee, exp, 1e-3, "ieee")
    assert not np.allclose(ieee, ref_mode)


def test_errors_are_reported(ctx, dev):
    import torch

    x = torch.zeros(300, device=dev)
    w = torch.zeros(10000, dtype=torch.uint8, device=dev)
    c = torch.zeros(4, device=dev)
    with pytest.raises(lc.LagunaError) as e:
        ctx.proj_q4k(x, w, c, 300, 4)  # k not a multiple of 256
    assert e.value.status == lc.LC_ERR_UNSUPPORTED
    with pytest.raises(lc.LagunaError) as e:
        ctx.proj_q4k(x, w.data_ptr() + 4, c, 256, 4)  # misaligned weights
    assert e.value.status == lc.LC_ERR_INVALID
    with pytest.raises(lc.LagunaError):
        ctx.proj_quant(99, x, w, c, 256, 4)
    ctx.proj_q4k(x, w, c, 256, 0)  # empty output is a no-op


# ---- dequant ---------------------------------------------------------------------------

@pytest.mark.parametrize("dtype,nel", [(orc.Q8_0, 4096), (orc.Q4_K, 4096), (orc.F32, 100), (orc.F16, 777),
                                       (orc.BF16, 777), (1012, 512)])
def test_dequant_vs_oracle(ctx, dev, oracle, dtype, nel):
    import torch

    rng = np.random.default_rng(dtype)
    if dtype == orc.Q8_0:
        raw = synth.q8_0_blocks(1, nel, rng).ravel()
    elif dtype in (orc.Q4_K, 1012):
        raw = synth.q4k_blocks(1, nel, rng).ravel()
    elif dtype == orc.F32:
        raw = rng.standard_normal(nel).astype(np.float32).view(np.uint8)
    else:
        raw = rng.integers(0, 65536, nel, dtype=np.int64).astype(np.uint16).view(np.uint8)
    for nbytes in (raw.size, raw.size - 7):
        out = torch.full((nel,), float("nan"), device=dev)
        ctx.dequant(dtype, to_dev(raw, dev), nbytes, nel, out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        if dtype == orc.Q4_K:
            exp = oracle.dequant_shader(raw[: nbytes // 144 * 144], orc.Q4_K, nbytes // 144 * 256)
            exp = np.concatenate([exp, np.zeros(nel - exp.size, np.float32)])
        else:
            # the reference CPU decoder's own "Q4_K" branch is GGUF id 12 in the
            # oracle (it restates dequant_to_f32), LC_Q4_K_DFLASH_CPU on the device
            exp = oracle.dequant_to_f32(raw[:nbytes], orc.Q4_K if dtype == 1012 else dtype, nel)
        # bit-exact; NaNs (random bf16 fields of the legacy decoder) compare as
        # NaN, since GPU arithmetic returns the canonical NaN payload
        nan = np.isnan(exp)
        assert np.array_equal(np.isnan(got), nan), (dtype, nbytes)
        assert np.array_equal(got[~nan].view(np.uint32), exp[~nan].view(np.uint32)), (dtype, nbytes)


# ---- interleaved ops -----------------------------------------------------------------

def test_golden_ops(ctx, dev, golden):
    import torch

    g = golden("ops")
    d = lambda a: to_dev(a, dev)  # noqa: E731
    y = torch.empty(4096, device=dev)
    ctx.rmsnorm(d(g["rms_w"]), d(g["rms_x"]), y, 1, 4096, 1e-5)
    torch.cuda.synchronize()
    check_tol(y.cpu().numpy(), g["rms_y"], 2e-6, "rmsnorm")
    for pos in (0, 1, 7, 2063):
        yq = torch.empty(512, device=dev)
        ctx.qk_norm_rope(d(g["qk_x"]), d(g["qk_w"]), d(g["qk_freq"]), yq, 1, 4, 128, 128, 1e-6, pos)
        torch.cuda.synchronize()
        check_tol(yq.cpu().numpy(), g[f"qk_y_pos{pos}"], 2e-5 if pos > 100 else 2e-6, f"qk_norm_rope pos {pos}")
    h = torch.empty(1000, device=dev)
    ctx.activation(d(g["act_gate"]), d(g["act_up"]), h, 1000)
    s = torch.empty(1000, device=dev)
    ctx.add(d(g["act_gate"]), d(g["act_up"]), s, 1000)
    gm = torch.empty(512, device=dev)
    ctx.gate_mul(d(g["gm_v"]), d(g["gm_gate"]), gm, 512, 4, 128)
    torch.cuda.synchronize()
    check_tol(h.cpu().numpy(), g["act_h"], 2e-6, "activation")
    assert np.array_equal(s.cpu().numpy(), g["add_c"])
    assert np.array_equal(gm.cpu().numpy(), g["gm_out"])
    for q_pos, causal in ((2, 1), (4, 1), (0, 1), (1, 0)):
        o = torch.empty(8 * 128, device=dev)
        ctx.mha_attn(d(g["att_q"]), d(g["att_k"]), d(g["att_v"]), o, 1, 8, 2, 128, 5, float(g["att_scale"]),
                     q_pos, causal)
        torch.cuda.synchronize()
        check_tol(o.cpu().numpy(), g[f"att_out_p{q_pos}_c{causal}"], 1e-5, f"attn {q_pos} {causal}")
    nf, naux, ntok = (int(v) for v in g["enc_dims"])
    ye = torch.empty(nf * naux * ntok, device=dev)
    ctx.enc_aux_norm(d(g["enc_x"]), d(g["enc_w"]), ye, nf, naux, ntok, 1e-5)
    torch.cuda.synchronize()
    check_tol(ye.cpu().numpy(), g["enc_y"], 2e-6, "enc_aux_norm")


def test_rmsnorm_rows_inplace(ctx, dev, oracle):
    import torch

    rng = np.random.default_rng(8)
    for m, n in ((3, 4096), (16, 4096), (2, 20480), (1, 5)):
        x = rng.standard_normal((m, n)).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        xd = to_dev(x, dev)
        ctx.rmsnorm(to_dev(w, dev), xd, xd, m, n, 1e-5)  # in place, like output_norm x -> x
        torch.cuda.synchronize()
        ref = oracle.rmsnorm(x, w, 1e-5)
        for r in range(m):
            check_tol(xd[r].cpu().numpy(), ref[r], 3e-6, "rmsnorm rows")


def test_qk_norm_rope_block(ctx, dev, oracle):
    import torch

    rng = np.random.default_rng(9)
    m, nh, hd = 16, 8, 128
    x = rng.standard_normal((m, nh * hd)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = oracle.rope_freq(hd, 500000.0)
    for rope_dim in (128, 0):
        y = torch.empty(m, nh * hd, device=dev)
        ctx.qk_norm_rope(to_dev(x, dev), to_dev(w, dev), to_dev(freq, dev), y, m, nh, hd, rope_dim, 1e-6, 2048)
        torch.cuda.synchronize()
        ref = oracle.qk_norm_rope(x, w, freq, nh, hd, rope_dim, 1e-6, np.arange(2048, 2048 + m))
        check_tol(y.cpu().numpy(), ref, 2e-5, f"qk_norm_rope rope_dim={rope_dim}")
    # partial rotary indexes outside the head in the reference: rejected
    with pytest.raises(lc.LagunaError) as e:
        ctx.qk_norm_rope(to_dev(x, dev), to_dev(w, dev), to_dev(freq, dev), y, m, nh, hd, 64, 1e-6, 0)
    assert e.value.status == lc.LC_ERR_UNSUPPORTED


def test_softplus(ctx, dev, oracle):
    import torch

    g = np.array([-30, -5, -0.5, 0, 0.5, 5, 19.9, 20, 20.1, 50], np.float32)
    out = torch.empty(g.size, device=dev)
    ctx.softplus(to_dev(g, dev), out, g.size)
    torch.cuda.synchronize()
    check_tol(out.cpu().numpy(), oracle.softplus(g), 2e-6, "softplus")


@pytest.mark.parametrize("m,seq,q_pos0,causal", [(1, 2, 1, 1), (16, 2064, 2048, 1), (16, 80, 64, 0),
                                                 (3, 40, 0, 1), (2, 0, 0, 1)])
def test_mha_attn_block(ctx, dev, oracle, m, seq, q_pos0, causal):
    import torch

    rng = np.random.default_rng(seq + m)
    nq, nkv, hd = 32, 8, 128
    q = rng.standard_normal((m, nq * hd)).astype(np.float32)
    k = rng.standard_normal((max(seq, 1), nkv * hd)).astype(np.float32)
    v = rng.standard_normal((max(seq, 1), nkv * hd)).astype(np.float32)
    scale = float(np.float32(1 / np.sqrt(hd)))
    out = torch.empty(m, nq * hd, device=dev)
    ctx.mha_attn(to_dev(q, dev), to_dev(k, dev), to_dev(v, dev), out, m, nq, nkv, hd, seq, scale, q_pos0, causal)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r in range(m):
        ref = oracle.mha_attn(q[r], k, v, nq, nkv, hd, seq, scale, q_pos0 + r, causal)
        check_tol(got[r], ref, 1e-5, f"attn row {r}")


# ---- argmax / lm_head ---------------------------------------------------------------

def test_argmax_rows_ties(ctx, dev, oracle):
    import torch

    rng = np.random.default_rng(10)
    m, n = 5, 50000
    logits = rng.standard_normal((m, n)).astype(np.float32)
    logits[1, 7] = logits[1, 4000] = 99.0  # tie -> last index
    logits[2, :] = 1.0  # all equal -> last index
    keys = torch.empty(m, dtype=torch.int64, device=dev)
    ctx.argmax_rows(to_dev(logits, dev), m, n, 1000, keys)
    torch.cuda.synchronize()
    for r, key in enumerate(keys.cpu().numpy()):
        k = int(np.int64(key).view(np.uint64))
        assert lc.key_index(k) == 1000 + oracle.argmax(logits[r])
        assert lc.key_value(k) == logits[r].max()


@pytest.mark.parametrize("dtype", [lc.Q8_0, lc.Q4_K])
def test_lm_head_argmax(ctx, dev, oracle, dtype):
    import torch

    rng = np.random.default_rng(12)
    m, k, n = 6, 512, 3000
    w = synth.q8_0_blocks(n, k, rng) if dtype == lc.Q8_0 else synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    keys = torch.empty(m, dtype=torch.int64, device=dev)
    logits = torch.empty(m, n, device=dev)
    ctx.lm_head_argmax(dtype, to_dev(x, dev), to_dev(w, dev), m, k, n, 0, keys, logits)
    torch.cuda.synchronize()
    ref = oracle.proj(dtype, x, w, k, n).reshape(m, n)
    lg = logits.cpu().numpy()
    for r in range(m):
        check_tol(lg[r], ref[r], 1e-3, "lm_head logits")
        kk = int(np.int64(keys[r].item()).view(np.uint64))
        idx = lc.key_index(kk)
        assert idx == n - 1 - int(np.argmax(lg[r][::-1]))  # last maximum of the returned logits
        # same token as the oracle unless the top two are within the error bound
        o = oracle.argmax(ref[r])
        if idx != o:
            srt = np.sort(ref[r])
            assert srt[-1] - srt[-2] <= 2e-3 * np.abs(ref[r]).max()


@pytest.mark.parametrize("dtype", [lc.Q8_0, lc.Q4_K])
def test_lm_head_argmax_tiles(ctx, dev, oracle, dtype):
    """More than 32 rows: the tensor-core tiles with the argmax in the epilogue
    (200 rows = a full and a partial 128-token tile; 3000 vocab rows = 23 full
    128-row tiles and a partial one; a shard offset)."""
    import torch

    rng = np.random.default_rng(13)
    m, k, n, off = 200, 512, 3000, 777
    w = synth.q8_0_blocks(n, k, rng) if dtype == lc.Q8_0 else synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    xd, wd = to_dev(x, dev), to_dev(w, dev)
    keys = torch.empty(m, dtype=torch.int64, device=dev)
    logits = torch.full((m, n), float("nan"), device=dev)
    ctx.lm_head_argmax(dtype, xd, wd, m, k, n, off, keys, logits)
    keys2 = torch.empty(m, dtype=torch.int64, device=dev)
    ctx.lm_head_argmax(dtype, xd, wd, m, k, n, off, keys2)  # without the logits output
    torch.cuda.synchronize()
    ctx.device_status()
    ref = oracle.proj(dtype, x, w, k, n).reshape(m, n)
    lg = logits.cpu().numpy()
    assert np.array_equal(keys.cpu().numpy(), keys2.cpu().numpy())
    for r in range(m):
        check_tol(lg[r], ref[r], 1e-3, "lm_head logits")
        kk = int(np.int64(keys[r].item()).view(np.uint64))
        idx = lc.key_index(kk)
        j = n - 1 - int(np.argmax(lg[r][::-1]))  # last maximum of the returned logits
        assert idx == off + j
        assert lc.key_value(kk) == lg[r][j]
        o = oracle.argmax(ref[r])
        if idx != off + o:
            srt = np.sort(ref[r])
            assert srt[-1] - srt[-2] <= 2e-3 * np.abs(ref[r]).max()


@pytest.mark.parametrize("dtype", [lc.Q4_K, lc.Q8_0])
def test_repeat_calls_consistent(ctx, dev, oracle, dtype):
    # The stream-K kernels sum split tiles in a scratch that each call must
    # leave zeroed; back-to-back calls (different n, then the same) agree.
    rng = np.random.default_rng(21)
    k = 4096
    for n in (4096, 777, 4096):
        w = synth.q4k_blocks(n, k, rng) if dtype == lc.Q4_K else synth.q8_0_blocks(n, k, rng)
        x = synth.activations(1, k, rng)
        ref = oracle.proj(dtype, x, w, k, n)
        a = run_proj(ctx, dev, dtype, x, w, 1, k, n)[0]
        b = run_proj(ctx, dev, dtype, x, w, 1, k, n)[0]
        check_tol(a, ref, 1e-3, "first call")
        check_tol(b, ref, 1e-3, "second call")
        assert np.abs(a - b).max() <= 1e-5 * np.abs(ref).max()
    ctx.device_status()  # no bounded device-side wait gave up


@pytest.mark.parametrize("dtype", [lc.Q4_K, lc.Q8_0])
@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("scale", [3e5, 1e-6])
def test_activation_range(ctx, dev, oracle, dtype, m, scale):
    # Activations far outside the f16 range (or deep in its subnormals) are
    # scaled by a per-token power of two before the f16 hi/lo split.
    rng = np.random.default_rng(int(m * 10 + (scale > 1)))
    k, n = 1024, 96
    w = synth.q4k_blocks(n, k, rng) if dtype == lc.Q4_K else synth.q8_0_blocks(n, k, rng)
    x = (synth.activations(m, k, rng) * np.float32(scale)).astype(np.float32)
    x[0, 5] *= 50  # one outlier
    c = run_proj(ctx, dev, dtype, x, w, m, k, n)
    ref = oracle.proj(dtype, x, w, k, n).reshape(m, n)
    assert np.isfinite(c).all()
    for r in range(m):
        check_tol(c[r], ref[r], 1e-3, f"range m={m} scale={scale} row {r}")


# ---- every projection route at every token count ------------------------------------

def _ctx_with_env(env):
    """A context created while the routing variables in `env` are set (they are
    read once, at lc_init)."""
    import os

    import torch

    old = {key: os.environ.get(key) for key in env}
    os.environ.update(env)
    try:
        c = lc.Context(0)
    finally:
        for key, v in old.items():
            if v is None:
                os.environ.pop(key, None)
            else:
                os.environ[key] = v
    c.set_stream(torch.cuda.current_stream())
    return c


@pytest.mark.parametrize("route", ["i8_all", "i8_none"])
@pytest.mark.parametrize("dtype", [lc.Q4_K, lc.Q8_0])
def test_proj_routes_all_m(dev, oracle, dtype, route):
    # i8_all: 1..16 tokens on the int8 tcgen05 GEMV; i8_none: 1..4 on the TMA
    # GEMV, 5..32 on the f16 tcgen05 GEMM, 33+ on the lm_head tiles.
    env = {"LC_GEMV_I8_MIN": "1", "LC_GEMV_I8_MAX": "16"} if route == "i8_all" else {"LC_GEMV_I8_MAX": "0"}
    c = _ctx_with_env(env)
    try:
        k, n = 2048, 300
        rng = np.random.default_rng(11 + (dtype == lc.Q8_0))
        w = synth.q4k_blocks(n, k, rng) if dtype == lc.Q4_K else synth.q8_0_blocks(n, k, rng)
        x_all = synth.activations(40, k, rng)
        ref_all = oracle.proj(dtype, x_all, w, k, n).reshape(40, n)
        for m in (list(range(1, 17)) if route == "i8_all" else [1, 4, 5, 9, 16, 32, 33, 40]):
            out = run_proj(c, dev, dtype, x_all[:m], w, m, k, n)
            for r in range(m):
                check_tol(out[r], ref_all[r], 1e-3, f"{route} m={m} row {r}")
        c.device_status()
    finally:
        c.close()


@pytest.mark.parametrize("m,seq,q_pos0,causal,nq,nkv,mag", [
    (16, 300, 284, 1, 32, 8, 1.0),      # partial last key tile
    (8, 129, 121, 1, 32, 8, 1.0),       # one key past a tile boundary
    (32, 200, 168, 1, 32, 8, 1.0),      # 128 query vectors: two query chunks
    (16, 257, 241, 1, 64, 8, 1.0),      # 8 query heads per KV head, two chunks
    (5, 70, 65, 1, 8, 8, 1.0),          # one query head per KV head
    (16, 150, 134, 0, 32, 8, 3e4),      # values far beyond the f16 range
    (16, 150, 134, 1, 32, 8, 1e-5),     # and deep in its subnormals
])
def test_mha_attn_shapes(ctx, dev, oracle, m, seq, q_pos0, causal, nq, nkv, mag):
    # The tensor-core kernel splits keys into 128-key tiles and query vectors
    # into chunks of 64, and scales rows / tiles by powers of two before its
    # f16 hi / lo split; tolerance 1e-5 of max|ref| per row, as above.  q, k, v
    # of magnitude `mag` leave the f16 range; the softmax scale divides by mag^2
    # so the logits stay O(1) (its scores carry ~22 significant bits, so their
    # absolute error grows with the logits' size).
    import torch

    rng = np.random.default_rng(seq * 7 + m + nq)
    hd = 128
    q = (rng.standard_normal((m, nq * hd)) * mag).astype(np.float32)
    k = (rng.standard_normal((seq, nkv * hd)) * mag).astype(np.float32)
    v = (rng.standard_normal((seq, nkv * hd)) * mag).astype(np.float32)
    scale = float(np.float32(1 / np.sqrt(hd) / (mag * mag)))
    out = torch.empty(m, nq * hd, device=dev)
    ctx.mha_attn(to_dev(q, dev), to_dev(k, dev), to_dev(v, dev), out, m, nq, nkv, hd, seq, scale, q_pos0, causal)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r in range(m):
        ref = oracle.mha_attn(q[r], k, v, nq, nkv, hd, seq, scale, q_pos0 + r, causal)
        check_tol(got[r], ref, 1e-5, f"attn row {r}")
    ctx.device_status()
