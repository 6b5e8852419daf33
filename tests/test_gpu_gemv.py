"""GPU parity of the f32-activation GEMV (lc_gemv.cu: one and two tokens) and of
the FFN block call, against the CPU oracle at BASELINE.json's full sizes.

Tolerances:
  * the spec's projection bound, max|err| <= 1e-3 * ||y||_inf, everywhere;
  * and, because these kernels keep the activations in f32 and accumulate
    in f32 (only the summation order differs from kernels/proj_q4k.comp:60-92
    and proj_q8_0.comp:47-67), max|err| <= 2e-5 * ||y||_inf -- including
    activations whose magnitudes span many decades inside one super-block.
"""
import numpy as np
import pytest

import oracle as orc
from conftest import check_tol, to_dev
from laguna_raw_halo_strix_b200 import lc, synth

pytestmark = pytest.mark.gpu

F32_TOL = 2e-5


def run(ctx, dev, dtype, x, w, m, k, n):
    import torch

    xd = to_dev(np.ascontiguousarray(x, np.float32).reshape(m, k), dev)
    wd = to_dev(np.ascontiguousarray(w).view(np.uint8).ravel(), dev)
    cd = torch.full((m, n), float("nan"), device=dev)
    ctx.proj_m(dtype, xd, wd, cd, m, k, n)
    torch.cuda.synchronize()
    return cd.cpu().numpy()


def ref_proj(oracle, dtype, x, w, k, n):
    return np.stack([oracle.proj(dtype, x[j:j + 1], w, k, n)[0] for j in range(x.shape[0])])


@pytest.mark.parametrize("m,k,n", [(1, 4096, 14336), (1, 14336, 4096), (2, 4096, 14336), (2, 14336, 4096),
                                   (1, 20480, 4096)])
def test_q4k_full_size(ctx, dev, oracle, m, k, n):
    """BASELINE config 1 (gate/up 4096->14336, down 14336->4096) and the encoder fc."""
    rng = np.random.default_rng(k + n + m)
    w = synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    c = run(ctx, dev, lc.Q4_K, x, w, m, k, n)
    ref = ref_proj(oracle, orc.Q4_K, x, w, k, n)
    for j in range(m):
        check_tol(c[j], ref[j], 1e-3, f"q4k {k}->{n} token {j}")
        check_tol(c[j], ref[j], F32_TOL, f"q4k {k}->{n} token {j} (f32)")


def test_q8_0_full_size(ctx, dev, oracle):
    """Q8_0 4096x4096, m = 1."""
    rng = np.random.default_rng(0)
    k = n = 4096
    w = synth.q8_0_blocks(n, k, rng)
    x = synth.activations(1, k, rng)
    c = run(ctx, dev, lc.Q8_0, x, w, 1, k, n)
    ref = oracle.proj(orc.Q8_0, x, w, k, n)[0]
    check_tol(c[0], ref, 1e-3, "q8_0 4096x4096")
    check_tol(c[0], ref, F32_TOL, "q8_0 4096x4096 (f32)")


@pytest.mark.parametrize("dtype,m,k,n", [(orc.Q4_K, 1, 256, 1), (orc.Q4_K, 1, 768, 150), (orc.Q4_K, 2, 1280, 7),
                                         (orc.Q4_K, 1, 2304, 333), (orc.Q4_K, 2, 256, 149),
                                         (orc.Q8_0, 1, 256, 1), (orc.Q8_0, 1, 2304, 149), (orc.Q8_0, 1, 6144, 600)])
def test_ragged_shapes(ctx, dev, oracle, dtype, m, k, n):
    """Partial k-slices (k not a multiple of the slice), fewer rows than SMs."""
    rng = np.random.default_rng(k * 3 + n)
    w = synth.weight_blocks(dtype, n, k, rng)
    x = synth.activations(m, k, rng)
    c = run(ctx, dev, dtype, x, w, m, k, n)
    ref = ref_proj(oracle, dtype, x, w, k, n)
    for j in range(m):
        check_tol(c[j], ref[j], F32_TOL, f"dtype {dtype} m={m} k={k} n={n} token {j}")


@pytest.mark.parametrize("dtype,m", [(orc.Q4_K, 1), (orc.Q4_K, 2), (orc.Q8_0, 1)])
def test_wide_dynamic_range(ctx, dev, oracle, dtype, m):
    """Activations spanning 1e-6 .. 1e4 inside every super-block, plus exact
    zeros and subnormals: a scale per block (or any fixed-point activation
    format) would lose the small elements; f32 activations keep them."""
    rng = np.random.default_rng(5 + m)
    k, n = 4096, 512
    w = synth.weight_blocks(dtype, n, k, rng)
    mag = 10.0 ** rng.uniform(-6, 4, size=(m, k))
    x = (rng.choice([-1.0, 1.0], size=(m, k)) * mag).astype(np.float32)
    x[:, ::97] = 0.0
    x[:, 5::131] = np.float32(1e-40)  # subnormal
    c = run(ctx, dev, dtype, x, w, m, k, n)
    ref = ref_proj(oracle, dtype, x, w, k, n)
    for j in range(m):
        check_tol(c[j], ref[j], F32_TOL, f"dtype {dtype} token {j}")


def test_small_elements_beside_large(ctx, dev, oracle):
    """In every super-block, sub-block 0 carries activations of 1e4 whose
    weights are zero (nibbles 0, min 0); the output comes only from the other
    sub-blocks' activations of ~1e-2, which must not be rounded to the large
    ones' precision."""
    rng = np.random.default_rng(9)
    k, n = 4096, 256
    S = k // 256
    sc = rng.integers(1, 64, size=(n * S, 8))
    mn = rng.integers(0, 64, size=(n * S, 8))
    mn[:, 0] = 0
    w = synth.q4k_blocks(n, k, rng).reshape(n * S, 144)
    w[:, 4:16] = synth.pack_scale_min_k4(sc, mn)
    qs = w[:, 16:].reshape(n * S, 4, 32)
    qs[:, 0, :] &= 0xF0  # sub-block 0 = low nibbles of group 0
    w = w.reshape(n, S * 144)
    x = (rng.standard_normal((1, k)) * 1e-2).astype(np.float32)
    x.reshape(S, 256)[:, :32] = 1e4
    c = run(ctx, dev, lc.Q4_K, x, w, 1, k, n)
    ref = oracle.proj(orc.Q4_K, x, w, k, n)[0]
    err = np.abs(c[0].astype(np.float64) - ref)
    assert err.max() <= F32_TOL * np.abs(ref).max(), err.max()


def test_repeat_bitwise(ctx, dev):
    """The k-slices are summed in a fixed order: two calls agree bit for bit."""
    rng = np.random.default_rng(3)
    k, n = 14336, 4096
    w = synth.q4k_blocks(n, k, rng)
    x = synth.activations(1, k, rng)
    a = run(ctx, dev, lc.Q4_K, x, w, 1, k, n)
    b = run(ctx, dev, lc.Q4_K, x, w, 1, k, n)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("dtype,m", [(orc.Q4_K, 1), (orc.Q4_K, 2), (orc.Q8_0, 1), (orc.Q4_K, 16)])
def test_ffn_block(ctx, dev, oracle, dtype, m):
    """lc_ffn = down(SiLU(gate x) * up x) (src/dflash.rs:965-968) at the DFlash
    FFN's full size, against the oracle's projections and activation kernel."""
    import torch

    rng = np.random.default_rng(21 + m)
    E, F = 4096, 14336
    wg = synth.weight_blocks(dtype, F, E, rng)
    wu = synth.weight_blocks(dtype, F, E, rng)
    wd = synth.weight_blocks(dtype, E, F, rng)
    x = synth.activations(m, E, rng)
    y = torch.full((m, E), float("nan"), device=dev)
    ctx.ffn(dtype, to_dev(x, dev), to_dev(wg, dev), to_dev(wu, dev), to_dev(wd, dev), y, m, E, F)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for j in range(m):
        g = oracle.proj(dtype, x[j:j + 1], wg, E, F)[0]
        u = oracle.proj(dtype, x[j:j + 1], wu, E, F)[0]
        h = oracle.activation(g, u)
        ref = oracle.proj(dtype, h[None, :], wd, F, E)[0]
        check_tol(got[j], ref, 1e-3, f"ffn dtype {dtype} token {j}")
        if m <= 2:
            check_tol(got[j], ref, F32_TOL, f"ffn dtype {dtype} token {j} (f32)")


@pytest.mark.parametrize("dtype,m,E,F", [(orc.Q4_K, 1, 512, 768), (orc.Q4_K, 2, 256, 1280), (orc.Q8_0, 1, 256, 256),
                                         (orc.Q4_K, 1, 256, 256), (orc.Q8_0, 1, 2048, 2304)])
def test_ffn_block_small(ctx, dev, oracle, dtype, m, E, F):
    """The interleaved gate/up launch at sizes where CTAs hold a few row pairs
    (2F rows over 148 CTAs, range bounds rounded to whole pairs, some CTAs
    with none): every SiLU(gate) * up pair formed once, as the oracle's."""
    import torch

    rng = np.random.default_rng(7 * F + m)
    wg = synth.weight_blocks(dtype, F, E, rng)
    wu = synth.weight_blocks(dtype, F, E, rng)
    wd = synth.weight_blocks(dtype, E, F, rng)
    x = synth.activations(m, E, rng)
    y = torch.full((m, E), float("nan"), device=dev)
    ctx.ffn(dtype, to_dev(x, dev), to_dev(wg, dev), to_dev(wu, dev), to_dev(wd, dev), y, m, E, F)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for j in range(m):
        h = oracle.activation(oracle.proj(dtype, x[j:j + 1], wg, E, F)[0], oracle.proj(dtype, x[j:j + 1], wu, E, F)[0])
        check_tol(got[j], oracle.proj(dtype, h[None, :], wd, F, E)[0], F32_TOL, f"ffn {dtype} m={m} {E}x{F} row {j}")


@pytest.mark.parametrize("dtype,m", [(orc.Q4_K, 1), (orc.Q8_0, 1), (orc.Q4_K, 16)])
def test_host_buffer_calls(ctx, dev, dtype, m):
    """lc_ffn_host / lc_proj_m_host (upload, compute, read back in one call)
    return what the device-pointer calls leave on the device: bit for bit at
    one token (fixed summation order), within f32 rounding at 16 (the tcgen05
    GEMM adds its split sums with atomics, in no fixed order)."""
    import torch

    def same(a, b):
        if m == 1:
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        else:
            check_tol(a, b, 1e-5, "host-buffer call")

    rng = np.random.default_rng(40 + m)
    E, F = 4096, 14336
    wg, wu, wd = (to_dev(synth.weight_blocks(dtype, r, c, rng), dev) for r, c in ((F, E), (F, E), (E, F)))
    x = synth.activations(m, E, rng)
    x_host = torch.from_numpy(x).pin_memory()
    y_host = torch.full((m, E), float("nan")).pin_memory()
    ctx.ffn_host(dtype, x_host, wg, wu, wd, y_host, m, E, F)
    y = torch.full((m, E), float("nan"), device=dev)
    ctx.ffn(dtype, to_dev(x, dev), wg, wu, wd, y, m, E, F)
    torch.cuda.synchronize()
    same(y_host.numpy(), y.cpu().numpy())
    c_host = torch.full((m, F), float("nan")).pin_memory()
    ctx.proj_m_host(dtype, x_host, wg, c_host, m, E, F)
    c = torch.full((m, F), float("nan"), device=dev)
    ctx.proj_m(dtype, to_dev(x, dev), wg, c, m, E, F)
    torch.cuda.synchronize()
    same(c_host.numpy(), c.cpu().numpy())
