"""lc_proj_q4k_static: the Q4_K projection that allocates no device memory
(m <= 4: the cluster GEMV, which needs no scratch; m = 5..16: the tiled path
with its packed activations in a static device array).  Compared through the
C ABI with the existing entry point (lc_proj_m, LC_Q4_K) and the CPU oracle,
on two calls in a row.  Named to be collected last; it also passes alone in a
fresh process."""
import numpy as np
import pytest

import oracle as orc
from conftest import check_tol, to_dev
from laguna_raw_halo_strix_b200 import lc, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max|err| <= TOL * ||ref||_inf, the projection tolerance


@pytest.mark.parametrize("m,k,n", [(1, 4096, 14336), (2, 1024, 777), (3, 512, 4096), (2, 14336, 4096),
                                   (4, 4096, 4096), (1, 256, 16), (8, 4096, 1000), (16, 14336, 4096),
                                   (5, 256, 40)])
def test_static_matches_existing_entry(ctx, dev, m, k, n):
    import torch

    rng = np.random.default_rng(1000 * m + n)
    w = synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    wd, xd = to_dev(w, dev), to_dev(x, dev)
    ref = torch.empty(m, n, device=dev)
    ctx.proj_m(lc.Q4_K, xd, wd, ref, m, k, n)
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    for call in range(2):
        got = torch.full((m, n), float("nan"), device=dev)
        free0 = torch.cuda.mem_get_info()[0]
        ctx.proj_q4k_static(xd, wd, got, m, k, n)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free0  # no device memory taken
        check_tol(got.cpu().numpy(), ref_h, TOL, f"call {call} vs lc_proj_m")


def test_static_matches_oracle(ctx, dev, oracle):
    import torch

    m, k, n = 2, 1024, 333
    rng = np.random.default_rng(7)
    w = synth.q4k_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    ref = oracle.proj(orc.Q4_K, x, w, k, n)
    got = torch.empty(m, n, device=dev)
    for _ in range(2):
        ctx.proj_q4k_static(to_dev(x, dev), to_dev(w, dev), got, m, k, n)
        torch.cuda.synchronize()
        check_tol(got.cpu().numpy(), ref, TOL, "vs oracle")


def test_static_rejects_out_of_range(ctx, dev):
    import torch

    rng = np.random.default_rng(3)
    w = to_dev(synth.q4k_blocks(16, 256, rng), dev)
    x = to_dev(synth.activations(17, 256, rng), dev)
    c = torch.empty(17, 16, device=dev)
    cases = [((17, 256, 16), "at most 16"),          # more than 16 tokens
             ((1, 320, 16), "multiple of 256"),       # k not a multiple of 256
             ((4, 32768, 16), "shared memory"),       # 4 x 32768 activation table exceeds shared memory
             ((16, 16384, 16), "static scratch")]     # packed activations exceed the 1 MiB array
    for (m, k, n), what in cases:  # all rejected on the host, before any launch
        with pytest.raises(lc.LagunaError) as e:
            ctx.proj_q4k_static(x, w, c, m, k, n)
        assert e.value.status == lc.LC_ERR_UNSUPPORTED and what in str(e.value), (m, k, n, str(e.value))
