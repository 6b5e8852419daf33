"""lc_proj_q4k_static: the Q4_K projection that allocates no device memory
(m <= 2: the f32-activation row GEMV and m = 3, 4: the cluster GEMV, which
need no scratch; m = 5..16: the tiled path with its packed activations in a
static device array).  Some callers cannot allocate on the call path -- a
serving loop whose memory plan has handed all of HBM to weights and K/V, or a
decode loop that must not pay cudaMalloc's device-wide synchronisation -- and
this entry point is for them.

Checked through the C ABI against the CPU oracle and against the existing entry
point (lc_proj_m, LC_Q4_K), on two calls in a row, on a fresh context whose
scratch has never been used: the context's scratch stays at 0 bytes and the
device's free memory does not move around either call (after one call on
another context has loaded the kernels' code).  Named to be collected
last; it also passes alone in a fresh process."""
import numpy as np
import pytest

import oracle as orc
from conftest import check_tol, to_dev
from laguna_raw_halo_strix_b200 import lc, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max|err| <= TOL * ||ref||_inf, the projection tolerance


@pytest.fixture(scope="module")
def fresh():
    """A context of its own: its scratch slots are never grown by other tests."""
    import torch

    c = lc.Context(0)
    c.set_stream(torch.cuda.current_stream())
    yield c
    c.close()


@pytest.mark.parametrize("m,k,n,eo", [(1, 4096, 14336, 0), (2, 1024, 777, 0), (3, 512, 4096, 0),
                                      (2, 14336, 4096, 0), (4, 4096, 4096, 0), (1, 256, 16, 0),
                                      (8, 4096, 1000, 0), (16, 14336, 4096, 0), (5, 256, 40, 0),
                                      (1, 512, 24, 2 * 24 * 512), (6, 512, 24, 24 * 512)])
def test_static_vs_oracle_and_existing_entry(ctx, fresh, dev, oracle, m, k, n, eo):
    import torch

    rng = np.random.default_rng(1000 * m + n)
    experts = 1 + eo // (n * k)
    w = synth.q4k_blocks(n * experts, k, rng)
    x = synth.activations(m, k, rng)
    ref = oracle.proj(orc.Q4_K, x, w, k, n, expert_offset=eo).reshape(m, n)
    wd, xd = to_dev(w, dev), to_dev(x, dev)
    exist = torch.empty(m, n, device=dev)
    ctx.proj_m(lc.Q4_K, xd, wd, exist, m, k, n, eo)  # the existing entry point, on the shared context
    torch.cuda.synchronize()
    exist_h = exist.cpu().numpy()
    outs = [torch.full((m, n), float("nan"), device=dev) for _ in range(3)]
    # one call on the shared context first: the driver loads a kernel's code on
    # its first launch (lazy module loading), which is not the entry point's doing
    ctx.proj_q4k_static(xd, wd, outs[2], m, k, n, eo)
    torch.cuda.synchronize()
    for call in range(2):
        free0 = torch.cuda.mem_get_info()[0]
        fresh.proj_q4k_static(xd, wd, outs[call], m, k, n, eo)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, f"call {call}: device memory taken"
        assert fresh.scratch_bytes() == 0, f"call {call}: scratch grown"
        got = outs[call].cpu().numpy()
        for r in range(m):
            check_tol(got[r], ref[r], TOL, f"call {call} row {r} vs oracle")
        check_tol(got, exist_h, TOL, f"call {call} vs lc_proj_m")


def test_static_rejects_out_of_range(fresh, dev):
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
            fresh.proj_q4k_static(x, w, c, m, k, n)
        assert e.value.status == lc.LC_ERR_UNSUPPORTED and what in str(e.value), (m, k, n, str(e.value))
    assert fresh.scratch_bytes() == 0
