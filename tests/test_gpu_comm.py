"""The library-owned reduction of the vocab-sharded lm_head (lc_comm, NCCL)
and the device-side bounded waits.

* lc_check_bounded_wait: a wait that nobody ends gives up, lc_device_status
  reports LC_ERR_TIMEOUT, and the context keeps working.
* One rank: lc_lm_head_argmax_sharded over a one-rank communicator equals the
  unsharded lc_lm_head_argmax.
* Two GPUs (skipped with fewer): two processes, one shard each; step 1 must
  equal the unsharded keys; in step 2 rank 1 does not take part (it stays
  between steps, nothing in flight) and rank 0's bounded wait must return
  LC_ERR_TIMEOUT with the communicator aborted -- and its context must still
  run a projection.  NVLS is off in NCCL for this test.
"""
import os
import time

import numpy as np
import pytest

from conftest import check_tol, to_dev
from laguna_raw_halo_strix_b200 import lc, synth
from laguna_raw_halo_strix_b200.lm_head import ShardedLmHead, key_indices, shard_range

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout(ctx, dev, oracle):
    import torch

    ctx.device_status()  # clear
    ctx.check_bounded_wait(4096)
    with pytest.raises(lc.LagunaError) as e:
        ctx.device_status()
    assert e.value.status == lc.LC_ERR_TIMEOUT
    ctx.device_status()  # cleared by the previous read
    # the context still works
    rng = np.random.default_rng(1)
    k, n = 512, 64
    w = synth.q8_0_blocks(n, k, rng)
    x = synth.activations(1, k, rng)
    y = torch.empty(1, n, device=dev)
    ctx.proj_q8_0(to_dev(x, dev), to_dev(w, dev), y, k, n)
    torch.cuda.synchronize()
    check_tol(y.cpu().numpy()[0], oracle.proj(8, x, w, k, n)[0], 1e-3, "after the timeout")


def test_one_rank_comm_matches_unsharded(ctx, dev):
    import torch

    rng = np.random.default_rng(5)
    m, k, n = 40, 512, 3001
    w = synth.q8_0_blocks(n, k, rng)
    x = to_dev(synth.activations(m, k, rng), dev)
    wd = to_dev(w, dev)
    ref = torch.empty(m, dtype=torch.int64, device=dev)
    ctx.lm_head_argmax(lc.Q8_0, x, wd, m, k, n, 0, ref)
    comm = lc.Comm(ctx, lc.comm_unique_id(), 1, 0, timeout_ms=10000)
    try:
        head = ShardedLmHead(ctx, lc.Q8_0, k, n, 0, 1, comm=comm)
        head.w = wd
        keys = torch.empty(m, dtype=torch.int64, device=dev)
        head(x, m, keys)
        comm.wait()
        assert np.array_equal(keys.cpu().numpy(), ref.cpu().numpy())
    finally:
        comm.close()


def _two_rank_main(rank, id_path, out_dir, n, k, m, seed):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    ctx = lc.Context(rank)
    ctx.set_stream(torch.cuda.current_stream(dev))
    result = "start"
    try:
        if rank == 0:
            uid = lc.comm_unique_id()
            with open(id_path + ".tmp", "wb") as f:
                f.write(uid)
            os.replace(id_path + ".tmp", id_path)
        else:
            t0 = time.time()
            while not os.path.exists(id_path):
                if time.time() - t0 > 60:
                    raise RuntimeError("no communicator id")
                time.sleep(0.05)
            uid = open(id_path, "rb").read()
        comm = lc.Comm(ctx, uid, 2, rank, timeout_ms=3000)
        rng = np.random.default_rng(seed)
        w = synth.q8_0_blocks(n, k, rng)
        x = to_dev(synth.activations(m, k, rng), dev)
        head = ShardedLmHead(ctx, lc.Q8_0, k, n, rank, 2, comm=comm).load_shard(
            ShardedLmHead(None, lc.Q8_0, k, n, rank, 2).shard_bytes(w), dev)
        keys = torch.empty(m, dtype=torch.int64, device=dev)
        head(x, m, keys)  # step 1: both ranks
        comm.wait()
        got = keys.cpu().numpy()
        ref = torch.empty(m, dtype=torch.int64, device=dev)
        ctx.lm_head_argmax(lc.Q8_0, x, to_dev(w, dev), m, k, n, 0, ref)
        torch.cuda.synchronize()
        assert np.array_equal(got, ref.cpu().numpy()), "step 1 differs from the unsharded keys"
        lo, hi = shard_range(n, rank, 2)
        assert np.any((key_indices(got) < lo) | (key_indices(got) >= hi)), "no token came from the other shard"
        result = "step1 ok"
        if rank == 1:
            # does not take part in step 2: waits (host only) until rank 0 has reported
            t0 = time.time()
            while not os.path.exists(os.path.join(out_dir, "rank0.txt")) and time.time() - t0 < 60:
                time.sleep(0.05)
            comm.h = None  # the peer aborted; leave without finalising against it
            return
        t0 = time.perf_counter()
        try:
            head(x, m, keys)
            comm.wait()
            result = "step2 completed without rank 1"
        except lc.LagunaError as e:
            result = f"status {e.status} after {time.perf_counter() - t0:.1f}s: {e}"
        comm.h = None  # aborted by the library
        # the context still works after the abort
        y = torch.empty(1, 64, device=dev)
        ctx.proj_q8_0(x, to_dev(w, dev), y, k, 64)
        torch.cuda.synchronize()
        result += " | context ok" if bool(torch.isfinite(y).all()) else " | context broken"
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        result = f"exception: {type(e).__name__}: {e}"
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(result)


def test_two_ranks_and_a_missing_rank(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mctx = mp.get_context("spawn")
    args = (str(tmp_path / "uid"), str(tmp_path), 5003, 1024, 40, 11)
    ps = [mctx.Process(target=_two_rank_main, args=(r,) + args) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=180)
    hung = [i for i, p in enumerate(ps) if p.is_alive()]
    for p in ps:
        if p.is_alive():
            p.kill()
    out = {r: open(tmp_path / f"rank{r}.txt").read() for r in range(2) if (tmp_path / f"rank{r}.txt").exists()}
    assert not hung, f"ranks {hung} hung: {out}"
    assert out.get(1) == "step1 ok", out
    r0 = out.get(0, "")
    assert r0.startswith(f"status {lc.LC_ERR_TIMEOUT} ") and "communicator aborted" in r0, out
    assert float(r0.split()[3].rstrip("s:")) < 15.0 and r0.endswith("context ok"), out
