"""Vocab sharding of lm_head + argmax (laguna_raw_halo_strix_b200/lm_head.py).

CPU: the shard split and the int64 MAX reduction across two gloo ranks, with
each rank's local keys built from the CPU oracle's logits of its shard; the
reduced token must be the full-vocab argmax of src/lib.rs:456-464 (last
maximum wins), including a tie planted across the shard boundary.
GPU: several shards run on one device through lc_lm_head_argmax (global row
offsets) combine to the unsharded result."""
import os
import socket

import numpy as np
import pytest

import oracle as orc
from laguna_raw_halo_strix_b200 import lc, synth
from laguna_raw_halo_strix_b200.lm_head import ShardedLmHead, key_indices, reduce_keys, shard_range


def test_shard_range_partitions():
    for n in (1, 7, 1000, 128256):
        for world in (1, 2, 3, 4, 8):
            if world > n:
                continue
            rs = [shard_range(n, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in rs]
            assert max(sizes) - min(sizes) <= 1


def _local_keys_cpu(logits_shard, lo):
    """Keys of the shard's last maximum per row (what lc_lm_head_argmax returns)."""
    keys = []
    for row in logits_shard:
        j = len(row) - 1 - int(np.argmax(row[::-1]))
        keys.append(np.int64(np.uint64(lc.pack_key(float(row[j]), lo + j)).view(np.int64)))
    return np.array(keys, np.int64)


def _rank_main(rank, world, port, x, w, k, n, out_path):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        o = orc.Oracle()
        head = ShardedLmHead(None, orc.Q8_0, k, n, rank, world)
        shard = head.shard_bytes(w)
        logits = o.proj(orc.Q8_0, x, shard, k, head.n_local).reshape(x.shape[0], head.n_local)
        keys = torch.from_numpy(_local_keys_cpu(logits, head.lo))
        reduce_keys(keys)
        if rank == 0:
            np.save(out_path, keys.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_reduction(tmp_path):
    import torch.multiprocessing as mp

    rng = np.random.default_rng(3)
    m, k, n = 5, 256, 301
    w = synth.q8_0_blocks(n, k, rng)
    x = synth.activations(m, k, rng)
    # plant an exact tie on both sides of the shard boundary: row lo1 - 2 gets
    # q = 127 * sign of the tokens' summed activations (a large logit for every
    # token row) and row lo1 + 3 is an identical copy of it
    lo1, _ = shard_range(n, 1, 2)
    wq = w.reshape(n, -1).copy()
    q = (np.sign(x.sum(0)) * 127).astype(np.int8).view(np.uint8)
    for b in range(k // 32):  # keep each block's f16 d, replace its 32 q bytes
        wq[lo1 - 2, 34 * b + 2:34 * b + 34] = q[32 * b:32 * b + 32]
    wq[lo1 + 3] = wq[lo1 - 2]
    w = wq.reshape(w.shape)
    full = orc.Oracle().proj(orc.Q8_0, x, w, k, n).reshape(m, n)
    out = str(tmp_path / "keys.npy")
    mp.spawn(_rank_main, args=(2, _free_port(), x, w, k, n, out), nprocs=2, join=True)
    got = key_indices(np.load(out))
    exp = np.array([n - 1 - int(np.argmax(r[::-1])) for r in full])
    assert np.array_equal(got, exp)
    # the planted pair ties exactly; wherever it is the maximum, the later row wins
    tied = [r for r in range(m) if full[r, lo1 - 2] == full[r].max()]
    assert tied, "the planted tie decides no row"
    assert all(got[r] == lo1 + 3 for r in tied)


@pytest.mark.gpu
@pytest.mark.parametrize("m", [9, 150])  # 150: the tensor-core tiles (m > 32), a partial token tile
@pytest.mark.parametrize("dtype", [lc.Q8_0, lc.Q4_K])
def test_shards_on_one_gpu_combine(ctx, dev, oracle, dtype, m):
    import torch

    rng = np.random.default_rng(17)
    k, n = 512, 2051
    w = synth.weight_blocks(dtype, n, k, rng)
    x = synth.activations(m, k, rng)
    xd = torch.from_numpy(x).to(dev)
    whole = ShardedLmHead(ctx, dtype, k, n).load_shard(w, dev)
    ref_keys = torch.empty(m, dtype=torch.int64, device=dev)
    whole(xd, m, ref_keys)
    torch.cuda.synchronize()
    ref = ref_keys.cpu().numpy()
    for world in (2, 3, 8):
        combined = np.full(m, np.iinfo(np.int64).min, np.int64)
        for rank in range(world):
            h = ShardedLmHead(ctx, dtype, k, n, rank, world)
            h.load_shard(h.shard_bytes(w), dev)
            keys = torch.empty(m, dtype=torch.int64, device=dev)
            h.local_keys(xd, m, keys)
            torch.cuda.synchronize()
            kk = keys.cpu().numpy()
            idx = key_indices(kk)
            assert np.all((idx >= h.lo) & (idx < h.hi))
            combined = np.maximum(combined, kk)
        assert np.array_equal(combined, ref), world
    # and the token is the oracle's unless the top two logits are within the error bound
    logits = oracle.proj(dtype, x, w, k, n).reshape(m, n)
    for r, t in enumerate(key_indices(ref)):
        o = oracle.argmax(logits[r])
        if t != o:
            s = np.sort(logits[r])
            assert s[-1] - s[-2] <= 2e-3 * np.abs(logits[r]).max()


# ---- failure detection on the host: a rank that is late or leaves -------------------

def _late_rank_main(rank, world, port, mode, out_dir):
    """Two gloo ranks reduce keys twice.  In step 2 rank 1 is late past the
    group's timeout ("late") or has left after step 1 ("leaves"); rank 0's
    reduction must end with an error within the timeout, not hang."""
    import time
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=2))
    outcome = "ok"
    try:
        keys = torch.full((4,), rank, dtype=torch.int64)
        reduce_keys(keys)  # step 1: both ranks
        assert keys.tolist() == [world - 1] * 4
        if rank == 1:
            if mode == "leaves":
                return  # leaves between steps, nothing in flight
            time.sleep(6)  # late past the timeout
        t0 = time.perf_counter()
        try:
            reduce_keys(torch.full((4,), rank, dtype=torch.int64))  # step 2
        except Exception as e:  # noqa: BLE001 -- the error is the outcome under test
            outcome = f"error after {time.perf_counter() - t0:.1f}s: {type(e).__name__}"
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(outcome)
        if outcome == "ok":
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["late", "leaves"])
def test_key_reduction_with_a_missing_rank(tmp_path, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_late_rank_main, args=(r, 2, _free_port_shared(tmp_path), mode, str(tmp_path)))
          for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
    for p in ps:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    out0 = open(tmp_path / "rank0.txt").read()
    assert out0.startswith("error after"), out0
    assert float(out0.split()[2].rstrip("s:")) < 10.0, out0


_PORTS = {}


def _free_port_shared(tmp_path):
    # one port per test invocation, shared by both ranks
    key = str(tmp_path)
    if key not in _PORTS:
        _PORTS[key] = _free_port()
    return _PORTS[key]
