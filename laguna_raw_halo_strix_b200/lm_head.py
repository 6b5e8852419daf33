"""Vocab-sharded lm_head + argmax over a process group.

TargetModel::project_normalized_hidden (src/target.rs:580-605) followed by
argmax (src/lib.rs:456-464), for m hidden rows at once.  The vocab rows of the
weight are split into contiguous shards, one per rank (each shard is a
contiguous byte range of the GGUF tensor); every rank runs lc_lm_head_argmax
on its shard, which yields per-row keys carrying the shard's best (logit,
global index), and one int64 MAX all-reduce combines them.  The keys are
order-preserving signed integers with ties broken toward the larger index, so
the reduced key is exactly the reference's max_by result over the whole vocab.

The reduction is the only exchange of the path: 8 bytes per row.  With a
library communicator (lc.Comm, NCCL owned by liblaguna_cuda.so, bounded
waits) the whole step is one C-ABI call, lc_lm_head_argmax_sharded -- what a
host binding the C ABI alone uses; without one, the keys are reduced through
the torch.distributed group (NCCL on GPU tensors, gloo on CPU tensors).
"""
from __future__ import annotations

import numpy as np

from . import lc, synth


def shard_range(n_vocab: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) of rank's shard: contiguous, sizes differing by at most one."""
    lo = n_vocab * rank // world
    hi = n_vocab * (rank + 1) // world
    return lo, hi


def reduce_keys(keys, group=None):
    """MAX all-reduce of int64 keys across the group (NCCL on GPU tensors, gloo
    on CPU tensors); a no-op without an initialised process group."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return keys


def key_indices(keys: np.ndarray) -> np.ndarray:
    """Token ids of int64 keys (the low 32 bits)."""
    return (np.asarray(keys, np.int64).view(np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.int64)


class ShardedLmHead:
    """lm_head of n_vocab rows x k columns (dtype LC_Q8_0, LC_Q4_K or LC_F32),
    this rank's shard on the context's device."""

    def __init__(self, ctx: lc.Context, dtype: int, k: int, n_vocab: int, rank: int = 0, world: int = 1,
                 group=None, comm: "lc.Comm | None" = None):
        self.ctx, self.dtype, self.k, self.n_vocab = ctx, dtype, k, n_vocab
        self.rank, self.world, self.group, self.comm = rank, world, group, comm
        self.lo, self.hi = shard_range(n_vocab, rank, world)
        self.row_bytes = synth.row_bytes(dtype, k)
        self.w = None

    @property
    def n_local(self) -> int:
        return self.hi - self.lo

    def shard_bytes(self, full: np.ndarray) -> np.ndarray:
        """This rank's rows of the whole weight given as raw GGUF bytes."""
        flat = np.ascontiguousarray(full).view(np.uint8).ravel()
        assert flat.size == self.n_vocab * self.row_bytes, "weight size does not match n_vocab x k"
        return flat[self.lo * self.row_bytes:self.hi * self.row_bytes]

    def load_shard(self, shard: np.ndarray, device):
        """Upload this rank's rows (raw bytes, row-major) unchanged."""
        import torch

        b = np.ascontiguousarray(shard).view(np.uint8).ravel()
        assert b.size == self.n_local * self.row_bytes
        self.w = torch.from_numpy(b).to(device)
        return self

    def local_keys(self, x, m: int, keys, logits=None):
        """keys[m] (device int64) <- the shard's best (logit, global index) per row."""
        self.ctx.lm_head_argmax(self.dtype, x, self.w, m, self.k, self.n_local, self.lo, keys, logits)
        return keys

    def __call__(self, x, m: int, keys):
        """Global argmax keys of x [m, k] (device): local keys, then the MAX all-reduce."""
        if self.comm is not None:
            self.comm.lm_head_argmax(self.dtype, x, self.w, m, self.k, self.n_local, self.lo, keys)
            return keys
        self.local_keys(x, m, keys)
        return reduce_keys(keys, self.group)


def make_comm(ctx: lc.Context, rank: int, world: int, timeout_ms: int = 30000, group=None) -> "lc.Comm":
    """The library communicator over an initialised torch.distributed group:
    rank 0 makes the NCCL id, the group carries it to the others."""
    import torch.distributed as dist

    obj = [lc.comm_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(obj, src=0, group=group)
    return lc.Comm(ctx, obj[0], world, rank, timeout_ms)
