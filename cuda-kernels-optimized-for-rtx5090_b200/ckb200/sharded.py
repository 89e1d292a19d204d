"""Multi-GPU plumbing: row sharding (no communication) and the vocab-sharded top-k (one all-gather).

One process per GPU (torchrun), torch.distributed over NCCL. The reference is single-GPU; these are the two
partitionings its row-wise ops admit:
  * rows (tokens, batch entries) are independent for softmax, RMSNorm, RoPE and top-k: rank r owns the contiguous
    rows row_range(rows, r, world) and runs the single-GPU kernel on them, with no data-path collective;
  * a vocab row split over GPUs (columns col_range(cols, r, world) on rank r) needs one exchange for top-k: each
    rank selects its local top k as sorted 64-bit composites carrying global column indices, an all-gather brings
    every rank's [rows, k] list to every rank ([world, rows, k], world * rows * k * 8 bytes), and the merge kernel
    ranks them into the final top k. Composites are distinct, so the merge is exact and ties still go to the lower
    global index.
"""

import torch
import torch.distributed as dist

from . import topk as _topk


def split_range(n, rank, world):
    """[start, stop) of part `rank` of n items split into `world` contiguous parts (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


row_range = split_range
col_range = split_range


def gather_lists(lists, group=None):
    """All-gather of every rank's [rows, k] int64 composite list into [world, rows, k] on every rank."""
    world = dist.get_world_size(group)
    out = torch.empty((world, *lists.shape), dtype=lists.dtype, device=lists.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, lists.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), lists.contiguous(), group=group)
    return out


def topk_vocab_sharded(x_shard, col_offset, k=_topk.K, group=None):
    """Top-k of rows whose columns are split over the ranks of `group`: x_shard [rows, local_cols] holds global
    columns [col_offset, col_offset + local_cols). Every rank returns the same (values, indices) [rows, k]."""
    lists = _topk.shard_lists(x_shard, col_offset, k)
    return _topk.merge_lists(gather_lists(lists, group), x_shard.dtype, k)


class VocabShardedTopK:
    """topk_vocab_sharded with every buffer allocated once (for repeated calls on one shape): the local lists, the
    gathered [world, rows, k] lists and the outputs. A call launches the shard kernel, one NCCL all-gather and the
    merge kernel on the current stream."""

    def __init__(self, rows, k=_topk.K, dtype=None, device=None, group=None):
        self.group = group
        self.k = k
        self.dtype = dtype
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.lists = torch.empty((rows, k), dtype=torch.int64, device=device)
        self.gathered = torch.empty((self.world, rows, k), dtype=torch.int64, device=device)

    def __call__(self, x_shard, col_offset):
        _topk.shard_lists(x_shard, col_offset, self.k, out=self.lists)
        if self.world == 1:
            self.gathered[0].copy_(self.lists)
        elif dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self.gathered, self.lists, group=self.group)
        else:
            dist.all_gather(list(self.gathered.unbind(0)), self.lists, group=self.group)
        return _topk.merge_lists(self.gathered, x_shard.dtype, self.k)
