"""Multi-GPU plumbing: row and token sharding (no communication) and the vocab-sharded top-k (one all-gather).

One process per GPU (torchrun), torch.distributed over NCCL. The reference is single-GPU; these are the two
partitionings its row-wise ops admit:
  * rows (tokens, batch entries) are independent for softmax, RMSNorm, RoPE and top-k: rank r owns the contiguous
    rows row_range(rows, r, world) and runs the single-GPU kernel on them, with no data-path collective (RoPE's
    rows are the batch x seq tokens, token_shard; its cos/sin cache is replicated);
  * a vocab row split over GPUs (columns col_range(cols, r, world) on rank r) needs one exchange for top-k: each
    rank selects its local top k as sorted 64-bit composites carrying global column indices, an all-gather brings
    every rank's [rows, k] list to every rank ([world, rows, k], world * rows * k * 8 bytes), and the merge kernel
    ranks them into the final top k. Composites are distinct, so the merge is exact and ties still go to the lower
    global index. PeerVocabShardedTopK does the same exchange without a collective call: the shard kernel stores
    its lists straight into every rank's memory over NVLink (CUDA IPC mappings) and raises per-row flags there, and
    the merge kernel waits on those flags.
"""

import ctypes


import torch
import torch.distributed as dist

from . import _native
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
token_range = split_range


def token_shard(t, rank, world):
    """Rank `rank`'s contiguous share of the tokens of a [batch, seq, ...] tensor (q, k, or position_ids [batch,
    seq]): the tokens batch * seq flattened and split by token_range, returned as a [1, n, ...] view (RoPE rotates
    tokens independently, and the cos/sin cache is replicated on every rank, so a shard needs no exchange)."""
    if t.dim() < 2 or not t.is_contiguous():
        raise ValueError(f"token_shard: a contiguous [batch, seq, ...] tensor, got {tuple(t.shape)}")
    flat = t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])
    lo, hi = token_range(flat.shape[0], rank, world)
    return flat[lo:hi].unsqueeze(0)


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


def exchange_layout(world, rows, k):
    """Byte layout of one parity half of a rank's exchange buffer: (half_bytes, lists_offset, flags_offset) for
    lists [world][rows][k] uint64 then flags [world][rows] uint32, the half padded to 256 bytes."""
    lists_bytes = world * rows * k * 8
    flags_bytes = world * rows * 4
    half = (lists_bytes + flags_bytes + 255) // 256 * 256
    return half, 0, lists_bytes


def next_epoch(epoch):
    """The epoch after `epoch` (32-bit, never 0, parity always alternating: 0xffffffff is followed by 2)."""
    e = epoch + 1
    return e if e <= 0xFFFFFFFF else 2


def graph_epochs(epoch):
    """For a graphed step after epoch `epoch`: the two eager warm-up epochs and the four epochs the graphs carry
    (replayed in rotation, every call alternates parity and calls two apart differ)."""
    seq = [epoch]
    for _ in range(6):
        seq.append(next_epoch(seq[-1]))
    return seq[1:3], seq[3:]


class PeerVocabShardedTopK:
    """The vocab-sharded top-k with its all-gather done by the kernels over peer memory.

    Every rank allocates one exchange buffer (two parity halves, exchange_layout) through the top-k library, and the
    ranks swap CUDA IPC handles once (a host all-gather of 64-byte handles), so each holds every rank's buffer
    address. A call with epoch e (counted from 1) uses half e & 1: ckb_topk_shard_push_launch stores this rank's
    row lists into slot `rank` of every rank's half and sets the row flags to e there; in the same kernel each row
    then waits on this rank's own flags and merges (a merge-wait kernel follows instead when the kernel's CTAs do
    not all fit the GPU at once). Two halves suffice: a rank starts call e + 2 only after its merge of call e + 1
    saw every rank's lists of e + 1, which those ranks pushed after finishing their merges of call e. The launch
    arguments are checked and packed once per shard shape, so a call costs one library call and the two output
    allocations. Call close() on every rank (it synchronises them) before the process group goes.

    Every wait on a peer's flag is bounded (2 s); a wait that runs out merges whatever the buffer holds, which can be
    an older call's lists, and records the timeout in the library's status word. check() reads that word (it
    synchronises the device) and raises; call it after a batch of calls, before trusting their outputs. After a
    timeout the two-halves invariant no longer holds, so the object refuses further calls: close it on every rank
    and build a new one (its exchange buffers start zeroed). The in-kernel wait is chosen when all of the kernel's
    CTAs fit the GPU at once, counted as if nothing else ran on the device; other kernels running beside it (another
    stream, a collective) delay its CTAs and make a timeout likelier, never a hang."""

    def __init__(self, rows, k=_topk.K, device=None, group=None):
        self.group = group
        self.rows, self.k = rows, k
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        distributed = dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if self.world > 8:
            raise ValueError(f"PeerVocabShardedTopK: at most 8 ranks, got {self.world}")
        self.half, self.lists_off, self.flags_off = exchange_layout(self.world, rows, k)
        lib = _native.load("topk")
        self._lib = lib
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.check(lib.ckb_p2p_alloc(ctypes.byref(own), 2 * self.half))
            handle = ctypes.create_string_buffer(64)
            _native.check(lib.ckb_p2p_export(own, handle))
        self._own = own.value
        handles = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
        self.bases, self._imported = [], []
        with torch.cuda.device(self.device):
            for p in range(self.world):
                if p == self.rank:
                    self.bases.append(self._own)
                    continue
                ptr = ctypes.c_void_p()
                _native.check(lib.ckb_p2p_import(ctypes.create_string_buffer(handles[p], 64), ctypes.byref(ptr)))
                self.bases.append(ptr.value)
                self._imported.append(ptr.value)
        self.epoch = 0
        self._graphs = []
        self._args = {}
        self.broken = False
        lib.ckb_topk_status(1)  # a timeout recorded before this object existed is not its own

    def __call__(self, x_shard, col_offset):
        """(values, int64 indices) [rows, k] of the full rows; x_shard [rows, local_cols] holds global columns
        [col_offset, col_offset + local_cols). One kernel on the current stream (two when its CTAs do not all fit
        the GPU at once), no collective call. The outputs are trusted only after check() passes."""
        if self.broken:
            raise RuntimeError("PeerVocabShardedTopK: a peer wait timed out earlier; close() and rebuild")
        self.epoch = next_epoch(self.epoch)
        return self._step(x_shard, col_offset, self.epoch)

    def _launch_args(self, x_shard):
        """Everything a call passes to ckb_topk_shard_push_launch but x, the outputs and the epoch, for this shard's
        shape (checked, planned and packed once): (dtype code, cols, chunk, work, counters, lists and flags pointer
        arrays per parity)."""
        key = (tuple(x_shard.shape), x_shard.dtype, x_shard.device)
        hit = self._args.get(key)
        if hit is not None:
            return hit
        if x_shard.shape[0] != self.rows:
            raise ValueError(f"PeerVocabShardedTopK: {x_shard.shape[0]} rows, built for {self.rows}")
        dtype = _topk._check_x(x_shard, self.k)
        rows, cols = x_shard.shape
        chunk, work = _topk._plan(x_shard, rows, cols, dtype, self.k)
        counters = _topk._row_counters(x_shard.device, rows)
        arrays = []
        for par in (0, 1):
            off = par * self.half
            lists = (ctypes.c_void_p * self.world)(*[b + off + self.lists_off for b in self.bases])
            flags = (ctypes.c_void_p * self.world)(*[b + off + self.flags_off for b in self.bases])
            arrays.append((lists, flags))
        hit = (dtype, cols, chunk, work, counters, arrays)
        self._args[key] = hit
        return hit

    def _step(self, x_shard, col_offset, epoch, values=None, indices=None):
        if not x_shard.is_contiguous():
            x_shard = x_shard.contiguous()
        dtype, cols, chunk, work, counters, arrays = self._launch_args(x_shard)
        if values is None:
            values = torch.empty((self.rows, self.k), dtype=x_shard.dtype, device=x_shard.device)
            indices = torch.empty((self.rows, self.k), dtype=torch.int64, device=x_shard.device)
        lists, flags = arrays[epoch & 1]
        err = self._lib.ckb_topk_shard_push_launch(x_shard.data_ptr(), values.data_ptr(), indices.data_ptr(),
                                                   work.data_ptr(), counters.data_ptr(), self.rows, cols,
                                                   int(col_offset), self.k, dtype, chunk, lists, flags, self.world,
                                                   self.rank, epoch, torch.cuda.current_stream(self.device).cuda_stream)
        _native.check(err)
        return values, indices

    def graphed(self, x_shards, col_offset):
        """A replayable step on fixed buffers: four CUDA graphs carrying the next four epochs of this object's
        sequence, replayed in rotation by the returned callable, which gives the (values, indices) tensors it
        rewrites. x_shards is one shard tensor or a list of 1, 2 or 4 of them (graph j reads x_shards[j % n], so two
        copies alternate). The rotation keeps what the equal-flag waits need: consecutive calls alternate parity and
        calls two apart carry different epochs. Every rank must capture and replay in step; no eager call may
        follow. check() covers the replays as it covers eager calls."""
        if self.broken:
            raise RuntimeError("PeerVocabShardedTopK: a peer wait timed out earlier; close() and rebuild")
        shards = list(x_shards) if isinstance(x_shards, (list, tuple)) else [x_shards]
        if len(shards) not in (1, 2, 4):
            raise ValueError(f"PeerVocabShardedTopK.graphed: 1, 2 or 4 inputs, got {len(shards)}")
        x0 = shards[0]
        values = torch.empty((self.rows, self.k), dtype=x0.dtype, device=x0.device)
        indices = torch.empty((self.rows, self.k), dtype=torch.int64, device=x0.device)
        warm, captured = graph_epochs(self.epoch)
        for j, e in enumerate(warm):  # two eager steps: plan, workspace and counters exist before capture
            self._step(shards[j % len(shards)], col_offset, e, values, indices)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        graphs = []
        for j, e in enumerate(captured):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._step(shards[j % len(shards)], col_offset, e, values, indices)
            graphs.append(g)
        self.epoch = captured[-1]
        self._graphs = graphs
        state = {"i": 0}

        def replay():
            graphs[state["i"] % 4].replay()
            state["i"] += 1
            return values, indices

        return replay

    def check(self):
        """Synchronises this device and raises RuntimeError when any peer-flag wait since the last check ran out (the
        outputs of the calls since then may hold stale lists); the object is then unusable (close and rebuild)."""
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            status = self._lib.ckb_topk_status(1)
        if status < 0:
            raise RuntimeError(f"PeerVocabShardedTopK: status read failed: CUDA error {-status}")
        if status:
            self.broken = True
            raise RuntimeError("PeerVocabShardedTopK: a peer-memory wait ran out (2 s); the outputs since the last "
                               "check may be stale; close() and rebuild on every rank")

    def close(self):
        """Unmaps the peers' buffers and frees this rank's once every rank is done with them."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        self._graphs = []
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._imported:
                self._lib.ckb_p2p_close(ctypes.c_void_p(ptr))
            if self.world > 1:
                dist.barrier(group=self.group)
            self._lib.ckb_p2p_free(ctypes.c_void_p(self._own))
        self._own, self._imported, self.bases = None, [], []
