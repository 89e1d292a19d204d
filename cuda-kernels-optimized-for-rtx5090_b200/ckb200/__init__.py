"""B200-native (sm_100a) row-wise inference kernels behind the entry points of
fengwang/cuda-kernels-optimized-for-rtx5090: softmax.run, rmsnorm.run, rope.run and topk.run take and return the same
dicts as the reference's softmax/baseline.py and {rmsnorm,rope,topk}/candidate.py. The CUDA libraries are built in
tree by ckb200.build (lib/<op>/libkernel.so); there is no CPU fallback. ckb200.hostpipe.RowPipeline streams pinned
host batches through any of them with the copies overlapped.
"""

from . import build, hostpipe, rmsnorm, rope, sharded, softmax, topk  # noqa: F401

__all__ = ["build", "hostpipe", "rmsnorm", "rope", "sharded", "softmax", "topk"]
