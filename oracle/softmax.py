"""Softmax oracle (test infrastructure only).

The reference's own implementation is torch.softmax(x, dim=-1) (softmax/baseline.py:12-13); its harness checks
candidates against it run in fp64 (softmax/baseline.py:5-6). Both are restated here on CPU torch.
"""

import torch


def softmax_f64(x):
    """The oracle: softmax over the last dim in fp64 of x's values (softmax/baseline.py:5-6,13)."""
    return torch.softmax(x.detach().cpu().to(torch.float64), dim=-1)


def softmax_cpu(x):
    """The reference's CPU path at x's own dtype (softmax/baseline.py:13), the timed CPU baseline."""
    return torch.softmax(x, dim=-1)
