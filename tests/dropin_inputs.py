"""Seeded inputs for the recorded drop-in calls (tests/golden/make_dropin_calls.py records the reference wrappers'
calls on them; tests/test_gpu_dropin_replay.py replays those calls on the GPU with the same inputs)."""

import torch

from ckb200 import workloads

OUTPUTS = {"rmsnorm": ("y",), "rope": ("q_out", "k_out"), "topk": ("values", "indices")}


def make_inputs(op):
    g = torch.Generator().manual_seed({"rmsnorm": 11, "rope": 12, "topk": 13}[op])
    if op == "rmsnorm":
        return {"x": torch.randn(512, 4096, generator=g).to(torch.bfloat16)}
    if op == "rope":
        base = workloads.rope_8x4096(batch=2, seq=64)
        return {"q": base["q"], "k": base["k"], "cos": base["cos"], "sin": base["sin"],
                "position_ids": torch.randint(0, 4096, (2, 64), generator=g)}
    if op == "topk":
        # 512 rows: one segment per row on any GPU, so the chunk the wrapper got from plan() on the CPU is valid
        return {"x": torch.randn(512, 2048, generator=g) * 3}
    raise ValueError(op)
