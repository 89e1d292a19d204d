"""Seeded inputs for the recorded drop-in calls (tests/golden/make_dropin_calls.py records the reference wrappers'
calls on them; tests/test_gpu_dropin_replay.py replays those calls on the GPU with the same inputs)."""

import torch

from ckb200 import workloads

OUTPUTS = {"rmsnorm": ("y",), "rope": ("q_out", "k_out"), "topk": ("values", "indices")}


CASES = {"rmsnorm": ("bf16", "fp16_odd_cols"), "rope": ("bf16", "fp16_bf16_cache"), "topk": ("fp32", "bf16")}


def make_inputs(op, case):
    g = torch.Generator().manual_seed({"rmsnorm": 11, "rope": 12, "topk": 13}[op] * 10 + CASES[op].index(case))
    if op == "rmsnorm":
        if case == "bf16":
            return {"x": torch.randn(512, 4096, generator=g).to(torch.bfloat16)}
        return {"x": torch.randn(33, 1000, generator=g).to(torch.float16)}  # 1000 columns: the scalar path
    if op == "rope":
        if case == "bf16":
            base = workloads.rope_8x4096(batch=2, seq=64)
        else:
            base = workloads.rope_8x4096(batch=2, seq=64, cache_dtype=torch.bfloat16)
            base["q"], base["k"] = base["q"].to(torch.float16), base["k"].to(torch.float16)
        return {"q": base["q"], "k": base["k"], "cos": base["cos"], "sin": base["sin"],
                "position_ids": torch.randint(0, 4096, (2, 64), generator=g)}
    if op == "topk":
        # 512 rows: one segment per row on any GPU, so the chunk the wrapper got from plan() on the CPU is valid
        x = torch.randn(512, 2048, generator=g) * 3
        return {"x": x if case == "fp32" else x.to(torch.bfloat16)}
    raise ValueError(op)
