"""CPU oracle for the four row-wise kernels -- TEST INFRASTRUCTURE ONLY.

Restatements of the reference's semantics (fengwang/cuda-kernels-optimized-for-rtx5090), each function citing the
reference file:line it follows. Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
`--impl reference` arm) may import this package, and only as the checker or the CPU baseline: the product
(ckb200) never calls it, and has no CPU fallback.

Pinning: softmax against fixtures produced by the reference's own softmax/baseline.py; RMSNorm, RoPE and top-k
against fixtures produced by the reference's own CUDA kernels rebuilt for sm_100a from their sources (oracle/_ref,
recipe in oracle/build_ref.sh) and run on a B200. tests/golden/make_golden.py makes both kinds.
"""
