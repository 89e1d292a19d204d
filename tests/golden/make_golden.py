"""Makes the golden fixtures that pin the oracle to the reference's own code.

  python tests/golden/make_golden.py --softmax --ref <reference checkout>
      imports the reference's softmax/baseline.py (its torch implementation) on the CPU and records its outputs in
      fp64 and at the input dtype for seeded inputs -> tests/golden/softmax.npz
  python tests/golden/make_golden.py --gpu [--out DIR]
      runs the reference's own RMSNorm, RoPE and top-k CUDA kernels, rebuilt for sm_100a from their sources by
      oracle/build_ref.sh (oracle/_ref/<op>/libkernel.so), on a GPU with seeded inputs, calling their C ABI with
      the arguments their candidate.py wrappers pass -> DIR/{rmsnorm,rope,topk}.npz (default tests/golden)

The fixtures hold the inputs and the outputs (bit patterns for 16-bit dtypes), so the CPU tests need neither the
reference nor a GPU.
"""

import argparse
import ctypes
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().copy()
    return t.numpy().copy()


def softmax_cases():
    g = torch.Generator().manual_seed(100)
    cases = [torch.randn(4, 37, generator=g), torch.randn(5, 128, generator=g) * 2,
             torch.randn(2, 4096, generator=g) * 4, torch.randn(3, 1000, generator=g)]
    cases[2][0, 17] += 20.0
    cases[2][1, 4000] += 20.0
    cases[3][0, 5] = float("-inf")
    cases[3][1, :] = float("-inf")
    cases[3][2, 9] = float("inf")
    return cases


def make_softmax(ref_root, out):
    spec = importlib.util.spec_from_file_location("ref_softmax_baseline", os.path.join(ref_root, "softmax",
                                                                                        "baseline.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    arrays = {}
    for i, x in enumerate(softmax_cases()):
        arrays[f"x{i}"] = x.numpy()
        arrays[f"y64_{i}"] = mod.run({"x": x.double()})["y"].numpy()
        arrays[f"y32_{i}"] = mod.run({"x": x})["y"].numpy()
        xb = x.to(torch.bfloat16)
        arrays[f"xbf16_{i}"] = bits(xb)
        arrays[f"ybf16_{i}"] = bits(mod.run({"x": xb})["y"])
    np.savez_compressed(os.path.join(out, "softmax.npz"), **arrays)


def _ref(op):
    path = os.path.join(ROOT, "oracle", "_ref", op, "libkernel.so")
    if not os.path.exists(path):
        raise SystemExit(f"{path} missing: run oracle/build_ref.sh where the reference is mounted")
    return ctypes.CDLL(path)


def make_rmsnorm(out):
    # Arguments as rmsnorm/candidate.py:48-49 passes them (eps 1e-6, threads 256).
    lib = _ref("rmsnorm")
    lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                           ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    g = torch.Generator().manual_seed(200)
    cases = [(torch.randn(8, 4096, generator=g), torch.bfloat16), (torch.randn(8, 1024, generator=g), torch.float16),
             (torch.randn(3, 1000, generator=g) * 5, torch.bfloat16), (torch.randn(6, 128, generator=g), torch.float16)]
    cases[0][0][2, 3] = float("nan")
    arrays = {}
    for i, (xf, dt) in enumerate(cases):
        x = xf.to(dt).cuda()
        y = torch.empty_like(x)
        err = lib.launch(x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1], 1 if dt == torch.bfloat16 else 2, 1e-6,
                         256, torch.cuda.current_stream().cuda_stream)
        assert err == 0, err
        torch.cuda.synchronize()
        arrays[f"x{i}"], arrays[f"y{i}"] = bits(x), bits(y)
        arrays[f"dtype{i}"] = np.array(1 if dt == torch.bfloat16 else 2)
    np.savez_compressed(os.path.join(out, "rmsnorm.npz"), **arrays)


def make_rope(out):
    # Arguments as rope/candidate.py:52-54 passes them (rows 40, splits 1), out of place.
    sys.path.insert(0, ROOT)
    from oracle.rope import cos_sin_cache
    lib = _ref("rope")
    lib.launch.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_longlong] + [ctypes.c_int] * 7 + [ctypes.c_void_p]
    g = torch.Generator().manual_seed(300)
    arrays = {}
    cases = [(torch.bfloat16, torch.float32, False, 64), (torch.bfloat16, torch.float32, True, 128),
             (torch.float16, torch.bfloat16, False, 64), (torch.bfloat16, torch.float16, False, 10)]
    for i, (qk, cd, integer, hd) in enumerate(cases):
        b, s, hq, hkv = 2, 16, 4, 2
        if integer:
            q = torch.randint(-8, 9, (b, s, hq, hd), generator=g).to(qk)
            k = torch.randint(-8, 9, (b, s, hkv, hd), generator=g).to(qk)
        else:
            q = torch.randn(b, s, hq, hd, generator=g).to(qk)
            k = torch.randn(b, s, hkv, hd, generator=g).to(qk)
        cos, sin = cos_sin_cache(10000.0, hd, 32, cd)
        ids = torch.randint(0, 32, (b, s), generator=g)
        d = [t.cuda() for t in (q, k, cos, sin, ids)]
        qo, ko = torch.empty_like(d[0]), torch.empty_like(d[1])
        err = lib.launch(*[t.data_ptr() for t in d], qo.data_ptr(), ko.data_ptr(), b * s, hq, hkv, hd,
                         1 if qk == torch.bfloat16 else 2, {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[cd],
                         40, 1, torch.cuda.current_stream().cuda_stream)
        assert err == 0, err
        torch.cuda.synchronize()
        for name, t in (("q", q), ("k", k), ("cos", cos), ("sin", sin), ("ids", ids), ("qo", qo), ("ko", ko)):
            arrays[f"{name}{i}"] = bits(t)
        arrays[f"qk{i}"] = np.array(1 if qk == torch.bfloat16 else 2)
        arrays[f"cache{i}"] = np.array({torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[cd])
    np.savez_compressed(os.path.join(out, "rope.npz"), **arrays)


def make_topk(out):
    # plan + launch as topk/candidate.py:58,77-78 call them (K 50, threads 256, depth 4, min_chunk 2048).
    lib = _ref("topk")
    lib.plan.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.plan.restype = ctypes.c_longlong
    lib.launch.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p]
    g = torch.Generator().manual_seed(400)
    cases = [torch.randn(4, 5000, generator=g) * 3, torch.randint(-3, 4, (4, 3000), generator=g).float(),
             (torch.randn(3, 2000, generator=g) * 3).to(torch.bfloat16), torch.randn(2, 40000, generator=g)]
    cases[0][1, 10] = float("inf")
    cases[0][2, 20] = float("nan")
    arrays = {}
    for i, x in enumerate(cases):
        xd = x.cuda()
        rows, cols = x.shape
        dt = 1 if x.dtype == torch.bfloat16 else 0
        chunk = lib.plan(rows, cols, dt, 256, 4, 2048)
        nch = -(-cols // chunk)
        work = torch.empty(max(1, rows * nch * 50), dtype=torch.int64, device="cuda")
        counters = torch.zeros(4096, dtype=torch.int32, device="cuda")
        v = torch.empty(rows, 50, dtype=x.dtype, device="cuda")
        ix = torch.empty(rows, 50, dtype=torch.int64, device="cuda")
        err = lib.launch(xd.data_ptr(), v.data_ptr(), ix.data_ptr(), work.data_ptr(), counters.data_ptr(), rows, cols,
                         50, dt, 256, 4, chunk, torch.cuda.current_stream().cuda_stream)
        assert err == 0, err
        torch.cuda.synchronize()
        arrays[f"x{i}"], arrays[f"v{i}"], arrays[f"i{i}"] = bits(x), bits(v), ix.cpu().numpy()
        arrays[f"dtype{i}"] = np.array(dt)
    np.savez_compressed(os.path.join(out, "topk.npz"), **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--softmax", action="store_true")
    ap.add_argument("--gpu", action="store_true")
    ap.add_argument("--ref", default=os.environ.get("CKB_REFERENCE_DIR"),
                    help="the reference checkout (default: $CKB_REFERENCE_DIR)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    if a.softmax:
        if not a.ref:
            raise SystemExit("make_golden --softmax: give --ref or set CKB_REFERENCE_DIR")
        make_softmax(a.ref, a.out)
    if a.gpu:
        make_rmsnorm(a.out)
        make_rope(a.out)
        make_topk(a.out)


if __name__ == "__main__":
    main()
