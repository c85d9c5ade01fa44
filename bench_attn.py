"""Attention micro-benchmark: the library's tcgen05 flash attention (forward, backward) vs
PyTorch SDPA (cuDNN / flash backend, a library kernel) on the Llama-3-8B attention shape.

    python bench_attn.py [--B 1 --T 4096 --Hq 32 --Hkv 8 --D 128 --iters 20]
    python bench_attn.py --sweep 'fwd=0,1'                 # forward kernels, one process

Causal FLOPs: forward 2 * 2 * B * Hq * T^2 * D / 2, backward 2.5x forward.  CUDA events on the
launching stream after warm-up.  The inputs (32 MB per tensor at the default shape) fit in the
126 MB L2, so these are warm-L2 numbers — attention is compute-bound, which is what they measure.
"""
import argparse
import json
import math

import torch
import torch.nn.functional as F


def timeit(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--Hq", type=int, default=32)
    ap.add_argument("--Hkv", type=int, default=8)
    ap.add_argument("--D", type=int, default=128)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", choices=["all", "ours_fwd", "ours_bwd"], default="all")
    ap.add_argument("--fwd-variant", type=int, default=0,
                    help="0: three warpgroups with whole score rows (default), 1: two softmax warpgroups")
    ap.add_argument("--sweep", default="",
                    help="time several forward kernels in one process, e.g. 'fwd=0,1' (checks each against "
                         "the default kernel's output first)")
    a = ap.parse_args()
    if a.sweep:
        return sweep(a)
    from my_muon_fsdp2_b200._ext import ext

    ext().set_attention_fwd_variant(a.fwd_variant)
    torch.manual_seed(0)
    q = torch.randn(a.B, a.T, a.Hq, a.D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(a.B, a.T, a.Hkv, a.D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(a.B, a.T, a.Hkv, a.D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(a.D)
    o, lse = ext().attention_fwd(q, k, v, scale)
    do = torch.randn_like(o)
    fl = 2 * 2 * a.B * a.Hq * a.T * a.T * a.D / 2
    res = {}
    res["ours_fwd_ms"] = timeit(lambda: ext().attention_fwd(q, k, v, scale), a.iters)
    if a.only == "ours_fwd":
        print(json.dumps(res))
        return
    res["ours_bwd_ms"] = timeit(lambda: ext().attention_bwd(do, q, k, v, o, lse, scale), a.iters)
    if a.only == "ours_bwd":
        print(json.dumps(res))
        return
    qt, kt, vt = (t.transpose(1, 2).requires_grad_() for t in (q, k, v))
    res["sdpa_fwd_ms"] = timeit(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True),
                                a.iters)
    out = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)
    dot = do.transpose(1, 2)
    res["sdpa_bwd_ms"] = timeit(lambda: torch.autograd.grad(out, (qt, kt, vt), dot, retain_graph=True), a.iters)
    for k_ in list(res):
        mult = 2.5 if "bwd" in k_ else 1.0
        res[k_.replace("_ms", "_tflops")] = fl * mult / (res[k_] / 1e3) / 1e12
    res["shape"] = dict(B=a.B, T=a.T, Hq=a.Hq, Hkv=a.Hkv, D=a.D)
    print(json.dumps(res))


def sweep(a):
    """Time the listed forward variants at one shape, interleaved twice, after checking that each
    gives the default kernel's result (relative Frobenius difference)."""
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    spec = dict(part.split("=") for part in a.sweep.split(";") if part)
    fwd = [int(v) for v in spec.get("fwd", "").split(",") if v != ""]
    torch.manual_seed(0)
    q = torch.randn(a.B, a.T, a.Hq, a.D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(a.B, a.T, a.Hkv, a.D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(a.B, a.T, a.Hkv, a.D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(a.D)
    ext().set_attention_fwd_variant(0)
    o0, lse0 = ext().attention_fwd(q, k, v, scale)
    torch.cuda.synchronize()

    def rel(x, y):
        return float((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-30))

    res = {}
    for rep in range(2):
        for fv in fwd:
            ext().set_attention_fwd_variant(fv)
            o, lse = ext().attention_fwd(q, k, v, scale)
            torch.cuda.synchronize()
            check_device_error(0)
            res.setdefault(f"fwd{fv}_rel_diff", rel(o, o0))
            res.setdefault(f"fwd{fv}_ms", []).append(timeit(lambda: ext().attention_fwd(q, k, v, scale), a.iters))
        ext().set_attention_fwd_variant(0)
    res["shape"] = dict(B=a.B, T=a.T, Hq=a.Hq, Hkv=a.Hkv, D=a.D)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
