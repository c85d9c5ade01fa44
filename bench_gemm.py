"""Transformer-linear GEMMs of the Llama-3-8B step on this library's tcgen05 kernel vs cuBLAS.

    python bench_gemm.py [--iters 20] [--variant 0|1|2] [--tokens 4096]

For every linear of one decoder block (and the LM head) at T tokens it times the three GEMMs of
a training step -- forward Y = X W^T (``nt``), input gradient dX = dY W (``nn``) and weight
gradient dW = dY^T X (``tn``) -- through the grouped transformer-linear kernel (``lin_*``,
``ops.linear.gemm``), through the Newton-Schulz GEMM kernel (``ext.tc_gemm_ws`` /
``ext.wgrad_out``) and through ``torch.mm`` (cuBLAS), with CUDA events after 3 warm-ups.  The operands of each case
are rotated over enough copies that the bytes touched between two launches of the same copy
exceed the 126 MB L2.  Reports ms, TFLOP/s and the fraction of the measured cuBLAS bf16 peak
(MEASURED_PEAKS.json ``bf16_tflops``; fallback 1590).  One JSON line per case.
"""
import argparse
import json
import os

import torch

L2_BYTES = 126 << 20


def peak_tflops() -> float:
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def timeit(fns, iters):
    """fns: list of callables over rotating operand copies; returns ms per call."""
    for i in range(3):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(iters):
        fns[i % len(fns)]()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def copies(nbytes: int) -> int:
    return max(1, min(8, -(-2 * L2_BYTES // max(nbytes, 1))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--variant", type=int, default=0, help="0 auto, 1 single-CTA tiles, 2 CTA-pair tiles")
    ap.add_argument("--only", default="", help="comma-separated case names")
    ap.add_argument("--lin-only", action="store_true", help="only the grouped transformer-linear kernel (and cuBLAS)")
    ap.add_argument("--no-split", action="store_true", help="grouped kernel: whole tiles only (no split last wave)")
    a = ap.parse_args()
    from my_muon_fsdp2_b200._ext import ext

    E = ext()
    E.set_gemm_variant(a.variant)
    E.set_linear_split_tail(not a.no_split)
    print(json.dumps({"resident_cta_pairs": int(E.linear_resident_pairs())}), flush=True)
    T = a.tokens
    bf = torch.bfloat16
    shapes = {  # name: (N out features, K in features)
        "wqkv": (6144, 4096), "wq": (4096, 4096), "wkv": (1024, 4096), "wo": (4096, 4096),
        "w13": (28672, 4096), "w1": (14336, 4096), "w2": (4096, 14336), "lm_head": (128256, 4096),
    }
    only = set(s for s in a.only.split(",") if s)
    peak = peak_tflops()
    for name, (N, K) in shapes.items():
        if only and name not in only:
            continue
        flops = 2.0 * T * N * K
        nb = 2 * (T * K + N * K + T * N)
        c = copies(nb)
        X = [torch.randn(1, T, K, device="cuda", dtype=bf) for _ in range(c)]
        W = [torch.randn(1, N, K, device="cuda", dtype=bf) * 0.02 for _ in range(c)]
        dY = [torch.randn(1, T, N, device="cuda", dtype=bf) for _ in range(c)]
        Y = torch.empty(1, T, N, device="cuda", dtype=bf)
        dX = torch.empty(1, T, K, device="cuda", dtype=bf)
        dW = torch.empty(N, K, device="cuda", dtype=bf)
        meta = torch.tensor([K, 0, N], dtype=torch.int64, device="cuda")
        ptr = E.ptr_table([dW])
        from my_muon_fsdp2_b200.ops import linear as L

        Y2, dX2 = Y[0], dX[0]
        cases = {
            "lin_nt": ([lambda i=i: L.gemm([X[i][0]], [W[i][0]], False, False, [Y2]) for i in range(c)],
                       [lambda i=i: torch.mm(X[i][0], W[i][0].t(), out=Y2) for i in range(c)]),
            "lin_nn": ([lambda i=i: L.gemm([dY[i][0]], [W[i][0]], False, True, [dX2]) for i in range(c)],
                       [lambda i=i: torch.mm(dY[i][0], W[i][0], out=dX2) for i in range(c)]),
            "lin_tn": ([lambda i=i: L.gemm([dY[i][0]], [X[i][0]], True, True, [dW]) for i in range(c)],
                       [lambda i=i: torch.mm(dY[i][0].t(), X[i][0], out=dW) for i in range(c)]),
            "nt": ([lambda i=i: E.tc_gemm_ws(X[i], W[i], False, Y, None, None, 1.0, None, 0.0, False) for i in range(c)],
                   [lambda i=i: torch.mm(X[i][0], W[i][0].t(), out=Y[0]) for i in range(c)]),
            "nn": ([lambda i=i: E.tc_gemm_ws(dY[i], W[i], True, dX, None, None, 1.0, None, 0.0, False) for i in range(c)],
                   [lambda i=i: torch.mm(dY[i][0], W[i][0], out=dX[0]) for i in range(c)]),
            "tn": ([lambda i=i: E.wgrad_out(dY[i][0], X[i][0], ptr, 1, meta, False, 0.0, None, 1.0) for i in range(c)],
                   [lambda i=i: torch.mm(dY[i][0].t(), X[i][0], out=dW) for i in range(c)]),
        }
        for kind, (ours, lib) in cases.items():
            if a.lin_only and not kind.startswith("lin_"):
                continue
            t_ours = timeit(ours, a.iters)
            t_lib = timeit(lib, a.iters)
            rec = {"case": f"{name}_{kind}", "T": T, "N": N, "K": K, "ms": round(t_ours, 4),
                   "cublas_ms": round(t_lib, 4), "tflops": round(flops / t_ours / 1e9, 1),
                   "cublas_tflops": round(flops / t_lib / 1e9, 1),
                   "frac_of_measured_peak": round(flops / t_ours / 1e9 / peak, 3),
                   "speedup_vs_cublas": round(t_lib / t_ours, 3), "variant": a.variant, "split_last_wave": not a.no_split}
            print(json.dumps(rec), flush=True)
        del X, W, dY
        torch.cuda.empty_cache()
    from my_muon_fsdp2_b200._ext import check_device_error

    check_device_error(torch.cuda.current_device())


if __name__ == "__main__":
    main()
