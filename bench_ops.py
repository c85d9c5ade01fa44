"""Memory-bound kernels of this library at the Llama-3-8B step's shapes: achieved bandwidth
against the measured HBM copy bandwidth (MEASURED_PEAKS.json `hbm_gbs`, else 6650 GB/s).

    python bench_ops.py [--iters 20] [--only rmsnorm_fwd,adamw,...]

Each op is timed with CUDA events on the launching stream after 3 warm-ups.  Its inputs are
larger than the 126 MB L2 where the op's shape allows; `l2_resident` in the output says where
they are not (then the number is an upper bound on DRAM bandwidth).  Bytes are algorithmic:
every input read once and every output written once.
"""
import argparse
import json
import math
import os

import torch

L2_BYTES = 126 << 20


def peak_gbs() -> float:
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


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


def cases(E):
    """name -> (callable, algorithmic bytes, bytes of the inputs)."""
    bf, f32, dev = torch.bfloat16, torch.float32, "cuda"
    T, D, F, V, H, KV, HD = 4096, 4096, 14336, 128256, 32, 8, 128
    out = {}

    x = torch.randn(T, D, device=dev, dtype=bf)
    w = torch.ones(D, device=dev, dtype=bf)
    y, rstd = E.rmsnorm_fwd(x, w, 1e-5)
    out["rmsnorm_fwd"] = (lambda: E.rmsnorm_fwd(x, w, 1e-5), 2 * x.numel() * 2, x.numel() * 2)
    dy = torch.randn_like(x)
    out["rmsnorm_bwd"] = (lambda: E.rmsnorm_bwd(dy, x, w, rstd), 3 * x.numel() * 2, 2 * x.numel() * 2)

    g = torch.randn(T, F, device=dev, dtype=bf)
    u = torch.randn(T, F, device=dev, dtype=bf)
    out["swiglu_fwd"] = (lambda: E.swiglu_fwd(g, u), 3 * g.numel() * 2, 2 * g.numel() * 2)
    d = torch.randn_like(g)
    out["swiglu_bwd"] = (lambda: E.swiglu_bwd(d, g, u), 5 * g.numel() * 2, 3 * g.numel() * 2)

    qk = torch.randn(T, (H + KV) * HD, device=dev, dtype=bf)
    out["rope_qk"] = (lambda: E.rope_(qk, T, H + KV, HD, T, 500000.0, False, (H + KV) * HD, HD),
                      2 * qk.numel() * 2, qk.numel() * 2)

    logits = torch.randn(T, V, device=dev, dtype=bf)
    tgt = torch.randint(0, V, (T,), device=dev)
    out["cross_entropy_fwd_bwd"] = (lambda: E.cross_entropy_(logits, tgt, V, 1.0 / T, -100),
                                    2 * logits.numel() * 2, logits.numel() * 2)

    xg = torch.randn(16 * 1024, 3072, device=dev, dtype=bf)
    out["gelu_fwd"] = (lambda: E.gelu_fwd(xg), 2 * xg.numel() * 2, xg.numel() * 2)

    # AdamW over the embedding and LM head of Llama-3-8B (2 x 128256 x 4096, bf16 params and grads)
    ps = [torch.randn(V, D, device=dev, dtype=bf) for _ in range(2)]
    gs = [torch.randn_like(p) for p in ps]
    ms = [torch.zeros(p.shape, device=dev, dtype=f32) for p in ps]
    vs = [torch.zeros(p.shape, device=dev, dtype=f32) for p in ps]
    n = sum(p.numel() for p in ps)
    out["adamw_embed_head"] = (lambda: E.adamw(ps, gs, ms, vs, 1e-3, 0.9, 0.999, 1e-8, 0.01, 0.1, 0.03),
                               n * (2 + 2 + 4 + 4 + 2 + 4 + 4), n * 12)

    # LM-head gradient scaled by a device scalar (128256 x 4096 bf16, in place)
    sc = torch.ones(1, device=dev, dtype=f32)
    out["scale_head_grad"] = (lambda: E.scale_(ps[1], sc), 2 * ps[1].numel() * 2, ps[1].numel() * 2)
    # embedding: gather of 4096 rows; dense table gradient (zeros + 4096 summed rows) in one pass
    tok = torch.randint(0, V, (T,), device=dev)
    out["embedding_fwd"] = (lambda: E.embedding_fwd(ps[0], tok), 2 * T * D * 2, T * D * 2)
    dy_e = torch.randn(T, D, device=dev, dtype=bf)
    out["embedding_bwd"] = (lambda: E.embedding_bwd(dy_e, tok, V), V * D * 2 + T * D * 2, T * D * 2)

    # P2P-style pull-reduce, 8 "ranks" whose buffers are local here (the kernel of the
    # overlapped gradient reduce-scatter): reads 8 x rows, writes 1 x rows
    ws, rows = 8, F * D // 8
    bufs = [torch.randn(rows * ws, device=dev, dtype=bf) for _ in range(ws)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    dst = torch.empty(rows, device=dev, dtype=bf)
    out["rs_pull_reduce_8"] = (lambda: E.rs_pull_reduce(ptrs, 0, dst, False, 1.0 / ws), (ws + 1) * rows * 2,
                               ws * rows * 2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    from my_muon_fsdp2_b200._ext import check_device_error, ext

    peak = peak_gbs()
    want = set(filter(None, a.only.split(",")))
    res = {"peak_hbm_gbs": peak}
    for name, (fn, nbytes, in_bytes) in cases(ext()).items():
        if want and name not in want:
            continue
        ms = timeit(fn, a.iters)
        check_device_error(0)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac_of_measured": round(gbs / peak, 3),
                     "l2_resident": in_bytes <= L2_BYTES}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
