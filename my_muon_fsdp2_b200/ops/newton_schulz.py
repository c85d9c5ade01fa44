"""Newton–Schulz quintic orthogonalisation (the Muon "zeropower" map).

Math (parity with the reference, ``src/muon_fsdp/utils.py:12-106`` and the duplicate
``src/fsdp2_utils/numerical.py:10-56``)::

    X0 = G / (||G||_F + 1e-7)
    repeat `steps` times:   A = X X^T ;  B = b A + c A A ;  X = a X + B X
    (a, b, c) = (3.4445, -4.7750, 2.0315)

The reference transposes so that X is *tall* and therefore forms the larger Gram matrix.
Because p(X X^T) X == X p(X^T X) for any polynomial p, we always iterate on the *wide*
orientation (rows <= cols), i.e. the smaller Gram matrix: same result in exact arithmetic,
up to (n/m)^2 fewer FLOPs.

Two execution paths, chosen by the device of the input (never silently mixed):

* CPU tensors: plain PyTorch in fp32 (fp64 if the input is fp64). This is the oracle that
  the GPU kernels are tested against.
* CUDA tensors: the batched sm_100a chain in ``csrc/ns_chain.cu`` — bf16 operands, fp32
  TMEM accumulation, tcgen05 GEMMs with the Frobenius scale, the ``bA + cA^2`` axpby and the
  ``aX + BX`` axpby fused into the GEMM epilogues, symmetric (SYRK-style) Gram products.
  If the native extension is missing on a CUDA input this raises instead of falling back.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

NS_COEFFICIENTS = (3.4445, -4.7750, 2.0315)
NS_EPS = 1e-7


def _validate(G: torch.Tensor, steps: int) -> None:
    if G.dim() < 2:
        raise ValueError(f"Input tensor must have at least 2 dimensions, got {G.dim()}")
    if steps < 0:
        raise ValueError(f"steps must be non-negative, got {steps}")


def newton_schulz_reference(G: torch.Tensor, steps: int = 5, compute_dtype=None) -> torch.Tensor:
    """Literal restatement of the reference loop (tall orientation, larger Gram).

    Used only by tests as an independent oracle (typically in float64).
    """
    _validate(G, steps)
    if G.numel() == 0:
        return G
    dtype = G.dtype
    if compute_dtype is None:
        compute_dtype = torch.float32 if dtype == torch.bfloat16 else dtype
    X = G.to(compute_dtype)
    transposed = G.size(-2) < G.size(-1)
    if transposed:
        X = X.transpose(-2, -1)
    X = X / (X.norm() + NS_EPS)
    a, b, c = NS_COEFFICIENTS
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = b * A + c * A @ A
        X = a * X + B @ X
    if transposed:
        X = X.transpose(-2, -1)
    return X.to(dtype)


def _ns_torch(G: torch.Tensor, steps: int) -> torch.Tensor:
    """CPU path: fp32 (or fp64) iteration on the wide orientation, per matrix."""
    dtype = G.dtype
    compute_dtype = torch.float64 if dtype == torch.float64 else torch.float32
    X = G.to(compute_dtype)
    tall = X.size(-2) > X.size(-1)
    if tall:
        X = X.transpose(-2, -1)
    norm = torch.linalg.vector_norm(X, dim=(-2, -1), keepdim=True)
    X = X / (norm + NS_EPS)
    a, b, c = NS_COEFFICIENTS
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = torch.addmm(A, A, A, beta=b, alpha=c) if A.dim() == 2 else b * A + c * (A @ A)
        X = torch.addmm(X, B, X, beta=a) if X.dim() == 2 else a * X + B @ X
    if tall:
        X = X.transpose(-2, -1)
    return X.to(dtype).contiguous()


def zeropower_via_newtonschulz5(
    G: torch.Tensor,
    steps: int = 5,
    dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Approximate the orthogonal polar factor of ``G`` with the quintic Newton–Schulz map.

    Signature and validation match ``muon_fsdp.utils.zeropower_via_newtonschulz5``
    (``src/muon_fsdp/utils.py:12-72``): at least 2 dims, ``steps >= 0``, an empty tensor is
    returned as is, the output has the input's shape and dtype (or ``dtype`` when given).
    Inputs with more than 2 dims are treated as a batch of matrices over the last two dims.
    """
    _validate(G, steps)
    if G.numel() == 0:
        return G
    out_dtype = dtype if dtype is not None else G.dtype
    if G.is_cuda:
        from . import ns_cuda

        lead = G.shape[:-2]
        mats = G.reshape(-1, G.size(-2), G.size(-1))
        outs = ns_cuda.newton_schulz_batched([mats[i] for i in range(mats.size(0))], steps, out_dtype=out_dtype)
        return torch.stack(outs).reshape(*lead, G.size(-2), G.size(-1)) if len(lead) else outs[0]
    return _ns_torch(G, steps).to(out_dtype)


def newton_schulz_many(mats: Sequence[torch.Tensor], steps: int = 5) -> List[torch.Tensor]:
    """Orthogonalise a list of 2-D matrices (any shapes), batching same-shape ones on GPU."""
    if not mats:
        return []
    if mats[0].is_cuda:
        from . import ns_cuda

        return ns_cuda.newton_schulz_batched(list(mats), steps)
    return [_ns_torch(m, steps) for m in mats]


def muon_lr_scale(shape) -> float:
    """The reference's dimension-based lr scale ``max(1, min/max) ** 0.5``.

    ``src/muon_fsdp/optimizer.py:157-163``. Since min/max <= 1 this is always 1.0; it is kept
    as a function so that the (documented) behaviour is explicit.
    """
    m, n = shape[0], shape[1]
    return max(1.0, min(m, n) / max(m, n)) ** 0.5


def hsdp_lr_scale(shape) -> float:
    """HSDP variant scale ``sqrt(max/min)`` (``src/muon_fsdp/hdsp.py:380-382``)."""
    d_out, d_in = shape[0], shape[1]
    return (max(d_out, d_in) / min(d_out, d_in)) ** 0.5
