"""The tcgen05 GEMM (``csrc/gemm_tc.cu``) for the model projections.

Three products cover a projection ``y = x . W`` (``W`` in the Flax ``[in, out]`` layout)
and its backward pass, each read straight from the row-major tensors:

* :func:`mm`          ``x @ W``            forward (bf16 out);
* :func:`mm_nt`       ``dy @ W^T``         input gradient (bf16 out);
* :func:`mm_tn_acc`   ``out += x^T @ dy``  weight gradient, reduce-added in fp32 into ``out``
  (normally the parameter's slice of the flat float32 gradient buffer).

The reference computes these as XLA dots inside ``nn.Dense``
(``src/base_model/models/mamba3.py:191-331``, ``src/base_model/models/layers.py:120-160``).
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from ._ext import ext

# S0_GEMM=cublas routes the model projections through torch.matmul instead (the comparison arm
# of the step benchmarks); the default is this package's kernel
USE_TC = os.environ.get("S0_GEMM", "tc") != "cublas"


def _rows(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def mm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x [M, K] @ w [K, N]`` in bf16 with fp32 accumulation."""
    return ext().gemm_tc(_rows(x), _rows(w), False, True)


def mm_nt(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``dy [M, N] @ w[K, N]^T`` -> ``[M, K]`` (bf16)."""
    return ext().gemm_tc(_rows(dy), _rows(w), False, False)


def mm_tn_acc(x: torch.Tensor, dy: torch.Tensor, out: torch.Tensor, split_k: int = 0) -> torch.Tensor:
    """``out += x[T, M]^T @ dy[T, N]`` with ``out`` fp32 of shape ``[<= M, <= N]`` (the
    rows / columns beyond it are dropped).  ``split_k`` 0 lets the launcher split the long
    token reduction so the output tiles fill every SM (the parts meet in the reduce-add)."""
    ext().gemm_tc(_rows(x), _rows(dy), True, True, 2, out, max(0, int(split_k)))
    return out


def use_pair(on: bool = True) -> None:
    """Two-SM (``cta_group::2``, 256 x 256) tiles (the default) or one-SM 128 x 256 tiles."""
    ext().gemm_use_pair(bool(on))


def status(like: torch.Tensor) -> int:
    """1 once a bounded wait of the GEMM gave up on this device (reads the device word)."""
    return int(ext().gemm_status(like).item())


# ---- the model's projection products (the kernel, or torch.matmul under S0_GEMM=cublas) --------
def proj(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w`` (bf16)."""
    return mm(x, w) if USE_TC else x @ w


def proj_dx(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``dy @ w^T`` (bf16)."""
    return mm_nt(dy, w) if USE_TC else dy @ w.t()


def _fusable(*ts: torch.Tensor) -> bool:
    return USE_TC and all(t.is_cuda and t.stride(-1) == 1 and t.data_ptr() % 16 == 0 for t in ts)


def proj_gelu(x: torch.Tensor, w: torch.Tensor):
    """``o = x @ w`` and ``g = gelu(o)`` (both bf16), one GEMM with the GELU in its epilogue."""
    if _fusable(x, w) and w.shape[1] % 64 == 0:
        o, g = ext().gemm_gelu_fwd(_rows(x), _rows(w))
        return o, g
    o = proj(x, w)
    return o, ext().gelu_fwd(o)


def _owns_grad(param: torch.Tensor) -> bool:
    g = param.grad
    return (getattr(param, "_s0_flat_grad", False) and g is not None and g.dtype == torch.float32
            and g.stride(-1) == 1 and g.data_ptr() % 16 == 0 and (g.stride(0) * 4) % 16 == 0)


def wgrad(param: torch.Tensor, x: torch.Tensor, dy: torch.Tensor) -> Optional[torch.Tensor]:
    """The weight gradient ``x^T @ dy`` of ``param`` (its leading ``param.shape`` block).

    For a parameter whose gradient lives in the flat float32 buffer of the optimizer (marked
    ``_s0_flat_grad`` by it) the product is reduce-added straight into ``param.grad`` in fp32 and
    None is returned: autograd has nothing left to accumulate.  Otherwise the gradient is returned
    as a new float32 tensor."""
    r, c = param.shape
    if not USE_TC:
        return (x.t() @ dy)[:r, :c].float()
    if _owns_grad(param):
        mm_tn_acc(x, dy, param.grad)
        return None
    # a separate fp32 result whose rows are padded to 16 bytes for the tensor map (odd widths such
    # as the 503-wide book layers); the leading block is returned
    cp = (c + 3) // 4 * 4
    if cp > dy.shape[1] or r > x.shape[1]:
        return (x.t() @ dy)[:r, :c].float()
    out = torch.zeros(r, cp, dtype=torch.float32, device=x.device)
    mm_tn_acc(x, dy, out)
    return out[:, :c]
