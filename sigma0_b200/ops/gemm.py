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

import torch

from ._ext import ext

# weight gradients whose output tiles cannot fill the GPU are split along the long reduction
# (tokens) into this many parts at most; the parts meet in the fp32 reduce-add
_MAX_SPLIT = 8


def _sms(t: torch.Tensor) -> int:
    return torch.cuda.get_device_properties(t.device).multi_processor_count


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
    rows / columns beyond it are dropped).  ``split_k`` 0 picks a split that gives every SM
    a share of the output tiles."""
    M, N = x.shape[1], dy.shape[1]
    if split_k <= 0:
        tiles = -(-M // 128) * -(-N // 256)
        sms = _sms(x)
        split_k = max(1, min(_MAX_SPLIT, sms // max(tiles, 1)))
        while split_k > 1 and x.shape[0] // split_k < 64 * 4:
            split_k -= 1
    ext().gemm_tc(_rows(x), _rows(dy), True, True, 2, out, split_k)
    return out


def status(like: torch.Tensor) -> int:
    """1 once a bounded wait of the GEMM gave up on this device (reads the device word)."""
    return int(ext().gemm_status(like).item())
