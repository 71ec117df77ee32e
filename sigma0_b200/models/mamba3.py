"""Mamba-3 SISO mixer (the flagship backbone).

Parameters and shapes follow the reference layer
(``src/base_model/models/mamba3.py:73-175``): one fused ``in_proj`` producing
``[z, x, B, C, dd_dt, dd_A, trap, angles]``, ``dt_bias``, per-head ``B_bias``
/ ``C_bias`` / ``D``, RMSNorms on B and C (``B_norm``/``C_norm``), and
``out_norm``/``out_proj`` held at full ``d_inner`` whatever the tensor-parallel
degree.  The small book pre-layers shrink ``headdim`` and the head count the
same way the reference does (``:111-123``).

Execution paths:

* ``impl="torch"``: the plain-torch oracle (CPU tests, reference numerics);
* ``impl="cuda"``: the fused sm_100a kernels (``sigma0_b200/csrc/mamba3_ssd.cu``)
  for the SSD and its pre/post processing, driven from
  :mod:`sigma0_b200.ops.mamba3_layer`.

``step`` is the recurrent decode (``__call_rnn__``, ``:466-578``); its state
is ``(angle (B,nh,R), ssm (B,nh,P,N), k_prev (B,nh,N), v_prev (B,nh,P))``.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .common import Dense, RMSNorm
from ..ops.reference import mamba3_ref as ref


@dataclass(frozen=True)
class Mamba3Dims:
    H: int
    d_state: int
    headdim: int
    n_heads: int
    d_inner: int
    R: int
    d_in_proj: int
    chunk_size: int


def mamba3_dims(H, d_state=128, expand=2, headdim=64, chunk_size=64, rope_fraction=0.5) -> Mamba3Dims:
    target = expand * H
    hd = min(headdim, target)
    nh = max(1, target // hd)
    d_inner = nh * hd
    split = int(d_state * rope_fraction)
    if split % 2:
        split -= 1
    R = split // 2
    return Mamba3Dims(H, d_state, hd, nh, d_inner, R, 2 * d_inner + 2 * d_state + 3 * nh + R, chunk_size)


class Mamba3(nn.Module):
    is_transformer = False

    def __init__(self, H, d_state=128, expand=2, headdim=64, chunk_size=64, rope_fraction=0.5,
                 A_floor=1e-4, dt_min=0.001, dt_max=0.1, tp_size=1, dtype=torch.float32,
                 impl="torch"):
        super().__init__()
        self.dims = d = mamba3_dims(H, d_state, expand, headdim, chunk_size, rope_fraction)
        self.H, self.A_floor, self.compute_dtype, self.impl = H, A_floor, dtype, impl
        self.tp_size = tp_size if (tp_size > 1 and d.n_heads % tp_size == 0) else 1
        self.in_proj = Dense(H, d.d_in_proj, bias=False)
        u = torch.rand(d.n_heads)
        dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.B_bias = nn.Parameter(torch.ones(d.n_heads, d.d_state))
        self.C_bias = nn.Parameter(torch.ones(d.n_heads, d.d_state))
        self.B_norm = RMSNorm(d.d_state)
        self.C_norm = RMSNorm(d.d_state)
        self.D = nn.Parameter(torch.ones(d.n_heads))
        self.out_norm = RMSNorm(d.d_inner)
        self.out_proj = Dense(d.d_inner, H, bias=False)

    # -- projection split ---------------------------------------------------------------
    def split_proj(self, proj: torch.Tensor):
        d = self.dims
        sizes = [d.d_inner, d.d_inner, d.d_state, d.d_state, d.n_heads, d.n_heads, d.n_heads, d.R]
        z, x, B, C, dd_dt, dd_A, trap, ang = torch.split(proj, sizes, dim=-1)
        return z, x, B, C, dd_dt, dd_A, trap, ang

    def _prep(self, proj):
        """proj (..., d_in_proj) -> SSD operands in float32 (shared B/C and angles)."""
        d = self.dims
        z, x, B, C, dd_dt, dd_A, trap, ang = self.split_proj(proj.float())
        lead = proj.shape[:-1]
        z = z.reshape(*lead, d.n_heads, d.headdim)
        x = x.reshape(*lead, d.n_heads, d.headdim)
        B = self.B_norm(B)
        C = self.C_norm(C)
        A = torch.clamp(-F.softplus(dd_A), max=-self.A_floor)
        DT = F.softplus(dd_dt + self.dt_bias)
        return z, x, B, C, A * DT, DT, trap, ang

    def _post(self, y):
        """y (..., nh, P) -> out_norm -> out_proj in the compute dtype."""
        d = self.dims
        y = y.reshape(*y.shape[:-2], d.d_inner)
        y = self.out_norm(y)
        return self.out_proj(y.to(self.compute_dtype), dtype=self.compute_dtype)

    # -- forward (training) ---------------------------------------------------------------
    def forward(self, u: torch.Tensor) -> torch.Tensor:
        """u (B, L, H) -> (B, L, H)."""
        if self.impl == "cuda" and u.is_cuda:
            from ..ops.mamba3_layer import mamba3_mixer
            return mamba3_mixer(u, self)
        proj = self.in_proj(u, dtype=self.compute_dtype)
        z, x, B, C, ADT, DT, trap, ang = self._prep(proj)
        nh = self.dims.n_heads
        Bh = B[:, :, None, :].expand(-1, -1, nh, -1)
        Ch = C[:, :, None, :].expand(-1, -1, nh, -1)
        y = ref.mamba3_ssd_chunked(Ch, Bh, x, ADT.transpose(1, 2), DT.transpose(1, 2),
                                   trap.transpose(1, 2), ang, self.C_bias, self.B_bias, self.D, z,
                                   chunk_size=self.dims.chunk_size)
        return self._post(y)

    # -- decode ------------------------------------------------------------------------
    def initial_state(self, batch: int, device=None):
        d = self.dims
        z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=device)
        return (z(batch, d.n_heads, d.R), z(batch, d.n_heads, d.headdim, d.d_state),
                z(batch, d.n_heads, d.d_state), z(batch, d.n_heads, d.headdim))

    def _cuda_ok(self, u) -> bool:
        d = self.dims
        return (self.impl == "cuda" and u.is_cuda and (d.d_state, d.headdim, d.chunk_size, d.R) == (128, 64, 64, 32))

    def step(self, state, u: torch.Tensor):
        """Run ``u`` (B, L, H) through the recurrence from ``state``; returns (state, out)."""
        if self._cuda_ok(u) and u.shape[1] <= 8:
            return self._step_cuda(state, u)
        proj = self.in_proj(u, dtype=self.compute_dtype)
        z, x, B, C, ADT, DT, trap, ang = self._prep(proj)
        nh = self.dims.n_heads
        Bh = B[:, :, None, :].expand(-1, -1, nh, -1)
        Ch = C[:, :, None, :].expand(-1, -1, nh, -1)
        y, state = ref.mamba3_recurrent(Ch, Bh, x, ADT.transpose(1, 2), DT.transpose(1, 2),
                                        trap.transpose(1, 2), ang, self.C_bias, self.B_bias,
                                        self.D, z, state)
        return state, self._post(y)

    # -- CUDA decode and prefill -------------------------------------------------------------
    def _proj_cuda(self, u2):
        from ..ops import weights as W
        d = self.dims
        ldp = (d.d_in_proj + 7) // 8 * 8
        return u2.to(torch.bfloat16).contiguous() @ W.bf16_padded(self.in_proj.kernel, ldp)

    def _post_cuda(self, y2):
        from ..ops._ext import ext
        from ..ops import weights as W
        yn, _ = ext().rms_fwd(y2, self.out_norm.scale, self.out_norm.eps)
        return yn @ W.bf16(self.out_proj.kernel)

    def _step_cuda(self, state, u):
        """1..8 tokens through the recurrence in one kernel (each head's state is read and
        written once for all the tokens); the state tensors are updated in place."""
        from ..ops._ext import ext
        d = self.dims
        B, L, H = u.shape
        proj = self._proj_cuda(u.reshape(B * L, H))
        ang, ssm, kp, vp = state
        y = torch.empty(B * L, d.d_inner, dtype=torch.bfloat16, device=u.device)
        ext().m3_decode_step(proj, d.n_heads, self.B_norm.scale, self.C_norm.scale, self.dt_bias, self.B_bias,
                             self.C_bias, self.D, self.A_floor, self.B_norm.eps, ang, ssm, kp, vp, y, L)
        return state, self._post_cuda(y).view(B, L, -1)

    @torch.no_grad()
    def prefill(self, u: torch.Tensor):
        """Chunked forward over ``u`` (B, L, H) that also returns the recurrent state
        after the last token (the decode carry), instead of stepping token by token."""
        d = self.dims
        B, L, H = u.shape
        if not self._cuda_ok(u):
            proj = self.in_proj(u, dtype=self.compute_dtype)
            z, x, Bn, Cn, ADT, DT, trap, ang = self._prep(proj)
            st0 = self.initial_state(B, u.device)
            nh = d.n_heads
            y, st = ref.mamba3_recurrent(Cn[:, :, None].expand(-1, -1, nh, -1), Bn[:, :, None].expand(-1, -1, nh, -1),
                                         x, ADT.transpose(1, 2), DT.transpose(1, 2), trap.transpose(1, 2), ang,
                                         self.C_bias, self.B_bias, self.D, z, st0)
            return st, self._post(y)
        from ..ops._ext import ext
        proj = self._proj_cuda(u.reshape(-1, H))
        y, _, fin, thf = ext().m3_fwd(proj, B, L, d.n_heads, self.B_norm.scale, self.C_norm.scale, self.dt_bias,
                                      self.B_bias, self.C_bias, self.D, self.A_floor, self.B_norm.eps, want_final=True)
        # k_prev / v_prev: the last token's rotated key and value
        last = proj.view(B, L, -1)[:, -1, :d.d_in_proj].float()
        z, x, Bn, Cn, ADT, DT, trap, angr = self._prep(last[:, None])
        cos, sin = torch.cos(thf), torch.sin(thf)
        Kb = Bn[:, 0][:, None, :] + self.B_bias[None]
        kp = ref.apply_rope(Kb, cos, sin)
        st = (thf.contiguous(), fin, kp.contiguous(), x[:, 0].contiguous())
        return st, self._post_cuda(y.view(-1, d.d_inner)).view(B, L, H)
