"""S5: diagonal complex state-space layer with HiPPO-LegS initialisation.

Parameters follow the reference ``S5SSM`` (``src/base_model/models/ssm.py:169-381``,
init in ``ssm_init.py``): ``Lambda_re``/``Lambda_im`` (P), ``B`` (P, H, 2) =
V^-1 B in real/imaginary parts, ``C`` (H, P, 2) (``C1``/``C2`` when
bidirectional), ``D`` (H), ``log_step`` (P, 1).  Discretisation is ZOH or
bilinear; with conjugate symmetry the output is ``2 Re(C x)``.

The scan is computed chunkwise: inside a chunk the Vandermonde matrix
``Lambda_bar^(t-s)`` turns the recurrence into one complex batched product,
and the chunk-final state is carried to the next chunk.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn as nn

from .common import lecun_normal_


def make_dplr_hippo(N: int):
    """Eigen-decomposition of the normal part of HiPPO-LegS (diagonal init of S5)."""
    p = np.sqrt(1 + 2 * np.arange(N))
    A = p[:, None] * p[None, :]
    A = -(np.tril(A) - np.diag(np.arange(N)))
    P = np.sqrt(np.arange(N) + 0.5)
    S = A + P[:, None] * P[None, :]
    lam_re = np.mean(np.diagonal(S)) * np.ones(N)
    lam_im, V = np.linalg.eigh(S * -1j)
    return lam_re + 1j * lam_im, V


class _S5Scan(torch.autograd.Function):
    """x_t = lam * x_{t-1} + Bu_t on the kernels of ``csrc/s5_scan.cu`` (complex64):
    returns every state and the final one; gradients for lam, Bu and x0."""

    @staticmethod
    def forward(ctx, lam, bu, x0):
        from ..ops._ext import ext
        c64 = lambda t: t.detach().to(torch.complex64).contiguous()
        lam_c, bu_c = c64(lam), c64(bu)
        x0_c = None if x0 is None else c64(x0)
        B, L, P = bu_c.shape
        xs = torch.empty_like(bu_c)
        xl = torch.empty(B, P, dtype=torch.complex64, device=bu.device)
        part = torch.empty(B, (L + 63) // 64, P, dtype=torch.complex64, device=bu.device)
        ext().s5_scan_fwd(lam_c, bu_c, x0_c, xs, xl, part)
        ctx.save_for_backward(lam_c, xs, x0_c)
        ctx.has_x0 = x0 is not None
        return xs, xl

    @staticmethod
    def backward(ctx, dxs, dxl):
        from ..ops._ext import ext
        lam_c, xs, x0_c = ctx.saved_tensors
        B, L, P = xs.shape
        dxs = torch.zeros_like(xs) if dxs is None else dxs.to(torch.complex64).contiguous()
        dxl = None if dxl is None else dxl.to(torch.complex64).contiguous()
        dbu = torch.empty_like(xs)
        dlam = torch.zeros(P, dtype=torch.complex64, device=xs.device)
        dx0 = torch.empty(B, P, dtype=torch.complex64, device=xs.device) if ctx.has_x0 else None
        part = torch.empty(B, (L + 63) // 64, P, dtype=torch.complex64, device=xs.device)
        ext().s5_scan_bwd(lam_c, xs, x0_c, dxs, dxl, dbu, dlam, dx0, part)
        return dlam, dbu, dx0


class S5(nn.Module):
    is_transformer = False

    def __init__(self, H, P, Lambda, V, Vinv, C_init="trunc_standard_normal", discretization="zoh",
                 dt_min=0.001, dt_max=0.1, conj_sym=True, clip_eigs=False, bidirectional=False,
                 step_rescale=1.0, chunk=64):
        super().__init__()
        self.H, self.P = H, P
        self.conj_sym, self.clip_eigs, self.bidirectional = conj_sym, clip_eigs, bidirectional
        self.discretization, self.step_rescale, self.chunk = discretization, step_rescale, chunk
        local_P = 2 * P if conj_sym else P
        self.Lambda_re = nn.Parameter(torch.tensor(Lambda.real, dtype=torch.float32))
        self.Lambda_im = nn.Parameter(torch.tensor(Lambda.imag, dtype=torch.float32))
        Bm = lecun_normal_(torch.empty(local_P, H), H).numpy()
        VB = Vinv @ Bm
        self.B = nn.Parameter(torch.tensor(np.stack([VB.real, VB.imag], -1), dtype=torch.float32))

        def c_param():
            if C_init == "complex_normal":
                return torch.randn(H, P, 2) * math.sqrt(0.5)
            Cm = (torch.randn(H, local_P).clamp(-2, 2) if C_init == "trunc_standard_normal"
                  else lecun_normal_(torch.empty(H, local_P), local_P)).numpy()
            CV = Cm @ V
            return torch.tensor(np.stack([CV.real, CV.imag], -1), dtype=torch.float32)
        if bidirectional:
            self.C1 = nn.Parameter(c_param())
            self.C2 = nn.Parameter(c_param())
        else:
            self.C = nn.Parameter(c_param())
        self.D = nn.Parameter(torch.randn(H))
        self.log_step = nn.Parameter(
            (torch.rand(P, 1) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)))

    def discrete(self):
        re = self.Lambda_re.clamp(max=-1e-4) if self.clip_eigs else self.Lambda_re
        lam = torch.complex(re, self.Lambda_im)
        Bt = torch.complex(self.B[..., 0], self.B[..., 1])
        dt = self.step_rescale * torch.exp(self.log_step[:, 0])
        if self.discretization == "zoh":
            lb = torch.exp(lam * dt)
            bb = ((1 / lam) * (lb - 1))[:, None] * Bt
        else:
            bl = 1 / (1 - dt / 2 * lam)
            lb = bl * (1 + dt / 2 * lam)
            bb = (bl * dt)[:, None] * Bt
        return lb, bb

    def _C(self):
        if self.bidirectional:
            return torch.cat([torch.complex(self.C1[..., 0], self.C1[..., 1]),
                              torch.complex(self.C2[..., 0], self.C2[..., 1])], -1)
        return torch.complex(self.C[..., 0], self.C[..., 1])

    use_kernel = True        # CUDA tensors take the s5_scan kernels (False: the chunked einsum)

    def _scan(self, lb, Bu, x0=None, reverse=False):
        """x_t = lb * x_{t-1} + Bu_t over (B, L, P) complex."""
        if reverse:
            xs, _ = self._scan(lb, Bu.flip(1))
            return xs.flip(1), None
        if Bu.is_cuda and self.use_kernel and Bu.shape[1] > 0:
            return _S5Scan.apply(lb, Bu, x0)
        B_, L, P = Bu.shape
        C = self.chunk
        t = torch.arange(C, device=Bu.device)
        dexp = (t[:, None] - t[None, :]).clamp(min=0)
        pw = lb[None, None, :] ** dexp[..., None].to(lb.dtype)                     # (C, C, P)
        pw = pw * (t[:, None] >= t[None, :])[..., None]
        pw_first = lb[None, :] ** (t + 1)[:, None].to(lb.dtype)                    # (C, P)
        x = torch.zeros(B_, P, dtype=Bu.dtype, device=Bu.device) if x0 is None else x0
        outs = []
        for s in range(0, L, C):
            e = min(L, s + C)
            n = e - s
            xc = torch.einsum("tsp,bsp->btp", pw[:n, :n], Bu[:, s:e]) + pw_first[:n][None] * x[:, None, :]
            outs.append(xc)
            x = xc[:, -1]
        return torch.cat(outs, 1), x

    def forward(self, u):
        lb, bb = self.discrete()
        Bu = torch.einsum("ph,blh->blp", bb, u.to(torch.complex64))
        xs, _ = self._scan(lb, Bu)
        if self.bidirectional:
            xs2, _ = self._scan(lb, Bu, reverse=True)
            xs = torch.cat([xs, xs2], -1)
        y = torch.einsum("hp,blp->blh", self._C(), xs).real
        if self.conj_sym:
            y = 2 * y
        return y + self.D * u

    def initial_state(self, batch, device=None):
        return torch.zeros(batch, self.P, dtype=torch.complex64, device=device)

    def step(self, state, u):
        if self.bidirectional:
            raise ValueError("Cannot expect a bidirectional view if doing rnn")
        lb, bb = self.discrete()
        Bu = torch.einsum("ph,blh->blp", bb, u.to(torch.complex64))
        xs, x = self._scan(lb, Bu, state)
        y = torch.einsum("hp,blp->blh", self._C(), xs).real
        if self.conj_sym:
            y = 2 * y
        return x, y + self.D * u


def make_s5_factory(state_size, blocks, conj_sym=True, **kw):
    block = state_size // blocks
    lam, V = make_dplr_hippo(block)
    P = state_size
    if conj_sym:
        block //= 2
        P //= 2
    lam = np.tile(lam[:block], blocks)
    Vb = V[:, :block]
    Vbig = np.zeros((blocks * Vb.shape[0], blocks * block), dtype=complex)
    for i in range(blocks):
        Vbig[i * Vb.shape[0]:(i + 1) * Vb.shape[0], i * block:(i + 1) * block] = Vb
    Vinv = Vbig.conj().T
    return lambda H: S5(H, P, lam, Vbig, Vinv, conj_sym=conj_sym, **kw)
