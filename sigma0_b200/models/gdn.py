"""Gated DeltaNet (GDN) and Kimi Delta Attention (KDA) mixers.

Parameters and computation follow the reference ``GDNSSM``
(``src/base_model/models/gdn.py:40-630``): q/k/v projections, optional causal
depthwise Conv1d(k=4) with SiLU, L2-normalised q and k (epsilon under the
square root), ``q *= head_dim**-0.5``, write gate ``beta = sigmoid(b_proj)``,
decay ``log alpha = log_sigmoid(gk_proj)`` (per head for GDN, per key dim for
KDA), output gate ``silu(g_proj)``, per-head RMSNorm, ``o_proj`` and the
``D * x`` feed-through.

The recurrence per head (state S: (hvd, hd)):
``S <- S * alpha;  S <- S + beta (v - S k) k^T;  o = S q``.
Training uses the exact chunkwise form: within a chunk the delta-rule
interactions are resolved with a unit-lower-triangular solve (the WY form of
Yang et al., "Gated Delta Networks"), across chunks the state is carried.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .common import Dense, RMSNorm, lecun_normal_


def l2_normalize(x, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)).to(x.dtype)


class CausalDepthwiseConv1d(nn.Module):
    def __init__(self, channels, kernel_size=4):
        super().__init__()
        self.k = kernel_size
        self.kernel = nn.Parameter(lecun_normal_(torch.empty(kernel_size, channels), kernel_size))
        self.bias = nn.Parameter(torch.zeros(channels))

    def _conv(self, xc):
        # xc (B, k-1+L, C) -> (B, L, C)
        L = xc.shape[1] - (self.k - 1)
        out = self.bias.to(xc.dtype).expand(xc.shape[0], L, -1).clone()
        for j in range(self.k):
            out = out + xc[:, j:j + L] * self.kernel[j].to(xc.dtype)
        return out

    def forward(self, x):
        return self._conv(F.pad(x, (0, 0, self.k - 1, 0)))

    def step(self, buf, x):
        xc = torch.cat([buf, x], dim=1)
        return xc[:, -(self.k - 1):], self._conv(xc)


class _GDNScan(torch.autograd.Function):
    """The cross-chunk state scan on the sm_100a kernels of ``csrc/gdn_scan.cu``.

    Inputs in (B, nh, nc, C, ...) layout: qe = q exp(G), kc = (I - L)^-1 (beta k exp(G)),
    kd = k exp(G_end - G), intra (lower-triangular scores), vc = (I - L)^-1 (beta v),
    tot = exp(G_end) per key column, S0 (or None).  Returns o (B, nh, nc, C, hvd) and the
    final state.  The kernel multiplies in bf16 with fp32 accumulation and keeps the
    state in fp32."""

    @staticmethod
    def forward(ctx, qe, kc, kd, intra, vc, tot, S0):
        from ..ops._ext import ext
        bf = lambda t: t.detach().to(torch.bfloat16).contiguous()
        qe_b, kc_b, kd_b, in_b = bf(qe), bf(kc), bf(kd), bf(intra)
        vc_c, tot_c = vc.detach().float().contiguous(), tot.detach().float().contiguous()
        B, nh, nc, C, hd = qe.shape
        hvd = vc.shape[-1]
        o = torch.empty(B, nh, nc, C, hvd, device=qe.device)
        vnew = torch.empty_like(o)
        S_all = torch.empty(B, nh, nc, hvd, hd, device=qe.device)
        S_fin = torch.empty(B, nh, hvd, hd, device=qe.device)
        s0 = S0.detach().float().contiguous() if S0 is not None else None
        ext().gdn_scan_fwd(qe_b, kc_b, kd_b, in_b, vc_c, tot_c, s0, o, S_all, vnew, S_fin)
        ctx.save_for_backward(qe_b, kc_b, kd_b, in_b, tot_c, S_all, vnew)
        ctx.has_s0 = S0 is not None
        return o, S_fin

    @staticmethod
    def backward(ctx, do, dS_fin):
        from ..ops._ext import ext
        qe_b, kc_b, kd_b, in_b, tot_c, S_all, vnew = ctx.saved_tensors
        B, nh, nc, C, hd = qe_b.shape
        hvd = vnew.shape[-1]
        nvb = hvd // ext().gdn_scan_bwd_value_block()
        do = torch.zeros_like(vnew) if do is None else do.float().contiguous()
        dS_fin = None if dS_fin is None else dS_fin.float().contiguous()
        dev = vnew.device
        dqe = torch.empty(nvb, B, nh, nc, C, hd, device=dev)
        dkc, dkd = torch.empty_like(dqe), torch.empty_like(dqe)
        din = torch.empty(nvb, B, nh, nc, C, C, device=dev)
        dtot = torch.empty(nvb, B, nh, nc, hd, device=dev)
        dvc = torch.empty_like(vnew)
        dS0 = torch.empty(B, nh, hvd, hd, device=dev)
        ext().gdn_scan_bwd(qe_b, kc_b, kd_b, in_b, tot_c, S_all, vnew, do, dS_fin, dqe, dkc, dkd, din, dtot, dvc, dS0)
        return (dqe.sum(0), dkc.sum(0), dkd.sum(0), din.sum(0), dvc, dtot.sum(0),
                dS0 if ctx.has_s0 else None)


class _KDAIntra(torch.autograd.Function):
    """intra = sum_d q k exp(G_i - G_j) (i >= j) and Lm = -sum_d kb k exp(G_i - G_j) (i > j)
    per 64-step chunk on the kernels of ``csrc/kda_intra.cu`` (no [C, C, hd] tensor)."""

    @staticmethod
    def forward(ctx, q, k, kb, G):
        from ..ops._ext import ext
        shp = q.shape
        f = lambda t: t.detach().float().reshape(-1, shp[-2], shp[-1]).contiguous()
        qf, kf, kbf, Gf = f(q), f(k), f(kb), f(G)
        N = qf.shape[0]
        intra = torch.empty(N, 64, 64, device=q.device)
        Lm = torch.empty_like(intra)
        ext().kda_intra_fwd(qf, kf, kbf, Gf, intra, Lm)
        ctx.save_for_backward(qf, kf, kbf, Gf)
        ctx.shp = shp
        return intra.reshape(*shp[:-1], 64), Lm.reshape(*shp[:-1], 64)

    @staticmethod
    def backward(ctx, gI, gL):
        from ..ops._ext import ext
        qf, kf, kbf, Gf = ctx.saved_tensors
        N = qf.shape[0]
        g = lambda t: torch.zeros(N, 64, 64, device=qf.device) if t is None else t.float().reshape(N, 64, 64).contiguous()
        dq, dk, dkb, dG = (torch.empty_like(qf) for _ in range(4))
        ext().kda_intra_bwd(qf, kf, kbf, Gf, g(gI), g(gL), dq, dk, dkb, dG)
        return tuple(t.reshape(ctx.shp) for t in (dq, dk, dkb, dG))


def _scan_kernel_ok(q, v, chunk) -> bool:
    return q.is_cuda and chunk == 64 and q.shape[-1] in (64, 128) and v.shape[-1] % 64 == 0


def chunk_transitions_product(M: torch.Tensor) -> torch.Tensor:
    """M (B, nc, nh, d, d) -> M_0 M_1 ... M_{nc-1} (B, nh, d, d) by a log-depth pairwise
    product (the order of the factors is kept)."""
    while M.shape[1] > 1:
        if M.shape[1] % 2:
            eye = torch.eye(M.shape[-1], dtype=M.dtype, device=M.device).expand(M.shape[0], 1, *M.shape[2:])
            M = torch.cat([M, eye], 1)
        M = M[:, 0::2] @ M[:, 1::2]
    return M[:, 0]


def gated_delta_chunked(q, k, v, beta, alog, chunk=64, S0=None, use_kernel=None, return_transition=False):
    """q,k (B,L,nh,hd); v (B,L,nh,hvd); beta (B,L,nh); alog (B,L,nh,hd or 1).

    Returns o (B,L,nh,hvd) and the final state (B,nh,hvd,hd).  On CUDA (chunk 64, key
    head dim 64 / 128, value head dim a multiple of 64) the cross-chunk scan runs the
    ``gdn_scan`` kernels; ``use_kernel=False`` keeps the host loop (the oracle).

    ``return_transition=True`` also returns the sequence's state transition T (B, nh, hd,
    hd): the final state is S0 T plus the final state from a zero start, since every chunk
    maps S -> S (diag(tot) - kc^T kd) + vc^T kd (context parallelism composes segments
    with it).
    """
    B, L, nh, hd = q.shape
    hvd = v.shape[-1]
    pad = (chunk - L % chunk) % chunk
    if pad:
        q, k, v = (F.pad(t, (0, 0, 0, 0, 0, pad)) for t in (q, k, v))
        beta = F.pad(beta, (0, 0, 0, pad))
        alog = F.pad(alog, (0, 0, 0, 0, 0, pad))
    nc = (L + pad) // chunk
    C = chunk
    f = lambda t: t.float().reshape(B, nc, C, *t.shape[2:]).transpose(2, 3)   # (B,nc,nh,C,...)
    q, k, v, alog = f(q), f(k), f(v), f(alog)
    beta = beta.float().reshape(B, nc, C, nh).transpose(2, 3)                   # (B,nc,nh,C)
    G = alog.cumsum(3)                                                          # (B,nc,nh,C,d|1)
    tri = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device))
    stri = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device), -1)
    kb = k * beta[..., None]
    vb = v * beta[..., None]
    if use_kernel is None:
        use_kernel = _scan_kernel_ok(q, v, chunk)
    if G.shape[-1] != 1 and use_kernel:
        intra, Lm = _KDAIntra.apply(q, k, kb, G)
    elif G.shape[-1] == 1:
        dG = (G[..., :, None, 0] - G[..., None, :, 0]).masked_fill(~tri, 0.0)
        W = torch.exp(dG) * tri
        intra = (q @ k.transpose(-1, -2)) * W
        Lm = -(kb @ k.transpose(-1, -2)) * W * stri
    else:
        dG = (G[..., :, None, :] - G[..., None, :, :]).masked_fill(~tri[..., None], 0.0)
        W = torch.exp(dG) * tri[..., None]
        intra = torch.einsum("...id,...jd,...ijd->...ij", q, k, W)
        Lm = -torch.einsum("...id,...jd,...ijd->...ij", kb, k, W) * stri
    I = torch.eye(C, device=q.device)
    A = I - Lm
    vc = torch.linalg.solve_triangular(A, vb, upper=False)                     # (B,nc,nh,C,hvd)
    kcd = torch.linalg.solve_triangular(A, kb * torch.exp(G), upper=False)    # (B,nc,nh,C,hd)
    dec_end = torch.exp(G[..., -1:, :] - G)                                     # (B,nc,nh,C,d|1)
    kdec = k * dec_end
    trans = None
    if return_transition:
        totd = torch.exp(G[..., -1, :]).expand(B, nc, nh, hd)
        Mc = torch.diag_embed(totd) - kcd.transpose(-1, -2) @ kdec                  # (B,nc,nh,hd,hd)
        trans = chunk_transitions_product(Mc)
    if use_kernel:
        P = lambda t: t.transpose(1, 2)                                         # -> (B,nh,nc,...)
        tot = P(torch.exp(G[..., -1, :])).expand(B, nh, nc, hd)
        o, S = _GDNScan.apply(P(q * torch.exp(G)), P(kcd), P(kdec), P(intra), P(vc), tot,
                              None if S0 is None else S0.float())
        o = P(o).transpose(2, 3).reshape(B, nc * C, nh, hvd)[:, :L]
        return (o, S, trans) if return_transition else (o, S)
    S = torch.zeros(B, nh, hvd, hd, device=q.device) if S0 is None else S0.float()
    outs = []
    for c in range(nc):
        qc = q[:, c] * torch.exp(G[:, c])
        vnew = vc[:, c] - kcd[:, c] @ S.transpose(-1, -2)                       # (B,nh,C,hvd)
        o = qc @ S.transpose(-1, -2) + intra[:, c] @ vnew
        outs.append(o)
        tot = torch.exp(G[:, c, :, -1, :])                                      # (B,nh,d|1)
        S = S * tot[:, :, None, :] + vnew.transpose(-1, -2) @ kdec[:, c]
    o = torch.stack(outs, 1).transpose(2, 3).reshape(B, nc * C, nh, hvd)[:, :L]
    return (o, S, trans) if return_transition else (o, S)


def gated_delta_recurrent(q, k, v, beta, alog, S=None, use_kernel=None):
    """Token-by-token recurrence: o (B,L,nh,hvd) and the new state (B,nh,hvd,hd).  On CUDA,
    head dim 64 / 128, when no gradient is needed (decode) it runs the ``gdn_decode`` kernel
    (``csrc/gdn_decode.cu``: one warp per state row, the state read and written once);
    ``use_kernel=False`` keeps the loop below (the oracle)."""
    B, L, nh, hd = q.shape
    hvd = v.shape[-1]
    if use_kernel is None:
        needs_grad = torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                                     for t in (q, k, v, beta, alog, S))
        use_kernel = q.is_cuda and hd in (64, 128) and not needs_grad
    if use_kernel:
        from ..ops._ext import ext
        c = lambda t: t.detach().float().contiguous()
        St = torch.zeros(B, nh, hvd, hd, device=q.device) if S is None else S.detach().float().clone().contiguous()
        o = torch.empty(B, L, nh, hvd, device=q.device)
        ext().gdn_decode(c(q), c(k), c(v), c(beta), c(alog), St, o)
        return o, St
    S = torch.zeros(B, nh, hvd, hd, device=q.device) if S is None else S.float()
    outs = []
    for t in range(L):
        a = torch.exp(alog[:, t].float())                                       # (B,nh,d|1)
        S = S * a[:, :, None, :]
        kt = k[:, t].float()
        Sk = torch.einsum("bnvk,bnk->bnv", S, kt)
        delta = v[:, t].float() - Sk
        S = S + torch.einsum("bnv,bnk->bnvk", beta[:, t].float()[..., None] * delta, kt)
        outs.append(torch.einsum("bnvk,bnk->bnv", S, q[:, t].float()))
    return torch.stack(outs, 1), S


class GDN(nn.Module):
    is_transformer = False

    def __init__(self, H, num_heads, head_dim=128, expand_v=2, chunk_size=64, use_conv=True, use_kda=False,
                 impl="torch"):
        super().__init__()
        self.H = H
        self.nh = min(num_heads, max(1, H // head_dim))
        self.hd = min(head_dim, H)
        self.hvd = self.hd * expand_v
        self.chunk = chunk_size
        self.use_conv, self.use_kda, self.impl = use_conv, use_kda, impl
        nh, hd, hvd = self.nh, self.hd, self.hvd
        self.q_proj = Dense(H, nh * hd, bias=False)
        self.k_proj = Dense(H, nh * hd, bias=False)
        self.v_proj = Dense(H, nh * hvd, bias=False)
        self.b_proj = Dense(H, nh, bias=True)
        self.gk_proj = Dense(H, nh * hd if use_kda else nh, bias=True)
        self.g_proj = Dense(H, nh * hvd, bias=False)
        self.o_proj = Dense(nh * hvd, H, bias=False)
        if use_conv:
            self.q_conv = CausalDepthwiseConv1d(nh * hd)
            self.k_conv = CausalDepthwiseConv1d(nh * hd)
            self.v_conv = CausalDepthwiseConv1d(nh * hvd)
        self.out_norm = RMSNorm(hvd)
        self.D = nn.Parameter(torch.randn(H))

    def _inputs(self, x, bufs=None):
        B, L, _ = x.shape
        nh, hd, hvd = self.nh, self.hd, self.hvd
        q, k, v = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        new_bufs = None
        if self.use_conv:
            if bufs is None:
                q, k, v = F.silu(self.q_conv(q)), F.silu(self.k_conv(k)), F.silu(self.v_conv(v))
            else:
                qb, q = self.q_conv.step(bufs[0], q)
                kb, k = self.k_conv.step(bufs[1], k)
                vb, v = self.v_conv.step(bufs[2], v)
                q, k, v = F.silu(q), F.silu(k), F.silu(v)
                new_bufs = (qb, kb, vb)
        q = l2_normalize(q.reshape(B, L, nh, hd)) * hd ** -0.5
        k = l2_normalize(k.reshape(B, L, nh, hd))
        v = v.reshape(B, L, nh, hvd)
        beta = torch.sigmoid(self.b_proj(x))
        alog = F.logsigmoid(self.gk_proj(x)).reshape(B, L, nh, hd if self.use_kda else 1)
        g = F.silu(self.g_proj(x)).reshape(B, L, nh, hvd)
        return q, k, v, beta, alog, g, new_bufs

    def _out(self, x, o, g):
        B, L = o.shape[:2]
        o = self.out_norm(o) * g
        return self.o_proj(o.reshape(B, L, self.nh * self.hvd)) + x * self.D

    def forward(self, x):
        q, k, v, beta, alog, g, _ = self._inputs(x)
        o, _ = gated_delta_chunked(q, k, v, beta, alog, self.chunk)
        return self._out(x, o, g)

    def initial_state(self, batch, device=None):
        S = torch.zeros(batch, self.nh, self.hvd, self.hd, device=device)
        if not self.use_conv:
            return S
        z = lambda c: torch.zeros(batch, 3, c, device=device)
        return (S, (z(self.nh * self.hd), z(self.nh * self.hd), z(self.nh * self.hvd)))

    def step(self, state, x):
        S, bufs = (state if self.use_conv else (state, None))
        q, k, v, beta, alog, g, nb = self._inputs(x, bufs)
        o, S = gated_delta_recurrent(q, k, v, beta, alog, S)
        out = self._out(x, o, g)
        return ((S, nb) if self.use_conv else S), out
