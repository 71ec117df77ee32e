"""Tensor parallelism (heads split over a tensor-parallel group) for the GDN / KDA mixer, the
transformer block and the NSA block.

The reference shards these over its ``tp`` mesh axis: the projections that produce a head's
inputs are column-parallel, the projection that consumes the heads' outputs is
row-parallel and followed by a psum (``src/base_model/models/gdn.py:87-243``,
``src/base_model/models/transformer.py``).  Here, as in ``Mamba3TP``:

* the input enters through ``copy_to_tp`` (identity forward, gradient all-reduce) and the
  row-parallel output leaves through ``reduce_from_tp`` (all-reduce forward, identity
  backward) -- or through the fused GEMM + all-reduce kernel (``use_fused_out_proj``);
* terms that do not depend on the heads (the GDN ``D * x`` feed-through, output biases)
  are added once, after the reduction, on the replicated activation;
* a replicated parameter that only sees this rank's heads (GDN's per-head RMSNorm scale)
  enters through ``copy_to_tp`` too, so its gradient is summed over the group.

``shard_heads(model, group)`` replaces every ``GDN`` mixer, ``TransformerBlock`` and
``NSABlock`` of a model in place with its slice.
"""
from __future__ import annotations


import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..models.common import gelu_tanh
from ..models.gdn import GDN, gated_delta_chunked, gated_delta_recurrent, l2_normalize
from ..models.nsa import NSABlock
from ..models.rope import apply_rope, rotary_embedding, sinusoidal
from ..models.transformer import TransformerBlock, causal_attention
from .tp import copy_to_tp, reduce_from_tp


def _cols(t: torch.Tensor, h0: int, n: int, per: int, dim: int = -1) -> nn.Parameter:
    return nn.Parameter(t.detach().narrow(dim, h0 * per, n * per).clone())


def _split(world: int, rank: int, heads: int, what: str):
    if heads % world:
        raise ValueError(f"{heads} {what} do not split over tensor-parallel size {world}")
    n = heads // world
    return n, rank * n


class _RowParallel:
    """The row-parallel output: NCCL all-reduce, or the fused kernel once enabled; and the
    consolidated state of the single-device block (``full_state_dict``)."""

    fused = None
    # (this module's parameter, the single-device block's parameter, split dim or None)
    _FULL: tuple = ()

    def full_state_dict(self) -> dict:
        """The single-device block's parameters, by its names, from every rank's slices (an
        all-gather along each split dimension; replicated parameters as they are).  Every
        rank of the group must call it."""
        own = dict(self.named_parameters())
        out = {}
        for local, full, dim in self._full_table():
            t = own[local].detach()
            if dim is not None:
                parts = [torch.empty_like(t) for _ in range(dist.get_world_size(self.group))]
                dist.all_gather(parts, t.contiguous(), group=self.group)
                t = torch.cat(parts, dim)
            out[full] = t
        return out

    def _full_table(self) -> tuple:
        return self._FULL

    def tp_sharded_parameters(self) -> list:
        """This rank's slices (their gradients are partial per rank; the rest is replicated)."""
        own = dict(self.named_parameters())
        return [own[local] for local, _, dim in self._full_table() if dim is not None]

    def _reduce(self, y: torch.Tensor, w: torch.Tensor, group) -> torch.Tensor:
        if self.fused is not None and y.is_cuda and y.numel() // y.shape[-1] <= self.fused.M:
            from .tp_fused import fused_row_parallel
            lead = y.shape[:-1]
            return fused_row_parallel(y.reshape(-1, y.shape[-1]), w, self.fused).reshape(*lead, -1)
        return reduce_from_tp(y @ w.to(y.dtype), group)

    def use_fused_out_proj(self, max_rows: int) -> None:
        """Route the output projection + all-reduce through the fused peer-memory kernel
        for inputs of up to ``max_rows`` tokens."""
        from .tp_fused import FusedRowParallel
        w = self._out_weight()
        self.fused = FusedRowParallel(max_rows, w.shape[1], self.group, w.device)


def _dconv(x: torch.Tensor, kernel: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """Causal depthwise convolution (the ``CausalDepthwiseConv1d`` math on this rank's
    channels); x (B, L, C)."""
    k = kernel.shape[0]
    xc = F.pad(x, (0, 0, k - 1, 0))
    L = x.shape[1]
    out = bias.to(x.dtype).expand(x.shape[0], L, -1)
    for j in range(k):
        out = out + xc[:, j:j + L] * kernel[j].to(x.dtype)
    return out


class GDNTP(nn.Module, _RowParallel):
    is_transformer = False

    def __init__(self, full: GDN, group=None):
        super().__init__()
        self.group = group
        T, r = dist.get_world_size(group), dist.get_rank(group)
        self.nhl, self.h0 = _split(T, r, full.nh, "GDN heads")
        nhl, h0, hd, hvd = self.nhl, self.h0, full.hd, full.hvd
        self.hd, self.hvd, self.chunk = hd, hvd, full.chunk
        self.use_conv, self.use_kda = full.use_conv, full.use_kda
        self.q_w = _cols(full.q_proj.kernel, h0, nhl, hd)
        self.k_w = _cols(full.k_proj.kernel, h0, nhl, hd)
        self.v_w = _cols(full.v_proj.kernel, h0, nhl, hvd)
        self.g_w = _cols(full.g_proj.kernel, h0, nhl, hvd)
        self.b_w, self.b_b = _cols(full.b_proj.kernel, h0, nhl, 1), _cols(full.b_proj.bias, h0, nhl, 1)
        gper = hd if full.use_kda else 1
        self.gk_w, self.gk_b = _cols(full.gk_proj.kernel, h0, nhl, gper), _cols(full.gk_proj.bias, h0, nhl, gper)
        if full.use_conv:
            self.qc_w, self.qc_b = _cols(full.q_conv.kernel, h0, nhl, hd), _cols(full.q_conv.bias, h0, nhl, hd)
            self.kc_w, self.kc_b = _cols(full.k_conv.kernel, h0, nhl, hd), _cols(full.k_conv.bias, h0, nhl, hd)
            self.vc_w, self.vc_b = _cols(full.v_conv.kernel, h0, nhl, hvd), _cols(full.v_conv.bias, h0, nhl, hvd)
        self.out_norm_scale = nn.Parameter(full.out_norm.scale.detach().clone())   # replicated, per-head norm
        self.out_norm_eps = full.out_norm.eps
        self.o_w = _cols(full.o_proj.kernel, h0, nhl, hvd, dim=0)                  # row-parallel
        self.D = nn.Parameter(full.D.detach().clone())                              # replicated

    _FULL = (("q_w", "q_proj.kernel", -1), ("k_w", "k_proj.kernel", -1), ("v_w", "v_proj.kernel", -1),
             ("g_w", "g_proj.kernel", -1), ("b_w", "b_proj.kernel", -1), ("b_b", "b_proj.bias", 0),
             ("gk_w", "gk_proj.kernel", -1), ("gk_b", "gk_proj.bias", 0), ("o_w", "o_proj.kernel", 0),
             ("out_norm_scale", "out_norm.scale", None), ("D", "D", None))
    _FULL_CONV = (("qc_w", "q_conv.kernel", -1), ("qc_b", "q_conv.bias", 0), ("kc_w", "k_conv.kernel", -1),
                  ("kc_b", "k_conv.bias", 0), ("vc_w", "v_conv.kernel", -1), ("vc_b", "v_conv.bias", 0))

    def _full_table(self) -> tuple:
        return self._FULL + (self._FULL_CONV if self.use_conv else ())

    def _out_weight(self):
        return self.o_w

    def _inputs(self, xin, bufs=None):
        B, L, _ = xin.shape
        nh, hd, hvd = self.nhl, self.hd, self.hvd
        q, k, v = xin @ self.q_w, xin @ self.k_w, xin @ self.v_w
        new_bufs = None
        if self.use_conv:
            if bufs is None:
                q, k, v = (F.silu(_dconv(t, w, b)) for t, w, b in
                           ((q, self.qc_w, self.qc_b), (k, self.kc_w, self.kc_b), (v, self.vc_w, self.vc_b)))
            else:
                outs, new_bufs = [], []
                for buf, t, w, b in ((bufs[0], q, self.qc_w, self.qc_b), (bufs[1], k, self.kc_w, self.kc_b),
                                     (bufs[2], v, self.vc_w, self.vc_b)):
                    xc = torch.cat([buf, t], dim=1)
                    new_bufs.append(xc[:, -(w.shape[0] - 1):])
                    outs.append(F.silu(_dconv(xc, w, b)[:, -L:]))
                q, k, v = outs
                new_bufs = tuple(new_bufs)
        q = l2_normalize(q.reshape(B, L, nh, hd)) * hd ** -0.5
        k = l2_normalize(k.reshape(B, L, nh, hd))
        v = v.reshape(B, L, nh, hvd)
        beta = torch.sigmoid(xin @ self.b_w + self.b_b)
        alog = F.logsigmoid(xin @ self.gk_w + self.gk_b).reshape(B, L, nh, hd if self.use_kda else 1)
        g = F.silu(xin @ self.g_w).reshape(B, L, nh, hvd)
        return q, k, v, beta, alog, g, new_bufs

    def _out(self, x, o, g):
        B, L = o.shape[:2]
        scale = copy_to_tp(self.out_norm_scale, self.group)
        of = o.float()
        o = of * torch.rsqrt((of * of).mean(-1, keepdim=True) + self.out_norm_eps) * scale * g
        return self._reduce(o.reshape(B, L, self.nhl * self.hvd), self.o_w, self.group) + x * self.D

    def forward(self, x):
        xin = copy_to_tp(x, self.group)
        q, k, v, beta, alog, g, _ = self._inputs(xin)
        o, _ = gated_delta_chunked(q, k, v, beta, alog, self.chunk)
        return self._out(x, o, g)

    def initial_state(self, batch, device=None):
        S = torch.zeros(batch, self.nhl, self.hvd, self.hd, device=device)
        if not self.use_conv:
            return S
        z = lambda c: torch.zeros(batch, 3, c, device=device)
        return (S, (z(self.nhl * self.hd), z(self.nhl * self.hd), z(self.nhl * self.hvd)))

    def step(self, state, x):
        S, bufs = (state if self.use_conv else (state, None))
        q, k, v, beta, alog, g, nb = self._inputs(x, bufs)
        o, S = gated_delta_recurrent(q, k, v, beta, alog, S)
        out = self._out(x, o, g)
        return ((S, nb) if self.use_conv else S), out


class TransformerBlockTP(nn.Module, _RowParallel):
    """Attention heads and FFN width split over the group; norms, position encoding and
    output biases replicated (biases added once after each reduction)."""
    is_transformer = True

    def __init__(self, full: TransformerBlock, group=None):
        super().__init__()
        self.group = group
        T, r = dist.get_world_size(group), dist.get_rank(group)
        self.nhl, self.h0 = _split(T, r, full.nh, "attention heads")
        self.fl, self.f0 = _split(T, r, full.d_ff, "FFN columns")
        nhl, h0 = self.nhl, self.h0
        self.H, self.hd, self.use_pe = full.H, full.hd, full.use_pe
        self.compute_dtype = full.compute_dtype
        a = full.attn
        self.wq, self.bq = _cols(a.query.kernel, h0, nhl, 1, dim=1), _cols(a.query.bias, h0, nhl, 1, dim=0)
        self.wk, self.bk = _cols(a.key.kernel, h0, nhl, 1, dim=1), _cols(a.key.bias, h0, nhl, 1, dim=0)
        self.wv, self.bv = _cols(a.value.kernel, h0, nhl, 1, dim=1), _cols(a.value.bias, h0, nhl, 1, dim=0)
        self.wo = nn.Parameter(a.out.kernel.detach()[h0:h0 + nhl].reshape(nhl * self.hd, self.H).clone())
        self.bo = nn.Parameter(a.out.bias.detach().clone())
        self.norm1, self.norm2 = full.norm1, full.norm2            # replicated
        self.w1, self.b1 = _cols(full.ff.layers_0.kernel, self.f0, self.fl, 1), _cols(full.ff.layers_0.bias, self.f0,
                                                                                     self.fl, 1)
        self.w2 = _cols(full.ff.layers_2.kernel, self.f0, self.fl, 1, dim=0)
        self.b2 = nn.Parameter(full.ff.layers_2.bias.detach().clone())

    _FULL = (("wq", "attn.query.kernel", 1), ("bq", "attn.query.bias", 0), ("wk", "attn.key.kernel", 1),
             ("bk", "attn.key.bias", 0), ("wv", "attn.value.kernel", 1), ("bv", "attn.value.bias", 0),
             ("wo", "attn.out.kernel", 0), ("bo", "attn.out.bias", None), ("norm1.scale", "norm1.scale", None),
             ("norm1.bias", "norm1.bias", None), ("norm2.scale", "norm2.scale", None), ("norm2.bias", "norm2.bias", None),
             ("w1", "ff.layers_0.kernel", -1), ("b1", "ff.layers_0.bias", 0), ("w2", "ff.layers_2.kernel", 0),
             ("b2", "ff.layers_2.bias", None))

    def full_state_dict(self) -> dict:
        out = super().full_state_dict()
        out["attn.out.kernel"] = out["attn.out.kernel"].reshape(-1, self.hd, self.H)     # (nh, hd, H)
        return out

    def _out_weight(self):
        return self.wo

    def forward(self, x):
        B, L, H = x.shape
        cd = self.compute_dtype
        if self.use_pe:
            x = x + sinusoidal(L, H, x.device)
        h = copy_to_tp(self.norm1(x), self.group).to(cd)
        proj = lambda w, b: torch.einsum("...d,dnk->...nk", h, w.to(cd)) + b.to(cd)
        q, k, v = proj(self.wq, self.bq), proj(self.wk, self.bk), proj(self.wv, self.bv)
        o = causal_attention(q, k, v)
        x = x + (self._reduce(o.reshape(B, L, -1), self.wo.to(cd), self.group) + self.bo.to(cd)).float()
        h2 = copy_to_tp(self.norm2(x), self.group).to(cd)
        f = gelu_tanh(h2 @ self.w1.to(cd) + self.b1.to(cd))
        return x + (reduce_from_tp(f @ self.w2.to(cd), self.group) + self.b2.to(cd)).float()


class NSABlockTP(nn.Module, _RowParallel):
    """NSA heads and FFN width split over the group.  The three branches are per head,
    except the block selection: it ranks blocks by importance summed over all heads, so each
    rank's per-head sum is summed over the group before the top-k (the current block's
    importance and the masked entries are then reset to their constants, as in the
    single-device block), and every rank selects the same blocks."""
    is_transformer = True

    def __init__(self, full: NSABlock, group=None):
        super().__init__()
        # the full block lends its branch methods and configuration; it is not registered as
        # a submodule, so its unsliced weights stay out of this module's parameters
        self.__dict__["inner"] = full
        self.group = group
        T, r = dist.get_world_size(group), dist.get_rank(group)
        self.nhl, self.h0 = _split(T, r, full.nh, "NSA heads")
        self.fl, self.f0 = _split(T, r, full.ff.layers_0.kernel.shape[1], "FFN columns")
        nhl, h0, hd = self.nhl, self.h0, full.hd
        self.wq = _cols(full.q_proj.kernel, h0, nhl, hd)
        self.wk = _cols(full.k_proj.kernel, h0, nhl, hd)
        self.wv = _cols(full.v_proj.kernel, h0, nhl, hd)
        self.wg = _cols(full.g_proj.kernel, h0, nhl, 3)
        self.wo = _cols(full.o_proj.kernel, h0, nhl, hd, dim=0)                        # row-parallel
        self.w1, self.b1 = _cols(full.ff.layers_0.kernel, self.f0, self.fl, 1), _cols(full.ff.layers_0.bias, self.f0,
                                                                                     self.fl, 1)
        self.w2 = _cols(full.ff.layers_2.kernel, self.f0, self.fl, 1, dim=0)
        self.b2 = nn.Parameter(full.ff.layers_2.bias.detach().clone())
        self.norm1, self.norm2 = full.norm1, full.norm2                                # replicated

    _FULL = (("wq", "q_proj.kernel", -1), ("wk", "k_proj.kernel", -1), ("wv", "v_proj.kernel", -1),
             ("wg", "g_proj.kernel", -1), ("wo", "o_proj.kernel", 0), ("norm1.scale", "norm1.scale", None),
             ("norm1.bias", "norm1.bias", None), ("norm2.scale", "norm2.scale", None), ("norm2.bias", "norm2.bias", None),
             ("w1", "ff.layers_0.kernel", -1), ("b1", "ff.layers_0.bias", 0), ("w2", "ff.layers_2.kernel", 0),
             ("b2", "ff.layers_2.bias", None))

    def _out_weight(self):
        return self.wo

    def forward(self, x):
        m, grp = self.inner, self.group
        B, L, H = x.shape
        cd = m.compute_dtype
        if m.pe != "rope":
            x = x + sinusoidal(L, H, x.device)
        h = copy_to_tp(self.norm1(x), grp).to(cd)
        q = (h @ self.wq.to(cd)).reshape(B, L, self.nhl, m.hd)
        k = (h @ self.wk.to(cd)).reshape(B, L, self.nhl, m.hd)
        v = (h @ self.wv.to(cd)).reshape(B, L, self.nhl, m.hd)
        if m.pe == "rope":
            cos, sin = rotary_embedding(m.hd, L, m.rope_base, x.device)
            q, k = apply_rope(q, k, cos, sin)
        g = torch.sigmoid((h @ self.wg.to(cd)).float()).reshape(B, L, self.nhl, 3)
        scale = m.hd ** -0.5
        o_cmp, imp = m._compressed(q, k, v, scale)
        with torch.no_grad():                                  # selection only: no gradient
            imp = imp.detach().clone()
            dist.all_reduce(imp, group=grp)
            BS, nb = m.block_size, imp.shape[-1]
            t = torch.arange(L, device=x.device)
            cmask = torch.arange(nb, device=x.device)[None, :] < torch.clamp((t - BS + 1) // BS + 1, min=0)[:, None]
            cur = (t // BS)[:, None] == torch.arange(nb, device=x.device)[None, :]
            imp = torch.where(cur[None], torch.ones_like(imp), imp).masked_fill(~cmask[None], -1e9)
        o_slc = m._select(q, k, v, imp, scale)
        o_win = causal_attention(q, k, v, scale=scale, window=m.window)
        o = g[..., 0:1] * o_cmp.float() + g[..., 1:2] * o_slc.float() + g[..., 2:3] * o_win.float()
        x = x + self._reduce(o.reshape(B, L, -1).to(cd), self.wo.to(cd), grp).float()
        h2 = copy_to_tp(self.norm2(x), grp).to(cd)
        f = gelu_tanh(h2 @ self.w1.to(cd) + self.b1.to(cd))
        return x + (reduce_from_tp(f @ self.w2.to(cd), grp) + self.b2.to(cd)).float()


def shard_heads(model: nn.Module, group=None) -> nn.Module:
    """Replace every ``GDN`` mixer, ``TransformerBlock`` and ``NSABlock`` of a model by its
    slice.  A GDN mixer whose head count does not divide over the group (the narrow book
    layers) stays whole and replicated: every rank computes it on the same input."""
    T = dist.get_world_size(group)
    for _, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, GDN) and child.nh % T:
                continue
            if isinstance(child, GDN):
                setattr(mod, cname, GDNTP(child, group))
            elif isinstance(child, NSABlock):
                setattr(mod, cname, NSABlockTP(child, group))
            elif isinstance(child, TransformerBlock):
                setattr(mod, cname, TransformerBlockTP(child, group))
    return model
