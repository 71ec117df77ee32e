"""Fully sharded data parallelism (ZeRO-3) for the projection kernels of the Mamba3 layers.

BASELINE's 350m recipe trains data-parallel with parameters sharded across the ranks; the
reference shards with XLA's FSDP-style shardings over the ``data`` mesh axis
(``src/base_model/sharding/sharding_utils.py:21-98``, the train step's gradient reduction at
``src/base_model/training/train_helpers.py:1395-1462,2123-2196``).  Here the unit of sharding
is one fused sequence layer (``ops.mamba3_layer`` ``_LayerFn``) and its three projection
kernels (in_proj, out_proj, the GLU gate): 99% of the model's parameters.

At rest a rank holds, for every layer, only its ``1/world`` slice of the layer's flattened
kernels: the fp32 master, the Adam moments, the accumulated gradient and the bf16 compute
copy.  The kernels' own ``Parameter`` objects keep their shapes but no storage of their own.

* forward of layer i: its bf16 kernels are all-gathered into one of two ping-pong buffers
  (prefetched on a side stream while layer i-1 computes; the buffer is reused two layers
  later, after the compute stream has passed the layer that read it);
* backward of layer i: the kernels are gathered again (the buffer of the layer just run is
  reused without a collective), the weight-gradient GEMMs reduce-add straight into a
  full-size fp32 gradient buffer of the layer, and right after the layer's backward that
  buffer is reduce-scattered on the side stream into the layer's gradient shard, overlapping
  the backward of layer i-1;
* the optimizer step is AdamW on the shards (the package's fused kernel, which also writes
  the bf16 shard the next step gathers), with the global gradient norm summed over shards.

The small parameters (biases, norms, the SSM vectors, embeddings, encoders and the decoder)
stay replicated under the ordinary flat optimizer and its all-reduce.  Collectives are
NCCL (``torch.distributed``); every rank issues them in the same order.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..ops import weights as W

ALIGN = 128


def fsdp_layers(model) -> List:
    """The sequence layers that run as one fused unit (CUDA Mamba3 ``half_glu1`` layers)."""
    from ..models.layers import SequenceLayer
    from ..models.mamba3 import Mamba3
    out = []
    for mod in model.modules():
        if isinstance(mod, SequenceLayer) and isinstance(mod.seq, Mamba3) and mod.seq.impl == "cuda" \
                and mod.prenorm and mod.activation == "half_glu1" and mod.dropout == 0.0 and mod.d_model % 8 == 0:
            out.append(mod)
    return out


def _kernels(layer) -> List[torch.nn.Parameter]:
    return [layer.seq.in_proj.kernel, layer.seq.out_proj.kernel, layer.out2.kernel]


class _Unit:
    def __init__(self, idx: int, layer, world: int, rank: int, device):
        self.idx, self.layer = idx, layer
        self.params = _kernels(layer)
        self.offsets = []
        off = 0
        for p in self.params:
            self.offsets.append(off)
            off += p.numel()
        self.numel = off
        q = world * ALIGN
        self.padded = -(-off // q) * q
        self.shard = self.padded // world
        lo = rank * self.shard
        full = torch.zeros(self.padded, dtype=torch.float32, device=device)
        for p, o in zip(self.params, self.offsets):
            full[o:o + p.numel()].copy_(p.detach().reshape(-1))
        self.master = full[lo:lo + self.shard].clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad = torch.zeros_like(self.master)
        self.bf16 = self.master.to(torch.bfloat16)
        del full


class FSDP:
    """ZeRO-3 over ``fsdp_layers(model)``; see the module docstring."""

    def __init__(self, model, world: int, rank: int, group=None, lr: float = 1e-3, weight_decay: float = 0.05,
                 betas=(0.9, 0.999), eps: float = 1e-8, wire_bf16: bool = False):
        self.world, self.rank, self.group = world, rank, group
        self.b1, self.b2 = betas
        self.eps, self.wd, self.base_lr = eps, weight_decay, lr
        self.wire_bf16 = wire_bf16
        layers = fsdp_layers(model)
        if not layers:
            raise ValueError("no fused CUDA Mamba3 layers to shard")
        dev = _kernels(layers[0])[0].device
        self.device = dev
        self.units = [_Unit(i, l, world, rank, dev) for i, l in enumerate(layers)]
        self.by_layer = {id(u.layer): u for u in self.units}
        big = max(u.padded for u in self.units)
        self.gbuf = [torch.empty(big, dtype=torch.bfloat16, device=dev) for _ in range(2)]   # gathered kernels
        self.gradbuf = [torch.zeros(big, dtype=torch.float32, device=dev) for _ in range(2)]  # full-size grads
        self.resident: List[Optional[int]] = [None, None]       # unit whose kernels each buffer holds
        cuda = dev.type == "cuda"
        self.stream = torch.cuda.Stream(device=dev) if cuda else None
        self.gather_ev: Dict[int, object] = {}
        self.rs_ev: List[Optional[object]] = [None, None]
        self.step_count = 0
        self._lr = torch.zeros(1, dtype=torch.float32, device=dev)
        for u in self.units:
            for p in u.params:
                # the Parameter keeps its shape, not its storage: a broadcast zero of the same shape
                p.data = torch.zeros((), dtype=p.dtype, device=dev).expand(p.shape)
                p.grad = None
                p._s0_flat_grad = True
            u.layer._s0_fsdp = self

    # ---- parameters of every unit ------------------------------------------------------------
    def sharded_parameters(self) -> List[torch.nn.Parameter]:
        return [p for u in self.units for p in u.params]

    def _views(self, u: _Unit, buf: torch.Tensor, dtype_buf=None) -> List[torch.Tensor]:
        return [buf[o:o + p.numel()].view(p.shape) for p, o in zip(u.params, u.offsets)]

    # ---- collectives (on the side stream on CUDA) -----------------------------------------------
    def _side(self):
        return torch.cuda.stream(self.stream) if self.stream is not None else _Null()

    def _gather(self, u: _Unit, b: int) -> None:
        """All-gather unit u's bf16 kernels into buffer b (ordered after the compute stream's
        current position: the kernels that last read buffer b have been enqueued before)."""
        if self.resident[b] == u.idx:
            return
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with self._side():
            dist.all_gather_into_tensor(self.gbuf[b][:u.padded], u.bf16, group=self.group)
            if self.stream is not None:
                ev = torch.cuda.Event()
                ev.record(self.stream)
                self.gather_ev[u.idx] = ev
        self.resident[b] = u.idx

    def _use(self, u: _Unit, b: int) -> None:
        ev = self.gather_ev.pop(u.idx, None)
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
        for p, view in zip(u.params, self._views(u, self.gbuf[b])):
            W.register(p, view)

    # ---- hooks called by the fused layer -------------------------------------------------------
    def before_forward(self, layer) -> None:
        u = self.by_layer[id(layer)]
        b = u.idx % 2
        self._gather(u, b)
        self._use(u, b)
        if u.idx + 1 < len(self.units):                       # prefetch the next layer
            self._gather(self.units[u.idx + 1], (u.idx + 1) % 2)

    def before_backward(self, layer) -> None:
        u = self.by_layer[id(layer)]
        b = u.idx % 2
        self._gather(u, b)
        self._use(u, b)
        if u.idx > 0:                                          # prefetch the previous layer
            self._gather(self.units[u.idx - 1], (u.idx - 1) % 2)
        ev = self.rs_ev[b]                                     # gradient buffer b is free again
        if ev is not None:
            torch.cuda.current_stream(self.device).wait_event(ev)
        g = self.gradbuf[b][:u.padded]
        g.zero_()
        for p, view in zip(u.params, self._views(u, g)):
            p.grad = view

    def after_backward(self, layer) -> None:
        u = self.by_layer[id(layer)]
        b = u.idx % 2
        g = self.gradbuf[b][:u.padded]
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with self._side():
            if self.wire_bf16:
                gs = torch.empty(u.shard, dtype=torch.bfloat16, device=self.device)
                dist.reduce_scatter_tensor(gs, g.to(torch.bfloat16), group=self.group)
                u.grad.add_(gs.float())
            else:
                gs = torch.empty(u.shard, dtype=torch.float32, device=self.device)
                dist.reduce_scatter_tensor(gs, g, group=self.group)
                u.grad.add_(gs)
            if self.stream is not None:
                ev = torch.cuda.Event()
                ev.record(self.stream)
                self.rs_ev[b] = ev
        for p in u.params:
            p.grad = None

    # ---- optimizer -------------------------------------------------------------------------------
    def zero_grad(self) -> None:
        for u in self.units:
            u.grad.zero_()

    def sync(self) -> None:
        """The compute stream waits for every collective issued so far."""
        if self.stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def grad_sumsq(self) -> torch.Tensor:
        """Sum of squares of the averaged sharded gradients over all ranks (a device scalar)."""
        s = torch.zeros(1, dtype=torch.float32, device=self.device)
        for u in self.units:
            s += (u.grad.float() / self.world).pow(2).sum()
        dist.all_reduce(s, group=self.group)
        return s

    def step(self, lr_scale: float, grad_sumsq: torch.Tensor, max_grad_norm: float) -> None:
        """AdamW on every shard; the gradients are sums over ranks (divided by world here);
        ``grad_sumsq`` is the global sum of squares of the averaged gradient (clipping)."""
        self.step_count += 1
        t = self.step_count
        bc1, bc2 = 1 - self.b1 ** t, 1 - self.b2 ** t
        lr = self.base_lr * lr_scale
        for u in self.units:
            u.grad.div_(self.world)
        if self.device.type == "cuda":
            from ..ops._ext import ext
            C = ext()
            self._lr.fill_(lr)
            for u in self.units:
                C.adam(u.master, u.grad, u.m, u.v, u.bf16, grad_sumsq, max_grad_norm, self._lr, self.b1, self.b2,
                       self.eps, self.wd, bc1, bc2)
        else:
            import math
            nrm = math.sqrt(float(grad_sumsq))
            scale = 1.0 if (max_grad_norm <= 0 or nrm < max_grad_norm) else max_grad_norm / nrm
            for u in self.units:
                g = u.grad * scale
                u.m.mul_(self.b1).add_(g, alpha=1 - self.b1)
                u.v.mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
                u.master.sub_(lr * ((u.m / bc1) / ((u.v / bc2).sqrt() + self.eps) + self.wd * u.master))
                u.bf16.copy_(u.master)
        self.resident = [None, None]          # the gathered copies are stale now

    # ---- full parameters (checkpoints, tests) ----------------------------------------------------
    def full_parameters(self) -> Dict[torch.nn.Parameter, torch.Tensor]:
        """Every sharded kernel as a full fp32 tensor (all ranks take part)."""
        out = {}
        for u in self.units:
            full = torch.empty(u.padded, dtype=torch.float32, device=self.device)
            dist.all_gather_into_tensor(full, u.master.contiguous(), group=self.group)
            for p, o in zip(u.params, u.offsets):
                out[p] = full[o:o + p.numel()].view(p.shape).clone()
        return out

    def load_full_parameters(self, full: Dict[torch.nn.Parameter, torch.Tensor]) -> None:
        for u in self.units:
            buf = torch.zeros(u.padded, dtype=torch.float32, device=self.device)
            for p, o in zip(u.params, u.offsets):
                buf[o:o + p.numel()].copy_(full[p].reshape(-1))
            lo = self.rank * u.shard
            u.master.copy_(buf[lo:lo + u.shard])
            u.bf16.copy_(u.master)
        self.resident = [None, None]


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
