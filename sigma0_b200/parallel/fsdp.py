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
  later, after the compute stream has passed the layer that read it).  With ``fused_ag``
  in_proj is not gathered by NCCL: the in_proj GEMM itself copies every rank's row block of
  the kernel into the buffer (peer loads from symmetric memory, by otherwise idle lanes of
  its producer warps, each remote byte crossing NVLink once) and starts on this rank's own
  block while the others arrive (``csrc/gemm_tc.cu`` ``ag_copy``);
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
    """One layer's kernels, sharded by row blocks: rank r holds rows [r R / W, (r + 1) R / W) of
    every kernel (R rows each); its shard is those blocks concatenated.  An all-gather per kernel
    then yields the kernel row-major in the gathered buffer, and the first one (in_proj) can be
    gathered by the GEMM itself (``gemm_ag``)."""

    def __init__(self, idx: int, layer, world: int, rank: int, device, bf16_shard: Optional[torch.Tensor] = None):
        self.idx, self.layer = idx, layer
        self.params = _kernels(layer)
        for p in self.params:
            if p.shape[0] % world:
                raise ValueError(f"kernel rows {p.shape[0]} do not split over {world} ranks")
        self.offsets, self.soffsets = [], []           # full-buffer and shard offsets per kernel
        off = soff = 0
        for p in self.params:
            self.offsets.append(off)
            self.soffsets.append(soff)
            off += p.numel()
            soff += p.numel() // world
        self.numel = off
        self.padded = -(-off // ALIGN) * ALIGN
        self.shard = soff
        self.master = torch.empty(soff, dtype=torch.float32, device=device)
        for p, so in zip(self.params, self.soffsets):
            rows = p.shape[0] // world
            self.master[so:so + rows * p.shape[1]].copy_(p.detach()[rank * rows:(rank + 1) * rows].reshape(-1))
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.grad = torch.zeros_like(self.master)
        self.bf16 = bf16_shard if bf16_shard is not None else torch.empty(soff, dtype=torch.bfloat16, device=device)
        self.bf16.copy_(self.master)

    def block(self, k: int, world: int) -> int:
        """Elements of kernel k in one rank's block."""
        return self.params[k].numel() // world


class FSDP:
    """ZeRO-3 over ``fsdp_layers(model)``; see the module docstring."""

    SPIN_LIMIT = 20_000_000        # polls (~100 ns): a peer missing for ~2 s makes the fused gather fail

    def __init__(self, model, world: int, rank: int, group=None, lr: float = 1e-3, weight_decay: float = 0.05,
                 betas=(0.9, 0.999), eps: float = 1e-8, wire_bf16: bool = False, fused_ag: bool = False):
        self.world, self.rank, self.group = world, rank, group
        self.b1, self.b2 = betas
        self.eps, self.wd, self.base_lr = eps, weight_decay, lr
        self.wire_bf16 = wire_bf16
        layers = fsdp_layers(model)
        if not layers:
            raise ValueError("no fused CUDA Mamba3 layers to shard")
        dev = _kernels(layers[0])[0].device
        self.device = dev
        self.fused_ag = bool(fused_ag) and dev.type == "cuda" and 2 <= world <= 8
        shards = [None] * len(layers)
        if self.fused_ag:
            # every unit's bf16 shard in one symmetric (peer-mapped) buffer: the fused in_proj GEMM
            # reads the other ranks' row blocks straight from their memory
            import torch.distributed._symmetric_memory as symm
            sizes = [sum(p.numel() // world for p in _kernels(l)) for l in layers]
            self._symm_bf16 = symm.empty(sum(sizes), dtype=torch.bfloat16, device=dev)
            self._ready = symm.empty(8, dtype=torch.int32, device=dev)
            self._ready.zero_()
            o = 0
            for i, n in enumerate(sizes):
                shards[i] = self._symm_bf16[o:o + n]
                o += n
        self.units = [_Unit(i, l, world, rank, dev, shards[i]) for i, l in enumerate(layers)]
        self.by_layer = {id(u.layer): u for u in self.units}
        big = max(u.padded for u in self.units)
        self.gbuf = [torch.empty(big, dtype=torch.bfloat16, device=dev) for _ in range(2)]   # gathered kernels
        self.gradbuf = [torch.zeros(big, dtype=torch.float32, device=dev) for _ in range(2)]  # full-size grads
        # per buffer: (unit, complete) -- the unit whose kernels it holds, and whether in_proj is
        # among them (the fused mode gathers in_proj inside its GEMM)
        self.resident: List[Optional[tuple]] = [None, None]
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
        if self.fused_ag:
            import torch.distributed._symmetric_memory as symm
            torch.cuda.synchronize(dev)
            g = group if group is not None else dist.group.WORLD
            h = symm.rendezvous(self._symm_bf16, g)
            hr = symm.rendezvous(self._ready, g)
            base = int(h.buffer_ptrs[h.rank])
            self._peer_bf16 = [int(ptr) for ptr in h.buffer_ptrs]
            self._peer_ready = [int(ptr) + 4 * r for r, ptr in enumerate(hr.buffer_ptrs)]
            self._sym_base = base
            self._handles = (h, hr)
            self._counters = torch.zeros(8, dtype=torch.int32, device=dev)
            self._publish()
            dist.barrier(group=group)         # every shard exists before anyone reads a peer's

    # ---- parameters of every unit ------------------------------------------------------------
    def sharded_parameters(self) -> List[torch.nn.Parameter]:
        return [p for u in self.units for p in u.params]

    def _views(self, u: _Unit, buf: torch.Tensor, dtype_buf=None) -> List[torch.Tensor]:
        return [buf[o:o + p.numel()].view(p.shape) for p, o in zip(u.params, u.offsets)]

    # ---- collectives (on the side stream on CUDA) -----------------------------------------------
    def _side(self):
        return torch.cuda.stream(self.stream) if self.stream is not None else _Null()

    def _gather(self, u: _Unit, b: int, skip_first: bool = False) -> None:
        """All-gather unit u's bf16 kernels into buffer b (ordered after the compute stream's
        current position: the kernels that last read buffer b have been enqueued before);
        with ``skip_first`` in_proj is left to the fused GEMM."""
        have = self.resident[b]
        if have is not None and have[0] == u.idx and (have[1] or skip_first):
            return
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with self._side():
            for k in range(1 if skip_first else 0, len(u.params)):
                n, o, so = u.params[k].numel(), u.offsets[k], u.soffsets[k]
                dist.all_gather_into_tensor(self.gbuf[b][o:o + n], u.bf16[so:so + n // self.world], group=self.group)
            if self.stream is not None:
                ev = torch.cuda.Event()
                ev.record(self.stream)
                self.gather_ev[u.idx] = ev
        self.resident[b] = (u.idx, not skip_first)

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
        self._gather(u, b, skip_first=self.fused_ag)
        self._use(u, b)
        if self.fused_ag:
            u.params[0]._s0_ag = lambda x, u=u, b=b: self._fused_in_proj(u, b, x)
        if u.idx + 1 < len(self.units):                       # prefetch the next layer
            self._gather(self.units[u.idx + 1], (u.idx + 1) % 2, skip_first=self.fused_ag)

    def _fused_in_proj(self, u: _Unit, b: int, x: torch.Tensor) -> torch.Tensor:
        """x @ in_proj with in_proj's row blocks gathered by the GEMM (``csrc/gemm_tc.cu``)."""
        from ..ops._ext import ext
        p = u.params[0]
        u.params[0]._s0_ag = None
        wfull = self.gbuf[b][u.offsets[0]:u.offsets[0] + p.numel()].view(p.shape)
        so = u.soffsets[0]
        off = (u.bf16.data_ptr() - self._sym_base) + so * 2        # this unit's in_proj block in the buffer
        src = [ptr + off for ptr in self._peer_bf16]
        y = ext().gemm_ag(x, wfull, src, self._peer_ready[:self.world], self._counters, self.rank,
                          self.step_count + 1, self.SPIN_LIMIT)
        self.resident[b] = (u.idx, True)             # the GEMM left the whole kernel in the buffer
        return y

    def _publish(self) -> None:
        """This rank's shards are current for version step_count + 1 (stream-ordered after the
        update that wrote them)."""
        self._ready[self.rank].fill_(self.step_count + 1)

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
            gs = torch.empty(u.shard, dtype=torch.bfloat16 if self.wire_bf16 else torch.float32, device=self.device)
            for k, p in enumerate(u.params):
                n, o, so = p.numel(), u.offsets[k], u.soffsets[k]
                src = g[o:o + n].to(torch.bfloat16) if self.wire_bf16 else g[o:o + n]
                dist.reduce_scatter_tensor(gs[so:so + n // self.world], src, group=self.group)
            u.grad.add_(gs.float() if self.wire_bf16 else gs)
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
        if self.fused_ag:
            self._publish()
            self._stage_status()

    # ---- errors of the fused gather (bounded waits in the kernel) --------------------------------
    def _stage_status(self) -> None:
        """Copy the GEMM status word to pinned host memory behind this step (no sync); the next
        step reads it."""
        from ..ops._ext import ext
        if not hasattr(self, "_status_host"):
            self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
            self._status_ev = torch.cuda.Event()
        self._check_status()
        self._status_host.copy_(ext().gemm_status(self._counters), non_blocking=True)
        self._status_ev.record()

    def _check_status(self) -> None:
        ev = getattr(self, "_status_ev", None)
        if ev is not None and ev.query() and int(self._status_host[0]) != 0:
            code = int(self._status_host[0])
            raise RuntimeError(f"fused FSDP all-gather: a bounded wait gave up (status {code}: "
                               f"{'a peer shard never became current' if code == 3 else 'pipeline wait'})")

    # ---- full parameters (checkpoints, tests) ----------------------------------------------------
    def full_parameters(self) -> Dict[torch.nn.Parameter, torch.Tensor]:
        """Every sharded kernel as a full fp32 tensor (all ranks take part)."""
        out = {}
        for u in self.units:
            for k, p in enumerate(u.params):
                n, so = p.numel(), u.soffsets[k]
                full = torch.empty(n, dtype=torch.float32, device=self.device)
                dist.all_gather_into_tensor(full, u.master[so:so + n // self.world].contiguous(), group=self.group)
                out[p] = full.view(p.shape)
        return out

    def load_full_parameters(self, full: Dict[torch.nn.Parameter, torch.Tensor]) -> None:
        for u in self.units:
            for k, p in enumerate(u.params):
                rows = p.shape[0] // self.world
                n, so = rows * p.shape[1], u.soffsets[k]
                u.master[so:so + n].copy_(full[p].to(self.device)[self.rank * rows:(self.rank + 1) * rows].reshape(-1))
            u.bf16.copy_(u.master)
        self.resident = [None, None]
        if self.fused_ag:
            self._publish()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
