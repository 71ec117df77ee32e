"""Training step and loop (the public training API).

``Trainer`` builds the model from a preset / argparse namespace, re-homes its
parameters into the flat optimizer buffers, and runs steps:

* ``step_device(tokens, labels, book)`` -- one optimizer step on device tensors,
  returns the loss as a device scalar (no host sync);
* ``train_step(batch)`` -- the end-to-end call a user makes: copies the batch
  from (pinned) host memory, runs the step, returns the loss as a Python float.

Data parallelism: with ``world > 1`` the flat gradient is averaged over ranks
(NCCL all-reduce) before the update -- the reference's ``pmean`` over
``data``/``gpus`` (``training/train_helpers.py:2123-2196``) -- or, with
``sharded=True``, reduce-scattered so each rank updates only its shard of the
flat buffer and the updated parameters are all-gathered (ZeRO-1/2 style).

Context parallelism (``context_parallel=True``, ``world > 1``): every rank receives the
whole batch and keeps one contiguous segment of every sequence (tokens and labels along
the sequence, book rows along the messages; segments start on a message boundary).  The
mixers and attention blocks are wrapped by ``parallel.cp.shard_model_cp``, which carries
the recurrent state (and the attention keys / values) across segment boundaries, so the
segment losses' mean is the full-sequence loss and the data-parallel gradient average
above is its exact gradient.  The returned loss is averaged over the ranks.  The
reference has no training-time context parallelism (its only sequence-parallel code is
the test-time Mamba3 phase split, ``src/base_model/models/mamba3_seqpar.py``).
"""
from __future__ import annotations

import math
import time
from typing import Dict, Optional

import numpy as np
import torch
import torch.distributed as dist

from ..encoding import get_tokenizer, set_token_mode
from ..models.registry import build_model, architecture_from_args, architecture_has_attention
from .optim import FlatAdam, cosine_schedule


class Trainer:
    def __init__(self, args, device: Optional[torch.device] = None, world: int = 1, rank: int = 0,
                 group=None, total_steps: int = 1000, seed: int = 0, sharded: bool = False,
                 accum_steps: int = 1, grad_wire_dtype: str = "float32", dp_impl: str = "nccl",
                 context_parallel: bool = False, tp: int = 1, hierarchical: bool = False,
                 gpus_per_node: Optional[int] = None, fsdp: bool = False, fsdp_fused_ag: bool = False,
                 tp_fused_out: Optional[bool] = None):
        self.args = args
        self.device = device or torch.device("cuda" if torch.cuda.is_available() else "cpu")
        from ..encoding.tok1 import encoding_mode
        set_token_mode(encoding_mode(args.token_mode))
        self.tok = get_tokenizer(encoding_mode(args.token_mode))
        torch.manual_seed(seed)
        self.model = build_model(args).to(self.device)
        arch = architecture_from_args(args)
        attn_only = arch in ("transformer", "nsa")
        if world > 1:
            # identical initial parameters on every rank (broadcast_one_to_all in the reference)
            for p in self.model.parameters():
                dist.broadcast(p.data, 0, group=group)
        # tensor parallelism: a (dp, tp) mesh over the default group; the mixers' heads (and
        # the attention blocks' FFN width) are split over the tp axis, the batch over dp
        self.tp, self.tp_group, tp_slices = 1, None, []
        self.tp_fused: list = []          # TP modules whose out_proj runs the fused GEMM + all-reduce
        if int(tp) > 1:
            if world <= 1 or group is not None or context_parallel:
                raise ValueError("tensor parallelism needs the default process group of >= 2 ranks and no "
                                 "context parallelism")
            from ..parallel.mesh import create_mesh
            from ..parallel.tp import shard_model
            from ..parallel.tp_heads import shard_heads
            if sharded:
                raise ValueError("tensor parallelism keeps replicated moments (no ZeRO sharding)")
            mesh = create_mesh(tp_size=int(tp), per_gpu_processes=True)
            self.mesh, self.tp, self.tp_group = mesh, int(tp), mesh.group("tp")
            shard_heads(shard_model(self.model, self.tp_group), self.tp_group)
            for mod in self.model.modules():
                if hasattr(mod, "tp_sharded_parameters"):
                    tp_slices += mod.tp_sharded_parameters()
            # the row-parallel output projections + their all-reduce as one peer-memory kernel
            # (csrc/tp_fused.cu); default on CUDA, a module whose width the kernel cannot tile
            # keeps GEMM + NCCL
            if tp_fused_out is None:
                tp_fused_out = self.device.type == "cuda"
            if tp_fused_out:
                rows = int(getattr(args, "micro_bsz", 1)) * int(getattr(args, "n_messages", 1)) * \
                    int(getattr(args, "msg_len", 1))
                for mod in self.model.modules():
                    if hasattr(mod, "use_fused_out_proj"):
                        try:
                            mod.use_fused_out_proj(rows)
                            self.tp_fused.append(mod)
                        except ValueError:
                            pass
            dp = mesh.size("dp") if "dp" in mesh.axis_names else 1
            group = mesh.group("dp") if dp > 1 else None
            world, rank = dp, (mesh.coord("dp") if dp > 1 else 0)
            if dp_impl == "fused":
                dp_impl = "nccl"          # the fused sync spans the default group only
        self.world, self.rank, self.group = world, rank, group
        # hierarchical data parallelism: a (nodes, gpus) mesh; the gradient is reduce-scattered
        # inside a node, all-reduced across nodes shard by shard, and all-gathered back
        self.hier = None
        if hierarchical and world > 1 and self.tp == 1:
            if group is not None or context_parallel or sharded or dp_impl == "fused":
                raise ValueError("the hierarchical step runs over the default group with replicated moments")
            from ..parallel.mesh import create_mesh
            mesh = create_mesh(hierarchical=True, gpus_per_node=gpus_per_node, allow_single_node_hierarchical=True)
            self.mesh = mesh
            self.hier = (mesh.group("nodes"), mesh.group("gpus"), mesh.size("gpus"))
        lr_base = float(getattr(args, "ssm_lr_base", 1e-3))
        lr = lr_base * float(getattr(args, "lr_factor", 1.0))
        # ZeRO-3 over the fused layers' projection kernels (parallel/fsdp.py); the rest of the
        # parameters stay replicated under the flat optimizer below
        self.fsdp = None
        if fsdp and world > 1:
            if self.tp > 1 or context_parallel or sharded or self.hier is not None or dp_impl == "fused" or \
                    accum_steps < 1:
                raise ValueError("FSDP runs plain data parallelism over the default group")
            if str(getattr(args, "opt_config", "standard")) == "muon":
                raise ValueError("FSDP shards the AdamW state of the kernels; Muon is not supported with it")
            from ..parallel.fsdp import FSDP
            self.fsdp = FSDP(self.model, world, rank, group, lr=lr,
                             weight_decay=float(getattr(args, "weight_decay", 0.05)),
                             wire_bf16=grad_wire_dtype == "bfloat16", fused_ag=fsdp_fused_ag)
        opt_cls = FlatAdam
        extra_opt = {}
        if str(getattr(args, "opt_config", "standard")) == "muon":
            from .muon import FlatMuon
            opt_cls = FlatMuon
            mwd = getattr(args, "muon_wd", None)
            extra_opt = dict(muon_lr=float(getattr(args, "muon_lr", 0.02)),
                             muon_wd=None if mwd is None else float(mwd))
        self.opt = opt_cls(self.model, lr=lr, ssm_lr=lr_base, **extra_opt,
                            weight_decay=float(getattr(args, "weight_decay", 0.05)),
                            max_grad_norm=float(getattr(args, "max_grad_norm", 1.0)),
                            opt_config=str(getattr(args, "opt_config", "standard")),
                            attention_model=attn_only,
                            pad_multiple=128 * (world if ((sharded or dp_impl == "fused" or hierarchical)
                                                          and world > 1) else 1),
                            alloc=self._alloc(dp_impl, world), last=tp_slices,
                            dt_global=bool(getattr(args, "dt_global", False)),
                            exclude=self.fsdp.sharded_parameters() if self.fsdp is not None else ())
        self.total_steps = total_steps
        self.warmup_steps = int(round(float(getattr(args, "warmup_end", 0.01)) * total_steps))
        lr_min = float(getattr(args, "lr_min", 0.0) or 0.0)
        self.lr_min_frac = (lr_min / lr) if lr_min > 0 else 0.05
        # cosine decay after the warmup (the reference's cosine_anneal), else a constant lr;
        # lr_mult is the reduce-on-plateau factor the loop lowers (lr_patience / reduce_factor)
        self.cosine = bool(getattr(args, "cosine_anneal", True))
        self.lr_mult = 1.0
        self.ignore_times = bool(getattr(args, "ignore_times", False))
        if dp_impl not in ("nccl", "fused"):
            raise ValueError(f"dp_impl must be 'nccl' or 'fused', not {dp_impl!r}")
        self.fused = None
        self.sharded = (sharded or dp_impl == "fused") and world > 1
        if self.sharded:
            self.opt.shard(world, rank)
            self._gshard = torch.empty(self.opt.hi - self.opt.lo, dtype=torch.float32, device=self.device)
        if grad_wire_dtype not in ("float32", "bfloat16"):
            raise ValueError(f"grad_wire_dtype must be float32 or bfloat16, not {grad_wire_dtype!r}")
        self.wire_bf16 = grad_wire_dtype == "bfloat16"
        if dp_impl == "fused" and world > 1:
            from ..parallel.fused_dp import FusedDPSync
            self.fused = FusedDPSync(self.opt, group)
        self.cp = bool(context_parallel) and world > 1
        if self.cp:
            from ..parallel.cp import shard_model_cp
            shard_model_cp(self.model, group)   # the wrappers share the re-homed parameters
        self.accum_steps = max(1, int(accum_steps))
        self.global_batch = int(getattr(args, "micro_bsz", 1)) * (1 if self.cp else world)
        self.step_idx = 0
        self._sumsq_all = torch.zeros(1, device=self.device)

    def _alloc(self, dp_impl, world):
        if dp_impl == "fused" and world > 1 and self.device.type == "cuda":
            from ..parallel.fused_dp import symmetric_alloc
            return symmetric_alloc()
        return None

    # -- one step -------------------------------------------------------------------------
    def _update(self, lr_scale: float):
        """Gradient reduction over ranks + optimizer update.

        * one rank: plain update;
        * replicated DP: all-reduce of the flat gradient (the reference's pmean,
          ``training/train_helpers.py:2123-2196``), optionally on a bf16 wire
          (``GRAD_ALLREDUCE_DTYPE=bfloat16``, ``:2045-2066``);
        * sharded DP (ZeRO-1/2): reduce-scatter so each rank gets the summed
          gradient of its shard, global-norm from the shards' sums of squares,
          Adam on the shard, then all-gather of the updated parameters."""
        opt = self.opt
        if self.tp > 1:
            self._update_tp(lr_scale)
            return
        if self.hier is not None:
            self._update_hier(lr_scale)
            return
        if self.fsdp is not None:
            self._update_fsdp(lr_scale)
            return
        if self.world == 1:
            opt.step(lr_scale=lr_scale)
            return
        g = opt.grad
        if not self.sharded:
            if self.wire_bf16:
                gb = g.to(torch.bfloat16)
                dist.all_reduce(gb, group=self.group)
                g.copy_(gb)
                g.div_(self.world)
            else:
                g.div_(self.world)
                dist.all_reduce(g, group=self.group)
            opt.step(lr_scale=lr_scale)
            return
        if self.fused is not None:
            self.fused.step(lr_scale)
            return
        gs = self._gshard
        if self.wire_bf16:
            out = torch.empty(gs.numel(), dtype=torch.bfloat16, device=self.device)
            dist.reduce_scatter_tensor(out, g.to(torch.bfloat16), group=self.group)
            gs.copy_(out)
        else:
            dist.reduce_scatter_tensor(gs, g, group=self.group)
        gs.div_(self.world)
        ss = self._sumsq_all
        if gs.is_cuda:
            from ..ops._ext import ext
            ss.zero_()
            ext().sumsq(gs, ss)
        else:
            ss.copy_((gs * gs).sum().reshape(1))
        dist.all_reduce(ss, group=self.group)
        opt.step_shard(gs, ss, lr_scale=lr_scale)
        dist.all_gather_into_tensor(opt.flat, opt.flat[opt.lo:opt.hi].clone(), group=self.group)
        opt.refresh_shadow()

    def _update_fsdp(self, lr_scale: float):
        """Replicated parameters: all-reduce and the flat AdamW; sharded kernels: their
        gradient shards (reduce-scattered during the backward) and the sharded AdamW; one global
        gradient norm over both for clipping."""
        fs = self.fsdp
        fs.sync()
        g = self.opt.grad
        if self.wire_bf16:
            gb = g.to(torch.bfloat16)
            dist.all_reduce(gb, group=self.group)
            g.copy_(gb)
        else:
            dist.all_reduce(g, group=self.group)
        g.div_(self.world)
        total = fs.grad_sumsq() + (g * g).sum().reshape(1)
        self.opt.step(lr_scale=lr_scale, grad_sumsq=total)
        fs.step(lr_scale, total, self.opt.max_grad_norm)

    def _update_hier(self, lr_scale: float):
        """Two-level gradient average (the reference's hierarchical step,
        ``training/train_helpers.py:2069-2200``): reduce-scatter over the GPUs of a node,
        all-reduce of each shard over the nodes (bf16 on the wire with
        ``grad_wire_dtype="bfloat16"``), all-gather inside the node, then the update."""
        nodes_g, gpus_g, gpn = self.hier
        g = self.opt.grad
        shard = torch.empty(g.numel() // gpn, dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(shard, g, group=gpus_g)
        if self.wire_bf16:
            sb = shard.to(torch.bfloat16)
            dist.all_reduce(sb, group=nodes_g)
            shard.copy_(sb)
        else:
            dist.all_reduce(shard, group=nodes_g)
        shard.div_(self.world)
        dist.all_gather_into_tensor(g, shard, group=gpus_g)
        self.opt.step(lr_scale=lr_scale)

    def _update_tp(self, lr_scale: float):
        """Tensor parallel: average over the dp axis, then the global gradient norm -- each
        rank's head slices summed over the tp axis, the replicated parameters (identical
        gradients on every tp rank) counted once -- and the update."""
        opt = self.opt
        g = opt.grad
        if self.world > 1:
            g.div_(self.world)
            dist.all_reduce(g, group=self.group)
        parts = torch.zeros(2, dtype=torch.float32, device=g.device)   # (slices, everything)
        if g.is_cuda:
            from ..ops._ext import ext
            C = ext()
            for lo, hi in opt.late_ranges:
                C.sumsq(g[lo:hi], parts[0:1])
            C.sumsq(g, parts[1:2])
        else:
            for lo, hi in opt.late_ranges:
                parts[0] += (g[lo:hi] * g[lo:hi]).sum()
            parts[1] = (g * g).sum()
        rep = parts[1:2] - parts[0:1]
        sl = parts[0:1].clone()
        dist.all_reduce(sl, group=self.tp_group)
        opt.step(lr_scale=lr_scale, grad_sumsq=sl + rep)

    def step_device(self, tokens, labels, book=None):
        """One optimizer step on device tensors; with ``accum_steps > 1`` the batch is
        split into micro-batches whose gradients accumulate before the update."""
        self.opt.zero_grad()
        if self.fsdp is not None:
            self.fsdp.zero_grad()
        if self.cp:
            tokens, labels, book = self._segment(tokens, labels, book)
        k = self.accum_steps
        if k == 1:
            loss, ce_pos = self.model.loss(tokens, book, labels, ignore_times=self.ignore_times, tokenizer=self.tok)
            loss.backward()
            total = loss.detach()
            self.last_ce_pos = ce_pos.detach()
        else:
            total = torch.zeros((), device=tokens.device)
            ce_sum = None
            for tc, lc, bc in zip(tokens.chunk(k), labels.chunk(k), book.chunk(k) if book is not None else [None] * k):
                loss, ce_pos = self.model.loss(tc, bc, lc, ignore_times=self.ignore_times, tokenizer=self.tok)
                (loss / k).backward()
                total = total + loss.detach() / k
                ce_sum = ce_pos.detach() / k if ce_sum is None else ce_sum + ce_pos.detach() / k
            self.last_ce_pos = ce_sum
        self._update(self.lr_scale(self.step_idx + 1))
        self.step_idx += 1
        if self.cp:
            dist.all_reduce(total, group=self.group)
            total = total / self.world
        return total

    def field_ce(self) -> Dict[str, float]:
        """Mean cross-entropy of the last step per message field (the reference logs it per
        field): the per-position CE of the last batch grouped by the field each position of
        a message belongs to.  Empty for encodings without per-token fields (1tok)."""
        ce = getattr(self, "last_ce_pos", None)
        tok = self.tok
        lens = np.asarray(getattr(tok, "TOK_LENS", []), np.int64)
        msg_len = int(getattr(self.model, "msg_len", 0))
        if ce is None or not len(lens) or int(lens.sum()) != msg_len:
            return {}
        field_of = np.repeat(np.arange(len(lens)), lens)               # offset in a message -> field
        offs = np.arange(msg_len)
        if self.ignore_times:
            offs = offs[(offs < tok.TIME_START_I) | (offs > tok.TIME_END_I)]
        vals = ce.float().cpu().numpy()
        if len(vals) % len(offs):
            return {}
        f = field_of[np.tile(offs, len(vals) // len(offs))]
        return {str(tok.FIELDS[i]): float(vals[f == i].mean()) for i in np.unique(f)}

    def current_lr(self) -> float:
        """The regular group's learning rate of the next step."""
        return float(self.opt.base_lr["regular"]) * self.lr_scale(self.step_idx + 1)

    def lr_scale(self, step: int) -> float:
        """The learning-rate multiple for optimizer step ``step`` (1-based)."""
        if self.cosine:
            s = cosine_schedule(step, self.warmup_steps, self.total_steps, self.lr_min_frac)
        else:
            s = step / self.warmup_steps if self.warmup_steps > 0 and step < self.warmup_steps else 1.0
        return s * self.lr_mult

    def _segment(self, tokens, labels, book):
        """This rank's segment of every sequence (context parallelism)."""
        from ..parallel.cp import split_sequence
        msg_len = self.model.msg_len
        if tokens.shape[1] % (self.world * msg_len):
            raise ValueError(f"{tokens.shape[1]} tokens do not split into whole messages over {self.world} ranks")
        book = split_sequence(book, self.group) if book is not None else None
        return split_sequence(tokens, self.group), split_sequence(labels, self.group), book

    def to_device(self, batch):
        return tuple(t.to(self.device, non_blocking=True) if t is not None else None for t in batch)

    def train_step(self, batch) -> float:
        """End-to-end step from host tensors ``(tokens, labels, book)``; returns the loss."""
        tokens, labels, book = self.to_device(batch)
        loss = self.step_device(tokens, labels, book)
        value = float(loss.item())
        if self.fused is not None:      # the loss read synchronised: the status copy has landed
            self.fused.poll()
        for mod in self.tp_fused:       # and every fused TP kernel's status word is final
            helper = getattr(mod, "fused_out", None) or getattr(mod, "fused", None)
            if helper is not None:
                helper.check()
        return value

    @torch.no_grad()
    def eval_loss(self, tokens, labels, book=None, sync: bool = True):
        """Mean loss of one batch without a parameter update (a float; a device scalar with
        ``sync=False``).  Under context parallelism each rank scores its segment and the
        segment means are averaged over the group."""
        tokens, labels, book = self.to_device((tokens, labels, book))
        was = self.model.training
        self.model.eval()
        try:
            if self.cp:
                tokens, labels, book = self._segment(tokens, labels, book)
            loss, _ = self.model.loss(tokens, book, labels, ignore_times=self.ignore_times, tokenizer=self.tok)
            loss = loss.detach().float()
            if self.cp:
                dist.all_reduce(loss, group=self.group)
                loss = loss / self.world
        finally:
            self.model.train(was)
        return float(loss) if sync else loss
