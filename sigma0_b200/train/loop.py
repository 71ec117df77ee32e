"""The training loop around ``Trainer``: logging, checkpoints, resume, and failure handling.

Mirrors the reference's ``train_epoch`` / ``train`` duties
(``src/base_model/training/train_helpers.py:27-95,1033-1346``,
``run/base_model/runtime/train.py:296-325,538-790``):

* ``StepWatchdog``: a daemon monitor armed for every step until the DEVICE has
  finished it (a CUDA event recorded behind the step, polled without syncing the
  host); if a step does not finish within ``timeout`` seconds (longer during
  warm-up) the process exits with status 1, so a hung kernel or collective cannot
  hold the job forever even on steps where the loop never reads the loss;
* NaN/Inf loss -> stop without overwriting the newest (good) checkpoint;
* a time limit (e.g. the scheduler's wall clock) -> save before it is reached;
* periodic checkpoints and resume from the newest intact checkpoint, skipping
  the batches already consumed (resume-by-step at the sampler level);
* periodic logs: loss, tokens/s, MFU, gradient norm, learning-rate scale;
* validation on held-out batches every ``eval_every`` steps and at the end, with early
  stopping and reduce-on-plateau of the learning rate (the reference's
  ``early_stop_patience`` / ``lr_patience`` / ``reduce_factor``);
* a profiler trace window over a range of steps and NVTX step ranges.

The step itself never syncs the host; the loop reads the loss only every
``log_every`` steps (and for the NaN check at that cadence).
"""
from __future__ import annotations

import math
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import torch


class StepWatchdog:
    """Arm before a step; disarm after it, or hand it a completion token with ``watch``.

    A step is covered until the host returns from it (``disarm``) or, on a GPU, until
    the device has finished it: ``watch(step, done)`` keeps the step armed until
    ``done()`` returns True (e.g. a CUDA event's ``query``), so a kernel or collective
    that hangs on the device fires the watchdog even though the host enqueued the
    step and moved on.  ``on_timeout`` (default: exit 1) fires once."""

    def __init__(self, timeout: float, warmup_timeout: Optional[float] = None, warmup_steps: int = 2,
                 on_timeout: Optional[Callable[[str], None]] = None, clock=time.monotonic,
                 poll_s: Optional[float] = None):
        self.timeout, self.warmup_timeout = timeout, warmup_timeout or 4 * timeout
        self.warmup_steps = warmup_steps
        self.on_timeout = on_timeout or self._exit
        self.clock = clock
        self.poll_s = poll_s if poll_s is not None else max(0.005, min(0.5, self.timeout / 8))
        self._lock = threading.Lock()
        self._host: Optional[tuple] = None          # (step, deadline) of the step on the host
        self._device: List[tuple] = []              # (step, deadline, done) enqueued, not finished
        self._thread: Optional[threading.Thread] = None
        self.fired = False

    @staticmethod
    def _exit(msg: str) -> None:
        print(f"[watchdog] {msg}; exiting", flush=True)
        os._exit(1)

    def _limit(self, step: int) -> float:
        return self.warmup_timeout if step < self.warmup_steps else self.timeout

    def _run(self) -> None:
        while not self.fired:
            time.sleep(self.poll_s)
            now = self.clock()
            with self._lock:
                self._device = [r for r in self._device if not r[2]()]
                late = [r for r in ([self._host] if self._host else []) + self._device if now > r[1]]
            if late:
                step = min(r[0] for r in late)
                self.fired = True
                self.on_timeout(f"step {step} exceeded {self._limit(step):.0f} s")
                return

    def _ensure_thread(self) -> None:
        if self._thread is None or not self._thread.is_alive():
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def arm(self, step: int) -> None:
        with self._lock:
            self._host = (step, self.clock() + self._limit(step))
        self._ensure_thread()

    def watch(self, step: int, done: Callable[[], bool]) -> None:
        """The host is done with ``step``; keep it armed until ``done()`` is True."""
        with self._lock:
            deadline = self._host[1] if self._host and self._host[0] == step else self.clock() + self._limit(step)
            self._host = None
            self._device.append((step, deadline, done))

    def disarm(self) -> None:
        with self._lock:
            self._host = None

    def pending(self) -> int:
        """Steps the device has not finished yet."""
        with self._lock:
            return len(self._device)


@dataclass
class LoopConfig:
    steps: int
    log_every: int = 100
    save_every: int = 0                 # 0 = only at the end
    ckpt_dir: Optional[str] = None
    resume: bool = True
    watchdog_timeout: float = 900.0
    time_limit_s: Optional[float] = None    # wall-clock budget; save this long before it
    save_margin_s: float = 300.0
    config: Dict = field(default_factory=dict)
    ckpt_format: str = "native"           # "native" flat buffers or the Orbax StandardSave layout
    # trace window [start, stop) in optimizer steps (the reference's --enable_profiler: 2..20)
    profile_steps: Optional[Tuple[int, int]] = None
    profile_dir: str = "profile"
    nvtx: bool = False                    # NVTX range around every step
    # validation every eval_every steps (0: only at the end) over the val_batches callable's
    # batches; early stop after early_stop_patience evaluations without improvement; the lr
    # multiple drops by reduce_factor after lr_patience evaluations without improvement
    eval_every: int = 0
    early_stop_patience: int = 0
    # resume from this step of ckpt_dir instead of the newest (the reference's
    # --resume_from_step); or, when ckpt_dir holds nothing, initialise from another run's
    # checkpoint (--restore / --restore_step), parameters only with partial_restore, with the
    # step counter and lr schedule started over with reset_schedule
    resume_step: Optional[int] = None
    restore_dir: Optional[str] = None
    restore_step: Optional[int] = None
    partial_restore: bool = False
    reset_schedule: bool = False
    lr_patience: int = 0
    reduce_factor: float = 0.9
    # log records also carry the gradient norm per optimizer group and the CE per message field
    detailed_logs: bool = True


@dataclass
class LoopResult:
    steps_done: int
    last_loss: float
    stopped: str                       # "done" | "nan" | "time_limit" | "early_stop"
    history: List[Dict] = field(default_factory=list)
    best_val: Optional[float] = None
    trace_path: Optional[str] = None


class _Plateau:
    """Evaluation bookkeeping: best loss, evaluations since it, and the lr multiple."""

    def __init__(self, early_stop_patience: int, lr_patience: int, reduce_factor: float):
        self.best, self.since, self.since_lr = None, 0, 0
        self.esp, self.lrp, self.factor = early_stop_patience, lr_patience, reduce_factor

    def update(self, val: float, trainer) -> bool:
        """Record one validation loss; returns True when training should stop."""
        if self.best is None or val < self.best:
            self.best, self.since, self.since_lr = val, 0, 0
            return False
        self.since += 1
        self.since_lr += 1
        if self.lrp > 0 and self.since_lr >= self.lrp:
            trainer.lr_mult *= self.factor
            self.since_lr = 0
        return self.esp > 0 and self.since >= self.esp


def evaluate(trainer, batches: Iterable) -> float:
    """Mean loss over ``batches`` (averaged over the data-parallel ranks)."""
    tot, n = None, 0
    for b in batches:
        loss = trainer.eval_loss(*b, sync=False)
        tot = loss if tot is None else tot + loss
        n += 1
    if n == 0:
        return float("nan")
    val = (tot / n).reshape(1)
    if trainer.world > 1 and not getattr(trainer, "cp", False):
        torch.distributed.all_reduce(val)
        val = val / torch.distributed.get_world_size()
    return float(val)


def fit(trainer, batches: Iterable, cfg: LoopConfig, log: Callable[[Dict], None] = None,
        watchdog: Optional[StepWatchdog] = None,
        val_batches: Optional[Callable[[], Iterable]] = None) -> LoopResult:
    """Train for ``cfg.steps`` optimizer steps over ``batches`` (host or device tuples);
    ``val_batches()`` yields the held-out batches of one evaluation."""
    from ..utils.step_profile import TraceWindow
    from ..ckpt import CheckpointManager
    from ..models.flops import lob_model_flops, measured_bf16_peak
    log = log or (lambda rec: print(rec, flush=True))
    barrier = (lambda: torch.distributed.barrier()) if trainer.world > 1 else None
    mgr = CheckpointManager(cfg.ckpt_dir, rank=trainer.rank, world=trainer.world, barrier=barrier,
                            fmt=cfg.ckpt_format) if cfg.ckpt_dir else None
    start = 0
    if mgr is not None and cfg.resume and mgr.latest_step() is not None:
        meta = mgr.restore(trainer, step=cfg.resume_step)
        start = trainer.step_idx
        log({"event": "resumed", "from_step": meta["restored_step"], "trainer_step": start})
    elif cfg.restore_dir:
        src = CheckpointManager(cfg.restore_dir, rank=trainer.rank, world=trainer.world, barrier=barrier)
        meta = src.restore(trainer, step=cfg.restore_step, params_only=cfg.partial_restore)
        if cfg.reset_schedule or cfg.partial_restore:
            trainer.step_idx = 0
        start = trainer.step_idx
        log({"event": "restored", "from": cfg.restore_dir, "step": meta["restored_step"],
             "params_only": cfg.partial_restore, "trainer_step": start})
    wd = watchdog or (StepWatchdog(cfg.watchdog_timeout) if cfg.watchdog_timeout > 0 else None)
    t_begin = time.time()
    flops_tok = lob_model_flops(trainer.args).train if hasattr(trainer.args, "mamba3_d_state") else None
    peak = measured_bf16_peak()
    it = iter(batches)
    for _ in range(start):                  # resume-by-step: skip consumed batches
        next(it)
    hist: List[Dict] = []
    last_loss = float("nan")
    t0, tok_count = time.time(), 0
    step = start
    stopped = "done"
    tw = None
    if cfg.profile_steps is not None or cfg.nvtx:
        a, b = cfg.profile_steps if cfg.profile_steps is not None else (cfg.steps + 1, cfg.steps + 2)
        tw = TraceWindow(a, b, cfg.profile_dir, rank=trainer.rank, nvtx=cfg.nvtx)
    plateau = _Plateau(cfg.early_stop_patience, cfg.lr_patience, cfg.reduce_factor)

    def validate():
        v = evaluate(trainer, val_batches())
        rec = {"step": step, "val_loss": v, "lr_mult": trainer.lr_mult}
        log(rec)
        hist.append(rec)
        return plateau.update(v, trainer) if math.isfinite(v) else False

    while step < cfg.steps:
        batch = next(it)
        if wd:
            wd.arm(step)
        if batch[0].device.type == "cpu" and trainer.device.type == "cuda":
            batch = trainer.to_device(batch)
        if tw:
            tw.before(step)
        loss = trainer.step_device(*batch)
        if tw:
            tw.after(step)
        if wd and trainer.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record()
            wd.watch(step, ev.query)        # armed until the device has finished the step
        step += 1
        tok_count += batch[0].numel() * trainer.world
        if step % cfg.log_every == 0 or step == cfg.steps:
            last_loss = float(loss)             # the one host sync per log interval
            dt = time.time() - t0
            gn = trainer.opt.last_grad_norm
            rec = {"step": step, "loss": last_loss, "tokens_per_s": tok_count / max(dt, 1e-9),
                   "grad_norm": math.sqrt(float(gn)) if gn is not None else None}
            if hasattr(trainer, "current_lr"):
                rec["lr"] = trainer.current_lr()
            if cfg.detailed_logs and hasattr(trainer, "field_ce"):
                rec["grad_norm_by_group"] = trainer.opt.group_grad_norms()
                rec["ce_by_field"] = trainer.field_ce()
            if flops_tok:
                rec["mfu"] = flops_tok * rec["tokens_per_s"] / (peak * trainer.world)
            log(rec)
            hist.append(rec)
            t0, tok_count = time.time(), 0
            if not math.isfinite(last_loss):
                stopped = "nan"
                log({"event": "non-finite loss: stopping without saving the corrupted state",
                     "step": step, "newest_checkpoint": mgr.latest_step() if mgr is not None else None})
                break
        if wd:
            wd.disarm()
        if val_batches is not None and cfg.eval_every and step % cfg.eval_every == 0 and step < cfg.steps:
            if validate():
                stopped = "early_stop"
                log({"event": "early stop", "step": step, "best_val_loss": plateau.best})
                break
        if mgr is not None and cfg.save_every and step % cfg.save_every == 0:
            mgr.save(step, trainer, metrics={"loss": last_loss}, config=cfg.config)
        if cfg.time_limit_s is not None and time.time() - t_begin > cfg.time_limit_s - cfg.save_margin_s:
            stopped = "time_limit"
            break
    if wd:
        wd.disarm()
    if tw:
        tw.close()
    if val_batches is not None and stopped in ("done", "time_limit"):
        validate()
    if mgr is not None and stopped != "nan":
        if not math.isfinite(last_loss):
            last_loss = float(loss)
        mgr.save(step, trainer, metrics={"loss": last_loss}, config=cfg.config, blocking=True)
        mgr.wait()
    return LoopResult(step, last_loss, stopped, hist, plateau.best, tw.path if tw else None)
