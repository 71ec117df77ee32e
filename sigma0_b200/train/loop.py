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
* periodic logs: loss, tokens/s, MFU, gradient norm, learning-rate scale.

The step itself never syncs the host; the loop reads the loss only every
``log_every`` steps (and for the NaN check at that cadence).
"""
from __future__ import annotations

import math
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional

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


@dataclass
class LoopResult:
    steps_done: int
    last_loss: float
    stopped: str                       # "done" | "nan" | "time_limit"
    history: List[Dict] = field(default_factory=list)


def fit(trainer, batches: Iterable, cfg: LoopConfig, log: Callable[[Dict], None] = None,
        watchdog: Optional[StepWatchdog] = None) -> LoopResult:
    """Train for ``cfg.steps`` optimizer steps over ``batches`` (host or device tuples)."""
    from ..ckpt import CheckpointManager
    from ..models.flops import lob_model_flops, measured_bf16_peak
    log = log or (lambda rec: print(rec, flush=True))
    barrier = (lambda: torch.distributed.barrier()) if trainer.world > 1 else None
    mgr = CheckpointManager(cfg.ckpt_dir, rank=trainer.rank, world=trainer.world, barrier=barrier,
                            fmt=cfg.ckpt_format) if cfg.ckpt_dir else None
    start = 0
    if mgr is not None and cfg.resume and mgr.latest_step() is not None:
        meta = mgr.restore(trainer)
        start = trainer.step_idx
        log({"event": "resumed", "from_step": meta["restored_step"], "trainer_step": start})
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
    while step < cfg.steps:
        batch = next(it)
        if wd:
            wd.arm(step)
        if batch[0].device.type == "cpu" and trainer.device.type == "cuda":
            batch = trainer.to_device(batch)
        loss = trainer.step_device(*batch)
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
        if mgr is not None and cfg.save_every and step % cfg.save_every == 0:
            mgr.save(step, trainer, metrics={"loss": last_loss}, config=cfg.config)
        if cfg.time_limit_s is not None and time.time() - t_begin > cfg.time_limit_s - cfg.save_margin_s:
            stopped = "time_limit"
            break
    if wd:
        wd.disarm()
    if mgr is not None and stopped != "nan":
        if not math.isfinite(last_loss):
            last_loss = float(loss)
        mgr.save(step, trainer, metrics={"loss": last_loss}, config=cfg.config, blocking=True)
        mgr.wait()
    return LoopResult(step, last_loss, stopped, hist)
