"""Auto-resuming launcher: run the training runtime under ``torchrun`` and restart it from
the newest checkpoint when it fails.

    python -m sigma0_b200.cli launch --ckpt_dir runs/a --nproc-per-node 8 -- \
        --preset 350m --steps 20000 --save_every 500

The reference's batch script re-submits a failed job up to 20 times, restoring the
newest step checkpoint of the job's directory and remapping the resume step when the
node count (global batch) changed (``run/base_model/train_full_autoreg.batch:605-700``).
Here one process drives the attempts:

* every attempt is ``python -m torch.distributed.run ... -m <module> <args> --ckpt_dir D``
  on a fresh rendezvous port; the runtime itself resumes from the newest intact
  checkpoint of ``D`` and remaps the step when the global batch changed (the checkpoint
  records it);
* exit 0 ends the loop, and so does a non-finite-loss stop (``run_status.json``, which the
  runtime writes into ``D`` as it ends: a restart would resume from the same checkpoint
  into the same divergence; torchrun reports every worker failure as exit 1, so the
  status file, not the exit code, carries the reason);
* any other exit restarts after ``--backoff_s`` unless ``--max_restarts`` attempts are
  used or ``--max_stalls`` consecutive attempts ended without a newer checkpoint;
* ``D/launch_history.json`` records every attempt (command, exit code, checkpoint step
  before and after, wall times, host) -- the provenance the reference's launcher tests
  check.

``NO_AUTO_RESUME=1`` in the environment runs a single attempt.
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import subprocess
import sys
import time
from typing import List, Optional


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def latest_checkpoint_step(ckpt_dir: str) -> Optional[int]:
    """Newest committed step directory of ``ckpt_dir`` (digits only; temporary ``.N.tmp``
    directories of an interrupted save are ignored)."""
    if not os.path.isdir(ckpt_dir):
        return None
    steps = [int(d) for d in os.listdir(ckpt_dir)
             if d.isdigit() and os.path.exists(os.path.join(ckpt_dir, d, "metadata", "metadata"))]
    return max(steps) if steps else None


def build_command(a, train_args: List[str], port: int) -> List[str]:
    cmd = [sys.executable, "-m", "torch.distributed.run", f"--nnodes={a.nnodes}",
           f"--nproc-per-node={a.nproc_per_node}"]
    if a.nnodes > 1:
        cmd += [f"--node-rank={a.node_rank}", f"--master-addr={a.master_addr}", f"--master-port={a.master_port}"]
    else:
        cmd += ["--master-addr=127.0.0.1", f"--master-port={port}"]
    return cmd + ["-m", a.module] + list(train_args) + ["--ckpt_dir", a.ckpt_dir]


def run(a, train_args: List[str], log=print) -> int:
    os.makedirs(a.ckpt_dir, exist_ok=True)
    hist_path = os.path.join(a.ckpt_dir, "launch_history.json")
    history = []
    if os.path.exists(hist_path):
        with open(hist_path) as f:
            history = json.load(f)
    single = os.environ.get("NO_AUTO_RESUME", "") not in ("", "0")
    stalls, rc = 0, 1
    for attempt in range(1 if single else a.max_restarts + 1):
        before = latest_checkpoint_step(a.ckpt_dir)
        status_path = os.path.join(a.ckpt_dir, "run_status.json")
        if os.path.exists(status_path):
            os.remove(status_path)
        cmd = build_command(a, train_args, _free_port())
        t0 = time.time()
        log(json.dumps({"event": "launch", "attempt": attempt, "resume_from": before}))
        rc = subprocess.call(cmd, env=dict(os.environ))
        after = latest_checkpoint_step(a.ckpt_dir)
        status = None
        if os.path.exists(status_path):
            with open(status_path) as f:
                status = json.load(f).get("stopped")
        rec = {"attempt": attempt, "cmd": cmd, "rc": rc, "status": status, "ckpt_before": before,
               "ckpt_after": after, "start": t0, "end": time.time(), "host": socket.gethostname()}
        history.append(rec)
        with open(hist_path + ".tmp", "w") as f:
            json.dump(history, f, indent=1)
        os.replace(hist_path + ".tmp", hist_path)
        if rc == 0:
            log(json.dumps({"event": "finished", "attempts": attempt + 1}))
            return 0
        if status == "nan":
            log(json.dumps({"event": "stopped: non-finite loss, not restarting", "attempt": attempt}))
            return rc
        progressed = after is not None and (before is None or after > before)
        stalls = 0 if progressed else stalls + 1
        if stalls >= a.max_stalls:
            log(json.dumps({"event": f"stopped: {stalls} attempts without a new checkpoint", "rc": rc}))
            return rc
        if single or attempt == a.max_restarts:
            break
        log(json.dumps({"event": "restart", "rc": rc, "newest_checkpoint": after, "backoff_s": a.backoff_s}))
        time.sleep(a.backoff_s)
    log(json.dumps({"event": "stopped: restart limit reached" if not single else "stopped", "rc": rc}))
    return rc


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--" in argv:
        i = argv.index("--")
        own, train_args = argv[:i], argv[i + 1:]
    else:
        own, train_args = argv, []
    p = argparse.ArgumentParser(description="auto-resuming training launcher")
    p.add_argument("--ckpt_dir", required=True)
    p.add_argument("--nproc-per-node", "--nproc_per_node", dest="nproc_per_node", type=int, default=1)
    p.add_argument("--nnodes", type=int, default=1)
    p.add_argument("--node_rank", type=int, default=0)
    p.add_argument("--master_addr", default="127.0.0.1")
    p.add_argument("--master_port", type=int, default=29500)
    p.add_argument("--module", default="sigma0_b200.cli.train", help="the runtime each attempt runs")
    p.add_argument("--max_restarts", type=int, default=20)
    p.add_argument("--max_stalls", type=int, default=3,
                   help="stop after this many consecutive attempts without a newer checkpoint")
    p.add_argument("--backoff_s", type=float, default=10.0)
    a = p.parse_args(own)
    return run(a, train_args)


if __name__ == "__main__":
    raise SystemExit(main())
