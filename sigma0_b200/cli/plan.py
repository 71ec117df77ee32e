"""Launch plans: a flat config -> the exact command that would run it (never executed).

``torchrun`` for one node; for several nodes an ``sbatch`` wrapper around
``srun torchrun`` with the rendezvous on the first node.  The config keys follow
the reference's train configs (``name``, ``sbatch_nodes``, ``sbatch_time``,
``sbatch_job_name``, ``env_*``; ``training/launch_plan.py:50``,
``inference/launch_plan.py:57``); ``gpus_per_node`` defaults to 8 (B200 HGX).
"""
from __future__ import annotations

import shlex
from dataclasses import dataclass, field
from typing import Dict, List, Tuple


@dataclass(frozen=True)
class LaunchPlan:
    name: str
    nodes: int
    gpus_per_node: int
    time_limit: str
    job_name: str
    environment: Dict[str, str]
    module: str
    args: Tuple[str, ...] = ()

    def torchrun(self, master_addr: str = "127.0.0.1", port: int = 29500) -> List[str]:
        cmd = ["env"] + [f"{k}={v}" for k, v in sorted(self.environment.items())]
        cmd += ["python", "-m", "torch.distributed.run", f"--nnodes={self.nodes}",
                f"--nproc-per-node={self.gpus_per_node}", f"--master-addr={master_addr}", f"--master-port={port}",
                "-m", self.module] + list(self.args)
        return cmd

    def sbatch(self, test_only: bool = False) -> List[str]:
        inner = ("srun --kill-on-bad-exit=1 python -m torch.distributed.run "
                 f"--nnodes={self.nodes} --nproc-per-node={self.gpus_per_node} "
                 "--rdzv-backend=c10d --rdzv-endpoint=$(scontrol show hostnames $SLURM_NODELIST | head -1):29500 "
                 f"-m {self.module} " + " ".join(shlex.quote(x) for x in self.args))
        cmd = ["env"] + [f"{k}={v}" for k, v in sorted(self.environment.items())] + ["sbatch", "--export=ALL"]
        if test_only:
            cmd.append("--test-only")
        cmd += [f"--nodes={self.nodes}", f"--gpus-per-node={self.gpus_per_node}", f"--time={self.time_limit}",
                f"--job-name={self.job_name}", f"--wrap={inner}"]
        return cmd

    def shell(self, kind: str = "auto") -> str:
        parts = self.torchrun() if (kind == "torchrun" or (kind == "auto" and self.nodes == 1)) else self.sbatch()
        return " ".join(shlex.quote(p) for p in parts)


def build_plan(config_path: str, kind: str = "train", extra_args: Tuple[str, ...] = ()) -> LaunchPlan:
    from ..utils.config import read_flat_config, with_prefix
    cfg = read_flat_config(config_path)
    nodes = int(cfg.get("sbatch_nodes", "1"))
    if nodes < 1:
        raise ValueError(f"{config_path}: sbatch_nodes must be >= 1")
    module = {"train": "sigma0_b200.cli.train", "infer": "sigma0_b200.cli.infer"}[kind]
    args = ("--config", config_path) + tuple(extra_args)
    return LaunchPlan(name=cfg.get("name", "job"), nodes=nodes, gpus_per_node=int(cfg.get("gpus_per_node", "8")),
                      time_limit=cfg.get("sbatch_time", "01:00:00"),
                      job_name=cfg.get("sbatch_job_name", f"sigma0-b200-{cfg.get('name', 'job')}"),
                      environment=with_prefix(cfg, "env_"), module=module, args=args)


def main(argv=None):
    import argparse
    p = argparse.ArgumentParser(description="print the launch command for a config (never submits)")
    p.add_argument("config")
    p.add_argument("--kind", choices=["train", "infer"], default="train")
    p.add_argument("--format", choices=["auto", "torchrun", "sbatch"], default="auto")
    a, rest = p.parse_known_args(argv)
    print(build_plan(a.config, a.kind, tuple(rest)).shell(a.format))
    return 0
