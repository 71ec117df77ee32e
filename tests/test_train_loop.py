"""Training loop: resume continuity, watchdog, NaN stop, time limit, config reader, FLOPs."""
import time

import pytest
import torch

from sigma0_b200.train.loop import LoopConfig, StepWatchdog, fit


def _args():
    from sigma0_b200.models import preset_args
    return preset_args("smoke", d_model=64, mamba3_d_state=16, mamba3_headdim=16, n_messages=4, micro_bsz=2,
                       warmup_end=0.0)


def _batches(n):
    from sigma0_b200.data import make_sequences, LobWindowDataset, collate
    ds = LobWindowDataset.from_days(make_sequences(2 * n, 5, seed=9), 4, token_mode="22tok")
    return [collate([ds[2 * i], ds[2 * i + 1]]) for i in range(n)]


def _trainer(seed=0):
    from sigma0_b200.train.trainer import Trainer
    return Trainer(_args(), device=torch.device("cpu"), total_steps=6, seed=seed)


def test_resume_matches_uninterrupted(tmp_path):
    data = _batches(6)
    a = _trainer()
    fit(a, data, LoopConfig(steps=6, log_every=3, watchdog_timeout=0), log=lambda r: None)
    b = _trainer()
    r1 = fit(b, data, LoopConfig(steps=4, log_every=2, save_every=2, ckpt_dir=str(tmp_path), watchdog_timeout=0),
             log=lambda r: None)
    assert r1.steps_done == 4
    c = _trainer(seed=3)
    events = []
    r2 = fit(c, data, LoopConfig(steps=6, log_every=2, ckpt_dir=str(tmp_path), watchdog_timeout=0), log=events.append)
    assert events[0]["event"] == "resumed" and events[0]["trainer_step"] == 4
    assert r2.steps_done == 6
    assert torch.equal(a.opt.flat, c.opt.flat)


class _Stub:
    """Trainer stand-in: configurable loss and step duration."""
    def __init__(self, losses, sleep=0.0):
        self.losses, self.sleep = list(losses), sleep
        self.world, self.rank, self.step_idx = 1, 0, 0
        self.device = torch.device("cpu")
        self.args = object()
        self.opt = type("O", (), {"last_grad_norm": None})()

    def step_device(self, *b):
        time.sleep(self.sleep)
        self.step_idx += 1
        return torch.tensor(self.losses.pop(0))


def test_nan_loss_stops():
    r = fit(_Stub([1.0, 2.0, float("nan"), 1.0]), [(torch.zeros(1, 2),)] * 4,
            LoopConfig(steps=4, log_every=1, watchdog_timeout=0), log=lambda r: None)
    assert r.stopped == "nan" and r.steps_done == 3


def test_time_limit_stops_early():
    r = fit(_Stub([1.0] * 50, sleep=0.02), [(torch.zeros(1, 2),)] * 50,
            LoopConfig(steps=50, log_every=5, watchdog_timeout=0, time_limit_s=0.2, save_margin_s=0.0),
            log=lambda r: None)
    assert r.stopped == "time_limit" and r.steps_done < 50


def test_watchdog_fires_on_a_hung_step():
    hits = []
    wd = StepWatchdog(timeout=0.05, warmup_timeout=0.05, on_timeout=hits.append)
    fit(_Stub([1.0, 1.0], sleep=0.3), [(torch.zeros(1, 2),)] * 2, LoopConfig(steps=2, log_every=1),
        log=lambda r: None, watchdog=wd)
    assert wd.fired and "exceeded" in hits[0]
    ok = []
    wd2 = StepWatchdog(timeout=5.0, on_timeout=ok.append)
    fit(_Stub([1.0, 1.0]), [(torch.zeros(1, 2),)] * 2, LoopConfig(steps=2, log_every=1), log=lambda r: None,
        watchdog=wd2)
    time.sleep(0.05)
    assert not ok


def test_flat_config_include_and_env(tmp_path):
    from sigma0_b200.utils.config import read_flat_config, env_from_config, coerce
    (tmp_path / "base.yaml").write_text("name: base\nenv_EPOCHS: 40\nsbatch_nodes: 8\n")
    (tmp_path / "child.yaml").write_text("# smoke\ninclude: base.yaml\nname: 'child'\nenv_EPOCHS: 1\n")
    c = read_flat_config(tmp_path / "child.yaml")
    assert c == {"name": "child", "env_EPOCHS": "1", "sbatch_nodes": "8"}
    assert env_from_config(c) == {"EPOCHS": "1"} and coerce("8") == 8 and coerce("True") is True
    (tmp_path / "a.yaml").write_text("include: b.yaml\n")
    (tmp_path / "b.yaml").write_text("include: a.yaml\n")
    with pytest.raises(ValueError, match="cycle"):
        read_flat_config(tmp_path / "a.yaml")


def test_flops_count_near_6n():
    from sigma0_b200.models import preset_args, build_model
    from sigma0_b200.models.flops import lob_model_flops
    a = preset_args("75m")
    n = sum(p.numel() for p in build_model(a).parameters())
    f = lob_model_flops(a)
    # projections dominate: within 2x of 6*N per token, and SSD adds a positive share
    assert 0.5 < f.train / (6 * n) < 2.0 and f.ssd_fwd > 0


def test_watchdog_covers_work_still_running_after_the_host_returns():
    """A step the host enqueued and left stays armed until its completion token turns True:
    a token that never does (a hung device) fires; one that does (a finished step) never fires."""
    hits = []
    wd = StepWatchdog(timeout=0.1, warmup_timeout=0.1, on_timeout=hits.append, poll_s=0.01)
    wd.arm(0)
    wd.watch(0, lambda: False)        # the device never finishes step 0
    time.sleep(0.3)
    assert wd.fired and "step 0 exceeded" in hits[0]
    ok = []
    wd2 = StepWatchdog(timeout=0.1, warmup_timeout=0.1, on_timeout=ok.append, poll_s=0.01)
    done = {"v": False}
    wd2.arm(0)
    wd2.watch(0, lambda: done["v"])
    time.sleep(0.03)
    assert wd2.pending() == 1
    done["v"] = True
    time.sleep(0.2)
    assert not ok and wd2.pending() == 0


def test_log_records_carry_lr_group_norms_and_field_ce():
    """Log records carry the learning rate, the gradient norm of each optimizer group and the
    cross-entropy per message field; the field means reproduce the step's mean loss."""
    import math
    import numpy as np
    recs = []
    tr = _trainer()
    fit(tr, _batches(2), LoopConfig(steps=2, log_every=1, watchdog_timeout=0), log=recs.append)
    r = recs[-1]
    assert r["lr"] > 0 and set(r["grad_norm_by_group"]) == {"ssm", "regular"}
    g = r["grad_norm_by_group"]
    assert all(math.isfinite(v) and v > 0 for v in g.values())
    fields = r["ce_by_field"]
    assert "event_type" in fields or len(fields) >= 5
    # per-field means weighted by the field widths give back the mean over positions
    lens = dict(zip(tr.tok.FIELDS, tr.tok.TOK_LENS))
    w = np.array([lens[f] for f in fields])
    mean = float((np.array(list(fields.values())) * w).sum() / w.sum())
    assert abs(mean - float(tr.last_ce_pos.mean())) < 1e-4
