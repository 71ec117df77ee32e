"""The auto-resuming launcher (``sigma0_b200/cli/launch.py``) on CPU: a runtime that dies
after its first checkpoints is restarted and resumes; deterministic failures stop."""
import json
import os
import sys
import textwrap

import pytest

FLAKY = textwrap.dedent('''
    import os, sys
    from sigma0_b200.cli.train import main
    marker = os.environ["FLAKY_MARKER"]
    args = sys.argv[1:]
    if not os.path.exists(marker):
        open(marker, "w").close()
        i = args.index("--steps")
        main(args[:i + 1] + ["2"] + args[i + 2:])     # trains 2 steps, checkpoints them, then the process dies
        raise SystemExit(1)
    raise SystemExit(main(args))
''')


def _launch(tmp_path, module, train_args, **kw):
    from sigma0_b200.cli.launch import main
    env_pp = os.environ.get("PYTHONPATH", "")
    os.environ["PYTHONPATH"] = os.pathsep.join([str(tmp_path), os.getcwd()] + ([env_pp] if env_pp else []))
    try:
        own = ["--ckpt_dir", str(tmp_path / "ck"), "--module", module, "--backoff_s", "0"]
        for k, v in kw.items():
            own += [f"--{k}", str(v)]
        return main(own + ["--"] + train_args)
    finally:
        os.environ["PYTHONPATH"] = env_pp


TRAIN = ["--preset", "smoke", "--impl", "torch", "--synthetic", "2", "--n_messages", "4", "--micro_bsz", "2",
         "--log_every", "1", "--watchdog_timeout", "0", "--no_validation", "--steps", "4", "--save_every", "1"]


def test_launcher_restarts_and_resumes(tmp_path, monkeypatch):
    (tmp_path / "flaky_train.py").write_text(FLAKY)
    monkeypatch.setenv("FLAKY_MARKER", str(tmp_path / "marker"))
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert _launch(tmp_path, "flaky_train", TRAIN) == 0
    hist = json.load(open(tmp_path / "ck" / "launch_history.json"))
    assert [h["rc"] for h in hist] == [1, 0]
    assert hist[0]["ckpt_before"] is None and hist[0]["ckpt_after"] == 2
    assert hist[1]["ckpt_before"] == 2 and hist[1]["ckpt_after"] == 4
    assert "--ckpt_dir" in hist[1]["cmd"]


def test_launcher_stops_on_repeated_failure_without_progress(tmp_path, monkeypatch):
    (tmp_path / "always_fail.py").write_text("raise SystemExit(3)\n")
    assert _launch(tmp_path, "always_fail", [], max_stalls=2, max_restarts=5) != 0
    hist = json.load(open(tmp_path / "ck" / "launch_history.json"))
    assert len(hist) == 2 and all(h["rc"] != 0 for h in hist)


def test_launcher_does_not_restart_a_nan_stop(tmp_path):
    (tmp_path / "nan_stop.py").write_text(
        "import json, sys\n"
        "d = sys.argv[sys.argv.index('--ckpt_dir') + 1]\n"
        "json.dump({'stopped': 'nan', 'steps': 3}, open(d + '/run_status.json', 'w'))\n"
        "raise SystemExit(2)\n")
    assert _launch(tmp_path, "nan_stop", [], max_restarts=5) != 0
    hist = json.load(open(tmp_path / "ck" / "launch_history.json"))
    assert len(hist) == 1 and hist[0]["status"] == "nan"


def test_no_auto_resume_runs_once(tmp_path, monkeypatch):
    (tmp_path / "always_fail.py").write_text("raise SystemExit(3)\n")
    monkeypatch.setenv("NO_AUTO_RESUME", "1")
    assert _launch(tmp_path, "always_fail", [], max_stalls=9, max_restarts=5) != 0
    assert len(json.load(open(tmp_path / "ck" / "launch_history.json"))) == 1
